// Internal include: the kernel launcher API lives in the public header.
#pragma once
#include "unified_fpn/kernels/interface.h"
