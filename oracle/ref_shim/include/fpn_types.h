/* Forwarding header (see fpn_kernels.h).  Oracle build only. */
#pragma once
#include "unified_fpn/core/types.h"
