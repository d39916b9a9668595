/* Forwarding header for compiling the reference's host bilinear reference
 * (benchmarks/upsample_benchmark.cu) from its own source.  The reference's
 * sources include "fpn_kernels.h" / "fpn_types.h", which its tree does not
 * contain; these shims forward to the headers it does contain and declare the
 * two C-ABI launchers (lib/kernels/memory/fast_upsample_kernels.cu:620-676)
 * that the benchmark file names before declaring them.  Oracle build only. */
#pragma once
#include "unified_fpn/core/types.h"
#include "unified_fpn/kernels/interface.h"
extern "C" {
cudaError_t launch_production_upsample_float(const float*, float*, int, int, int, int, int, int,
                                             int, float*, float*);
cudaError_t launch_production_upsample_half(const half*, half*, int, int, int, int, int, int,
                                            int, float*, float*);
}
