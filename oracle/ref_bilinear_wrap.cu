// Compiles the reference's own host bilinear reference
// (benchmarks/upsample_benchmark.cu:24-108, cpu_bilinear_upsample_reference<T>)
// from its source file and exports it with a C symbol, so the oracle's
// restatement can be checked against the reference itself.  Test
// infrastructure: built by oracle/Makefile into oracle/_ref/.
#define main ufpn_ref_upsample_benchmark_main
#include REF_UPSAMPLE_BENCH
#undef main

extern "C" __attribute__((visibility("default"))) void ref_cpu_bilinear_upsample_f32(
    const float* in, float* out, int b, int c, int ih, int iw, int oh, int ow, int align_corners) {
  cpu_bilinear_upsample_reference<float>(in, out, b, c, ih, iw, oh, ow, align_corners != 0);
}
