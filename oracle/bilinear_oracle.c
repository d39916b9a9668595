/* C restatement of the reference's host bilinear upsample -- TEST INFRASTRUCTURE.
 *
 * Follows cpu_bilinear_upsample_reference (benchmarks/upsample_benchmark.cu:24-108
 * of sanowl/-UnifiedFPN): NCHW fp32, scale = in/out (or (in-1)/(out-1) with
 * align_corners), source (o + 0.5) * scale - 0.5 clamped to [0, in-1],
 * y1 = min(y0 + 1, in - 1), weights (1-wy)(1-wx), (1-wy)wx, wy(1-wx), wy*wx.
 * Used by the tests as a second, compiled oracle and by bench.py as the
 * single-threaded CPU baseline of the upsample op; never by the library. */
#include <math.h>

static float src_coord(int o, int in, int out, int align_corners) {
  float s;
  if (align_corners) {
    const float scale = out > 1 ? (float)(in - 1) / (float)(out - 1) : 0.0f;
    s = out > 1 ? (float)o * scale : 0.0f;
  } else {
    const float scale = (float)in / (float)out;
    s = ((float)o + 0.5f) * scale - 0.5f;
  }
  if (s > (float)(in - 1)) s = (float)(in - 1);
  if (s < 0.0f) s = 0.0f;
  return s;
}

void oracle_bilinear_upsample_f32(const float* in, float* out, int n_img, int channels, int ih,
                                  int iw, int oh, int ow, int align_corners) {
  for (long plane = 0; plane < (long)n_img * channels; ++plane) {
    const float* src = in + plane * (long)ih * iw;
    float* dst = out + plane * (long)oh * ow;
    for (int y = 0; y < oh; ++y) {
      const float sy = src_coord(y, ih, oh, align_corners);
      const int y0 = (int)floorf(sy);
      const int y1 = y0 + 1 < ih ? y0 + 1 : ih - 1;
      const float wy = sy - (float)y0;
      for (int x = 0; x < ow; ++x) {
        const float sx = src_coord(x, iw, ow, align_corners);
        const int x0 = (int)floorf(sx);
        const int x1 = x0 + 1 < iw ? x0 + 1 : iw - 1;
        const float wx = sx - (float)x0;
        dst[(long)y * ow + x] = src[(long)y0 * iw + x0] * (1.0f - wy) * (1.0f - wx) +
                                src[(long)y0 * iw + x1] * (1.0f - wy) * wx +
                                src[(long)y1 * iw + x0] * wy * (1.0f - wx) +
                                src[(long)y1 * iw + x1] * wy * wx;
      }
    }
  }
}
