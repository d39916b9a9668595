// Output activations applied in the 3x3 epilogues (fp32, after the bias), numbered as
// FPNActivation: 0 none, 1 ReLU, 2 LeakyReLU(alpha), 3 Swish -- the formulas of the reference's
// activation_kernel (lib/kernels/compute/fpn_compute_kernels.cu:373-395): max(0, v),
// v > 0 ? v : alpha v, v / (1 + exp(-v)).
#pragma once

namespace ufpn {

enum : int { kActNone = 0, kActRelu = 1, kActLeakyRelu = 2, kActSwish = 3 };

__device__ __forceinline__ float epilogue_act(float v, int act, float alpha) {
  if (act == kActRelu) return fmaxf(0.f, v);
  if (act == kActLeakyRelu) return v > 0.f ? v : alpha * v;
  if (act == kActSwish) return v / (1.f + expf(-v));
  return v;
}

template <int kN>
__device__ __forceinline__ void epilogue_act(float (&v)[kN], int act, float alpha) {
  if (act == kActNone) return;
#pragma unroll
  for (int i = 0; i < kN; ++i) v[i] = epilogue_act(v[i], act, alpha);
}

}  // namespace ufpn
