"""CPU oracle for the FPN neck -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
may import this module, and only as the checker (or as the timed CPU baseline).
The library never routes through it.

What it restates (paths relative to the sanowl/-UnifiedFPN source tree):

* ``bilinear_upsample_nchw`` -- the reference's host reference implementation
  ``cpu_bilinear_upsample_reference`` (benchmarks/upsample_benchmark.cu:24-108):
  scale = in/out (or (in-1)/(out-1) with align_corners), source coordinate
  (o + 0.5) * scale - 0.5 clamped to [0, in-1], y1 = min(y0 + 1, in - 1),
  corner weights (1-wy)(1-wx), (1-wy)wx, wy(1-wx), wy*wx.  Vectorised numpy,
  fp32 arithmetic in the same order.  Pinned against the reference's own
  compiled function (oracle/_ref, built by oracle/Makefile) through the golden
  vectors in tests/golden/.
* ``lateral_conv`` -- lateral_conv_kernel (lib/kernels/compute/fpn_compute_kernels.cu:127-230):
  out[o, p] = sum_c in[c, p] * W[o, c] + bias[o].
* ``fpn_neck`` -- the top-down schedule of UnifiedFPNCore::forward
  (lib/core/fpn_engine.cu:191-245) with the standard-neck semantics the library
  implements: M5 = lat(C5); M_l = lat(C_l) + up(M_{l+1}); P_l = conv3x3(M_l)
  (full 256->256, pad 1, bias); P6 = max_pool2d(P5, 1, 2).  The 3x3 conv and
  max-pool use torch's CPU kernels (the reference has no CPU version of them;
  its device kernel is a depthwise 3x3, fpn_compute_kernels.cu:277-340).
* ``fpn_neck_e4m3`` -- the same neck with e4m3 inputs/weights (per-tensor and
  per-output-channel scales = absmax / 448), quantising each merged map before its
  3x3 and storing bf16 where the CUDA schedule does; ``e4m3_round`` is the
  nearest-even e4m3fn rounding, pinned against torch's float8_e4m3fn conversion.
* ``activation`` -- activation_kernel (lib/kernels/compute/fpn_compute_kernels.cu:373-395):
  ReLU max(0, v), LeakyReLU v > 0 ? v : alpha v, Swish v / (1 + exp(-v)); the LeakyReLU
  formula is the one the reference's unit test checks (tests/unit/test_fpn_kernels.cu:270-300).
  ``fpn_neck(act=...)`` applies it to every 3x3 output (P6 taken after it).
* ``batch_norm`` -- batch_norm_kernel (fpn_compute_kernels.cu:342-371):
  (v - mean) / sqrt(var + eps) * gamma + beta per channel (eps 1e-5 at fpn_engine.cu:343-353).

Tolerances (fp32 <= 1e-4, bf16/fp16 <= 1e-2, FP8 <= 3e-2) are relative to the
largest magnitude of the reference output: ``rel_err(y, ref) = max|y - ref| / max|ref|``;
beside it every element must satisfy ``|y - ref| <= atol * rms(ref) + rtol * |ref|``
(``elem_err`` / ``check_close``, ``ELEM_TOL`` per dtype).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

TOL = {"f32": 1e-4, "f16": 1e-2, "bf16": 1e-2, "e4m3": 3e-2}


# ----------------------------------------------------------------------------- bilinear
def _src_index(out_size: int, in_size: int, align_corners: bool) -> tuple[np.ndarray, ...]:
    """Per output index: (i0, i1, w) following upsample_benchmark.cu:37-69."""
    o = np.arange(out_size, dtype=np.float32)
    if align_corners:
        scale = np.float32((in_size - 1) / (out_size - 1)) if out_size > 1 else np.float32(0)
        src = o * scale if out_size > 1 else np.zeros_like(o)
    else:
        scale = np.float32(np.float32(in_size) / np.float32(out_size))
        src = (o + np.float32(0.5)) * scale - np.float32(0.5)
    src = np.maximum(np.float32(0), np.minimum(src, np.float32(in_size - 1))).astype(np.float32)
    i0 = np.floor(src).astype(np.int64)
    i1 = np.minimum(i0 + 1, in_size - 1)
    w = (src - i0.astype(np.float32)).astype(np.float32)
    return i0, i1, w


def bilinear_upsample_nchw(x: np.ndarray, out_h: int, out_w: int, align_corners: bool = False) -> np.ndarray:
    """fp32 NCHW bilinear resize, restating upsample_benchmark.cu:24-108."""
    x = np.asarray(x, dtype=np.float32)
    _, _, H, W = x.shape
    y0, y1, wy = _src_index(out_h, H, align_corners)
    x0, x1, wx = _src_index(out_w, W, align_corners)
    wy = wy[:, None]
    wx = wx[None, :]
    v00 = x[:, :, y0][:, :, :, x0]
    v01 = x[:, :, y0][:, :, :, x1]
    v10 = x[:, :, y1][:, :, :, x0]
    v11 = x[:, :, y1][:, :, :, x1]
    one = np.float32(1)
    # same association as the reference: v00*(1-wy)*(1-wx) + v01*(1-wy)*wx + ...
    return (v00 * (one - wy) * (one - wx) + v01 * (one - wy) * wx + v10 * wy * (one - wx)
            + v11 * wy * wx).astype(np.float32)


def bilinear_upsample_t(x: torch.Tensor, size) -> torch.Tensor:
    """torch-CPU bilinear (align_corners=False), used inside the neck oracle."""
    return F.interpolate(x, size=size, mode="bilinear", align_corners=False)


# ----------------------------------------------------------------------------- neck
def lateral_conv(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """out[n, o, y, x] = sum_c x[n, c, y, x] * w[o, c] + b[o] (fpn_compute_kernels.cu:127-230)."""
    return F.conv2d(x, w.reshape(w.shape[0], -1, 1, 1), b)


def conv3x3(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return F.conv2d(x, w, b, padding=1)


def p6_maxpool(p5: torch.Tensor) -> torch.Tensor:
    return F.max_pool2d(p5, kernel_size=1, stride=2)


def activation(x: torch.Tensor, kind: str | None, alpha: float = 0.01) -> torch.Tensor:
    """activation_kernel (fpn_compute_kernels.cu:373-395), elementwise in x's dtype."""
    if kind in (None, "none"):
        return x
    if kind == "relu":
        return torch.clamp_min(x, 0.0)
    if kind == "leaky_relu":
        return torch.where(x > 0, x, alpha * x)
    if kind == "swish":
        return x / (1.0 + torch.exp(-x))
    raise ValueError(kind)


def batch_norm(x: torch.Tensor, gamma, beta, mean, var, eps: float = 1e-5) -> torch.Tensor:
    """batch_norm_kernel (fpn_compute_kernels.cu:342-371) on NCHW: per channel c,
    (x - mean[c]) / sqrt(var[c] + eps) * gamma[c] + beta[c] (gamma / beta None: 1 / 0)."""
    sh = (1, -1, 1, 1)
    y = (x - mean.reshape(sh)) / torch.sqrt(var.reshape(sh) + eps)
    if gamma is not None:
        y = y * gamma.reshape(sh)
    if beta is not None:
        y = y + beta.reshape(sh)
    return y


@dataclass
class NeckWeights:
    lat_w: list  # [256, Cin] fp32
    lat_b: list  # [256]
    out_w: list  # [256, 256, 3, 3]
    out_b: list  # [256]


def fpn_neck(feats, wts: NeckWeights, return_merged: bool = False, act: str | None = None,
             alpha: float = 0.01):
    """fp32 CPU neck.  feats: C2..C5 (NCHW float tensors).  Returns [P2, P3, P4, P5, P6];
    ``act`` is applied to each 3x3 output before P6 is taken."""
    feats = [f.float() for f in feats]
    merged = [None] * 4
    for l in (3, 2, 1, 0):
        m = lateral_conv(feats[l], wts.lat_w[l].float(), wts.lat_b[l].float())
        if l < 3:
            m = m + bilinear_upsample_t(merged[l + 1], m.shape[-2:])
        merged[l] = m
    outs = [activation(conv3x3(merged[l], wts.out_w[l].float(), wts.out_b[l].float()), act, alpha)
            for l in range(4)]
    outs.append(p6_maxpool(outs[3]))
    return (outs, merged) if return_merged else outs


def fused_lateral_upsample(c3: torch.Tensor, p4: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Single-level op: conv1x1(C3) + bilinear_upsample(P4, C3's size)."""
    return lateral_conv(c3.float(), w.float(), b.float()) + bilinear_upsample_t(p4.float(), c3.shape[-2:])


# ----------------------------------------------------------------------------- synthetic inputs
R50_CHANNELS = (256, 512, 1024, 2048)
SWIN_CHANNELS = (128, 256, 512, 1024)


def level_sizes(h: int, w: int):
    """Spatial sizes of C2..C5 for an image: strides 4, 8, 16, 32 (ceil division)."""
    return [(math.ceil(h / s), math.ceil(w / s)) for s in (4, 8, 16, 32)]


def make_features(batch, channels, sizes, seed=0, dist="relu_normal"):
    """C2..C5 as fp32 NCHW CPU tensors (generation order C2 -> C5)."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for c, (h, w) in zip(channels, sizes):
        x = torch.randn(batch, c, h, w, generator=g)
        if dist == "relu_normal":
            x = x.clamp_min(0)
        out.append(x)
    return out


def make_weights(channels, seed=1, bias_scale=0.0) -> NeckWeights:
    """Kaiming-normal (fan_in) weights, per level lateral then 3x3; biases U(-s, s) or zero."""
    g = torch.Generator().manual_seed(seed)
    lw, lb, ow, ob = [], [], [], []
    for c in channels:
        lw.append(torch.randn(256, c, generator=g) * math.sqrt(2.0 / c))
        lb.append((torch.rand(256, generator=g) * 2 - 1) * bias_scale)
        ow.append(torch.randn(256, 256, 3, 3, generator=g) * math.sqrt(2.0 / (256 * 9)))
        ob.append((torch.rand(256, generator=g) * 2 - 1) * bias_scale)
    return NeckWeights(lw, lb, ow, ob)


def config1_inputs(seed=0):
    """fp32 NCHW b1: C3 [1,512,64,64] ~N(0,1), P4 [1,256,32,32] ~N(0,1); W [256,512]
    Kaiming-normal (fan_in); bias U(-0.1, 0.1)."""
    g = torch.Generator().manual_seed(seed)
    c3 = torch.randn(1, 512, 64, 64, generator=g)
    p4 = torch.randn(1, 256, 32, 32, generator=g)
    w = torch.randn(256, 512, generator=g) * math.sqrt(2.0 / 512)
    b = (torch.rand(256, generator=g) * 2 - 1) * 0.1
    return c3, p4, w, b


# ----------------------------------------------------------------------------- FP8 (e4m3)
# The reference declares FPNDataType::FP8_E4M3 (include/unified_fpn/core/types.h:208-223)
# but has no FP8 arithmetic; the FP8 neck follows the quantisation the benchmark
# configuration states (e4m3 weights with per-output-channel scale = absmax / 448,
# activations e4m3 with a per-tensor scale = absmax / 448, fp32 accumulate, bf16 out),
# made exact so the CUDA path can be checked element by element:
#   amax > 0: inv = fp32(448 / amax), scale = fp32(amax / 448); amax == 0: inv = scale = 1
#   q = e4m3(fp32(x * inv)), round to nearest even, saturate to +-448
E4M3_MAX = 448.0


def e4m3_round(v: np.ndarray) -> np.ndarray:
    """Nearest-even rounding of fp32 values onto the e4m3fn grid (saturating at +-448):
    normals 2^-6 <= |v| have 3 fraction bits, below that the grid step is 2^-9."""
    v = np.asarray(v, dtype=np.float64)
    a = np.abs(v)
    _, ex = np.frexp(a)                      # a = m * 2^ex, m in [0.5, 1)
    step = np.ldexp(1.0, np.maximum(ex - 4, -9))
    q = np.rint(a / step) * step             # rint: ties to even
    q = np.minimum(q, E4M3_MAX)
    return (np.sign(v) * q).astype(np.float32)


def _e4m3_inv_scale(amax: np.float32):
    if amax > 0:
        return np.float32(np.float32(448.0) / amax), np.float32(amax / np.float32(448.0))
    return np.float32(1.0), np.float32(1.0)


def quantize_e4m3_tensor(x):
    """Per-tensor quantisation: returns (codes as fp32 values, scale as np.float32)."""
    x = np.asarray(torch.as_tensor(x).float().numpy(), dtype=np.float32)
    amax = np.float32(np.abs(x).max()) if x.size else np.float32(0)
    inv, scale = _e4m3_inv_scale(amax)
    return e4m3_round((x * inv).astype(np.float32)), scale


def quantize_e4m3_images(x):
    """Per-image (dim 0) quantisation: (codes fp32 like x, scales [N] fp32)."""
    x = torch.as_tensor(x).float()
    qs, ss = zip(*[quantize_e4m3_tensor(x[n]) for n in range(x.shape[0])])
    return np.stack(qs), np.array(ss, dtype=np.float32)


def quantize_e4m3_rows(w):
    """Per-output-channel (dim 0) quantisation: (codes [rows, ...] fp32, scales [rows] fp32)."""
    w = np.asarray(torch.as_tensor(w).float().numpy(), dtype=np.float32)
    rows = w.reshape(w.shape[0], -1)
    q = np.empty_like(rows)
    scales = np.empty(rows.shape[0], dtype=np.float32)
    for r in range(rows.shape[0]):
        amax = np.float32(np.abs(rows[r]).max())
        inv, scales[r] = _e4m3_inv_scale(amax)
        q[r] = e4m3_round((rows[r] * inv).astype(np.float32))
    return q.reshape(w.shape), scales


def quantize_e4m3(x: torch.Tensor, per_channel_dim: int | None = None):
    """Dequantised fp32 tensor and scale(s) of the quantisation above (per tensor, or per
    output channel for ``per_channel_dim=0``)."""
    if per_channel_dim is None:
        q, s = quantize_e4m3_tensor(x)
        return torch.from_numpy(q * s), torch.tensor(s)
    if per_channel_dim != 0:
        raise ValueError("per-channel quantisation is along dim 0 (output channels)")
    q, s = quantize_e4m3_rows(x)
    shape = [-1] + [1] * (q.ndim - 1)
    return torch.from_numpy(q * s.reshape(shape)), torch.from_numpy(s).reshape(shape)


@dataclass
class NeckWeightsE4M3:
    lat_q: list   # e4m3 codes [256, Cin] (fp32 values)
    lat_s: list   # [256] fp32
    lat_b: list
    out_q: list   # e4m3 codes [256, 256, 3, 3]
    out_s: list
    out_b: list


def quantize_neck_weights(wts: NeckWeights) -> NeckWeightsE4M3:
    lq, ls, oq, os_ = [], [], [], []
    for l in range(4):
        q, sc = quantize_e4m3_rows(wts.lat_w[l])
        lq.append(torch.from_numpy(q))
        ls.append(torch.from_numpy(sc))
        q, sc = quantize_e4m3_rows(wts.out_w[l])
        oq.append(torch.from_numpy(q))
        os_.append(torch.from_numpy(sc))
    return NeckWeightsE4M3(lq, ls, [b.float() for b in wts.lat_b], oq, os_, [b.float() for b in wts.out_b])


def _bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


def fpn_neck_e4m3(q_feats, in_scales, qw: NeckWeightsE4M3, return_merged: bool = False,
                  act: str | None = None, alpha: float = 0.01):
    """FP8 neck with the storage points of the CUDA schedule: e4m3 inputs C_l = q_l * s_l;
    laterals in fp64 from the codes, scaled by s_l * w_scale[o] (+ bias) and stored bf16;
    M_l = bf16(L_l + up(M_{l+1})) (P2: one rounding of L_2 + up(M_3)); each M_l quantised
    per image to e4m3 before its 3x3; P_l = bf16(3x3 of the dequantised codes + bias);
    P6 = P5[::2, ::2].  Returns [P2, P3, P4, P5, P6] as fp32 tensors (bf16 values)."""
    merged = [None] * 4
    for l in (3, 2, 1, 0):
        x = q_feats[l].double()
        acc = F.conv2d(x, qw.lat_q[l].double().reshape(256, -1, 1, 1))
        cs32 = torch.tensor(np.float32(in_scales[l])).float() * qw.lat_s[l]  # fp32 product
        cs = cs32.double()
        m = acc * cs.reshape(1, -1, 1, 1) + qw.lat_b[l].double().reshape(1, -1, 1, 1)
        if l == 0:
            # The P2 top-down term enters the unscaled accumulator as bilinear(M3s) with
            # M3s = bf16(M3 * fp32(1 / cs)) per channel; the epilogue's scale restores it.
            inv = (torch.ones(256) / cs32).reshape(1, -1, 1, 1)
            m3s = _bf16(merged[1] * inv)
            up = bilinear_upsample_t(m3s.double(), m.shape[-2:]) * cs.reshape(1, -1, 1, 1)
            m = _bf16((m + up).float())
        elif l < 3:
            m = _bf16((_bf16(m.float()).double() + bilinear_upsample_t(merged[l + 1].double(),
                                                                        m.shape[-2:])).float())
        else:
            m = _bf16(m.float())
        merged[l] = m
    outs = []
    for l in range(4):
        q, s = quantize_e4m3_images(merged[l])
        acc = F.conv2d(torch.from_numpy(q).double(), qw.out_q[l].double(), padding=1)
        cs = (torch.from_numpy(s).reshape(-1, 1) * qw.out_s[l].reshape(1, -1)).double()  # fp32
        outs.append(_bf16(activation((acc * cs.reshape(cs.shape[0], -1, 1, 1)
                                      + qw.out_b[l].double().reshape(1, -1, 1, 1)).float(), act, alpha)))
    outs.append(p6_maxpool(outs[3]))
    return (outs, merged) if return_merged else outs


# ----------------------------------------------------------------------------- checking
def rel_err(y, ref) -> float:
    y = torch.as_tensor(y).float()
    ref = torch.as_tensor(ref).float()
    denom = ref.abs().max().item()
    return (y - ref).abs().max().item() / (denom if denom > 0 else 1.0)


# Per-element tolerances (atol, rtol): |y - ref| <= atol * rms(ref) + rtol * |ref| for every
# element of an output level, beside the max-norm ratio above.  The floor is relative to the
# level's RMS so that one rule serves every level and scale; rtol covers the output's own
# rounding.  bf16 / fp16: 2^-6 / 2^-8 (4x the unit roundoff of the 16-bit merged maps the
# CUDA path stores between its kernels); e4m3: a code step of the e4m3 merged maps (a
# one-ulp bf16 difference before quantisation can move a code by 2^-3 relative); fp32: 2e-5.
# Measured worst case on the test configurations (B200): bf16 0.79, fp16 ~0.5, e4m3 0.48,
# fp32 0.2 of the bound.
# Gradients (grad16): 16-bit gradient maps and fp32 weight gradients summed over every pixel
# from 16-bit operands, 2^-5.
ELEM_TOL = {"f32": (2e-5, 2e-5), "f16": (2.0 ** -8, 2.0 ** -8), "bf16": (2.0 ** -6, 2.0 ** -6),
            "e4m3": (2.0 ** -3, 2.0 ** -4), "grad16": (2.0 ** -5, 2.0 ** -5)}
_TOL_KIND = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}


def elem_err(y, ref, kind: str = "bf16") -> float:
    """max over elements of |y - ref| / (atol * rms(ref) + rtol * |ref|); <= 1 passes."""
    y = torch.as_tensor(y).float()
    ref = torch.as_tensor(ref).float()
    atol, rtol = ELEM_TOL[kind]
    rms = ref.pow(2).mean().sqrt().item()
    bound = atol * (rms if rms > 0 else 1.0) + rtol * ref.abs()
    return ((y - ref).abs() / bound).max().item()


def check_close(y, ref, kind: str = "bf16", tol: float | None = None) -> tuple[float, float]:
    """Both parity metrics of one output: the max-norm ratio (<= TOL[kind], or ``tol``) and the
    per-element bound (elem_err <= 1).  Raises AssertionError naming the failing metric."""
    if isinstance(kind, torch.dtype):
        kind = _TOL_KIND[kind]
    m = rel_err(y, ref)
    e = elem_err(y, ref, kind)
    limit = TOL.get(kind, 0.0) if tol is None else tol
    if not (m <= limit and e <= 1.0):
        raise AssertionError(f"{kind}: max-norm rel err {m:.3e} (limit {limit:.1e}), "
                             f"per-element {e:.3f} of the bound (limit 1)")
    return m, e


def round_to(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Rounds fp32 values to ``dtype`` and back (the oracle's inputs for 16-bit runs)."""
    return x.to(dtype).float()
