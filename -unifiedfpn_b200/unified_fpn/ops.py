"""Standalone FPN operators over the C ABI (the free functions of the reference's
extension module, python/fpn_pytorch.cpp:293-367, plus the ops it lacked).

All ops run on the tensors' CUDA device, on torch's current stream, and never
block the host.  16-bit tensors use the tensor-core / vectorised NHWC kernels
(channels_last tensors); fp32 tensors use the NCHW CUDA-core kernels.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib

_DT = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}: expected float32, float16 or bfloat16") from None


def layout_of(t: torch.Tensor) -> int:
    """NHWC if the 4-D tensor is channels_last-contiguous, NCHW if contiguous."""
    if t.dim() == 4 and t.is_contiguous(memory_format=torch.channels_last) and not (
            t.is_contiguous() and t.shape[1] > 1 and t.shape[2] * t.shape[3] > 1):
        return _lib.LAYOUT_NHWC
    if t.is_contiguous():
        return _lib.LAYOUT_NCHW
    raise ValueError("tensor must be contiguous (NCHW) or channels_last (NHWC)")


def _empty_like_layout(shape, ref: torch.Tensor, layout: int, dtype=None) -> torch.Tensor:
    mf = torch.channels_last if layout == _lib.LAYOUT_NHWC else torch.contiguous_format
    return torch.empty(shape, dtype=dtype or ref.dtype, device=ref.device, memory_format=mf)


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("all tensors must be CUDA tensors")


def fpn_lateral_conv(input: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                     coarse: torch.Tensor | None = None, cta_pair: bool = False) -> torch.Tensor:
    """1x1 lateral conv + bias, optionally fused with the top-down upsample-add:
    ``out = conv1x1(input, weight) + bias [+ bilinear_upsample(coarse, input size)]``.

    Reference: fpn_lateral_conv (python/fpn_pytorch.cpp:293-326) ->
    lateral_conv_kernel (lib/kernels/compute/fpn_compute_kernels.cu:127-230).
    ``weight`` is [Cout, Cin] or [Cout, Cin, 1, 1]; ``bias`` [Cout] (fp32).
    fp32 input: NCHW, any Cout.  16-bit input: channels_last, Cout = 256.
    ``cta_pair`` (16-bit, Cin <= 256): the CTA-pair kernel with resident weights.
    """
    _check_cuda(input, weight, bias, coarse)
    if input.dim() != 4:
        raise ValueError("input must be 4-D [N, C, H, W]")
    N, Cin, H, W = input.shape
    Cout = weight.shape[0]
    if weight.numel() != Cout * Cin:
        raise ValueError("weight must be [Cout, Cin] or [Cout, Cin, 1, 1]")
    dt = dtype_code(input)
    if dt == _lib.DTYPE_F32:
        input = input.contiguous()
        lay = _lib.LAYOUT_NCHW
    else:
        input = input.contiguous(memory_format=torch.channels_last)
        lay = _lib.LAYOUT_NHWC
    w = weight.reshape(Cout, Cin).to(device=input.device, dtype=input.dtype).contiguous()
    b = bias.to(device=input.device, dtype=torch.float32).contiguous()
    Hc = Wc = 0
    if coarse is not None:
        if coarse.dtype != input.dtype or coarse.shape[0] != N or coarse.shape[1] != Cout:
            raise ValueError("coarse must match the output's dtype, batch and channels")
        coarse = coarse.contiguous(memory_format=torch.channels_last if lay == _lib.LAYOUT_NHWC
                                   else torch.contiguous_format)
        Hc, Wc = coarse.shape[2], coarse.shape[3]
    out = _empty_like_layout((N, Cout, H, W), input, lay)
    if cta_pair:
        if dt == _lib.DTYPE_F32 or Cout != 256:
            raise ValueError("the CTA-pair lateral takes bf16 / fp16 input and Cout = 256")
        check(lib.ufpn_lateral_conv_pair(dt, input.data_ptr(), w.data_ptr(), b.data_ptr(),
                                         coarse.data_ptr() if coarse is not None else None,
                                         out.data_ptr(), N, Cin, H, W, Hc, Wc, _stream(input)),
              "ufpn_lateral_conv_pair")
        return out
    check(lib.ufpn_lateral_conv(dt, lay, input.data_ptr(), w.data_ptr(), b.data_ptr(),
                                coarse.data_ptr() if coarse is not None else None, out.data_ptr(),
                                N, Cin, H, W, Cout, Hc, Wc, _stream(input)), "ufpn_lateral_conv")
    return out


def pack_conv3x3_weight(weight: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """[256, 256, 3, 3] fp32 -> [256, 9, 256] (K-major) in ``dtype`` for the tensor-core 3x3."""
    Cout, Cin = weight.shape[0], weight.shape[1]
    w32 = weight.to(dtype=torch.float32).contiguous()
    out = torch.empty((Cout, 9, Cin), dtype=dtype, device=weight.device)
    check(lib.ufpn_pack_conv3x3_weights(_DT[dtype], w32.data_ptr(), out.data_ptr(), Cout, Cin,
                                        _stream(weight)), "ufpn_pack_conv3x3_weights")
    return out


_ACTIVATIONS = {None: 0, "none": 0, "relu": 1, "leaky_relu": 2, "swish": 3}


def fpn_conv3x3(input: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, p6: bool = False,
                tile_w: int = 0, activation: str | None = None, alpha: float = 0.01):
    """3x3 pad-1 output conv (256 -> 256) + bias; with ``p6=True`` also returns
    P6 = max_pool2d(out, 1, 2).  ``weight`` is [256, 256, 3, 3] (any float dtype)
    or, for 16-bit inputs, already packed [256, 9, 256] by :func:`pack_conv3x3_weight`.
    ``tile_w``: 0 = 8x16 halo tiles, -1 = halo tiles on CTA pairs, -2 / -3 = the same on the
    map's transposed view (16 columns x 8 rows per tile; not with ``p6``), -4 / -5 = a mixed
    tiling (the own view for the whole 16-row tile rows, the transposed view for the last
    1..8 rows; not with ``p6``), 8..128 = plain tiles.
    ``activation`` ("relu", "leaky_relu" with negative slope ``alpha``, "swish") is applied
    in the epilogue after the bias (P6 comes from the activated output); reference:
    activation_kernel (lib/kernels/compute/fpn_compute_kernels.cu:373-395).
    """
    if activation not in _ACTIVATIONS:
        raise ValueError(f"unknown activation {activation!r}")
    _check_cuda(input, weight, bias)
    N, C, H, W = input.shape
    if C != 256:
        raise ValueError("the output conv maps 256 -> 256 channels")
    dt = dtype_code(input)
    if dt == _lib.DTYPE_F32:
        x = input.contiguous()
        w = weight.to(torch.float32).contiguous()
        lay = _lib.LAYOUT_NCHW
    else:
        x = input.contiguous(memory_format=torch.channels_last)
        w = weight if (weight.dim() == 3 and weight.dtype == input.dtype) else pack_conv3x3_weight(
            weight, input.dtype)
        lay = _lib.LAYOUT_NHWC
    b = bias.to(device=input.device, dtype=torch.float32).contiguous()
    out = _empty_like_layout((N, 256, H, W), x, lay)
    p6t = _empty_like_layout((N, 256, (H - 1) // 2 + 1, (W - 1) // 2 + 1), x, lay) if p6 else None
    check(lib.ufpn_conv3x3_act(dt, x.data_ptr(), w.data_ptr(), b.data_ptr(), out.data_ptr(),
                               p6t.data_ptr() if p6t is not None else None, N, H, W, tile_w,
                               _ACTIVATIONS[activation], float(alpha), _stream(x)), "ufpn_conv3x3")
    return (out, p6t) if p6 else out


def fold_batch_norm(weight: torch.Tensor, bias: torch.Tensor | None, bn_weight: torch.Tensor | None,
                    bn_bias: torch.Tensor | None, running_mean: torch.Tensor, running_var: torch.Tensor,
                    eps: float = 1e-5) -> tuple[torch.Tensor, torch.Tensor]:
    """Folds an inference BatchNorm that follows a conv into the conv's weight and bias:
    ``conv(x, W', b') == batch_norm(conv(x, W, b))`` with W' = W * s, b' = (b - mean) * s + beta,
    s = gamma / sqrt(var + eps) per output channel (fp32 results on the CPU, computed in double
    by the library's host code).  Reference: batch_norm_kernel
    (lib/kernels/compute/fpn_compute_kernels.cu:342-371), run with eps 1e-5 after every output
    conv (lib/core/fpn_engine.cu:343-353)."""
    cout = weight.shape[0]

    def host(t):
        return None if t is None else t.detach().to(device="cpu", dtype=torch.float32).contiguous()

    w = host(weight)
    vecs = [host(t) for t in (bias, bn_weight, bn_bias, running_mean, running_var)]
    for v in vecs:
        if v is not None and v.numel() != cout:
            raise ValueError("bias and BatchNorm parameters need one value per output channel")
    out_w = torch.empty_like(w)
    out_b = torch.empty(cout, dtype=torch.float32)
    ptr = [None if v is None else v.data_ptr() for v in vecs]
    check(lib.ufpn_fold_batch_norm(w.data_ptr(), ptr[0], ptr[1], ptr[2], ptr[3], ptr[4], float(eps), cout,
                                   w.numel() // cout, out_w.data_ptr(), out_b.data_ptr()),
          "ufpn_fold_batch_norm")
    return out_w, out_b


def fpn_upsample_add(coarse: torch.Tensor, lateral: torch.Tensor | None = None,
                     size: tuple[int, int] | None = None, align_corners: bool = False) -> torch.Tensor:
    """``lateral + bilinear_upsample(coarse, lateral's H x W)`` (or a pure upsample to
    ``size`` when ``lateral`` is None).  Reference: launch_upsample_and_add
    (lib/core/fpn_engine.cu:274-313)."""
    _check_cuda(coarse, lateral)
    dt = dtype_code(coarse)
    lay = layout_of(coarse)
    N, C, Hc, Wc = coarse.shape
    if lateral is not None:
        if lateral.dtype != coarse.dtype or lateral.shape[:2] != coarse.shape[:2]:
            raise ValueError("lateral must match coarse in dtype, batch and channels")
        H, W = lateral.shape[2], lateral.shape[3]
        lateral = lateral.contiguous(memory_format=torch.channels_last if lay == _lib.LAYOUT_NHWC
                                     else torch.contiguous_format)
    else:
        if size is None:
            raise ValueError("size is required without a lateral tensor")
        H, W = size
    out = _empty_like_layout((N, C, H, W), coarse, lay)
    check(lib.ufpn_upsample_add(dt, lay, coarse.data_ptr(),
                                lateral.data_ptr() if lateral is not None else None, out.data_ptr(),
                                N, C, Hc, Wc, H, W, int(align_corners), _stream(coarse)),
          "ufpn_upsample_add")
    return out


def fpn_merge_two_levels(m5: torch.Tensor, l4: torch.Tensor, l3: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Two top-down steps in one launch: ``M4 = l4 + up(m5)``, ``M3 = l3 + up(M4)``
    (channels-last, 256 channels, bf16 / fp16, each map upsampling to the next).  Returns
    (M4, M3); bitwise the same as two ``fpn_upsample_add`` calls.  Reference: two iterations
    of the top-down loop, lib/core/fpn_engine.cu:230-245 with launch_upsample_and_add
    (:274-313)."""
    _check_cuda(m5, l4, l3)
    dt = dtype_code(m5)
    for t in (m5, l4, l3):
        if t.dtype != m5.dtype or t.shape[1] != 256 or t.shape[0] != m5.shape[0]:
            raise ValueError("m5, l4, l3 must share dtype and batch and have 256 channels")
    cl = torch.channels_last
    m5, l4 = m5.contiguous(memory_format=cl), l4.contiguous(memory_format=cl)
    m3 = l3.contiguous(memory_format=cl).clone(memory_format=cl)
    m4 = torch.empty_like(l4, memory_format=cl)
    N = m5.shape[0]
    check(lib.ufpn_merge_two_levels(dt, m5.data_ptr(), l4.data_ptr(), m4.data_ptr(), m3.data_ptr(), N,
                                    m5.shape[2], m5.shape[3], l4.shape[2], l4.shape[3], l3.shape[2],
                                    l3.shape[3], _stream(m5)), "ufpn_merge_two_levels")
    return m4, m3


# ----------------------------------------------------------------------------- backward
def _cl16(t: torch.Tensor, what: str) -> torch.Tensor:
    if t.dtype not in (torch.bfloat16, torch.float16):
        raise ValueError(f"{what} must be bfloat16 or float16")
    return t.contiguous(memory_format=torch.channels_last)


def fpn_lateral_conv_backward(input: torch.Tensor, weight: torch.Tensor, grad_output: torch.Tensor,
                              need_input_grad: bool = True, weight_t: torch.Tensor | None = None):
    """Gradients of ``fpn_lateral_conv(input, weight, bias)`` (16-bit, channels_last,
    Cout = 256): ``(grad_input, grad_weight [256, Cin] fp32, grad_bias [256] fp32)``;
    grad_input is None without ``need_input_grad``.  Reference: backward_lateral_conv_kernel
    (src/training/backward/lateral_conv_backward.cu:7-143), here deterministic: the weight
    gradient is a tensor-core GEMM over pixels, the input gradient the forward kernel with
    the transposed weights.  ``weight_t``: the weights already in that transposed layout
    ([ceil(Cin/256)*256, 256] in the input's dtype, ``prepare_neck_weights``); ``weight`` is
    then not read."""
    _check_cuda(input, weight, grad_output, weight_t)
    x = _cl16(input, "input")
    g = _cl16(grad_output, "grad_output")
    N, Cin, H, W = x.shape
    if g.dtype != x.dtype or tuple(g.shape) != (N, 256, H, W):
        raise ValueError("grad_output must be [N, 256, H, W] in the input's dtype")
    gx = torch.empty_like(x, memory_format=torch.channels_last) if need_input_grad else None
    gw = torch.empty(256, Cin, device=x.device, dtype=torch.float32)
    gb = torch.empty(256, device=x.device, dtype=torch.float32)
    if weight_t is not None:
        if weight_t.dtype != x.dtype or tuple(weight_t.shape) != ((Cin + 255) // 256 * 256, 256):
            raise ValueError("weight_t must be [ceil(Cin/256)*256, 256] in the input's dtype")
        check(lib.ufpn_lateral_conv_backward_t(dtype_code(x), x.data_ptr(), weight_t.contiguous().data_ptr(),
                                               g.data_ptr(), gx.data_ptr() if gx is not None else None,
                                               gw.data_ptr(), gb.data_ptr(), N, Cin, H, W, _stream(x)),
              "ufpn_lateral_conv_backward_t")
        return gx, gw, gb
    w = weight.reshape(256, Cin).to(device=x.device, dtype=x.dtype).contiguous()
    check(lib.ufpn_lateral_conv_backward(dtype_code(x), x.data_ptr(), w.data_ptr(), g.data_ptr(),
                                         gx.data_ptr() if gx is not None else None, gw.data_ptr(),
                                         gb.data_ptr(), N, Cin, H, W, _stream(x)),
          "ufpn_lateral_conv_backward")
    return gx, gw, gb


def fpn_conv3x3_backward(input: torch.Tensor, weight: torch.Tensor, grad_output: torch.Tensor,
                         need_input_grad: bool = True, weight_flipped: torch.Tensor | None = None):
    """Gradients of the 256 -> 256 pad-1 3x3 conv (``fpn_conv3x3``; 16-bit, channels_last):
    ``(grad_input, grad_weight [256, 256, 3, 3] fp32, grad_bias [256] fp32)``.  ``weight`` is
    [256, 256, 3, 3] (any float dtype) or packed [256, 9, 256] by ``pack_conv3x3_weight``.  The input
    gradient is the forward 3x3 kernel with the weights transposed in channels and flipped in
    space; the weight gradient is a tensor-core GEMM over pixels (nine shifted taps).
    ``weight_flipped``: the weights already in that flipped layout ([256 c, 9, 256 o] in the
    input's dtype, ``prepare_neck_weights``); ``weight`` is then not read."""
    _check_cuda(input, weight, grad_output, weight_flipped)
    x = _cl16(input, "input")
    g = _cl16(grad_output, "grad_output")
    N, C, H, W = x.shape
    if C != 256 or g.dtype != x.dtype or tuple(g.shape) != (N, 256, H, W):
        raise ValueError("input and grad_output must be [N, 256, H, W] of one dtype")
    gx = torch.empty_like(x, memory_format=torch.channels_last) if need_input_grad else None
    gw = torch.empty(256, 256, 3, 3, device=x.device, dtype=torch.float32)
    gb = torch.empty(256, device=x.device, dtype=torch.float32)
    if weight_flipped is not None:
        if weight_flipped.dtype != x.dtype or tuple(weight_flipped.shape) != (256, 9, 256):
            raise ValueError("weight_flipped must be [256, 9, 256] in the input's dtype")
        check(lib.ufpn_conv3x3_backward_f(dtype_code(x), x.data_ptr(), weight_flipped.contiguous().data_ptr(),
                                          g.data_ptr(), gx.data_ptr() if gx is not None else None,
                                          gw.data_ptr(), gb.data_ptr(), N, H, W, _stream(x)),
              "ufpn_conv3x3_backward_f")
        return gx, gw, gb
    wp = weight if (weight.dim() == 3 and weight.dtype == x.dtype) else pack_conv3x3_weight(weight, x.dtype)
    wp = wp.contiguous()
    check(lib.ufpn_conv3x3_backward(dtype_code(x), x.data_ptr(), wp.data_ptr(), g.data_ptr(),
                                    gx.data_ptr() if gx is not None else None, gw.data_ptr(),
                                    gb.data_ptr(), N, H, W, _stream(x)), "ufpn_conv3x3_backward")
    return gx, gw, gb


def prepare_neck_weights(lateral_w, output_w, dtype: torch.dtype, backward: bool = True):
    """Every per-step layout of the training path's weights from the fp32 masters in ONE
    launch: ``(lateral [256, Cin], lateral_t [ceil(Cin/256)*256, 256], packed 3x3 [256, 9,
    256], flipped 3x3 [256, 9, 256])`` as lists over the levels, in ``dtype`` (the last two
    lists are None without ``backward``).  ``lateral_w``: [256, Cin] (or [256, Cin, 1, 1]),
    ``output_w``: [256, 256, 3, 3]; fp32 CUDA tensors."""
    if dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("weights are prepared in bf16 or fp16")
    n = len(lateral_w)
    if n != len(output_w) or not 1 <= n <= 4:
        raise ValueError("one lateral and one 3x3 weight per level (1..4 levels)")
    lat = [w.detach().reshape(256, -1).to(torch.float32).contiguous() for w in lateral_w]
    conv = [w.detach().to(torch.float32).contiguous() for w in output_w]
    _check_cuda(*lat, *conv)
    dev = lat[0].device
    cin = [w.shape[1] for w in lat]
    if any(tuple(w.shape) != (256, 256, 3, 3) for w in conv):
        raise ValueError("3x3 weights must be [256, 256, 3, 3]")
    lat16 = [torch.empty(256, c, device=dev, dtype=dtype) for c in cin]
    packed = [torch.empty(256, 9, 256, device=dev, dtype=dtype) for _ in conv]
    lat_t = [torch.empty((c + 255) // 256 * 256, 256, device=dev, dtype=dtype) for c in cin] if backward else None
    flipped = [torch.empty(256, 9, 256, device=dev, dtype=dtype) for _ in conv] if backward else None
    P = _lib.c_void_p * n

    def ptrs(ts):
        return P(*[t.data_ptr() for t in ts]) if ts is not None else None
    check(lib.ufpn_prepare_neck_weights(_DT[dtype], n, ptrs(lat), (_lib.c_int * n)(*cin), ptrs(conv),
                                        ptrs(lat16), ptrs(lat_t), ptrs(packed), ptrs(flipped),
                                        _stream(lat[0])), "ufpn_prepare_neck_weights")
    return lat16, lat_t, packed, flipped


def fpn_upsample_add_backward(grad_output: torch.Tensor, coarse_size: tuple[int, int],
                              base: torch.Tensor | None = None) -> torch.Tensor:
    """Gradient of the coarse input of ``fpn_upsample_add(coarse, lateral)``:
    ``base + bilinear^T(grad_output)`` (the lateral's gradient is grad_output itself).
    channels_last; the exact adjoint of the forward's clamped half-pixel taps.  Reference:
    backward_upsample_add_kernel (src/training/backward/upsample_backward.cu:4-80)."""
    _check_cuda(grad_output, base)
    g = grad_output.contiguous(memory_format=torch.channels_last)
    N, C, H, W = g.shape
    Hc, Wc = coarse_size
    out = torch.empty(N, C, Hc, Wc, device=g.device, dtype=g.dtype, memory_format=torch.channels_last)
    if base is not None:
        base = base.to(dtype=g.dtype).contiguous(memory_format=torch.channels_last)
        if tuple(base.shape) != (N, C, Hc, Wc):
            raise ValueError("base must have the coarse map's shape")
    check(lib.ufpn_upsample_add_backward(dtype_code(g), g.data_ptr(),
                                         base.data_ptr() if base is not None else None, out.data_ptr(),
                                         N, C, Hc, Wc, H, W, _stream(g)), "ufpn_upsample_add_backward")
    return out


def fpn_p6_backward(grad_p6: torch.Tensor, grad_p5: torch.Tensor) -> torch.Tensor:
    """Adds the gradient of P6 = P5[:, :, ::2, ::2] into ``grad_p5`` (channels_last, in place;
    returned)."""
    _check_cuda(grad_p6, grad_p5)
    if not grad_p5.is_contiguous(memory_format=torch.channels_last):
        raise ValueError("grad_p5 must be channels_last (it is updated in place)")
    g6 = grad_p6.to(dtype=grad_p5.dtype).contiguous(memory_format=torch.channels_last)
    N, C, H5, W5 = grad_p5.shape
    check(lib.ufpn_p6_backward(dtype_code(grad_p5), g6.data_ptr(), grad_p5.data_ptr(), N, C, H5, W5,
                               _stream(grad_p5)), "ufpn_p6_backward")
    return grad_p5


def fpn_upsample_bilinear(input: torch.Tensor, scale_factor: float) -> torch.Tensor:
    """Bilinear upsample by ``scale_factor``; output size = int(in * scale), sampled
    with scale = in / out (half-pixel, align_corners=False).
    Reference: fpn_upsample_bilinear (python/fpn_pytorch.cpp:328-358)."""
    H = int(input.shape[2] * scale_factor)
    W = int(input.shape[3] * scale_factor)
    return fpn_upsample_add(input, None, size=(H, W))


def fpn_p6(p5: torch.Tensor) -> torch.Tensor:
    """P6 = max_pool2d(P5, kernel_size=1, stride=2)."""
    _check_cuda(p5)
    dt = dtype_code(p5)
    lay = layout_of(p5)
    N, C, H, W = p5.shape
    out = _empty_like_layout((N, C, (H - 1) // 2 + 1, (W - 1) // 2 + 1), p5, lay)
    check(lib.ufpn_p6_maxpool(dt, lay, p5.data_ptr(), out.data_ptr(), N, C, H, W, _stream(p5)),
          "ufpn_p6_maxpool")
    return out


# ----------------------------------------------------------------------------- e4m3 (FP8)
E4M3 = torch.float8_e4m3fn


def quantize_fp8(x: torch.Tensor, per_image: bool = False):
    """Symmetric e4m3 quantisation on the device: returns ``(q, scale)`` with ``q``
    float8_e4m3fn in ``x``'s memory format and ``scale`` fp32 on the device, one element
    (per tensor) or one per image along dim 0 (``per_image``); ``x ~ q * scale`` with
    scale = absmax / 448 and q = e4m3(x * 448 / absmax), rounded to nearest even and
    saturated."""
    _check_cuda(x)
    dt = dtype_code(x)
    nhwc = x.dim() == 4 and layout_of(x) == _lib.LAYOUT_NHWC
    mf = torch.channels_last if nhwc else torch.contiguous_format
    x = x.contiguous(memory_format=mf)
    groups = int(x.shape[0]) if per_image else 1
    q = torch.empty_like(x, dtype=E4M3, memory_format=mf)
    amax = torch.empty(groups, dtype=torch.int32, device=x.device)
    scale = torch.empty(groups, dtype=torch.float32, device=x.device)
    check(lib.ufpn_quantize_e4m3(dt, x.data_ptr(), x.numel(), groups, amax.data_ptr(), q.data_ptr(),
                                 scale.data_ptr(), _stream(x)), "ufpn_quantize_e4m3")
    return q, scale


def quantize_fp8_rows(weight: torch.Tensor, pack3x3: bool = False):
    """Per-output-channel e4m3 quantisation of fp32 weights: ``(q, scales)``.  Lateral
    [Cout, Cin] (or [Cout, Cin, 1, 1]) -> q [Cout, Cin]; with ``pack3x3`` a 3x3 kernel
    [Cout, Cin, 3, 3] -> q [Cout, 9, Cin] (the K order of :func:`fpn_conv3x3_fp8`)."""
    _check_cuda(weight)
    Cout = weight.shape[0]
    w = weight.to(torch.float32).contiguous()
    cols = w.numel() // Cout
    if pack3x3:
        if w.dim() != 4 or w.shape[2:] != (3, 3):
            raise ValueError("pack3x3 needs a [Cout, Cin, 3, 3] kernel")
        cin = w.shape[1]
        q = torch.empty((Cout, 9, cin), dtype=E4M3, device=w.device)
    else:
        cin = 0
        q = torch.empty((Cout, cols), dtype=E4M3, device=w.device)
    scales = torch.empty(Cout, dtype=torch.float32, device=w.device)
    check(lib.ufpn_quantize_e4m3_rows(w.data_ptr(), Cout, cols, cin, q.data_ptr(), scales.data_ptr(),
                                      _stream(w)), "ufpn_quantize_e4m3_rows")
    return q, scales


def _fp8_nhwc(x: torch.Tensor) -> torch.Tensor:
    if x.dtype != E4M3:
        raise TypeError("expected a float8_e4m3fn tensor")
    return x.contiguous(memory_format=torch.channels_last)


def _scale_ptr(scale, device, n_images):
    """(scale tensor, per_image flag): one element = per tensor, n_images = per image."""
    s = torch.as_tensor(scale, dtype=torch.float32).to(device).reshape(-1).contiguous()
    if s.numel() == 1:
        return s, 0
    if s.numel() == n_images:
        return s, 1
    raise ValueError("an activation scale has 1 element (per tensor) or N (per image)")


def fpn_lateral_conv_fp8(input: torch.Tensor, input_scale, weight: torch.Tensor,
                         weight_scales: torch.Tensor, bias: torch.Tensor,
                         coarse: torch.Tensor | None = None,
                         amax_out: torch.Tensor | None = None) -> torch.Tensor:
    """FP8 lateral: ``out = (q_x . q_w^T) * (scale_x * scale_w[o]) + bias[o]
    [+ bilinear(coarse)]`` on the e4m3 tensor cores, bf16 out (channels_last).
    ``input`` e4m3 [N, Cin, H, W]; ``weight`` e4m3 [256, Cin] with ``weight_scales`` [256];
    ``coarse`` bf16 [N, 256, Hc, Wc] or None; ``input_scale`` 1 (per tensor) or N (per
    image) elements; ``amax_out`` (int32 CUDA [N], optional, zeroed by the caller) receives
    the per-image atomicMax of |out| as fp32 bits."""
    _check_cuda(input, weight, weight_scales, bias, coarse, amax_out)
    x = _fp8_nhwc(input)
    N, Cin, H, W = x.shape
    w = weight.reshape(weight.shape[0], -1).contiguous()
    if w.dtype != E4M3 or w.shape != (256, Cin):
        raise ValueError("weight must be e4m3 [256, Cin]")
    ws = weight_scales.to(torch.float32).contiguous()
    b = bias.to(device=x.device, dtype=torch.float32).contiguous()
    xs, per_img = _scale_ptr(input_scale, x.device, N)
    Hc = Wc = 0
    if coarse is not None:
        if coarse.dtype != torch.bfloat16 or coarse.shape[:2] != (N, 256):
            raise ValueError("coarse must be bf16 [N, 256, Hc, Wc]")
        coarse = coarse.contiguous(memory_format=torch.channels_last)
        Hc, Wc = coarse.shape[2], coarse.shape[3]
    out = torch.empty((N, 256, H, W), dtype=torch.bfloat16, device=x.device,
                      memory_format=torch.channels_last)
    check(lib.ufpn_lateral_conv_e4m3(x.data_ptr(), xs.data_ptr(), per_img, w.data_ptr(), ws.data_ptr(),
                                     b.data_ptr(), coarse.data_ptr() if coarse is not None else None,
                                     out.data_ptr(), N, Cin, H, W, Hc, Wc,
                                     amax_out.data_ptr() if amax_out is not None else None,
                                     _stream(x)), "ufpn_lateral_conv_e4m3")
    return out


def fpn_conv3x3_fp8(input: torch.Tensor, input_scale, weight: torch.Tensor,
                    weight_scales: torch.Tensor, bias: torch.Tensor, p6: bool = False,
                    tile_w: int = 0):
    """FP8 3x3 pad-1 conv 256 -> 256 (+ optional P6): ``input`` e4m3 [N, 256, H, W];
    ``weight`` e4m3 packed [256, 9, 256] from :func:`quantize_fp8_rows` (pack3x3=True) with
    ``weight_scales`` [256]; ``input_scale`` 1 (per tensor) or N (per image) elements;
    bf16 channels_last out."""
    _check_cuda(input, weight, weight_scales, bias)
    x = _fp8_nhwc(input)
    N, C, H, W = x.shape
    if C != 256 or weight.dtype != E4M3 or tuple(weight.shape) != (256, 9, 256):
        raise ValueError("expects 256 channels and an e4m3 weight packed [256, 9, 256]")
    ws = weight_scales.to(torch.float32).contiguous()
    b = bias.to(device=x.device, dtype=torch.float32).contiguous()
    xs, per_img = _scale_ptr(input_scale, x.device, N)
    out = torch.empty((N, 256, H, W), dtype=torch.bfloat16, device=x.device,
                      memory_format=torch.channels_last)
    p6t = torch.empty((N, 256, (H - 1) // 2 + 1, (W - 1) // 2 + 1), dtype=torch.bfloat16,
                      device=x.device, memory_format=torch.channels_last) if p6 else None
    check(lib.ufpn_conv3x3_e4m3(x.data_ptr(), xs.data_ptr(), per_img, weight.contiguous().data_ptr(),
                                ws.data_ptr(), b.data_ptr(), out.data_ptr(),
                                p6t.data_ptr() if p6t is not None else None, N, H, W, tile_w,
                                None, _stream(x)), "ufpn_conv3x3_e4m3")
    return (out, p6t) if p6 else out


def fpn_conv3x3_fp8_from_bf16(input: torch.Tensor, amax_bits: torch.Tensor, weight: torch.Tensor,
                              weight_scales: torch.Tensor, bias: torch.Tensor, p6: bool = False):
    """FP8 3x3 on CTA pairs that quantises its bf16 ``input`` per image inside the kernel:
    ``amax_bits`` (int32 [N]) holds each image's absmax as fp32 bits; the result equals
    ``fpn_conv3x3_fp8(*quantize_fp8(input, per_image=True), ...)`` bit for bit."""
    _check_cuda(input, amax_bits, weight, weight_scales, bias)
    x = input.contiguous(memory_format=torch.channels_last)
    N, C, H, W = x.shape
    if x.dtype != torch.bfloat16 or C != 256 or weight.dtype != E4M3:
        raise ValueError("expects a bf16 [N, 256, H, W] input and an e4m3 packed weight")
    ws = weight_scales.to(torch.float32).contiguous()
    b = bias.to(device=x.device, dtype=torch.float32).contiguous()
    out = torch.empty((N, 256, H, W), dtype=torch.bfloat16, device=x.device,
                      memory_format=torch.channels_last)
    p6t = torch.empty((N, 256, (H - 1) // 2 + 1, (W - 1) // 2 + 1), dtype=torch.bfloat16,
                      device=x.device, memory_format=torch.channels_last) if p6 else None
    check(lib.ufpn_conv3x3_e4m3_from_bf16(x.data_ptr(), amax_bits.contiguous().data_ptr(),
                                          weight.contiguous().data_ptr(), ws.data_ptr(), b.data_ptr(),
                                          out.data_ptr(), p6t.data_ptr() if p6t is not None else None,
                                          N, H, W, _stream(x)), "ufpn_conv3x3_e4m3_from_bf16")
    return (out, p6t) if p6 else out


def device_status(reset: bool = True) -> int:
    """Status word of the standalone tensor-core ops on the current device (0 = ok)."""
    v = _lib.c_int(0)
    check(lib.ufpn_device_status(int(reset), _lib.ctypes.byref(v)), "ufpn_device_status")
    return v.value
