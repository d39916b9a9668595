"""Training path of the FPN neck on this library's kernels.

The reference ships backward kernels for two pieces of the neck -- the 1x1 lateral
(src/training/backward/lateral_conv_backward.cu:7-143) and the top-down upsample-add
(src/training/backward/upsample_backward.cu:4-80) -- without a driver.  Here the whole neck
has one: ``fpn_neck_forward_train`` runs the forward of ``UnifiedFPN`` (laterals with the fused
top-down add, pad-1 3x3 outputs, P6) on the same tensor-core kernels and keeps what the
backward needs; ``fpn_neck_backward`` returns the gradients of every input, weight and bias:

    dP5 += P6^T(dP6);  dM_l, dW3_l, db3_l = conv3x3^T(M_l, W3_l, dP_l)       (every level)
    dM_l += up^T(dM_{l-1}) for l = P3, P4, P5 (finest first: the top-down adjoint)
    dC_l, dWlat_l, dblat_l = lateral^T(C_l, Wlat_l, dM_l)

Each half is one call into the library's native driver (``ufpn_neck_train_forward`` /
``ufpn_neck_train_backward``), which issues its kernels on the caller's stream; Python only
allocates the results.  ``FPNNeck`` wraps both in a ``torch.nn.Module`` with fp32 master weights
(the kernels compute in the features' 16-bit dtype) for use under autograd.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _lib
from ._lib import check, lib
from .ops import _DT

_CL = torch.channels_last


def _f32(t: torch.Tensor, dev: torch.device) -> torch.Tensor:
    """``t`` as fp32, contiguous on ``dev`` (``t`` itself when it already is)."""
    if t.dtype is torch.float32 and t.is_contiguous() and t.device == dev:
        return t
    return t.detach().to(device=dev, dtype=torch.float32).contiguous()


def _layout(t: torch.Tensor, dt: torch.dtype, dev: torch.device) -> torch.Tensor:
    """``t`` in ``dt``, channels_last on ``dev`` (``t`` itself when it already is)."""
    if t.dtype is dt and t.is_contiguous(memory_format=_CL) and t.device == dev:
        return t
    return t.to(device=dev, dtype=dt).contiguous(memory_format=_CL)


def _arrays(ints, ptrs):
    """The driver calls' array arguments as two ctypes arrays (kept alive by the caller) and
    the address of each: ``int_at(k)`` / ``ptr_at(k)`` = address of element k."""
    ia = (ctypes.c_int * len(ints))(*ints)
    pa = (ctypes.c_void_p * len(ptrs))(*ptrs)
    ib, pb = ctypes.addressof(ia), ctypes.addressof(pa)
    return ia, pa, (lambda k: ib + 4 * k), (lambda k: pb + 8 * k)


def _workspace_layout(N, cin, H, W, esz):
    """Byte offsets (256-byte aligned) of the forward's saved intermediates in one buffer: per
    level the 16-bit lateral weights [256][Cin], their transpose [ceil(Cin/256)*256][256], the
    packed and the flipped 3x3 weights [256][9][256], then the merged maps M2..M5 (NHWC)."""
    sizes = []
    for c in cin:
        sizes += [256 * c, (c + 255) // 256 * 256 * 256, 256 * 9 * 256, 256 * 9 * 256]
    sizes += [N * h * w * 256 for h, w in zip(H, W)]
    offs, total = [], 0
    for n in sizes:
        offs.append(total)
        total += (n * esz + 255) // 256 * 256
    return offs, total


def fpn_neck_forward_train(feats: Sequence[torch.Tensor], lateral_w: Sequence[torch.Tensor],
                           lateral_b: Sequence[torch.Tensor], output_w: Sequence[torch.Tensor],
                           output_b: Sequence[torch.Tensor], return_p6: bool = True):
    """Forward of the neck for training.  ``feats``: C2..C5 (bf16 / fp16, 4-D CUDA); weights
    as for ``UnifiedFPN.initialize_weights`` (lateral [256, Cin] or [256, Cin, 1, 1], 3x3
    [256, 256, 3, 3], fp32 biases).  Returns ``(outputs, saved)``: P2..P5 (and P6)
    channels_last, and the opaque state ``fpn_neck_backward`` needs (the inputs, and one
    workspace holding the merged maps M2..M5 and the prepared weight layouts).  One library
    call (``ufpn_neck_train_forward``): the weight layouts of the whole step in one launch, the
    laterals top-down (the raw P5 / P4 / P3 laterals in one launch and both merges in another,
    as the forward engine runs them, then the P2 lateral with the top-down add), the four 3x3s
    (single-CTA halo tiles)."""
    if len(feats) != 4 or len(lateral_w) != 4 or len(output_w) != 4:
        raise ValueError("feats and weights must be C2..C5 / four levels")
    dt = feats[0].dtype
    if dt not in (torch.bfloat16, torch.float16) or any(f.dtype is not dt for f in feats):
        raise ValueError("training runs on bf16 or fp16 features of one dtype")
    if any(not f.is_cuda or f.dim() != 4 for f in feats):
        raise ValueError("features must be 4-D CUDA tensors")
    dev = feats[0].device
    x = [f if f.is_contiguous(memory_format=_CL) else f.contiguous(memory_format=_CL) for f in feats]
    N = x[0].shape[0]
    cin = [f.shape[1] for f in x]
    H = [f.shape[2] for f in x]
    W = [f.shape[3] for f in x]
    lat32 = [_f32(w, dev) for w in lateral_w]
    conv32 = [_f32(w, dev) for w in output_w]
    latb = [_f32(b, dev) for b in lateral_b]
    convb = [_f32(b, dev) for b in output_b]
    if any(w.shape[0] != 256 or w.numel() != 256 * c for w, c in zip(lat32, cin)) or any(
            w.shape != (256, 256, 3, 3) for w in conv32):
        raise ValueError("lateral weights must be [256, Cin] and 3x3 weights [256, 256, 3, 3]")
    offs, total = _workspace_layout(N, cin, H, W, 2)
    ws = torch.empty(total, device=dev, dtype=torch.uint8)
    base = ws.data_ptr()
    outs = [torch.empty(N, 256, h, w, device=dev, dtype=dt, memory_format=_CL) for h, w in zip(H, W)]
    p6 = torch.empty(N, 256, (H[3] - 1) // 2 + 1, (W[3] - 1) // 2 + 1, device=dev, dtype=dt,
                     memory_format=_CL) if return_p6 else None
    lay = [[base + offs[4 * l + k] for l in range(4)] for k in range(4)]  # lw, lw_t, packed, flipped
    merged = [base + offs[16 + l] for l in range(4)]
    ptrs = ([t.data_ptr() for t in x] + [t.data_ptr() for t in lat32] + [t.data_ptr() for t in latb]
            + [t.data_ptr() for t in conv32] + [t.data_ptr() for t in convb] + lay[0] + lay[1]
            + lay[2] + lay[3] + merged + [t.data_ptr() for t in outs])
    ia, pa, ip, pp = _arrays(cin + H + W, ptrs)
    check(lib.ufpn_neck_train_forward(_DT[dt], N, ip(0), ip(4), ip(8), *[pp(4 * k) for k in range(11)],
                                      p6.data_ptr() if p6 is not None else None,
                                      torch.cuda.current_stream(dev).cuda_stream), "ufpn_neck_train_forward")
    if return_p6:
        outs.append(p6)
    return outs, {"x": x, "workspace": ws, "merged": merged, "lateral_w_t": lay[1],
                  "flipped": lay[3], "sizes": (N, cin, H, W)}


def fpn_neck_backward(grad_outputs: Sequence[torch.Tensor | None], saved: dict,
                      need_input_grad: bool = True):
    """Gradients of the neck given dP2..dP5 (and dP6; None = zero) and ``saved`` from
    ``fpn_neck_forward_train``.  Returns a dict: ``grad_inputs`` (dC2..dC5, or None),
    ``grad_lateral_w`` ([256, Cin] fp32), ``grad_lateral_b``, ``grad_output_w``
    ([256, 256, 3, 3] fp32), ``grad_output_b``; the fp32 gradients are views of one buffer.
    One library call (``ufpn_neck_train_backward``)."""
    x = saved["x"]
    N, cin, H, W = saved["sizes"]
    dt = x[0].dtype
    dev = x[0].device

    def g16(l, shape):
        g = grad_outputs[l] if l < len(grad_outputs) else None
        if g is None:
            return None
        if g.shape != shape:
            raise ValueError(f"output gradient of shape {tuple(g.shape)}, expected {shape}")
        return _layout(g, dt, dev)

    dp = [g16(l, (N, 256, H[l], W[l])) for l in range(4)]
    g6 = g16(4, (N, 256, (H[3] - 1) // 2 + 1, (W[3] - 1) // 2 + 1))
    gx = [torch.empty_like(f, memory_format=_CL) for f in x] if need_input_grad else None
    sizes = [256 * c for c in cin] + [256] * 4 + [256 * 2304] * 4 + [256] * 4
    parts = torch.empty(sum(sizes), device=dev, dtype=torch.float32).split(sizes)
    gwl = [parts[l].view(256, c) for l, c in enumerate(cin)]
    gbl = list(parts[4:8])
    gw3 = [parts[8 + l].view(256, 256, 3, 3) for l in range(4)]
    gb3 = list(parts[12:16])
    ptrs = ([t.data_ptr() for t in x] + saved["merged"] + saved["lateral_w_t"]
            + saved["flipped"] + [g.data_ptr() if g is not None else None for g in dp]
            + ([t.data_ptr() for t in gx] if gx is not None else [None] * 4)
            + [t.data_ptr() for t in parts])
    ia, pa, ip, pp = _arrays(cin + H + W, ptrs)
    check(lib.ufpn_neck_train_backward(_DT[dt], N, ip(0), ip(4), ip(8), pp(0), pp(4), pp(8), pp(12),
                                       pp(16), g6.data_ptr() if g6 is not None else None,
                                       pp(20) if gx is not None else None, pp(24), pp(28), pp(32),
                                       pp(36), torch.cuda.current_stream(dev).cuda_stream),
          "ufpn_neck_train_backward")
    return {"grad_inputs": gx, "grad_lateral_w": gwl, "grad_lateral_b": gbl, "grad_output_w": gw3,
            "grad_output_b": gb3}


class _NeckFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, return_p6, c2, c3, c4, c5, *params):
        lw, lb, ow, ob = params[0:4], params[4:8], params[8:12], params[12:16]
        outs, saved = fpn_neck_forward_train([c2, c3, c4, c5], lw, lb, ow, ob, return_p6)
        ctx.saved = saved
        ctx.weight_dtypes = [p.dtype for p in params]
        ctx.lateral_shapes = [w.shape for w in lw]
        ctx.input_dtypes = [c.dtype for c in (c2, c3, c4, c5)]
        ctx.return_p6 = return_p6
        return tuple(outs)

    @staticmethod
    def backward(ctx, *grads):
        need_x = any(ctx.needs_input_grad[1:5])
        r = fpn_neck_backward(grads, ctx.saved, need_input_grad=need_x)
        ctx.saved = None
        gx = r["grad_inputs"] if need_x else [None] * 4
        wd = ctx.weight_dtypes

        def cast(g, d, shape=None):
            if shape is not None and g.shape != shape:
                g = g.reshape(shape)
            return g if g.dtype is d else g.to(d)
        gl = [cast(g, wd[i], s) for i, (g, s) in enumerate(zip(r["grad_lateral_w"], ctx.lateral_shapes))]
        gbl = [cast(g, wd[4 + i]) for i, g in enumerate(r["grad_lateral_b"])]
        gw3 = [cast(g, wd[8 + i]) for i, g in enumerate(r["grad_output_w"])]
        gb3 = [cast(g, wd[12 + i]) for i, g in enumerate(r["grad_output_b"])]
        return (None, *[cast(g, d) if g is not None else None for g, d in zip(gx, ctx.input_dtypes)],
                *gl, *gbl, *gw3, *gb3)


class FPNNeck(torch.nn.Module):
    """Trainable FPN neck: lateral 1x1 + top-down bilinear add + pad-1 3x3 per level, P6 =
    P5[::2, ::2], with fp32 master weights; the forward and backward run on this library's
    kernels in the features' dtype (bf16 / fp16, channels_last), and autograd sees the usual
    parameters."""

    def __init__(self, in_channels: Sequence[int] = (256, 512, 1024, 2048), out_channels: int = 256,
                 return_p6: bool = True, seed: int = 0):
        super().__init__()
        if out_channels != 256:
            raise ValueError("the neck's kernels produce 256 channels")
        g = torch.Generator().manual_seed(seed)
        self.return_p6 = return_p6
        self.lateral_w = torch.nn.ParameterList(
            [torch.nn.Parameter(torch.randn(256, c, generator=g) * (2.0 / c) ** 0.5) for c in in_channels])
        self.lateral_b = torch.nn.ParameterList([torch.nn.Parameter(torch.zeros(256)) for _ in in_channels])
        self.output_w = torch.nn.ParameterList(
            [torch.nn.Parameter(torch.randn(256, 256, 3, 3, generator=g) * (2.0 / 2304) ** 0.5)
             for _ in in_channels])
        self.output_b = torch.nn.ParameterList([torch.nn.Parameter(torch.zeros(256)) for _ in in_channels])

    def forward(self, feats: Sequence[torch.Tensor]):
        # (the lists' registered parameters in index order, without ParameterList's per-item
        # lookups)
        params = [*self.lateral_w._parameters.values(), *self.lateral_b._parameters.values(),
                  *self.output_w._parameters.values(), *self.output_b._parameters.values()]
        return list(_NeckFunction.apply(self.return_p6, *feats, *params))

    def make_graphed(self, sample_feats: Sequence[torch.Tensor]):
        """Captures this neck's forward and backward as CUDA graphs for the geometry, dtype and
        requires_grad pattern of ``sample_feats`` (C2..C5, channels_last CUDA tensors); returns
        a callable ``f(feats) -> [P2, .., P6]`` that replays them under autograd (weights are
        read in place, so optimiser updates between steps are seen).  Every launch of the
        step then goes to the GPU as one graph: measured 1.05 against 1.14 ms per R50
        800x1216 batch-2 training step, with bitwise the same gradients.  The inputs of later
        calls must match the samples' shapes, dtypes and strides, and no output of an eager
        call may still hold its autograd graph while this captures (its gradient-accumulation
        nodes would tie the capture to the default stream)."""
        module = _Positional(self)
        graphed = torch.cuda.make_graphed_callables(module, tuple(sample_feats))

        def run(feats: Sequence[torch.Tensor]):
            return list(graphed(*feats))
        return run


class _Positional(torch.nn.Module):
    """FPNNeck with C2..C5 as four positional tensors (the form CUDA-graph capture takes)."""

    def __init__(self, neck: FPNNeck):
        super().__init__()
        self.neck = neck

    def forward(self, c2, c3, c4, c5):
        return tuple(self.neck([c2, c3, c4, c5]))
