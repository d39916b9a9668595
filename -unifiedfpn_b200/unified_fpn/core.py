"""``UnifiedFPN``: the FPN neck module (drop-in for the reference's extension class).

Reference: class PyTorchFPNWrapper bound as ``UnifiedFPN`` in python/fpn_pytorch.cpp:9-393
(constructor ``UnifiedFPN(output_channels=256, workspace_size_mb=512)`` and methods
forward / initialize_weights / benchmark / get_performance_breakdown / set_kernel_config /
get_memory_usage), driving class UnifiedFPNCore (lib/core/fpn_engine.cu).

Differences from the reference (whose sources do not build as shipped):
  * forward takes C2..C5 (a fifth tensor C6 is accepted and ignored) in float32,
    float16 or bfloat16, NCHW-contiguous or channels_last, and returns P2..P5
    (plus P6 = max_pool2d(P5, 1, 2) with ``return_p6=True``).  Outputs keep the
    inputs' memory format.
  * float8_e4m3fn inputs (with per-tensor ``input_scales``) run the FP8 neck on the
    e4m3 tensor cores and return bf16 channels_last outputs.
  * The neck is the standard one: lateral 1x1 + bias, top-down bilinear
    upsample (align_corners=False) + add, full 3x3 output conv + bias.
  * Weights left uninitialised are filled deterministically (Kaiming-normal,
    fan_in, zero bias, seed 0) instead of from std::random_device.
"""
from __future__ import annotations

import ctypes
import math
from typing import Sequence

import torch

from . import _lib
from ._lib import check, lib
from .ops import _DT, E4M3, _stream

_ACT = {"none": 0, "relu": 1, "leaky_relu": 2, "swish": 3}


def _ptr_array(ptrs):
    arr = (ctypes.c_void_p * len(ptrs))()
    for i, p in enumerate(ptrs):
        arr[i] = p
    return arr


class UnifiedFPN:
    """FPN neck on one CUDA device."""

    def __init__(self, output_channels: int = 256, workspace_size_mb: int = 512, device=None):
        if output_channels != 256:
            raise ValueError("output_channels must be 256 (the tensor-core tile width)")
        self.output_channels = output_channels
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        h = ctypes.c_void_p()
        check(lib.ufpn_core_create(self.device.index or 0, workspace_size_mb << 20, ctypes.byref(h)),
              "ufpn_core_create")
        self._h = h
        self._channels = None       # Cin of C2..C5 the weights were allocated for
        self._weights_ready = False
        self._weight_refs = []      # keeps host/device weight tensors alive until copied
        self._config = None
        self._scale_buf = None      # e4m3 input scales, a stable device address per engine

    def __del__(self):
        h = getattr(self, "_h", None)
        # (at interpreter exit the module globals may already be cleared: the process's
        # teardown then releases the engine with the CUDA context)
        if h is not None and h.value and lib is not None:
            lib.ufpn_core_destroy(h)
            self._h = None

    # ------------------------------------------------------------------ weights
    def initialize_weights(self, lateral_weights: Sequence[torch.Tensor], lateral_bias: Sequence[torch.Tensor],
                           output_weights: Sequence[torch.Tensor], output_bias: Sequence[torch.Tensor],
                           lateral_scales: Sequence[torch.Tensor] | None = None,
                           output_scales: Sequence[torch.Tensor] | None = None) -> None:
        """Set the neck's fp32 weights (reference: fpn_pytorch.cpp:24-81).

        lateral_weights[l]: [256, Cin_l] or [256, Cin_l, 1, 1]; lateral_bias[l]: [256];
        output_weights[l]: [256, 256, 3, 3]; output_bias[l]: [256]; l = 0..3 for P2..P5.
        CPU or CUDA tensors; they are copied (and packed to the compute dtype) here.
        Weights may also be float8_e4m3fn with per-output-channel ``lateral_scales`` /
        ``output_scales`` ([256] each, w = q * scale); they are dequantised to fp32 here.
        """
        def deq(ws, scales):
            out = []
            for l, w in enumerate(ws):
                if w.dtype == E4M3:
                    if scales is None:
                        raise ValueError("float8_e4m3fn weights need their per-channel scales")
                    sc = scales[l].to(device=w.device, dtype=torch.float32).reshape(-1)
                    w = w.float() * sc.reshape([-1] + [1] * (w.dim() - 1))
                out.append(w)
            return out
        lateral_weights = deq(lateral_weights, lateral_scales)
        output_weights = deq(output_weights, output_scales)
        for name, seq in (("lateral_weights", lateral_weights), ("lateral_bias", lateral_bias),
                          ("output_weights", output_weights), ("output_bias", output_bias)):
            if len(seq) != 4:
                raise ValueError(f"Expected 4 weight tensors for each type (P2-P5): {name}")
        chans = []
        for l in range(4):
            lw = lateral_weights[l]
            if lw.dim() not in (2, 4) or (lw.dim() == 4 and tuple(lw.shape[2:]) != (1, 1)):
                raise ValueError("Lateral weights must be [out_channels, in_channels] (or [out, in, 1, 1])")
            if lw.shape[0] != self.output_channels:
                raise ValueError("Lateral weight output channels must match FPN output channels")
            if tuple(output_weights[l].shape) != (256, 256, 3, 3):
                raise ValueError("Output weights must be [256, 256, 3, 3]")
            if lateral_bias[l].numel() != 256 or output_bias[l].numel() != 256:
                raise ValueError("biases must have 256 elements")
            chans.append(int(lw.shape[1]))
        if chans != self._channels:
            arr = (ctypes.c_int * 4)(*chans)
            check(lib.ufpn_core_allocate_weights(self._h, arr, self.output_channels), "allocate_weights")
            self._channels = chans
        for l in range(4):
            ts = [t.detach().to(torch.float32).contiguous() for t in
                  (lateral_weights[l], lateral_bias[l], output_weights[l], output_bias[l])]
            if any(t.is_cuda and t.device != self.device for t in ts):
                ts = [t.to(self.device) for t in ts]
            if any(t.is_cuda for t in ts):
                # the engine copies on its own stream: finish the producers first
                torch.cuda.current_stream(self.device).synchronize()
            check(lib.ufpn_core_set_weights(self._h, l, *[t.data_ptr() for t in ts]), "set_weights")
        self._weights_ready = True

    def _default_weights(self, chans):
        g = torch.Generator().manual_seed(0)
        lw, lb, ow, ob = [], [], [], []
        for cin in chans:
            lw.append(torch.randn(256, cin, generator=g) * math.sqrt(2.0 / cin))
            lb.append(torch.zeros(256))
            ow.append(torch.randn(256, 256, 3, 3, generator=g) * math.sqrt(2.0 / (256 * 9)))
            ob.append(torch.zeros(256))
        self.initialize_weights(lw, lb, ow, ob)

    # ------------------------------------------------------------------ forward
    def _configure(self, feats):
        x0 = feats[0]
        if x0.dtype not in _DT and x0.dtype != E4M3:
            raise TypeError("inputs must be float32, float16, bfloat16 or float8_e4m3fn")
        for t in feats:
            if not t.is_cuda or t.device != self.device:
                raise ValueError("All input tensors must be on the engine's CUDA device")
            if t.dim() != 4:
                raise ValueError("All input tensors must be 4D [N, C, H, W]")
            if t.dtype != x0.dtype:
                raise ValueError("All input tensors must share one dtype")
            if t.shape[0] != x0.shape[0]:
                raise ValueError("All input tensors must share the batch size")
        if x0.dtype == E4M3 or (x0.dtype != torch.float32 and all(
                t.is_contiguous(memory_format=torch.channels_last) for t in feats)):
            layout = _lib.LAYOUT_NHWC
        else:
            layout = _lib.LAYOUT_NCHW
        chans = [int(t.shape[1]) for t in feats]
        cfg = (tuple(tuple(t.shape) for t in feats), x0.dtype, layout)
        if cfg != self._config:
            N = int(x0.shape[0])
            ci = (ctypes.c_int * 4)(*chans)
            hi = (ctypes.c_int * 4)(*[int(t.shape[2]) for t in feats])
            wi = (ctypes.c_int * 4)(*[int(t.shape[3]) for t in feats])
            code = _lib.DTYPE_E4M3 if x0.dtype == E4M3 else _DT[x0.dtype]
            check(lib.ufpn_core_configure_levels(self._h, N, ci, hi, wi, self.output_channels,
                                                 code, layout), "configure_levels")
            self._config = cfg
        if not self._weights_ready or chans != self._channels:
            if self._weights_ready:
                raise ValueError(f"weights were initialised for input channels {self._channels}, got {chans}")
            self._default_weights(chans)
        return layout

    def _prepare(self, backbone_features):
        if len(backbone_features) not in (4, 5):
            raise ValueError("Expected C2..C5 (or C2..C6) backbone feature tensors")
        feats = list(backbone_features[:4])
        layout = self._configure(feats)
        mf = torch.channels_last if layout == _lib.LAYOUT_NHWC else torch.contiguous_format
        feats = [t.contiguous(memory_format=mf) for t in feats]
        return feats, layout, mf

    def _alloc_outputs(self, feats, mf, return_p6):
        N = feats[0].shape[0]
        odt = torch.bfloat16 if feats[0].dtype == E4M3 else feats[0].dtype
        outs = [torch.empty((N, 256, t.shape[2], t.shape[3]), dtype=odt, device=t.device, memory_format=mf)
                for t in feats]
        p6 = None
        if return_p6:
            H5, W5 = feats[3].shape[2], feats[3].shape[3]
            p6 = torch.empty((N, 256, (H5 - 1) // 2 + 1, (W5 - 1) // 2 + 1), dtype=odt,
                             device=feats[0].device, memory_format=mf)
        return outs, p6

    def _scale_ptrs(self, input_scales):
        """Copies the 4 per-tensor input scales into the engine's device buffer (stream
        ordered, so a captured graph sees the same address every call)."""
        if input_scales is None or len(input_scales) < 4:
            raise ValueError("float8_e4m3fn inputs need input_scales for C2..C5")
        if (isinstance(input_scales, torch.Tensor) and input_scales.is_cuda
                and input_scales.device == self.device and input_scales.dtype == torch.float32
                and input_scales.numel() == 4 and input_scales.is_contiguous()):
            base = input_scales.data_ptr()  # the caller's own device array, used in place
            return _ptr_array([base + 4 * l for l in range(4)])
        if self._scale_buf is None:
            self._scale_buf = torch.empty(4, dtype=torch.float32, device=self.device)
        vals = torch.stack([torch.as_tensor(s, dtype=torch.float32).reshape(()).to(self.device)
                            for s in input_scales[:4]])
        self._scale_buf.copy_(vals)
        base = self._scale_buf.data_ptr()
        return _ptr_array([base + 4 * l for l in range(4)])

    def forward(self, backbone_features: Sequence[torch.Tensor], return_p6: bool = False,
                out: Sequence[torch.Tensor] | None = None, input_scales=None,
                output_fp8: bool = False):
        """P2..P5 (and P6) of the neck; stream-ordered on torch's current stream.
        float8_e4m3fn inputs need ``input_scales`` (4 per-tensor dequantisation scales,
        floats or 1-element tensors; x = q * scale) and produce bf16 outputs.
        ``output_fp8`` (16-bit outputs): each level comes back as ``(q, scale)`` for a
        downstream FP8 consumer -- float8_e4m3fn codes in the output's memory format and one
        fp32 scale per image (absmax / 448; P ~ q * scale), quantised on the device by the
        library's quantiser, exactly as ``quantize_fp8(P, per_image=True)``."""
        if output_fp8:
            if out is not None:
                raise ValueError("output_fp8 returns new tensors; out is not supported with it")
            res = self.forward(backbone_features, return_p6=return_p6, input_scales=input_scales)
            if res[0].dtype not in (torch.float16, torch.bfloat16):
                raise ValueError("output_fp8 needs 16-bit outputs (bf16 / fp16 or e4m3 inputs)")
            from .ops import quantize_fp8
            return [quantize_fp8(t, per_image=True) for t in res]
        feats, layout, mf = self._prepare(backbone_features)
        if out is not None:
            outs = list(out[:4])
            p6 = out[4] if (return_p6 and len(out) > 4) else None
            if return_p6 and p6 is None:
                raise ValueError("out must hold 5 tensors when return_p6=True")
        else:
            outs, p6 = self._alloc_outputs(feats, mf, return_p6)
        ins = _ptr_array([t.data_ptr() for t in feats])
        os_ = _ptr_array([t.data_ptr() for t in outs])
        if feats[0].dtype == E4M3:
            sp = self._scale_ptrs(input_scales)
            check(lib.ufpn_core_forward_e4m3(self._h, ins, sp, os_,
                                             p6.data_ptr() if p6 is not None else None,
                                             _stream(feats[0])), "forward")
        else:
            if input_scales is not None:
                raise ValueError("input_scales apply to float8_e4m3fn inputs only")
            check(lib.ufpn_core_forward(self._h, ins, os_, p6.data_ptr() if p6 is not None else None,
                                        _stream(feats[0])), "forward")
        return outs + [p6] if return_p6 else outs

    __call__ = forward

    # ------------------------------------------------------------------ tooling
    def benchmark(self, backbone_features, num_iterations: int = 100, input_scales=None):
        """(avg_ms, GB/s, compute utilisation) of the neck, timed with CUDA events
        on the current stream (reference: fpn_pytorch.cpp:139-169 timed with the
        host clock)."""
        feats, layout, mf = self._prepare(backbone_features)
        outs, p6 = self._alloc_outputs(feats, mf, True)
        out = outs + [p6]
        for _ in range(10):
            self.forward(feats, return_p6=True, out=out, input_scales=input_scales)
        s = torch.cuda.current_stream(self.device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(num_iterations):
            self.forward(feats, return_p6=True, out=out, input_scales=input_scales)
        e1.record(s)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / num_iterations
        esz = feats[0].element_size()
        osz = out[0].element_size()
        nbytes = 0.0
        flops = 0.0
        for t in feats:
            px = t.shape[0] * t.shape[2] * t.shape[3]
            nbytes += px * (t.shape[1] * esz + 256 * osz)
            flops += 2.0 * px * 256 * (t.shape[1] + 9 * 256)
        # against the peaks set for the library (measured ones when a peaks file is present,
        # else nominal B200 figures; see unified_fpn.set_peaks); e4m3 counts twice the 16-bit rate
        from .helpers import get_peaks
        pk = get_peaks()
        peak = {torch.float32: pk["fp32_tflops"] * 1e12,
                E4M3: 2.0 * pk["tensor_tflops"] * 1e12}.get(feats[0].dtype, pk["tensor_tflops"] * 1e12)
        return ms, nbytes / (ms * 1e-3) / 1e9, flops / (ms * 1e-3) / peak

    def get_performance_breakdown(self, backbone_features=None, input_scales=None):
        """[kernel_times_ms(8), metrics(5)] as in fpn_pytorch.cpp:171-187.  With
        ``backbone_features`` given, first runs one profiled (serialised) forward."""
        if backbone_features is not None:
            check(lib.ufpn_core_set_profiling(self._h, 1), "set_profiling")
            self.forward(backbone_features, return_p6=True, input_scales=input_scales)
        kt = (ctypes.c_float * 8)()
        mt = (ctypes.c_float * 5)()
        check(lib.ufpn_core_get_performance_metrics(self._h, kt, mt), "get_performance_metrics")
        return [torch.tensor(list(kt), dtype=torch.float32), torch.tensor(list(mt), dtype=torch.float32)]

    def set_kernel_config(self, tile_size: int = 0, channels_per_thread: int = 8, use_tensor_cores: bool = True,
                          activation: str = "none", enable_graph_capture: bool = True) -> None:
        """Reference: fpn_pytorch.cpp:189-209.  tile_size is the 3x3 tile width
        (8..128; 0 = tuned/heuristic).  ``activation`` ("relu", "leaky_relu", "swish"; any other
        string means none, as in the reference's mapping) is applied to every level's 3x3
        output in its epilogue; LeakyReLU uses the slope set by :meth:`set_activation`
        (0.01 by default)."""
        check(lib.ufpn_core_set_kernel_config(self._h, tile_size, channels_per_thread, int(use_tensor_cores),
                                              _ACT.get(activation, 0), int(enable_graph_capture)),
              "set_kernel_config")

    def set_activation(self, activation: str = "none", alpha: float = 0.01) -> None:
        """Output activation of every level's 3x3 (and so of P6): "none", "relu",
        "leaky_relu" (negative slope ``alpha``) or "swish" (v / (1 + exp(-v)))."""
        if activation not in _ACT:
            raise ValueError(f"unknown activation {activation!r}")
        check(lib.ufpn_core_set_activation(self._h, _ACT[activation], float(alpha)), "set_activation")

    def set_schedule(self, fused_neck_kernel: bool = False, single_stream: bool = False,
                     programmatic_launch: bool = True, chain_priority: bool = False,
                     merge_two_levels: bool = False, fp8_two_pass_p2: bool = False) -> None:
        """Tensor-core schedule: one persistent kernel for the whole neck, or per-level
        kernels on several streams (default) or, with ``single_stream``, one after the other
        on the caller's stream (bitwise the same results as the default).
        ``programmatic_launch`` (16-bit split schedule): kernels that follow a kernel on the
        main stream start during its tail and wait on the device for its results (same
        results, less launch latency).  ``chain_priority`` (16-bit split schedule): the
        main-stream chain gets the device's highest launch priority.  ``merge_two_levels``:
        the P4 and P3 top-down merges in one launch (when the maps upsample; set it before
        the first forward of a geometry).  ``fp8_two_pass_p2`` (e4m3 inputs): the P2 lateral
        runs an absmax pass and then stores M2 as e4m3 itself, instead of storing bf16 M2 for
        a separate quantisation pass (bitwise the same results; slower at the 640x640 batch-16
        workload, so off by default)."""
        mode = 1 if fused_neck_kernel else (2 if single_stream else 0)
        check(lib.ufpn_core_set_schedule(self._h, mode), "set_schedule")
        check(lib.ufpn_core_set_schedule_options(self._h, int(programmatic_launch), int(chain_priority),
                                                 int(merge_two_levels)), "set_schedule_options")
        check(lib.ufpn_core_set_fp8_options(self._h, int(fp8_two_pass_p2)), "set_fp8_options")

    def set_option(self, name: str, value: int) -> None:
        """Named option of the schedule or a per-level kernel shape (``ufpn_core_set_option``
        lists them): "lateral_tile_p2".."lateral_tile_p5" (8..128), "conv3x3_p2".."conv3x3_p5"
        (-1 halo tiles on CTA pairs, 0 halo tiles, 8..128 plain tiles), "p2_lateral_pair",
        "merge_units", "grouped_topdown", "ksplit_p3".."ksplit_p5" (1, 2 or 4), and the
        switches of :meth:`set_schedule`."""
        check(lib.ufpn_core_set_option(self._h, name.encode(), int(value)), f"set_option({name})")

    def get_option(self, name: str) -> int:
        v = ctypes.c_int(0)
        check(lib.ufpn_core_get_option(self._h, name.encode(), ctypes.byref(v)), f"get_option({name})")
        return v.value

    def neck_timeline(self, backbone_features) -> dict:
        """Runs one forward with the fused neck kernel's device timeline recorded and
        returns microseconds since the kernel started: when each level's laterals were
        complete, when the first P2 3x3 tile started, and the end."""
        check(lib.ufpn_core_trace_next_forward(self._h), "trace_next_forward")
        self.forward(backbone_features, return_p6=True)
        tr = (ctypes.c_ulonglong * 8)()
        check(lib.ufpn_core_get_neck_trace(self._h, tr), "get_neck_trace")
        t0 = tr[0]
        us = lambda v: (v - t0) / 1e3 if v else None  # noqa: E731
        return {"lat_P5_done": us(tr[4]), "lat_P4_done": us(tr[3]), "lat_P3_done": us(tr[2]),
                "lat_P2_done": us(tr[1]), "conv_P2_first_tile": us(tr[6]), "end": us(tr[5])}

    def graph_stats(self) -> dict:
        """Graph cache counters: pointer sets captured (on their second use), graph replays,
        forwards launched directly (a pointer set's first use) and graphs cached now."""
        v = (ctypes.c_longlong * 4)()
        check(lib.ufpn_core_graph_stats(self._h, v), "graph_stats")
        return {"captures": v[0], "replays": v[1], "direct": v[2], "cached": v[3]}

    def get_memory_usage(self) -> int:
        return int(lib.ufpn_core_get_memory_usage(self._h))

    def autotune(self, backbone_features, iterations: int = 10, input_scales=None) -> str:
        """Tunes the schedule for these features' geometry: every knob of :meth:`set_option`
        that applies (per level: 3x3 tiling, lateral tile shape; the P2 lateral on CTA pairs,
        the grouped lateral launch's top-down adds and split-K, the merge grid, programmatic
        launches, the two-level merge; e4m3: pair / single 3x3, the two-pass P2 lateral) is
        set to each candidate in turn, each timed as the whole forward; the fastest values
        are applied and kept for the geometry (save_tuning).  Returns the report.
        float8_e4m3fn inputs need ``input_scales`` as for forward."""
        feats, layout, mf = self._prepare(backbone_features)
        outs, p6 = self._alloc_outputs(feats, mf, True)
        sp = self._scale_ptrs(input_scales) if feats[0].dtype == E4M3 else None
        check(lib.ufpn_core_autotune_scaled(self._h, _ptr_array([t.data_ptr() for t in feats]), sp,
                                            _ptr_array([t.data_ptr() for t in outs]), p6.data_ptr(),
                                            _stream(feats[0]), iterations), "autotune")
        return lib.ufpn_last_error().decode()

    def save_tuning(self, path: str) -> None:
        check(lib.ufpn_core_save_tuning(self._h, str(path).encode()), "save_tuning")

    def load_tuning(self, path: str) -> None:
        check(lib.ufpn_core_load_tuning(self._h, str(path).encode()), "load_tuning")

    def device_status(self, reset: bool = True) -> int:
        v = ctypes.c_int(0)
        check(lib.ufpn_core_device_status(self._h, int(reset), ctypes.byref(v)), "device_status")
        return v.value


_SINGLETON: dict = {}


def fpn_forward_pytorch(backbone_features, lateral_weights, output_weights, lateral_bias=None,
                        output_bias=None):
    """Whole-neck forward with the given weights (reference: fpn_pytorch.cpp:360-367,
    which used a static engine and ignored its weight arguments).  Biases default to zero."""
    dev = backbone_features[0].device
    key = dev.index
    fpn = _SINGLETON.get(key)
    if fpn is None:
        fpn = _SINGLETON[key] = UnifiedFPN(device=dev)
    lb = lateral_bias if lateral_bias is not None else [torch.zeros(256) for _ in range(4)]
    ob = output_bias if output_bias is not None else [torch.zeros(256) for _ in range(4)]
    fpn.initialize_weights(lateral_weights, lb, output_weights, ob)
    return fpn.forward(backbone_features)
