"""User-facing helpers of the reference package (python/__init__.py:82-257),
rebuilt over this library with the reference's signatures and result keys:
benchmark_fpn, profile_fpn, get_device_info, check_installation; plus the peaks that
utilisation figures are reported against (set_peaks / get_peaks / load_measured_peaks)."""
from __future__ import annotations

import ctypes
import json
import os
from pathlib import Path

import torch

from . import _lib

# Stage names of get_performance_breakdown()'s eight kernel times.
STAGES_TC = ["laterals_P5_P4_P3", "conv3x3_P5", "merge_P4", "conv3x3_P4", "merge_P3", "conv3x3_P3",
             "lateral_P2_fused_add", "conv3x3_P2"]
STAGES_FP32 = ["lateral_P5", "conv3x3_P5", "lateral_P4", "conv3x3_P4", "lateral_P3", "conv3x3_P3",
               "lateral_P2", "conv3x3_P2"]

# Repository-root file of measured peaks (keys bf16_tflops, hbm_gbs), read at import when
# present; UFPN_PEAKS_JSON names another file.
_PEAKS_FILE = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"


def set_peaks(bf16_tflops: float | None = None, hbm_gbs: float | None = None,
              fp32_tflops: float | None = None) -> None:
    """Peaks that utilisation figures are reported against (the engine's profiled forward,
    UnifiedFPN.benchmark, benchmark_fpn, profile_fpn): dense 16-bit tensor TFLOP/s (e4m3
    counts twice it), HBM GB/s, fp32 CUDA-core TFLOP/s.  None keeps the current value."""
    _lib.check(_lib.lib.ufpn_set_peaks(float(bf16_tflops or 0.0), float(fp32_tflops or 0.0),
                                       float(hbm_gbs or 0.0)), "ufpn_set_peaks")


def get_peaks() -> dict:
    v = (ctypes.c_double * 3)()
    _lib.check(_lib.lib.ufpn_get_peaks(v), "ufpn_get_peaks")
    return {"tensor_tflops": v[0], "fp32_tflops": v[1], "hbm_gbs": v[2]}


def load_measured_peaks(path: str | os.PathLike | None = None) -> bool:
    """Sets the peaks from a JSON file with ``bf16_tflops`` and ``hbm_gbs`` (measured on the
    machine: a cuBLAS bf16 GEMM and a device copy).  Default: $UFPN_PEAKS_JSON, else the
    repository root's MEASURED_PEAKS.json.  Returns False (peaks unchanged) if there is none."""
    p = Path(path or os.environ.get("UFPN_PEAKS_JSON") or _PEAKS_FILE)
    if not p.is_file():
        return False
    d = json.loads(p.read_text())
    set_peaks(bf16_tflops=d.get("bf16_tflops"), hbm_gbs=d.get("hbm_gbs"))
    return True


def benchmark_fpn(backbone_features, num_iterations: int = 100, warmup_iterations: int = 10, fpn=None):
    """Times the neck with CUDA events (reference: python/__init__.py:82-133): the plain call
    ``fpn(backbone_features)`` (fresh outputs each call, as a drop-in caller makes it), then
    UnifiedFPN.benchmark's bandwidth and utilisation.

    Returns the reference's keys -- avg_time_ms, throughput_fps (forward calls per second),
    memory_bandwidth_gb_s, compute_utilization (of the peaks, see set_peaks),
    memory_usage_mb (inputs + outputs), detailed_metrics (UnifiedFPN.benchmark's tuple) --
    plus images_per_s and engine_memory_mb (weights + workspace)."""
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA not available for benchmarking")
    from .core import UnifiedFPN
    fpn = fpn or UnifiedFPN(device=backbone_features[0].device)
    for _ in range(warmup_iterations):
        fpn(backbone_features)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream(backbone_features[0].device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(num_iterations):
        outs = fpn(backbone_features)
    e1.record(s)
    e1.synchronize()
    avg_ms = e0.elapsed_time(e1) / num_iterations
    detailed = fpn.benchmark(backbone_features, num_iterations)
    mb = (sum(t.numel() * t.element_size() for t in backbone_features[:4]) +
          sum(t.numel() * t.element_size() for t in outs)) / (1024.0 * 1024.0)
    batch = backbone_features[0].shape[0]
    return {
        "avg_time_ms": avg_ms,
        "throughput_fps": 1000.0 / avg_ms,
        "memory_bandwidth_gb_s": detailed[1],
        "compute_utilization": detailed[2],
        "memory_usage_mb": mb,
        "detailed_metrics": detailed,
        "images_per_s": batch * 1000.0 / avg_ms,
        "engine_memory_mb": fpn.get_memory_usage() / (1024.0 * 1024.0),
    }


def profile_fpn(backbone_features, output_file: str | os.PathLike | None = "fpn_profile.json", fpn=None):
    """Per-stage device times of one serialised forward, saved as JSON to ``output_file``
    (None: not saved) and returned (reference: python/__init__.py:135-174, which wrapped the
    forward in cudaProfilerStart/Stop; here the engine times each stage with CUDA events).

    Keys as the reference's: kernel_times_ms (8 stage times), total_time_ms,
    memory_bandwidth_gb_s, compute_utilization, peak_memory_mb, num_kernel_launches; plus
    kernel_stages (the names of the 8 stages) and device."""
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA not available for profiling")
    from .core import UnifiedFPN
    fpn = fpn or UnifiedFPN(device=backbone_features[0].device)
    fpn(backbone_features)  # configure + weights
    kt, mt = fpn.get_performance_breakdown(backbone_features)
    names = STAGES_FP32 if backbone_features[0].dtype == torch.float32 else STAGES_TC
    data = {
        "kernel_times_ms": [float(v) for v in kt.tolist()],
        "total_time_ms": float(mt[0]),
        "memory_bandwidth_gb_s": float(mt[1]),
        "compute_utilization": float(mt[2]),
        "peak_memory_mb": float(mt[3]),
        "num_kernel_launches": int(mt[4]),
        "kernel_stages": names,
        "device": torch.cuda.get_device_name(backbone_features[0].device),
    }
    if output_file is not None:
        with open(output_file, "w") as f:
            json.dump(data, f, indent=2)
        print(f"Profiling results saved to {output_file}")
    return data


def get_device_info(device: int | None = None):
    """Device properties (reference: python/__init__.py:176-200, same keys; its property
    names max_threads_per_multiprocessor / l2_cache_size are torch's
    max_threads_per_multi_processor / L2_cache_size) plus what this library uses."""
    if not torch.cuda.is_available():
        return {"error": "CUDA not available", "cuda_available": False}
    device = torch.cuda.current_device() if device is None else device
    p = torch.cuda.get_device_properties(device)
    return {
        "device_name": p.name,
        "compute_capability": f"{p.major}.{p.minor}",
        "total_memory_gb": p.total_memory / (1024 ** 3),
        "multiprocessor_count": p.multi_processor_count,
        "max_threads_per_block": p.max_threads_per_block,
        "max_threads_per_multiprocessor": p.max_threads_per_multi_processor,
        "memory_clock_rate_mhz": p.memory_clock_rate / 1000,
        "memory_bus_width_bits": p.memory_bus_width,
        "l2_cache_size_mb": p.L2_cache_size / (1024 * 1024),
        "theoretical_bandwidth_gb_s": 2 * p.memory_clock_rate * p.memory_bus_width / 8 / 1e6,
        "cuda_available": True,
        "sm_count": p.multi_processor_count,
        "tensor_core_path": (p.major, p.minor) == (10, 0),
        "library": str(_lib.LIB_PATH),
        "library_version": _lib.lib.ufpn_version(),
        "peaks": get_peaks(),
    }


def check_installation() -> bool:
    """Runs a tiny neck and checks the output shapes and values (reference:
    python/__init__.py:202-257: CUDA, device, a forward on small features, P2..P5 shapes)."""
    try:
        if not torch.cuda.is_available():
            print("CUDA not available")
            return False
        info = get_device_info()
        print(f"GPU: {info['device_name']} (compute capability {info['compute_capability']})")
        from .core import UnifiedFPN
        dev = torch.device("cuda", torch.cuda.current_device())
        feats = [torch.randn(1, c, s, s, device=dev, dtype=torch.bfloat16).contiguous(memory_format=torch.channels_last)
                 for c, s in ((256, 32), (512, 16), (1024, 8), (2048, 4))]
        outs = UnifiedFPN(device=dev)(feats, return_p6=True)
        torch.cuda.synchronize()
        want = [(1, 256, 32, 32), (1, 256, 16, 16), (1, 256, 8, 8), (1, 256, 4, 4), (1, 256, 2, 2)]
        ok = [tuple(o.shape) for o in outs] == want and all(torch.isfinite(o.float()).all().item() for o in outs)
        print("unified_fpn installation", "OK" if ok else "FAILED")
        return ok
    except Exception as e:  # reported like the reference: a failed check, not an exception
        print(f"unified_fpn installation check failed: {e}")
        return False
