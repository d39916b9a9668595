"""User-facing helpers of the reference package (python/__init__.py:82-257),
rebuilt over this library: benchmark_fpn, profile_fpn, get_device_info,
check_installation."""
from __future__ import annotations

import torch

from . import _lib

# Stage names of get_performance_breakdown()'s eight kernel times.
STAGES_TC = ["laterals_P5_P4_P3", "conv3x3_P5", "merge_P4", "conv3x3_P4", "merge_P3", "conv3x3_P3",
             "lateral_P2_fused_add", "conv3x3_P2"]
STAGES_FP32 = ["lateral_P5", "conv3x3_P5", "lateral_P4", "conv3x3_P4", "lateral_P3", "conv3x3_P3",
               "lateral_P2", "conv3x3_P2"]


def benchmark_fpn(backbone_features, num_iterations: int = 100, warmup_iterations: int = 10, fpn=None):
    """Times the neck with CUDA events (reference: python/__init__.py:82-133).

    Returns a dict with avg_time_ms, fps (images/s), memory_bandwidth_gb_s,
    compute_utilization and memory_usage_mb."""
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA not available for benchmarking")
    from .core import UnifiedFPN
    fpn = fpn or UnifiedFPN(device=backbone_features[0].device)
    for _ in range(warmup_iterations):
        fpn(backbone_features)
    torch.cuda.synchronize()
    avg_ms, gbs, util = fpn.benchmark(backbone_features, num_iterations)
    batch = backbone_features[0].shape[0]
    return {
        "avg_time_ms": avg_ms,
        "fps": batch * 1000.0 / avg_ms,
        "memory_bandwidth_gb_s": gbs,
        "compute_utilization": util,
        "memory_usage_mb": fpn.get_memory_usage() / (1024.0 * 1024.0),
    }


def profile_fpn(backbone_features, fpn=None):
    """Per-kernel device times of one serialised forward (reference:
    python/__init__.py:135-174, which wrapped cudaProfilerStart/Stop)."""
    from .core import UnifiedFPN
    fpn = fpn or UnifiedFPN(device=backbone_features[0].device)
    fpn(backbone_features)  # configure + weights
    kt, mt = fpn.get_performance_breakdown(backbone_features)
    names = STAGES_FP32 if backbone_features[0].dtype == torch.float32 else STAGES_TC
    return {
        "kernel_times_ms": dict(zip(names, kt.tolist())),
        "forward_time_ms": float(mt[0]),
        "memory_bandwidth_gb_s": float(mt[1]),
        "compute_utilization": float(mt[2]),
        "peak_memory_mb": float(mt[3]),
        "num_kernel_launches": int(mt[4]),
    }


def get_device_info(device: int = 0):
    """Device properties relevant to the kernels (reference: python/__init__.py:176-200)."""
    if not torch.cuda.is_available():
        return {"cuda_available": False}
    p = torch.cuda.get_device_properties(device)
    return {
        "cuda_available": True,
        "name": p.name,
        "compute_capability": f"{p.major}.{p.minor}",
        "sm_count": p.multi_processor_count,
        "total_memory_gb": p.total_memory / 1e9,
        "tensor_core_path": (p.major, p.minor) == (10, 0),
        "library": str(_lib.LIB_PATH),
        "library_version": _lib.lib.ufpn_version(),
    }


def check_installation() -> bool:
    """Runs a tiny neck and checks output shapes (reference: python/__init__.py:202-257)."""
    if not torch.cuda.is_available():
        print("CUDA not available")
        return False
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
