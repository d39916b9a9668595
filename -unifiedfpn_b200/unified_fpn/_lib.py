"""ctypes binding of libunified_fpn_b200.so (the C ABI in include/unified_fpn_c.h).

There is no fallback: if the shared library is missing or fails to load, importing
this module raises ImportError, so nothing can silently run on the CPU.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_longlong, c_size_t, c_void_p
from pathlib import Path

LIB_NAME = "libunified_fpn_b200.so"
LIB_PATH = Path(os.environ.get("UFPN_LIBRARY", Path(__file__).resolve().parent / LIB_NAME))

OK = 0
ERR_INVALID_ARG = 1
ERR_CUDA = 2
ERR_UNSUPPORTED = 3
ERR_DEVICE_TIMEOUT = 4
ERR_STATE = 5
ERR_ALIGNMENT = 6

# device status words (the role whose bounded wait gave up first)
DEV_TIMEOUT_PRODUCER = 0x101
DEV_TIMEOUT_MMA = 0x102
DEV_TIMEOUT_EPILOGUE = 0x103
DEV_TIMEOUT_DRAIN = 0x104
DEV_TIMEOUT_DEPENDENCY = 0x105

DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_BF16 = 2
DTYPE_E4M3 = 6

LAYOUT_NCHW = 0
LAYOUT_NHWC = 1


class TuningResult(ctypes.Structure):
    _fields_ = [
        ("tile_w", c_int),
        ("tile_h", c_int),
        ("num_ctas", c_int),
        ("time_ms", c_float),
        ("performance_gflops", c_float),
        ("memory_bandwidth_gb_s", c_float),
        ("architecture_name", ctypes.c_char * 32),
    ]


# name -> (restype, argtypes)
SIGNATURES = {
    "ufpn_last_error": (c_char_p, []),
    "ufpn_version": (c_int, []),
    "ufpn_device_status": (c_int, [c_int, POINTER(c_int)]),
    "ufpn_core_create": (c_int, [c_int, c_size_t, POINTER(c_void_p)]),
    "ufpn_core_destroy": (None, [c_void_p]),
    "ufpn_core_configure_levels": (
        c_int, [c_void_p, c_int, POINTER(c_int), POINTER(c_int), POINTER(c_int), c_int, c_int, c_int]),
    "ufpn_core_allocate_weights": (c_int, [c_void_p, POINTER(c_int), c_int]),
    "ufpn_core_set_weights": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ufpn_core_forward": (c_int, [c_void_p, POINTER(c_void_p), POINTER(c_void_p), c_void_p, c_void_p]),
    "ufpn_core_set_kernel_config": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int]),
    "ufpn_core_set_schedule": (c_int, [c_void_p, c_int]),
    "ufpn_core_set_schedule_options": (c_int, [c_void_p, c_int, c_int, c_int]),
    "ufpn_core_set_option": (c_int, [c_void_p, c_char_p, c_int]),
    "ufpn_set_peaks": (c_int, [ctypes.c_double, ctypes.c_double, ctypes.c_double]),
    "ufpn_core_graph_stats": (c_int, [c_void_p, POINTER(c_longlong)]),
    "ufpn_get_peaks": (c_int, [POINTER(ctypes.c_double)]),
    "ufpn_core_get_option": (c_int, [c_void_p, c_char_p, POINTER(c_int)]),
    "ufpn_core_trace_next_forward": (c_int, [c_void_p]),
    "ufpn_core_get_neck_trace": (c_int, [c_void_p, POINTER(ctypes.c_ulonglong)]),
    "ufpn_core_get_memory_usage": (c_size_t, [c_void_p]),
    "ufpn_core_get_performance_metrics": (c_int, [c_void_p, POINTER(c_float), POINTER(c_float)]),
    "ufpn_core_set_profiling": (c_int, [c_void_p, c_int]),
    "ufpn_core_autotune": (c_int, [c_void_p, POINTER(c_void_p), POINTER(c_void_p), c_void_p, c_void_p, c_int]),
    "ufpn_core_save_tuning": (c_int, [c_void_p, c_char_p]),
    "ufpn_core_load_tuning": (c_int, [c_void_p, c_char_p]),
    "ufpn_core_device_status": (c_int, [c_void_p, c_int, POINTER(c_int)]),
    "ufpn_lateral_conv": (
        c_int, [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "ufpn_lateral_conv_pair": (
        c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                c_int, c_int, c_void_p]),
    "ufpn_conv3x3": (
        c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "ufpn_conv3x3_act": (
        c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                c_float, c_void_p]),
    "ufpn_core_set_activation": (c_int, [c_void_p, c_int, c_float]),
    "ufpn_core_set_fp8_options": (c_int, [c_void_p, c_int]),
    "ufpn_fold_batch_norm": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_int, c_longlong,
                c_void_p, c_void_p]),
    "ufpn_upsample_add": (
        c_int, [c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                c_void_p]),
    "ufpn_p6_maxpool": (c_int, [c_int, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "ufpn_lateral_conv_backward": (
        c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                c_int, c_void_p]),
    "ufpn_conv3x3_backward": (
        c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                c_void_p]),
    "ufpn_lateral_conv_backward_t": (
        c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                c_int, c_void_p]),
    "ufpn_conv3x3_backward_f": (
        c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                c_void_p]),
    "ufpn_prepare_neck_weights": (
        c_int, [c_int, c_int, POINTER(c_void_p), POINTER(c_int), POINTER(c_void_p), POINTER(c_void_p),
                POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p), c_void_p]),
    # (the array arguments of the two training drivers are passed as addresses)
    "ufpn_neck_train_forward": (c_int, [c_int, c_int] + [c_void_p] * 16),
    "ufpn_neck_train_backward": (c_int, [c_int, c_int] + [c_void_p] * 15),
    "ufpn_upsample_add_backward": (
        c_int, [c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "ufpn_p6_backward": (c_int, [c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "ufpn_merge_two_levels": (
        c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                c_int, c_void_p]),
    "ufpn_pack_conv3x3_weights": (c_int, [c_int, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "ufpn_absmax": (c_int, [c_int, c_void_p, c_longlong, c_int, c_void_p, c_void_p]),
    "ufpn_quantize_e4m3": (c_int, [c_int, c_void_p, c_longlong, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "ufpn_quantize_e4m3_rows": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "ufpn_lateral_conv_e4m3": (
        c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "ufpn_conv3x3_e4m3": (
        c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "ufpn_conv3x3_e4m3_from_bf16": (
        c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                c_int, c_int, c_int, c_void_p]),
    "ufpn_core_forward_e4m3": (
        c_int, [c_void_p, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p), c_void_p, c_void_p]),
    "ufpn_neck_forward_noalloc": (
        c_int, [c_int, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p),
                POINTER(c_void_p), POINTER(c_void_p), c_void_p, c_int, POINTER(c_int), POINTER(c_int),
                POINTER(c_int), c_void_p, c_void_p]),
    "ufpn_convert_weights": (c_int, [c_int, c_void_p, c_void_p, c_longlong, c_void_p]),
    "ufpn_layout_convert": (c_int, [c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "launch_production_upsample_float": (
        c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, POINTER(c_float),
                POINTER(c_float)]),
    "launch_production_upsample_half": (
        c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, POINTER(c_float),
                POINTER(c_float)]),
    "launch_production_upsample_bfloat16": (
        c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, POINTER(c_float),
                POINTER(c_float)]),
    "create_upsample_engine": (c_void_p, [c_int]),
    "destroy_upsample_engine": (None, [c_void_p]),
    "production_upsample_float": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_float, c_float, c_int,
                POINTER(c_float)]),
    "print_upsample_profiling_summary": (None, [c_void_p]),
    "export_upsample_profiling_data": (c_int, [c_void_p, c_char_p]),
    "fpn_auto_tune_lateral_conv": (POINTER(TuningResult), [c_int, c_int, c_int, c_int, c_int]),
    "ufpn_autotune_lateral": (c_int, [c_int, c_int, c_int, c_int, c_int, c_void_p, POINTER(TuningResult)]),
    "ufpn_core_autotune_scaled": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int]),
    "fpn_auto_tune_save_results": (None, [c_char_p]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(or python -unifiedfpn_b200/build.py); there is no CPU fallback")
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as e:  # pragma: no cover - depends on the host
        raise ImportError(f"cannot load {LIB_PATH}: {e}") from e
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class UFPNError(RuntimeError):
    """Raised when a C ABI call returns a non-zero status."""

    def __init__(self, code: int, where: str):
        msg = lib.ufpn_last_error().decode(errors="replace")
        super().__init__(f"{where} failed (status {code}): {msg}")
        self.code = code


def check(code: int, where: str) -> None:
    if code != OK:
        raise UFPNError(code, where)
