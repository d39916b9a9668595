"""unified_fpn: B200-native FPN neck (lateral 1x1 -> top-down bilinear upsample-add
-> 3x3 output conv, plus P6), a drop-in for the reference package's public API
(python/__init__.py:47-59 of sanowl/-UnifiedFPN): ``UnifiedFPN``,
``fpn_lateral_conv``, ``fpn_upsample_bilinear``, ``fpn_forward_pytorch``,
``benchmark_fpn``, ``profile_fpn``, ``get_device_info``, ``check_installation``.

The compute runs in libunified_fpn_b200.so (hand-written sm_100a kernels).  If
that library cannot be loaded the import fails: there is no CPU fallback.
"""
from ._lib import UFPNError, lib  # noqa: F401  (raises ImportError without the library)
from .core import UnifiedFPN, fpn_forward_pytorch
from .ops import (device_status, fold_batch_norm, fpn_conv3x3, prepare_neck_weights, fpn_conv3x3_backward, fpn_conv3x3_fp8, fpn_conv3x3_fp8_from_bf16,
                  fpn_lateral_conv, fpn_lateral_conv_backward, fpn_lateral_conv_fp8, fpn_merge_two_levels, fpn_p6,
                  fpn_p6_backward, fpn_upsample_add, fpn_upsample_add_backward, fpn_upsample_bilinear,
                  pack_conv3x3_weight, quantize_fp8, quantize_fp8_rows)
from .training import FPNNeck, fpn_neck_backward, fpn_neck_forward_train
from .helpers import (benchmark_fpn, check_installation, get_device_info, get_peaks, load_measured_peaks,
                      profile_fpn, set_peaks)
from .pipeline import HostPipeline

__version__ = "1.0.0"

# Utilisation figures are reported against measured peaks when a peaks file is present.
load_measured_peaks()

__all__ = [
    "UnifiedFPN", "fpn_lateral_conv", "fpn_upsample_bilinear", "fpn_forward_pytorch",
    "fpn_upsample_add", "fpn_merge_two_levels", "fpn_p6", "fpn_conv3x3", "fold_batch_norm", "prepare_neck_weights", "pack_conv3x3_weight", "device_status",
    "quantize_fp8", "quantize_fp8_rows", "fpn_lateral_conv_fp8", "fpn_conv3x3_fp8", "fpn_conv3x3_fp8_from_bf16", "HostPipeline",
    "benchmark_fpn", "profile_fpn", "get_device_info", "check_installation", "UFPNError",
    "set_peaks", "get_peaks", "load_measured_peaks",
    "fpn_lateral_conv_backward", "fpn_conv3x3_backward", "fpn_upsample_add_backward", "fpn_p6_backward",
    "FPNNeck", "fpn_neck_forward_train", "fpn_neck_backward",
]
