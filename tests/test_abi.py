"""CPU tests of the C ABI boundary: the library loads, exports every symbol
declared in include/*.h, and rejects bad arguments on the host (no GPU work)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M):
            name = m.group(1)
            if name not in ("if", "defined"):
                names.add(name)
    return sorted(names)


def test_header_declares_the_reference_entry_points():
    names = declared_functions()
    for ref_name in ("launch_production_upsample_float", "launch_production_upsample_half",
                     "launch_production_upsample_bfloat16", "create_upsample_engine",
                     "destroy_upsample_engine", "production_upsample_float",
                     "print_upsample_profiling_summary", "export_upsample_profiling_data",
                     "fpn_auto_tune_lateral_conv", "fpn_auto_tune_save_results"):
        assert ref_name in names
    assert len(names) >= 30


def test_library_exports_every_declared_symbol():
    from unified_fpn import _lib
    missing = [n for n in declared_functions() if not hasattr(_lib.lib, n)]
    assert not missing, missing
    # and every binding in the Python layer refers to a declared symbol
    assert set(_lib.SIGNATURES) <= set(declared_functions())


def test_library_is_built_for_sm100a():
    from unified_fpn import _lib
    data = _lib.LIB_PATH.read_bytes()
    assert b"sm_100a" in data


def test_host_side_argument_validation():
    from unified_fpn import _lib
    lib = _lib.lib
    # unsupported dtype code
    assert lib.ufpn_upsample_add(99, 1, 1, None, 1, 1, 1, 1, 1, 2, 2, 0, None) == _lib.ERR_UNSUPPORTED
    assert b"dtype" in lib.ufpn_last_error()
    # null tensors
    assert lib.ufpn_lateral_conv(2, 1, None, None, None, None, None, 1, 64, 4, 4, 256, 0, 0, None) == \
        _lib.ERR_INVALID_ARG
    # bad layout code
    assert lib.ufpn_p6_maxpool(2, 7, 16, 16, 1, 1, 2, 2, None) == _lib.ERR_INVALID_ARG
    # fp32 lateral must be NCHW
    assert lib.ufpn_lateral_conv(0, 1, 16, 16, 16, None, 16, 1, 8, 2, 2, 4, 0, 0, None) == _lib.ERR_UNSUPPORTED
    # tensor-core lateral needs Cout = 256 and 16-byte aligned pointers
    assert lib.ufpn_lateral_conv(2, 1, 16, 16, 16, None, 16, 1, 64, 2, 2, 128, 0, 0, None) == _lib.ERR_UNSUPPORTED
    assert lib.ufpn_lateral_conv(2, 1, 18, 16, 16, None, 16, 1, 64, 2, 2, 256, 0, 0, None) == _lib.ERR_ALIGNMENT
    # negative sizes
    assert lib.ufpn_upsample_add(2, 1, 16, None, 16, 1, 256, -1, 2, 4, 4, 0, None) == _lib.ERR_INVALID_ARG
    # conv3x3 tile width must divide 128
    assert lib.ufpn_conv3x3(2, 16, 16, 16, 16, None, 1, 8, 8, 24, None) == _lib.ERR_INVALID_ARG
    # backward: 16-bit only, NULL gradients, Cin a multiple of 8, alignment, shapes (all checked
    # on the host before any launch)
    assert lib.ufpn_lateral_conv_backward(0, 16, 16, 16, 16, None, None, 1, 64, 2, 2, None) == _lib.ERR_UNSUPPORTED
    assert lib.ufpn_lateral_conv_backward(2, None, None, None, None, None, None, 1, 64, 2, 2, None) == \
        _lib.ERR_INVALID_ARG
    assert lib.ufpn_lateral_conv_backward(2, None, None, 16, None, None, None, 1, 12, 2, 2, None) == \
        _lib.ERR_UNSUPPORTED
    assert lib.ufpn_conv3x3_backward(2, 16, 16, 18, 16, None, None, 1, 4, 4, None) == _lib.ERR_ALIGNMENT
    assert lib.ufpn_upsample_add_backward(2, 16, None, 16, 1, 256, 8, 8, 4, 4, None) == _lib.ERR_UNSUPPORTED
    assert lib.ufpn_p6_backward(2, 16, 16, 1, 256, -3, 4, None) == _lib.ERR_INVALID_ARG
    # training drivers: 16-bit only, every level argument required
    assert lib.ufpn_neck_train_forward(0, 1, None, None, None, None, None, None, None, None, None, None,
                                       None, None, None, None, None, None) == _lib.ERR_UNSUPPORTED
    assert lib.ufpn_neck_train_forward(2, 1, None, None, None, None, None, None, None, None, None, None,
                                       None, None, None, None, None, None) == _lib.ERR_INVALID_ARG
    assert lib.ufpn_neck_train_backward(2, 0, None, None, None, None, None, None, None, None, None,
                                        None, None, None, None, None, None) == _lib.ERR_INVALID_ARG
    assert lib.ufpn_prepare_neck_weights(2, 5, None, None, None, None, None, None, None, None) == \
        _lib.ERR_INVALID_ARG
    # activation codes are 0..3
    assert lib.ufpn_conv3x3_act(2, 16, 16, 16, 16, None, 1, 8, 8, 0, 7, 0.01, None) == _lib.ERR_INVALID_ARG
    assert lib.ufpn_core_set_activation(None, 1, 0.01) == _lib.ERR_INVALID_ARG
    # engine calls on a NULL handle
    assert lib.ufpn_core_forward(None, None, None, None, None) == _lib.ERR_INVALID_ARG
    assert lib.ufpn_core_get_memory_usage(None) == 0
    # reference autotuner rejects Cout != 256 before touching the device
    assert not lib.fpn_auto_tune_lateral_conv(1, 64, 128, 8, 8)


def test_version():
    from unified_fpn import _lib
    assert _lib.lib.ufpn_version() == 100


def test_package_exports_reference_api():
    import unified_fpn
    for name in ("UnifiedFPN", "fpn_lateral_conv", "fpn_upsample_bilinear", "fpn_forward_pytorch",
                 "benchmark_fpn", "profile_fpn", "get_device_info", "check_installation"):
        assert hasattr(unified_fpn, name)


def test_training_workspace_layout_and_pointer_arrays():
    """Host side of the training path: the forward's one workspace holds the 16 weight layouts
    and the four merged maps 256-byte aligned, in order and without overlap; the driver calls'
    int and pointer arrays sit at the addresses handed to the library."""
    from unified_fpn import training as T
    cin, H, W, N = [256, 512, 1024, 2048], [200, 100, 50, 25], [304, 152, 76, 38], 2
    offs, total = T._workspace_layout(N, cin, H, W, 2)
    sizes = []
    for c in cin:
        sizes += [256 * c, (c + 255) // 256 * 256 * 256, 256 * 9 * 256, 256 * 9 * 256]
    sizes += [N * h * w * 256 for h, w in zip(H, W)]
    assert len(offs) == 20 and offs[0] == 0
    assert all(o % 256 == 0 for o in offs)
    ends = [o + 2 * n for o, n in zip(offs, sizes)]
    assert all(e <= o for e, o in zip(ends, offs[1:])) and ends[-1] <= total
    assert total - ends[-1] < 256
    ints, ptrs = [3, 1, 4, 1, 5, 9], [0x1000, None, 0x3000]
    ia, pa, ip, pp = T._arrays(ints, ptrs)
    assert [ctypes.c_int.from_address(ip(k)).value for k in range(len(ints))] == ints
    assert [ctypes.c_void_p.from_address(pp(k)).value for k in range(len(ptrs))] == ptrs
