"""The no-allocation entry point, ufpn_neck_forward_noalloc, called through the C ABI.

It serves callers that cannot call cudaMalloc on their hot path (a server that owns
all device memory through its own arena, a real-time loop that must not enter the
driver's allocator): they pass every input, weight and output, and the library keeps
its scratch in a fixed device array.  These tests check it against the regular engine
entry point (UnifiedFPN -> ufpn_core_forward) and against the CPU oracle, for bf16 and
fp16 inputs at ResNet-50 and Swin-style odd sizes, on two calls in a row -- the second
call reuses the scratch array left by the first -- and that oversized or misordered
problems are refused before anything runs.

The file name sorts last so that a run stopping at the first failure has already run
every other test.
"""
import ctypes

import pytest
import torch

from oracle import fpn_oracle as O


def _ptrs(ts):
    arr = (ctypes.c_void_p * len(ts))()
    for i, t in enumerate(ts):
        arr[i] = t.data_ptr() if isinstance(t, torch.Tensor) else t
    return arr


def _ints(vals):
    return (ctypes.c_int * len(vals))(*vals)


CASES = [
    ("r50_256x384_b2", O.R50_CHANNELS, O.level_sizes(256, 384), 2, "relu_normal"),
    ("swin_1333x800_b1", O.SWIN_CHANNELS, [(200, 334), (100, 167), (50, 84), (25, 42)], 1, "normal"),
]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_noalloc_neck_matches_engine_and_oracle_on_two_calls(cuda_device, dtype, case):
    import unified_fpn as U
    from unified_fpn import _lib

    _, chans, sizes, batch, dist = case
    host = O.make_features(batch, chans, sizes, seed=5, dist=dist)
    feats = [f.to(dtype).to(cuda_device).contiguous(memory_format=torch.channels_last) for f in host]
    wts = O.make_weights(chans, seed=6, bias_scale=0.1)

    fpn = U.UnifiedFPN(device=cuda_device)
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    engine = [o.clone() for o in fpn(feats, return_p6=True)]
    torch.cuda.synchronize()

    rw = O.NeckWeights([O.round_to(w, dtype) for w in wts.lat_w], wts.lat_b,
                       [O.round_to(w, dtype) for w in wts.out_w], wts.out_b)
    ref = O.fpn_neck([O.round_to(f[:1], dtype) for f in host], rw)

    # Caller-owned weights in the compute dtype (the no-allocation call packs nothing).
    lat_w = [w.to(cuda_device).to(dtype).contiguous() for w in wts.lat_w]
    out_w = [U.pack_conv3x3_weight(w.to(cuda_device), dtype) for w in wts.out_w]
    lat_b = [b.to(cuda_device).float().contiguous() for b in wts.lat_b]
    out_b = [b.to(cuda_device).float().contiguous() for b in wts.out_b]
    outs = [torch.empty_like(e) for e in engine]
    status = torch.full((1,), 7, dtype=torch.int32, device=cuda_device)  # the call zeroes it
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    code = _lib.DTYPE_BF16 if dtype == torch.bfloat16 else _lib.DTYPE_F16
    torch.cuda.synchronize()

    for call in range(2):
        for o in outs:
            o.fill_(float("nan"))
        rc = _lib.lib.ufpn_neck_forward_noalloc(
            code, _ptrs(feats), _ptrs(lat_w), _ptrs(lat_b), _ptrs(out_w), _ptrs(out_b),
            _ptrs(outs[:4]), outs[4].data_ptr(), batch, _ints(chans), _ints([h for h, _ in sizes]),
            _ints([w for _, w in sizes]), status.data_ptr(), stream)
        assert rc == 0, _lib.lib.ufpn_last_error()
        torch.cuda.synchronize()
        assert status.item() == 0, f"call {call}: pipeline status {status.item():#x}"
        for k, (a, e, r) in enumerate(zip(outs, engine, ref)):
            assert a.shape == e.shape
            # the engine's split schedule rounds L4 / L3 to 16 bits before their top-down add,
            # the one-launch neck does not: both within the tolerance of the oracle
            O.check_close(a.float().cpu(), e.float().cpu(), dtype)
            O.check_close(a[:1].float().cpu(), r, dtype)


@pytest.mark.gpu
def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    from unified_fpn import _lib

    dummy = [torch.empty(16, dtype=torch.bfloat16, device=cuda_device) for _ in range(4)]
    bias = [torch.empty(256, device=cuda_device) for _ in range(4)]
    big = O.level_sizes(2048, 2048)  # 8 images: ~2.8 GB of merged maps
    rc = _lib.lib.ufpn_neck_forward_noalloc(
        _lib.DTYPE_BF16, _ptrs(dummy), _ptrs(dummy), _ptrs(bias), _ptrs(dummy), _ptrs(bias),
        _ptrs(dummy), None, 8, _ints(O.R50_CHANNELS), _ints([h for h, _ in big]),
        _ints([w for _, w in big]), None, None)
    assert rc == _lib.ERR_INVALID_ARG
    assert b"scratch" in _lib.lib.ufpn_last_error()


def test_noalloc_rejects_misordered_levels_before_any_launch():
    """Levels must go fine (C2) to coarse (C5), as for the engine.  The check runs before the
    entry point touches a device, so dummy (never dereferenced) pointers suffice here."""
    from unified_fpn import _lib

    fake = [0x1000 + 0x100 * i for i in range(4)]
    sizes = O.level_sizes(128, 192)
    swapped = [sizes[0], sizes[2], sizes[1], sizes[3]]  # C3 smaller than C4
    rc = _lib.lib.ufpn_neck_forward_noalloc(
        _lib.DTYPE_BF16, _ptrs(fake), _ptrs(fake), _ptrs(fake), _ptrs(fake), _ptrs(fake),
        _ptrs(fake), None, 1, _ints(O.R50_CHANNELS), _ints([h for h, _ in swapped]),
        _ints([w for _, w in swapped]), None, None)
    assert rc == _lib.ERR_INVALID_ARG
    assert b"ordered" in _lib.lib.ufpn_last_error()
