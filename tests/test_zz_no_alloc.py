"""The no-allocation entry point, ufpn_neck_forward_noalloc, called through the C ABI.

It serves callers that cannot call cudaMalloc on their hot path (a server that owns
all device memory through its own arena, a real-time loop that must not enter the
driver's allocator): they pass every input, weight and output, and the library keeps
its scratch in a fixed device array.  This test checks it against the regular engine
entry point (UnifiedFPN -> ufpn_core_forward) on two calls in a row -- the second call
reuses the scratch array left by the first -- and that oversized problems are refused.

The file name sorts last so that a run stopping at the first failure has already run
every other test.
"""
import ctypes

import pytest
import torch

from oracle import fpn_oracle as O

pytestmark = pytest.mark.gpu


def _ptrs(ts):
    arr = (ctypes.c_void_p * len(ts))()
    for i, t in enumerate(ts):
        arr[i] = t.data_ptr()
    return arr


def _ints(vals):
    return (ctypes.c_int * len(vals))(*vals)


def test_noalloc_neck_matches_engine_on_two_calls(cuda_device):
    import unified_fpn as U
    from unified_fpn import _lib

    chans = O.R50_CHANNELS
    sizes = O.level_sizes(256, 384)
    batch = 2
    feats = [f.to(torch.bfloat16).to(cuda_device).contiguous(memory_format=torch.channels_last)
             for f in O.make_features(batch, chans, sizes, seed=5)]
    wts = O.make_weights(chans, seed=6, bias_scale=0.1)

    fpn = U.UnifiedFPN(device=cuda_device)
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    ref = fpn(feats, return_p6=True)
    torch.cuda.synchronize()

    # Caller-owned weights in the compute dtype (the no-allocation call packs nothing).
    lat_w = [w.to(cuda_device).to(torch.bfloat16).contiguous() for w in wts.lat_w]
    out_w = [U.pack_conv3x3_weight(w.to(cuda_device), torch.bfloat16) for w in wts.out_w]
    lat_b = [b.to(cuda_device).float().contiguous() for b in wts.lat_b]
    out_b = [b.to(cuda_device).float().contiguous() for b in wts.out_b]
    outs = [torch.empty_like(r) for r in ref]
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    torch.cuda.synchronize()

    for call in range(2):
        for o in outs:
            o.fill_(float("nan"))
        rc = _lib.lib.ufpn_neck_forward_noalloc(
            _lib.DTYPE_BF16, _ptrs(feats), _ptrs(lat_w), _ptrs(lat_b), _ptrs(out_w), _ptrs(out_b),
            _ptrs(outs[:4]), outs[4].data_ptr(), batch, _ints(chans), _ints([h for h, _ in sizes]),
            _ints([w for _, w in sizes]), status.data_ptr(), stream)
        assert rc == 0, _lib.lib.ufpn_last_error()
        torch.cuda.synchronize()
        assert status.item() == 0, f"call {call}: pipeline status {status.item():#x}"
        for k, (a, b) in enumerate(zip(outs, ref)):
            assert a.shape == b.shape
            err = O.rel_err(a.float().cpu(), b.float().cpu())
            assert err <= O.TOL["bf16"], f"call {call}, P{k + 2}: rel err {err}"


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
