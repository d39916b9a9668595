"""GPU parity tests of the standalone kernels, called through the C ABI
(libunified_fpn_b200.so via ctypes), against the CPU oracle."""
import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fpn_oracle as O

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _golden_bilinear():
    z = np.load(GOLDEN / "bilinear_ref.npz")
    n = len([k for k in z.files if k.endswith("_shape")])
    return [(z[f"case{i}_shape"], z[f"case{i}_in"], z[f"case{i}_out"]) for i in range(n)]


def _cl(x):
    return x.contiguous(memory_format=torch.channels_last)


# ----------------------------------------------------------------------------- upsample
@pytest.mark.parametrize("case", range(9))
def test_reference_abi_upsample_float_matches_reference_golden(cuda_device, case):
    """launch_production_upsample_float (NHWC, reference C ABI) vs the reference's own
    host implementation's outputs."""
    from unified_fpn import _lib
    shape, x, ref = _golden_bilinear()[case]
    n, c, ih, iw, oh, ow, ac = [int(v) for v in shape]
    xd = _cl(torch.from_numpy(x).to(cuda_device))
    out = _cl(torch.empty(n, c, oh, ow, device=cuda_device))
    ms, gbs = ctypes.c_float(), ctypes.c_float()
    rc = _lib.lib.launch_production_upsample_float(xd.data_ptr(), out.data_ptr(), n, c, ih, iw, oh, ow, ac,
                                                   ctypes.byref(ms), ctypes.byref(gbs))
    assert rc == 0
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=0, atol=1e-5)  # fp32 FMA rounding; reference validator: 1e-3


@pytest.mark.parametrize("case", range(9))
def test_upsample_nchw_fp32_matches_reference_golden(cuda_device, case):
    import unified_fpn as U
    shape, x, ref = _golden_bilinear()[case]
    n, c, ih, iw, oh, ow, ac = [int(v) for v in shape]
    y = U.fpn_upsample_add(torch.from_numpy(x).to(cuda_device), None, size=(oh, ow), align_corners=bool(ac))
    np.testing.assert_allclose(y.cpu().numpy(), ref, rtol=0, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("layout", ["nhwc", "nchw"])
@pytest.mark.parametrize("sizes", [((2, 256, 25, 38), (50, 76)), ((1, 256, 84, 50), (167, 100)),
                                   ((1, 40, 7, 9), (13, 18)),
                                   ((2, 64, 20, 24), (40, 48)),      # NCHW rows of 8-element vectors
                                   ((1, 32, 13, 21), (25, 40)),      # ... with a non-2x width
                                   ((4, 256, 100, 77), (200, 153)),  # 256 ch, W % 8 = 1
                                   ((2, 64, 100, 152), (200, 304)),  # NCHW 8-element vectors
                                   ((1, 16, 64, 64), (24, 32)),      # ... downsampling (8 : 3)
                                   ((2, 256, 200, 152), (400, 304))])  # 124 MB lateral > L2 / 2:
def test_upsample_add(cuda_device, dtype, layout, sizes):          # interleaved NHWC batches
    import unified_fpn as U
    (n, c, hc, wc), (h, w) = sizes
    g = torch.Generator().manual_seed(5)
    coarse = torch.randn(n, c, hc, wc, generator=g).to(dtype)
    lat = torch.randn(n, c, h, w, generator=g).to(dtype)
    cd, ld = coarse.to(cuda_device), lat.to(cuda_device)
    if layout == "nhwc":
        cd, ld = _cl(cd), _cl(ld)
    y = U.fpn_upsample_add(cd, ld)
    ref = lat.float() + O.bilinear_upsample_t(coarse.float(), (h, w))
    O.check_close(y.cpu(), ref, dtype)
    if layout == "nhwc":
        assert y.is_contiguous(memory_format=torch.channels_last)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("geom", [
    (2, (25, 38), (50, 76), (100, 152)),   # R50 800x1216 P5 / P4 / P3
    (3, (42, 25), (84, 50), (167, 100)),   # 1333x800 (odd sizes, ratio not exactly 2)
    (1, (5, 7), (9, 13), (17, 26)),        # small, ragged tiles on both edges
    (2, (20, 20), (20, 20), (40, 40)),     # equal-size step (scale 1) then x2
])
def test_merge_two_levels_bitwise_equals_two_merges(cuda_device, dtype, geom):
    import unified_fpn as U
    n, (h5, w5), (h4, w4), (h3, w3) = geom
    g = torch.Generator().manual_seed(11)
    m5, l4, l3 = (_cl(torch.randn(n, 256, h, w, generator=g).to(dtype).to(cuda_device))
                  for h, w in ((h5, w5), (h4, w4), (h3, w3)))
    m4, m3 = U.fpn_merge_two_levels(m5, l4, l3)
    m4_ref = U.fpn_upsample_add(m5, l4)
    m3_ref = U.fpn_upsample_add(m4_ref, l3)
    assert torch.equal(m4, m4_ref)
    assert torch.equal(m3, m3_ref)
    # and against the oracle's two top-down steps
    r4 = l4.cpu().float() + O.bilinear_upsample_t(m5.cpu().float(), (h4, w4))
    r3 = l3.cpu().float() + O.bilinear_upsample_t(r4.to(dtype).float(), (h3, w3))
    O.check_close(m4.cpu(), r4, dtype)
    O.check_close(m3.cpu(), r3, dtype)


def test_reference_abi_upsample_half_and_bf16(cuda_device):
    from unified_fpn import _lib
    x = torch.randn(2, 64, 13, 19)
    ref = O.bilinear_upsample_t(x, (25, 38))
    for dt, fn in ((torch.float16, _lib.lib.launch_production_upsample_half),
                   (torch.bfloat16, _lib.lib.launch_production_upsample_bfloat16)):
        xd = _cl(x.to(dt).to(cuda_device))
        out = _cl(torch.empty(2, 64, 25, 38, dtype=dt, device=cuda_device))
        assert fn(xd.data_ptr(), out.data_ptr(), 2, 64, 13, 19, 25, 38, 0, None, None) == 0
        O.check_close(out.cpu(), O.bilinear_upsample_t(x.to(dt).float(), (25, 38)), dt)


def test_upsample_engine_abi(cuda_device, tmp_path):
    from unified_fpn import _lib
    lib = _lib.lib
    eng = lib.create_upsample_engine(0)
    assert eng
    x = _cl(torch.randn(1, 32, 8, 8, device=cuda_device))
    out = _cl(torch.empty(1, 32, 16, 16, device=cuda_device))
    m = (ctypes.c_float * 4)()
    assert lib.production_upsample_float(eng, x.data_ptr(), out.data_ptr(), 1, 32, 8, 8, 16, 16, 0.5, 0.5, 0, m) == 0
    assert m[3] > 0
    csv = tmp_path / "prof.csv"
    assert lib.export_upsample_profiling_data(eng, str(csv).encode()) == 0
    assert "bilinear_upsample_f32" in csv.read_text()
    lib.destroy_upsample_engine(eng)
    ref = O.bilinear_upsample_t(x.cpu().contiguous(), (16, 16))
    O.check_close(out.cpu(), ref, "f32")


# ----------------------------------------------------------------------------- P6
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("layout", ["nhwc", "nchw"])
@pytest.mark.parametrize("hw", [(25, 38), (20, 32), (7, 48)])  # (20, 32), (7, 48): NCHW 16-wide rows
def test_p6_exact(cuda_device, dtype, layout, hw):
    import unified_fpn as U
    h, w = hw
    p5 = torch.randn(2, 256, h, w).to(dtype).to(cuda_device)
    if layout == "nhwc":
        p5 = _cl(p5)
    p6 = U.fpn_p6(p5)
    assert p6.shape == (2, 256, (h + 1) // 2, (w + 1) // 2)
    assert torch.equal(p6.cpu(), O.p6_maxpool(p5.cpu().float()).to(dtype))


# ----------------------------------------------------------------------------- lateral (tcgen05)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(1, 64, 7, 9), (2, 256, 20, 30), (1, 96, 16, 16), (2, 2048, 5, 7),
                                   (1, 512, 33, 40)])
def test_lateral_tc(cuda_device, dtype, shape):
    import unified_fpn as U
    n, cin, h, w = shape
    g = torch.Generator().manual_seed(cin + h)
    x = torch.randn(n, cin, h, w, generator=g).to(dtype)
    wt = (torch.randn(256, cin, generator=g) * (2.0 / cin) ** 0.5)
    b = torch.rand(256, generator=g) * 0.2 - 0.1
    y = U.fpn_lateral_conv(_cl(x.to(cuda_device)), wt.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    assert U.device_status() == 0
    ref = O.lateral_conv(x.float(), wt.to(dtype).float(), b)
    O.check_close(y.cpu(), ref, dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("geom", [((2, 256, 20, 30), (10, 15)), ((1, 512, 25, 42), (13, 21)),
                                  ((1, 128, 100, 167), (50, 84)), ((2, 64, 9, 5), (9, 5))])
def test_lateral_tc_fused_upsample_add(cuda_device, dtype, geom):
    import unified_fpn as U
    (n, cin, h, w), (hc, wc) = geom
    g = torch.Generator().manual_seed(hc * 7 + wc)
    x = torch.randn(n, cin, h, w, generator=g).to(dtype)
    coarse = torch.randn(n, 256, hc, wc, generator=g).to(dtype)
    wt = torch.randn(256, cin, generator=g) * (2.0 / cin) ** 0.5
    b = torch.rand(256, generator=g) * 0.2 - 0.1
    y = U.fpn_lateral_conv(_cl(x.to(cuda_device)), wt.to(cuda_device), b.to(cuda_device),
                           coarse=_cl(coarse.to(cuda_device)))
    ref = O.lateral_conv(x.float(), wt.to(dtype).float(), b) + O.bilinear_upsample_t(coarse.float(), (h, w))
    O.check_close(y.cpu(), ref, dtype)
    assert U.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("geom", [
    ((2, 256, 200, 304), (100, 152)),  # R50 800x1216 P2 lateral (950 tiles, even)
    ((1, 256, 20, 30), (10, 15)),      # odd tile count: the pair's second tile is virtual
    ((3, 192, 40, 61), (20, 31)),      # ragged tiles, ratio not exactly 2
    ((2, 64, 9, 5), (9, 5)),           # scale 1, one k-block
    ((1, 256, 33, 40), None),          # no top-down add
])
def test_lateral_cta_pair(cuda_device, dtype, geom):
    """The CTA-pair lateral (resident weight halves, fp32 epilogue taps) against the oracle:
    one rounding of the fp32 result to the 16-bit output (the single-CTA lateral's tensor-core
    top-down add uses 16-bit bilinear weights, so it is only within the looser tolerance)."""
    import unified_fpn as U
    (n, cin, h, w), cg = geom
    g = torch.Generator().manual_seed(cin + h + w)
    x = torch.randn(n, cin, h, w, generator=g).to(dtype)
    wt = torch.randn(256, cin, generator=g) * (2.0 / cin) ** 0.5
    b = torch.rand(256, generator=g) * 0.2 - 0.1
    coarse = torch.randn(n, 256, *cg, generator=g).to(dtype) if cg else None
    args = (_cl(x.to(cuda_device)), wt.to(cuda_device), b.to(cuda_device))
    cd = _cl(coarse.to(cuda_device)) if cg else None
    y = U.fpn_lateral_conv(*args, coarse=cd, cta_pair=True)
    torch.cuda.synchronize()
    assert U.device_status() == 0
    ref = O.lateral_conv(x.float(), wt.to(dtype).float(), b)
    if cg:
        ref = ref + O.bilinear_upsample_t(coarse.float(), (h, w))
    O.check_close(y.cpu(), ref, dtype)
    ulp = ref.abs() * (2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11)  # half an ulp, at most
    assert ((y.cpu().float() - ref).abs() <= 2.01 * ulp + 1e-5 * ref.abs().max()).all()


def test_lateral_cta_pair_unsupported_raises(cuda_device):
    """Cin > 256 (weights no longer fit resident) and tiles whose tap box exceeds 64 coarse
    pixels are refused, not computed wrongly."""
    import unified_fpn as U
    x = _cl(torch.randn(1, 512, 16, 16, device=cuda_device, dtype=torch.bfloat16))
    with pytest.raises(U.UFPNError):
        U.fpn_lateral_conv(x, torch.randn(256, 512, device=cuda_device), torch.zeros(256, device=cuda_device),
                           cta_pair=True)
    x = _cl(torch.randn(1, 64, 41, 57, device=cuda_device, dtype=torch.bfloat16))
    c = _cl(torch.randn(1, 256, 21, 29, device=cuda_device, dtype=torch.bfloat16))
    with pytest.raises(U.UFPNError):
        U.fpn_lateral_conv(x, torch.randn(256, 64, device=cuda_device), torch.zeros(256, device=cuda_device),
                           coarse=c, cta_pair=True)


def test_lateral_fp32_config1(cuda_device):
    """Single-level fused op, fp32 NCHW b1: conv1x1(C3 [1,512,64,64]) + up2x(P4 [1,256,32,32])."""
    import unified_fpn as U
    c3, p4, w, b = O.config1_inputs(seed=0)
    y = U.fpn_lateral_conv(c3.to(cuda_device), w.to(cuda_device), b.to(cuda_device), coarse=p4.to(cuda_device))
    ref = O.fused_lateral_upsample(c3, p4, w, b)
    O.check_close(y.cpu(), ref, "f32")


# ----------------------------------------------------------------------------- 3x3 (tcgen05)
@pytest.mark.parametrize("tile_w", [8, 16, 32, 64, 128])
def test_conv3x3_tc_tilings(cuda_device, tile_w):
    import unified_fpn as U
    g = torch.Generator().manual_seed(tile_w)
    x = torch.randn(1, 256, 9, 13, generator=g).to(torch.bfloat16)
    w = torch.randn(256, 256, 3, 3, generator=g) * (2.0 / 2304) ** 0.5
    b = torch.rand(256, generator=g) * 0.2 - 0.1
    y = U.fpn_conv3x3(_cl(x.to(cuda_device)), w.to(cuda_device), b.to(cuda_device), tile_w=tile_w)
    ref = O.conv3x3(x.float(), w.to(torch.bfloat16).float(), b)
    O.check_close(y.cpu(), ref, "bf16")
    assert U.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 25, 38), (1, 50, 84), (1, 1, 1), (3, 17, 5)])
def test_conv3x3_tc_with_p6(cuda_device, dtype, shape):
    import unified_fpn as U
    n, h, w_ = shape
    g = torch.Generator().manual_seed(h * 100 + w_)
    x = torch.randn(n, 256, h, w_, generator=g).to(dtype)
    w = torch.randn(256, 256, 3, 3, generator=g) * (2.0 / 2304) ** 0.5
    b = torch.rand(256, generator=g) * 0.2 - 0.1
    y, p6 = U.fpn_conv3x3(_cl(x.to(cuda_device)), w.to(cuda_device), b.to(cuda_device), p6=True)
    ref = O.conv3x3(x.float(), w.to(dtype).float(), b)
    O.check_close(y.cpu(), ref, dtype)
    assert torch.equal(p6.cpu(), y.cpu()[:, :, ::2, ::2])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(1, 16, 8), (1, 13, 21), (2, 25, 38), (3, 17, 5), (1, 1, 1),
                                   (2, 200, 304), (1, 200, 304)])
def test_conv3x3_cta_pair_equals_single(cuda_device, dtype, shape):
    """Halo tiles on CTA pairs (tcgen05 cta_group::2, M = 256: two tiles per MMA stream, each
    CTA streaming half of the weights) give bitwise the results of single-CTA halo tiles:
    every output's K summation runs in the same order.  Odd tile counts exercise the
    virtual (never stored) second tile of the last pair; (2, 200, 304) is the R50 P2 map.
    On 148 SMs (74 pairs) the 1 x 200 x 304 map ends with a short round (247 units: 25 left)
    that runs as channel halves (N = 128 items); 2 x 200 x 304 (494 units: 50 left) does
    not."""
    import unified_fpn as U
    n, h, w_ = shape
    g = torch.Generator().manual_seed(h * 31 + w_)
    x = torch.randn(n, 256, h, w_, generator=g).to(dtype)
    w = torch.randn(256, 256, 3, 3, generator=g) * (2.0 / 2304) ** 0.5
    b = torch.rand(256, generator=g) * 0.2 - 0.1
    xd = _cl(x.to(cuda_device))
    wp = U.pack_conv3x3_weight(w.to(cuda_device), dtype)
    y1, p1 = U.fpn_conv3x3(xd, wp, b.to(cuda_device), p6=True, tile_w=0)
    y2, p2 = U.fpn_conv3x3(xd, wp, b.to(cuda_device), p6=True, tile_w=-1)
    torch.cuda.synchronize()
    assert U.device_status() == 0
    assert torch.equal(y1, y2) and torch.equal(p1, p2)
    if n * h * w_ <= 4096:
        ref = O.conv3x3(x.float(), w.to(dtype).float(), b)
        O.check_close(y2.cpu(), ref, dtype)


def _mixed_forms(n, h, w_):
    """tile_w codes of the mixed tiling that apply to n x h x w_ (-4 single CTA, -5 pairs)."""
    if h < 16 or h % 16 == 0 or h % 16 > 8:
        return []
    own = n * ((w_ + 7) // 8) * (h // 16)
    return [-4] + ([-5] if own % 2 == 0 else [])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(1, 16, 8), (1, 8, 16), (1, 13, 21), (3, 17, 5), (1, 1, 1),
                                   (2, 37, 50), (1, 200, 334), (2, 200, 304), (1, 24, 9)])
def test_conv3x3_transposed_view_equals_plain(cuda_device, dtype, shape):
    """Halo tiles on the map's transposed view (tile_w -2 on single CTAs, -3 on CTA pairs:
    16 columns x 8 rows per tile through tensor maps with the two axes swapped, each tap's
    halo shift mirrored) and the mixed tiling (-4 / -5: the own view for the whole 16-row
    tile rows, the transposed view for the last 1..8 rows, where it applies) give bitwise the
    results of the plain halo tiles, and match the oracle.  Ragged edges fall on other axes
    than with plain tiles.  (2, 200, 304), the R50 P2 map: 950 tiles instead of 988 either
    way (mixed: 912 own-view + 38 strip tiles), 475 pair units on 74 pairs whose last 31 run
    as channel halves; on single CTAs its last 62 of 950 tiles (100 of 988 on the own view)
    run as channel halves on 148 SMs.  (3, 17, 5): an odd own-view count, single CTAs only; (1, 24, 9): an
    odd one on pairs too."""
    import unified_fpn as U
    n, h, w_ = shape
    g = torch.Generator().manual_seed(h * 37 + w_)
    x = torch.randn(n, 256, h, w_, generator=g).to(dtype)
    w = torch.randn(256, 256, 3, 3, generator=g) * (2.0 / 2304) ** 0.5
    b = torch.rand(256, generator=g) * 0.2 - 0.1
    xd = _cl(x.to(cuda_device))
    wp = U.pack_conv3x3_weight(w.to(cuda_device), dtype)
    bd = b.to(cuda_device)
    ys = [U.fpn_conv3x3(xd, wp, bd, tile_w=t) for t in [0, -2, -1, -3] + _mixed_forms(n, h, w_)]
    torch.cuda.synchronize()
    assert U.device_status() == 0
    assert all(torch.equal(ys[0], y) for y in ys[1:])
    if n * h * w_ <= 4096:
        ref = O.conv3x3(x.float(), w.to(dtype).float(), b)
        O.check_close(ys[1].cpu(), ref, dtype)
    else:  # first and last image rows of the large maps against the oracle
        ref = O.conv3x3(x[:1, :, :12].float(), w.to(dtype).float(), b)
        O.check_close(ys[3][:1, :, :11].cpu(), ref[:, :, :11], dtype)
        ref = O.conv3x3(x[-1:, :, -12:].float(), w.to(dtype).float(), b)
        O.check_close(ys[3][-1:, :, -11:].cpu(), ref[:, :, -11:], dtype)


def test_conv3x3_transposed_view_refuses_p6(cuda_device):
    """The fused P6 output indexes the map's own rows: the transposed view and the mixed
    tiling refuse it on the host (no launch), as the mixed tiling refuses maps it does not
    apply to."""
    import unified_fpn as U
    x = _cl(torch.randn(1, 256, 8, 8, device=cuda_device).to(torch.bfloat16))
    w = U.pack_conv3x3_weight(torch.randn(256, 256, 3, 3, device=cuda_device), torch.bfloat16)
    b = torch.zeros(256, device=cuda_device)
    for t in (-2, -3, -4, -5):
        with pytest.raises(Exception):
            U.fpn_conv3x3(x, w, b, p6=True, tile_w=t)
    with pytest.raises(Exception):
        U.fpn_conv3x3(x, w, b, tile_w=-6)
    # the mixed tiling needs 1..8 rows past the last whole 16-row tile row, and on CTA pairs
    # an even number of own-view tiles
    for shape, t in (((1, 256, 32, 8), -4), ((1, 256, 8, 8), -4), ((1, 256, 28, 8), -4),
                     ((3, 256, 17, 5), -5)):
        xs = _cl(torch.randn(*shape, device=cuda_device).to(torch.bfloat16))
        with pytest.raises(Exception):
            U.fpn_conv3x3(xs, w, b, tile_w=t)
    assert U.device_status() == 0


def test_conv3x3_fp32(cuda_device):
    import unified_fpn as U
    g = torch.Generator().manual_seed(3)
    x = torch.randn(1, 256, 11, 14, generator=g)
    w = torch.randn(256, 256, 3, 3, generator=g) * (2.0 / 2304) ** 0.5
    b = torch.rand(256, generator=g) * 0.2 - 0.1
    y = U.fpn_conv3x3(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device))
    O.check_close(y.cpu(), O.conv3x3(x, w, b), "f32")


def test_layout_convert_roundtrip(cuda_device):
    from unified_fpn import _lib
    x = torch.randn(2, 40, 7, 9, device=cuda_device, dtype=torch.bfloat16)
    y = torch.empty(2, 7, 9, 40, device=cuda_device, dtype=torch.bfloat16)
    z = torch.empty_like(x)
    s = torch.cuda.current_stream().cuda_stream
    assert _lib.lib.ufpn_layout_convert(2, x.data_ptr(), y.data_ptr(), 2, 40, 7, 9, 1, s) == 0
    assert _lib.lib.ufpn_layout_convert(2, y.data_ptr(), z.data_ptr(), 2, 40, 7, 9, 0, s) == 0
    assert torch.equal(y, x.permute(0, 2, 3, 1))
    assert torch.equal(z, x)


@pytest.mark.parametrize("dtype,tile_w", [(torch.bfloat16, 0), (torch.bfloat16, -1), (torch.float16, 16),
                                          (torch.float32, 0)])
@pytest.mark.parametrize("act,alpha", [("relu", 0.01), ("leaky_relu", 0.2), ("swish", 0.01)])
def test_conv3x3_activation_epilogue(cuda_device, dtype, tile_w, act, alpha):
    """The activation fused into the 3x3 epilogue after the bias (P6 taken from the activated
    output) against the oracle's conv3x3 followed by the reference's activation formula."""
    import unified_fpn as U
    g = torch.Generator().manual_seed(len(act) * 7 + tile_w)
    x = torch.randn(2, 256, 13, 21, generator=g).to(dtype)
    w = torch.randn(256, 256, 3, 3, generator=g) * (2.0 / 2304) ** 0.5
    b = torch.rand(256, generator=g) * 0.2 - 0.1
    xd = x.to(cuda_device)
    if dtype != torch.float32:
        xd = _cl(xd)
    y, p6 = U.fpn_conv3x3(xd, w.to(cuda_device), b.to(cuda_device), p6=True, tile_w=tile_w,
                          activation=act, alpha=alpha)
    torch.cuda.synchronize()
    assert U.device_status() == 0
    ref = O.activation(O.conv3x3(x.float(), w.to(dtype).float(), b), act, alpha)
    O.check_close(y.float().cpu(), ref, dtype)
    assert torch.equal(p6.cpu(), y.cpu()[:, :, ::2, ::2])
    if act == "relu":
        assert y.min().item() >= 0
    with pytest.raises(ValueError):
        U.fpn_conv3x3(xd, w.to(cuda_device), b.to(cuda_device), activation="gelu")
