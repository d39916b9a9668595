"""GPU parity tests of the FP8 (e4m3) path against the CPU oracle: quantisers bit for bit,
the e4m3 lateral and 3x3 kernels, and the whole FP8 neck (UnifiedFPN with
float8_e4m3fn inputs) including the FP8 benchmark's per-GPU shape."""
import numpy as np
import pytest
import torch

from oracle import fpn_oracle as O

pytestmark = pytest.mark.gpu
TOL8 = O.TOL["e4m3"]   # 3e-2, max-norm relative
E4M3 = torch.float8_e4m3fn


def _cl(x):
    return x.contiguous(memory_format=torch.channels_last)


def _codes(q: torch.Tensor) -> np.ndarray:
    """e4m3 tensor (any layout) -> its values as fp32 numpy in logical NCHW order."""
    return q.float().cpu().numpy()


def _upload_codes(codes, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(codes)).to(E4M3).to(device)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(2, 64, 9, 13), (3, 1001)])
def test_quantize_fp8_bitexact(cuda_device, dtype, shape):
    import unified_fpn as U
    g = torch.Generator().manual_seed(11)
    x = (torch.randn(*shape, generator=g) * 3).to(dtype)
    xd = x.cuda()
    if xd.dim() == 4:
        xd = _cl(xd)
    q, s = U.quantize_fp8(xd)
    qo, so = O.quantize_e4m3_tensor(x.float())
    np.testing.assert_array_equal(_codes(q), qo)
    assert s.item() == float(so)
    # per-image groups
    q2, s2 = U.quantize_fp8(xd, per_image=True)
    qo2, so2 = O.quantize_e4m3_images(x.float())
    np.testing.assert_array_equal(_codes(q2), qo2)
    np.testing.assert_array_equal(s2.cpu().numpy(), so2)


def test_quantize_fp8_zero_tensor(cuda_device):
    import unified_fpn as U
    q, s = U.quantize_fp8(torch.zeros(4, 64, device="cuda", dtype=torch.bfloat16))
    assert s.item() == 1.0 and not q.float().any()


def test_quantize_fp8_rows_bitexact(cuda_device):
    import unified_fpn as U
    g = torch.Generator().manual_seed(12)
    wl = torch.randn(256, 512, generator=g) * 0.06
    w3 = torch.randn(256, 256, 3, 3, generator=g) * 0.03
    ql, sl = U.quantize_fp8_rows(wl.cuda())
    qo, so = O.quantize_e4m3_rows(wl)
    np.testing.assert_array_equal(_codes(ql), qo)
    np.testing.assert_array_equal(sl.cpu().numpy(), so)
    q3, s3 = U.quantize_fp8_rows(w3.cuda(), pack3x3=True)
    qo3, so3 = O.quantize_e4m3_rows(w3)
    packed = qo3.reshape(256, 256, 9).transpose(0, 2, 1)        # [o][tap][c]
    np.testing.assert_array_equal(_codes(q3), packed)
    np.testing.assert_array_equal(s3.cpu().numpy(), so3)


def _lateral_oracle(qx, sx, qw, sw, b, coarse=None):
    acc = torch.nn.functional.conv2d(torch.from_numpy(qx).double(),
                                     torch.from_numpy(qw).double().reshape(256, -1, 1, 1))
    sx = np.asarray(sx, dtype=np.float32).reshape(-1)
    cs = (torch.from_numpy(sx).reshape(-1, 1) * torch.from_numpy(sw).reshape(1, -1)).double()
    y = acc * cs.reshape(cs.shape[0], -1, 1, 1) + b.double().reshape(1, -1, 1, 1)
    if coarse is not None:
        y = y + O.bilinear_upsample_t(coarse.double(), y.shape[-2:])
    return y.float().to(torch.bfloat16).float()


@pytest.mark.parametrize("geom", [
    (2, 512, (40, 56), None),
    (2, 256, (50, 76), (25, 38)),      # 2x top-down
    (1, 128, (100, 167), (50, 84)),    # Swin odd, non-2x
    (1, 2048, (20, 20), None),
])
def test_lateral_fp8_matches_oracle(cuda_device, geom):
    import unified_fpn as U
    N, Cin, (H, W), csz = geom
    g = torch.Generator().manual_seed(13)
    x = torch.randn(N, Cin, H, W, generator=g)
    w = torch.randn(256, Cin, generator=g) * (2.0 / Cin) ** 0.5
    b = (torch.rand(256, generator=g) * 2 - 1) * 0.1
    qx, sx = O.quantize_e4m3_tensor(x)
    qw, sw = O.quantize_e4m3_rows(w)
    coarse = None if csz is None else torch.randn(N, 256, *csz, generator=g).to(torch.bfloat16).float()
    amax = torch.zeros(N, dtype=torch.int32, device="cuda")
    out = U.fpn_lateral_conv_fp8(_cl(_upload_codes(qx)), torch.tensor([float(sx)]),
                                 _upload_codes(qw), torch.from_numpy(sw).cuda(), b.cuda(),
                                 None if coarse is None else _cl(coarse.to(torch.bfloat16).cuda()),
                                 amax_out=amax)
    torch.cuda.synchronize()
    assert U.device_status() == 0
    ref = _lateral_oracle(qx, sx, qw, sw, b, coarse)
    O.check_close(out.float().cpu(), ref, "bf16")  # bf16 output of exact e4m3 products
    # per-image absmax of the stored bf16 output, bit for bit
    per_img = out.float().abs().amax(dim=(1, 2, 3)).cpu()
    got = amax.cpu().view(torch.float32)
    assert torch.equal(got, per_img)


@pytest.mark.parametrize("per_image", [False, True])
@pytest.mark.parametrize("shape", [(2, 40, 56), (1, 25, 38), (3, 13, 21), (1, 200, 304)])
def test_conv3x3_fp8_matches_oracle(cuda_device, shape, per_image):
    import unified_fpn as U
    N, H, W = shape
    g = torch.Generator().manual_seed(14)
    m = torch.randn(N, 256, H, W, generator=g)
    w3 = torch.randn(256, 256, 3, 3, generator=g) * (2.0 / 2304) ** 0.5
    b = (torch.rand(256, generator=g) * 2 - 1) * 0.1
    if per_image:
        qm, sm = O.quantize_e4m3_images(m)
    else:
        qm, s1 = O.quantize_e4m3_tensor(m)
        sm = np.array([s1], dtype=np.float32)
    qw, sw = O.quantize_e4m3_rows(w3)
    qwd, swd = U.quantize_fp8_rows(w3.cuda(), pack3x3=True)
    out, p6 = U.fpn_conv3x3_fp8(_cl(_upload_codes(qm)), torch.from_numpy(sm), qwd, swd, b.cuda(),
                                p6=True)
    out2, p62 = U.fpn_conv3x3_fp8(_cl(_upload_codes(qm)), torch.from_numpy(sm), qwd, swd, b.cuda(),
                                  p6=True, tile_w=-1)   # the same tiles on CTA pairs
    torch.cuda.synchronize()
    assert U.device_status() == 0
    assert torch.equal(out, out2) and torch.equal(p6, p62)
    acc = torch.nn.functional.conv2d(torch.from_numpy(qm).double(), torch.from_numpy(qw).double(),
                                     padding=1)
    cs = (torch.from_numpy(sm).reshape(-1, 1) * torch.from_numpy(sw).reshape(1, -1)).double()
    ref = (acc * cs.reshape(cs.shape[0], -1, 1, 1) + b.double().reshape(1, -1, 1, 1)).float()
    ref = ref.to(torch.bfloat16).float()
    O.check_close(out.float().cpu(), ref, "bf16")  # bf16 output of exact e4m3 products
    assert torch.equal(p6.cpu(), out[:, :, ::2, ::2].cpu())


@pytest.mark.parametrize("shape", [(3, 13, 21), (2, 37, 50), (1, 200, 304)])
def test_conv3x3_fp8_transposed_view_equals_plain(cuda_device, shape):
    """e4m3 3x3 halo tiles on the map's transposed view (tile_w -2, and -3 on CTA pairs) and
    with the mixed tiling (-4, -5) give bitwise the plain halo tiles' results."""
    import unified_fpn as U
    N, H, W = shape
    g = torch.Generator(device="cuda").manual_seed(16)
    m = _cl(torch.randn(N, 256, H, W, device="cuda", generator=g).to(torch.bfloat16))
    w3 = torch.randn(256, 256, 3, 3, device="cuda", generator=g) * (2.0 / 2304) ** 0.5
    b = (torch.rand(256, device="cuda", generator=g) * 2 - 1) * 0.1
    qw, sw = U.quantize_fp8_rows(w3, pack3x3=True)
    qm, sm = U.quantize_fp8(m, per_image=True)
    mixed = [-4, -5] if H >= 16 and 0 < H % 16 <= 8 and (N * ((W + 7) // 8) * (H // 16)) % 2 == 0 \
        else []
    ys = [U.fpn_conv3x3_fp8(qm, sm, qw, sw, b, tile_w=t) for t in [0, -2, -1, -3] + mixed]
    torch.cuda.synchronize()
    assert U.device_status() == 0
    assert all(torch.equal(ys[0], y) for y in ys[1:])


@pytest.mark.parametrize("shape", [(2, 40, 56), (1, 25, 38), (3, 13, 21), (16, 160, 160),
                                   (1, 200, 304)])
def test_conv3x3_fp8_in_kernel_quantisation(cuda_device, shape):
    """The CTA-pair e4m3 3x3 that quantises its bf16 input per image in shared memory gives
    bitwise what quantising first (the standalone quantiser) and convolving gives (1 x 200 x
    304: 247 pair units, the last 25 as channel halves on 148 SMs)."""
    import unified_fpn as U
    N, H, W = shape
    g = torch.Generator(device="cuda").manual_seed(15)
    m = _cl(torch.randn(N, 256, H, W, device="cuda", generator=g).to(torch.bfloat16))
    w3 = torch.randn(256, 256, 3, 3, device="cuda", generator=g) * (2.0 / 2304) ** 0.5
    b = (torch.rand(256, device="cuda", generator=g) * 2 - 1) * 0.1
    qw, sw = U.quantize_fp8_rows(w3, pack3x3=True)
    qm, sm = U.quantize_fp8(m, per_image=True)
    ref, ref6 = U.fpn_conv3x3_fp8(qm, sm, qw, sw, b, p6=True, tile_w=-1)
    amax = m.float().abs().amax(dim=(1, 2, 3)).contiguous().view(torch.int32)
    out, p6 = U.fpn_conv3x3_fp8_from_bf16(m, amax, qw, sw, b, p6=True)
    torch.cuda.synchronize()
    assert U.device_status() == 0
    assert torch.equal(out, ref) and torch.equal(p6, ref6)


def _fp8_case(batch, chans, sizes, seed, bias_scale=0.1):
    feats = O.make_features(batch, chans, sizes, seed=seed, dist="normal")
    wts = O.make_weights(chans, seed=seed + 1, bias_scale=bias_scale)
    qf, sc = zip(*[O.quantize_e4m3_tensor(f) for f in feats])
    return feats, wts, [torch.from_numpy(q) for q in qf], list(sc)


def _run_fp8_neck(chans, wts, qf, sc, fpn=None):
    import unified_fpn as U
    fpn = fpn or U.UnifiedFPN()
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    xin = [_cl(q.to(E4M3).cuda()) for q in qf]
    outs = fpn(xin, return_p6=True, input_scales=[float(s) for s in sc])
    torch.cuda.synchronize()
    assert fpn.device_status() == 0
    return fpn, xin, outs


@pytest.mark.parametrize("geom", [
    (2, O.R50_CHANNELS, O.level_sizes(128, 192)),
    (1, O.SWIN_CHANNELS, [(100, 167), (50, 84), (25, 42), (13, 21)]),
    (2, O.R50_CHANNELS, O.level_sizes(640, 640)),   # the FP8 benchmark's image size
])
def test_fp8_neck_matches_oracle(cuda_device, geom):
    batch, chans, sizes = geom
    feats, wts, qf, sc = _fp8_case(batch, chans, sizes, seed=21)
    fpn, _, outs = _run_fp8_neck(chans, wts, qf, sc)
    ref = O.fpn_neck_e4m3(qf, sc, O.quantize_neck_weights(wts))
    for o, r in zip(outs, ref):
        assert o.dtype == torch.bfloat16 and tuple(o.shape) == tuple(r.shape)
        assert o.is_contiguous(memory_format=torch.channels_last)
        O.check_close(o.float().cpu(), r, "e4m3")
    # accuracy against the unquantised fp32 neck, reported by the assertion message only
    full = O.fpn_neck(feats, wts)
    drift = [round(O.rel_err(o.float().cpu(), r), 4) for o, r in zip(outs, full)]
    assert max(drift) < 0.15, drift


def test_fp8_neck_batch_sharding_is_exact(cuda_device):
    """M_l is quantised per image, so each image's outputs are independent of the rest of
    the batch: a batch slice (one GPU's shard) gives bit-identical results."""
    chans, sizes = O.R50_CHANNELS, O.level_sizes(160, 224)
    _, wts, qf, sc = _fp8_case(4, chans, sizes, seed=31)
    fpn, xin, full = _run_fp8_neck(chans, wts, qf, sc)
    for lo, hi in ((0, 1), (1, 3), (3, 4)):
        part = fpn([_cl(x[lo:hi]) for x in xin], return_p6=True, input_scales=[float(s) for s in sc])
        torch.cuda.synchronize()
        for a, b in zip(full, part):
            assert torch.equal(a[lo:hi], b)


def test_fp8_neck_benchmark_shard_full_size(cuda_device):
    """One GPU's shard of the FP8 benchmark at full size: R50 neck, 16 images at 640x640,
    e4m3 inputs.  Size-independent properties: graph replay == direct launch bitwise,
    repeat determinism, and image 0 equals the oracle on that image alone."""
    import unified_fpn as U
    chans, sizes = O.R50_CHANNELS, O.level_sizes(640, 640)
    g = torch.Generator(device="cuda").manual_seed(5)
    feats = [torch.randn(16, c, h, w, generator=g, device="cuda") for c, (h, w) in zip(chans, sizes)]
    qs = [U.quantize_fp8(_cl(f)) for f in feats]
    xin = [q for q, _ in qs]
    scales = [s for _, s in qs]
    wts = O.make_weights(chans, seed=6)
    fpn = U.UnifiedFPN()
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    outs = fpn(xin, return_p6=True, input_scales=scales)
    again = fpn(xin, return_p6=True, input_scales=scales)
    fpn.set_kernel_config(enable_graph_capture=False)
    direct = fpn(xin, return_p6=True, input_scales=scales)
    torch.cuda.synchronize()
    assert fpn.device_status() == 0
    for a, b, c in zip(outs, again, direct):
        assert torch.equal(a, b) and torch.equal(a, c)
    qf0 = [torch.from_numpy(_codes(x[:1])) for x in xin]
    ref = O.fpn_neck_e4m3(qf0, [np.float32(s.item()) for s in scales], O.quantize_neck_weights(wts))
    for o, r in zip(outs, ref):
        O.check_close(o[:1].float().cpu(), r, "e4m3")


def test_fp8_errors(cuda_device):
    import unified_fpn as U
    fpn = U.UnifiedFPN()
    x = [_cl(torch.zeros(1, c, 8, 8, device="cuda").to(E4M3)) for c in O.R50_CHANNELS]
    with pytest.raises(ValueError):
        fpn(x)                                  # no input scales
    with pytest.raises(ValueError):
        fpn([torch.zeros(1, c, 8, 8, device="cuda", dtype=torch.bfloat16) for c in O.R50_CHANNELS],
            input_scales=[1.0] * 4)             # scales for a 16-bit neck


def test_fp8_neck_activation(cuda_device):
    """LeakyReLU on the e4m3 neck's 3x3 outputs (applied to the scaled fp32 value before the
    bf16 store) against the e4m3 oracle with the same activation."""
    import unified_fpn as U
    feats, wts, qf, sc = _fp8_case(2, O.R50_CHANNELS, O.level_sizes(128, 192), seed=31)
    fpn = U.UnifiedFPN()
    fpn.set_activation("leaky_relu", 0.1)
    _, _, outs = _run_fp8_neck(O.R50_CHANNELS, wts, qf, sc, fpn=fpn)
    ref = O.fpn_neck_e4m3(qf, sc, O.quantize_neck_weights(wts), act="leaky_relu", alpha=0.1)
    for o, r in zip(outs, ref):
        O.check_close(o.float().cpu(), r, "e4m3")


@pytest.mark.parametrize("geom", [(2, O.R50_CHANNELS, O.level_sizes(128, 192)),
                                  (16, O.R50_CHANNELS, O.level_sizes(640, 640))])
def test_fp8_two_pass_p2_lateral_is_bitwise_equal(cuda_device, geom):
    """The P2 lateral's absmax pass + quantised store against storing bf16 M2 and quantising it
    in a separate pass (the default): the same e4m3 codes and scales, so bitwise the same
    outputs; at the benchmark's 640x640 batch-16 size too."""
    import unified_fpn as U
    batch, chans, sizes = geom
    feats, wts, qf, sc = _fp8_case(batch, chans, sizes, seed=41)
    outs = {}
    for two_pass in (False, True):
        fpn = U.UnifiedFPN()
        fpn.set_schedule(fp8_two_pass_p2=two_pass)
        _, _, outs[two_pass] = _run_fp8_neck(chans, wts, qf, sc, fpn=fpn)
    for a, b in zip(outs[False], outs[True]):
        assert torch.equal(a, b)


def test_fp8_neck_transposed_view_and_claims_are_bitwise_equal(cuda_device):
    """e4m3 neck at the Swin 1333x800 level sizes, whose 3x3s tile the P2 / P3 / P4 maps on
    their transposed views by default (143 instead of 147 tiles at 100 x 167): bitwise what
    plain tiles give, and what CTA-pair 3x3s that claim their items at run time give, with the
    separate quantisation pass and with the 3x3 that quantises its input itself, repeated
    launches included (the claim counters reset themselves); the merges (with their
    per-image absmax and scaled copy) one warp per pixel instead of per 8-pixel unit; and the
    3x3s on other CTA counts (the P3 3x3 on all SMs instead of its e4m3 default of 96/148,
    the P2 3x3 on 60)."""
    import unified_fpn as U
    chans, sizes = O.SWIN_CHANNELS, [(100, 167), (50, 84), (25, 42), (13, 21)]
    _, wts, qf, sc = _fp8_case(2, chans, sizes, seed=43)
    outs = []
    for opts in ({}, {"conv3x3_transpose": 0}, {"conv3x3_dynamic": 1},
                 {"fp8_quantise_in_conv": 1}, {"fp8_quantise_in_conv": 1, "conv3x3_dynamic": 1},
                 {"merge_units": -1}, {"conv3x3_ctas_p3": 0}, {"conv3x3_ctas_p2": 60}):
        fpn = U.UnifiedFPN()
        for k, v in opts.items():
            fpn.set_option(k, v)
        fpn, xin, o = _run_fp8_neck(chans, wts, qf, sc, fpn=fpn)
        outs.append(o)
        again = fpn(xin, return_p6=True, input_scales=[float(s) for s in sc])
        torch.cuda.synchronize()
        assert fpn.device_status() == 0
        assert all(torch.equal(a, b) for a, b in zip(o, again))
    for r in outs[1:]:
        assert all(torch.equal(a, b) for a, b in zip(outs[0], r))


@pytest.mark.parametrize("fp8_in", [False, True])
def test_neck_fp8_outputs_for_a_downstream_head(cuda_device, fp8_in):
    """forward(output_fp8=True): every level as e4m3 codes with per-image scales, bitwise
    equal to quantising the 16-bit outputs, and within e4m3 rounding of them."""
    import unified_fpn as U
    chans, sizes = O.R50_CHANNELS, O.level_sizes(128, 192)
    feats, wts, qf, sc = _fp8_case(2, chans, sizes, seed=81)
    fpn = U.UnifiedFPN()
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    if fp8_in:
        xin = [_cl(q.to(E4M3).cuda()) for q in qf]
        kw = {"input_scales": [float(s) for s in sc]}
    else:
        xin = [_cl(f.to(torch.bfloat16).cuda()) for f in feats]
        kw = {}
    plain = fpn(xin, return_p6=True, **kw)
    quant = fpn(xin, return_p6=True, output_fp8=True, **kw)
    torch.cuda.synchronize()
    assert len(quant) == 5
    for p, (q, s) in zip(plain, quant):
        q_ref, s_ref = U.quantize_fp8(p, per_image=True)
        assert q.dtype == E4M3 and s.shape == (2,)
        assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8)) and torch.equal(s, s_ref)
        back = q.float() * s.reshape(-1, 1, 1, 1)
        assert O.rel_err(back.cpu(), p.float().cpu()) < 0.07  # e4m3: 3 mantissa bits


def test_fp8_neck_config5_full_batch(cuda_device):
    """Config 5 at its full batch on one GPU: FP8 R50 640x640, 128 images (3.4 GB of bf16
    outputs); the first and last images against the e4m3 oracle (per-tensor input scales of
    the whole batch, merged maps quantised per image)."""
    import unified_fpn as U
    chans, sizes, batch = O.R50_CHANNELS, O.level_sizes(640, 640), 128
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(35)
    qs = [U.quantize_fp8(torch.randn(batch, c, h, w, device=dev, generator=gen)
                         .contiguous(memory_format=torch.channels_last))
          for c, (h, w) in zip(chans, sizes)]
    wts = O.make_weights(chans, seed=36, bias_scale=0.1)
    fpn = U.UnifiedFPN()
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    outs = fpn([q for q, _ in qs], return_p6=True, input_scales=torch.cat([s for _, s in qs]))
    torch.cuda.synchronize()
    assert fpn.device_status() == 0
    qw = O.quantize_neck_weights(wts)
    scales = [np.float32(s.item()) for _, s in qs]
    for n in (0, batch - 1):
        codes = [q[n:n + 1].float().cpu() for q, _ in qs]  # the e4m3 code values, exactly
        ref = O.fpn_neck_e4m3(codes, scales, qw)
        for o, r in zip(outs, ref):
            O.check_close(o[n:n + 1].float().cpu(), r, "e4m3")
