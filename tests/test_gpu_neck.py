"""GPU parity tests of the whole neck (UnifiedFPN -> C ABI engine) against the
CPU oracle, including the R50 800x1216 batch-2 workload at full size."""
import math

import pytest
import torch

from oracle import fpn_oracle as O

pytestmark = pytest.mark.gpu
TOL16 = O.TOL["bf16"]
TOL32 = O.TOL["f32"]


def _cl(x):
    return x.contiguous(memory_format=torch.channels_last)


def _run(fpn, feats_dev, **kw):
    outs = fpn(feats_dev, return_p6=True, **kw)
    torch.cuda.synchronize()
    return outs


def _check(outs, ref, kind):
    """Both parity metrics per output level: max-norm ratio and the per-element bound
    (oracle.check_close); kind = the compute dtype (or its tolerance name)."""
    assert len(outs) == 5
    for k, (o, r) in enumerate(zip(outs, ref)):
        assert tuple(o.shape) == tuple(r.shape)
        try:
            O.check_close(o.float().cpu(), r, kind)
        except AssertionError as e:
            raise AssertionError(f"P{k + 2} {tuple(o.shape)}: {e}") from None


def _neck_case(dtype, batch, chans, sizes, layout, seed=0, dist="relu_normal"):
    import unified_fpn as U
    feats = O.make_features(batch, chans, sizes, seed=seed, dist=dist)
    wts = O.make_weights(chans, seed=seed + 1, bias_scale=0.1)
    fpn = U.UnifiedFPN()
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    dev = torch.device("cuda", 0)
    xin = [f.to(dtype).to(dev) for f in feats]
    if layout == "nhwc":
        xin = [_cl(x) for x in xin]
    outs = _run(fpn, xin)
    assert fpn.device_status() == 0
    if dtype == torch.float32:
        ref = O.fpn_neck(feats, wts)
    else:
        rw = O.NeckWeights([O.round_to(w, dtype) for w in wts.lat_w], wts.lat_b,
                           [O.round_to(w, dtype) for w in wts.out_w], wts.out_b)
        ref = O.fpn_neck([O.round_to(f, dtype) for f in feats], rw)
    _check(outs, ref, dtype)
    if layout == "nhwc":
        assert all(o.is_contiguous(memory_format=torch.channels_last) for o in outs)
    return fpn, xin, outs


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("layout", ["nhwc", "nchw"])
def test_neck_small_r50(cuda_device, dtype, layout):
    _neck_case(dtype, 2, O.R50_CHANNELS, O.level_sizes(128, 192), layout)


def test_neck_swin_odd_sizes(cuda_device):
    """Swin-B channels, 1333x800-style non-2x top-down sizes 25x42 -> 50x84 -> 100x167 -> 200x334."""
    _neck_case(torch.bfloat16, 1, O.SWIN_CHANNELS, [(200, 334), (100, 167), (50, 84), (25, 42)], "nhwc",
               dist="normal")


def test_neck_fp32(cuda_device):
    _neck_case(torch.float32, 1, (64, 128, 256, 256), O.level_sizes(96, 160), "nchw", dist="normal")


@pytest.mark.parametrize("dtype,layout", [(torch.bfloat16, "nhwc"), (torch.float16, "nhwc"),
                                          (torch.bfloat16, "nchw")])
def test_neck_r50_800x1216_batch2_full_size(cuda_device, dtype, layout):
    """The benchmark workload at full size: R50 FPN neck, 800x1216, batch 2 (bf16 NHWC as
    benchmarked; fp16, and NCHW inputs transposed on the device, too)."""
    fpn, xin, outs = _neck_case(dtype, 2, O.R50_CHANNELS, O.level_sizes(800, 1216), layout)
    # size-independent properties: bitwise determinism and graph replay == direct launch
    again = _run(fpn, xin)
    for a, b in zip(outs, again):
        assert torch.equal(a, b)
    fpn.set_kernel_config(enable_graph_capture=False)
    direct = _run(fpn, xin)
    for a, b in zip(outs, direct):
        assert torch.equal(a, b)


@pytest.mark.parametrize("geom", [(O.R50_CHANNELS, O.level_sizes(128, 192), 2),
                                  (O.SWIN_CHANNELS, [(100, 167), (50, 84), (25, 42), (13, 21)], 1),
                                  (O.R50_CHANNELS, O.level_sizes(800, 1216), 2)])
def test_fused_neck_kernel_matches_per_level_kernels(cuda_device, geom):
    """The single persistent neck kernel (device-side level dependencies) and the split
    schedule (grouped small laterals, in-place merges, fused P2 lateral, per-level 3x3s)
    each match the oracle (at the R50 800x1216 batch-2 workload too, on its first image), and
    repeated fused launches are bitwise identical."""
    import unified_fpn as U
    chans, sizes, batch = geom
    host = O.make_features(batch, chans, sizes, seed=33)
    feats = [_cl(f.to(torch.bfloat16).cuda()) for f in host]
    wts = O.make_weights(chans, seed=34, bias_scale=0.1)
    fpn = U.UnifiedFPN()
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    fpn.set_schedule(fused_neck_kernel=True)
    fused = [o.clone() for o in _run(fpn, feats)]
    assert fpn.device_status() == 0
    fpn.set_schedule(fused_neck_kernel=False)
    split = [o.clone() for o in _run(fpn, feats)]
    assert fpn.device_status() == 0
    rw = O.NeckWeights([O.round_to(w, torch.bfloat16) for w in wts.lat_w], wts.lat_b,
                       [O.round_to(w, torch.bfloat16) for w in wts.out_w], wts.out_b)
    ref = O.fpn_neck([O.round_to(f[:1], torch.bfloat16) for f in host], rw)
    _check([o[:1] for o in fused], ref, torch.bfloat16)
    _check([o[:1] for o in split], ref, torch.bfloat16)
    fpn.set_schedule(fused_neck_kernel=True)
    for _ in range(3):  # repeated launches: the schedule counters must reset themselves
        again = _run(fpn, feats)
        for a, b in zip(fused, again):
            assert torch.equal(a, b)
    assert fpn.device_status() == 0


@pytest.mark.parametrize("fused", [False, True])
def test_both_schedules_match_oracle_swin_odd(cuda_device, fused):
    import unified_fpn as U
    chans, sizes = O.SWIN_CHANNELS, [(100, 167), (50, 84), (25, 42), (13, 21)]
    feats = O.make_features(1, chans, sizes, seed=41, dist="normal")
    wts = O.make_weights(chans, seed=42, bias_scale=0.1)
    fpn = U.UnifiedFPN()
    fpn.set_schedule(fused_neck_kernel=fused)
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    outs = _run(fpn, [_cl(f.to(torch.bfloat16).cuda()) for f in feats])
    assert fpn.device_status() == 0
    rw = O.NeckWeights([O.round_to(w, torch.bfloat16) for w in wts.lat_w], wts.lat_b,
                       [O.round_to(w, torch.bfloat16) for w in wts.out_w], wts.out_b)
    _check(outs, O.fpn_neck([O.round_to(f, torch.bfloat16) for f in feats], rw), torch.bfloat16)


def test_neck_batch_linearity_and_sharding(cuda_device):
    """Images are independent: the neck on a batch equals the neck on each slice
    (the property multi-GPU batch sharding relies on)."""
    import unified_fpn as U
    chans, sizes = O.R50_CHANNELS, O.level_sizes(160, 224)
    feats = [_cl(f.to(torch.bfloat16).cuda()) for f in O.make_features(4, chans, sizes, seed=21)]
    fpn = U.UnifiedFPN()
    full = _run(fpn, feats)
    for lo, hi in ((0, 1), (1, 3), (3, 4)):
        part = _run(fpn, [_cl(f[lo:hi]) for f in feats])
        for a, b in zip(full, part):
            assert torch.equal(a[lo:hi], b)


def test_profiled_forward_breakdown(cuda_device):
    import unified_fpn as U
    feats = [_cl(f.to(torch.bfloat16).cuda()) for f in O.make_features(1, O.R50_CHANNELS, O.level_sizes(256, 256))]
    fpn = U.UnifiedFPN()
    base = _run(fpn, feats)
    kt, mt = fpn.get_performance_breakdown(feats)
    assert (kt > 0).all()
    # grouped P5/P4/P3 laterals, P4 and P3 merges, P2 lateral, 4 x 3x3
    assert mt[0] > 0 and mt[4] == 8
    prof = _run(fpn, feats)  # profiling is one-shot; results must match
    for a, b in zip(base, prof):
        assert torch.equal(a, b)


def test_autotune_and_cache(cuda_device, tmp_path):
    import unified_fpn as U
    host = O.make_features(1, O.R50_CHANNELS, O.level_sizes(256, 384))
    feats = [_cl(f.to(torch.bfloat16).cuda()) for f in host]
    fpn = U.UnifiedFPN()
    base = [o.clone() for o in _run(fpn, feats)]
    report = fpn.autotune(feats, iterations=2)
    assert "tile" in report
    path = tmp_path / "tune.txt"
    fpn.save_tuning(path)
    fpn2 = U.UnifiedFPN()
    fpn2.load_tuning(path)
    tuned = _run(fpn2, feats)
    # Halo tiles sum K channel-block-major, plain tiles tap-major: the same values up to
    # fp32 summation order; tuned and untuned outputs both match the oracle (the engine's
    # default weights: seeded Kaiming-normal, zero biases).
    g = torch.Generator().manual_seed(0)
    lw, ow = [], []
    for cin in O.R50_CHANNELS:
        lw.append(torch.randn(256, cin, generator=g) * math.sqrt(2.0 / cin))
        ow.append(torch.randn(256, 256, 3, 3, generator=g) * math.sqrt(2.0 / (256 * 9)))
    zb = [torch.zeros(256) for _ in range(4)]
    rw = O.NeckWeights([O.round_to(w, torch.bfloat16) for w in lw], zb,
                       [O.round_to(w, torch.bfloat16) for w in ow], zb)
    ref = O.fpn_neck([O.round_to(f, torch.bfloat16) for f in host], rw)
    _check(base, ref, torch.bfloat16)
    _check(tuned, ref, torch.bfloat16)


def test_errors_are_raised_not_exit(cuda_device):
    import unified_fpn as U
    fpn = U.UnifiedFPN()
    with pytest.raises(ValueError):
        fpn([torch.randn(1, 8, 4, 4, device="cuda")] * 3)
    with pytest.raises(RuntimeError):
        fpn.set_kernel_config(tile_size=24)
    with pytest.raises(ValueError):
        U.UnifiedFPN(output_channels=128)
    # an empty batch is refused on the host, before anything is allocated or launched
    empty = [torch.empty(0, c, 64 >> l, 96 >> l, device="cuda", dtype=torch.bfloat16)
             .contiguous(memory_format=torch.channels_last) for l, c in enumerate(O.R50_CHANNELS)]
    with pytest.raises(U.UFPNError):
        fpn(empty)
    assert fpn.device_status() == 0


@pytest.mark.parametrize("fp8", [False, True])
def test_host_pipeline_matches_forward(cuda_device, fp8):
    """HostPipeline (copy-in / neck / copy-out overlapped across batches) returns, for
    every batch, exactly what a plain forward of that batch returns."""
    import unified_fpn as U
    chans, sizes = O.R50_CHANNELS, O.level_sizes(128, 160)
    fpn = U.UnifiedFPN()
    batches, scales = [], []
    for k in range(5):
        fs = [_cl(f.cuda()) for f in O.make_features(2, chans, sizes, seed=50 + k, dist="normal")]
        if fp8:
            qs = [U.quantize_fp8(f) for f in fs]
            batches.append([q for q, _ in qs])
            scales.append(torch.cat([s for _, s in qs]))
        else:
            batches.append([f.to(torch.bfloat16) for f in fs])
            scales.append(None)
    expect = [[o.cpu() for o in fpn(b, return_p6=True, input_scales=s)] for b, s in zip(batches, scales)]
    pipe = U.HostPipeline(fpn, batches[0], return_p6=True, depth=2)
    outs = [pipe.host_buffers() for _ in batches]
    for b, s, o in zip(batches, scales, outs):
        pipe.submit([t.cpu().pin_memory() for t in b], o,
                    s.cpu().pin_memory() if s is not None else None)
    pipe.synchronize()
    assert fpn.device_status() == 0
    for e, o in zip(expect, outs):
        for a, b in zip(e, o):
            assert torch.equal(a, b)


@pytest.mark.parametrize("fp8", [False, True])
def test_single_stream_schedule_is_bitwise_equal(cuda_device, fp8):
    """The split schedule's kernels run one after the other on one stream give exactly the
    two-stream results."""
    import unified_fpn as U
    chans, sizes = O.R50_CHANNELS, O.level_sizes(160, 224)
    fs = [_cl(f.cuda()) for f in O.make_features(2, chans, sizes, seed=61, dist="normal")]
    if fp8:
        qs = [U.quantize_fp8(f) for f in fs]
        feats, sc = [q for q, _ in qs], torch.cat([s for _, s in qs])
    else:
        feats, sc = [f.to(torch.bfloat16) for f in fs], None
    fpn = U.UnifiedFPN()
    two = _run(fpn, feats, input_scales=sc)
    fpn.set_schedule(single_stream=True)
    one = _run(fpn, feats, input_scales=sc)
    assert fpn.device_status() == 0
    for a, b in zip(two, one):
        assert torch.equal(a, b)


@pytest.mark.parametrize("fp8", [False, True])
def test_schedule_options_are_bitwise_equal(cuda_device, fp8):
    """Programmatic launches, chain priority and the one-launch P4 + P3 merge change only
    when kernels run, not what they compute."""
    import unified_fpn as U
    chans, sizes = O.R50_CHANNELS, O.level_sizes(160, 224)
    fs = [_cl(f.cuda()) for f in O.make_features(2, chans, sizes, seed=62, dist="normal")]
    if fp8:
        qs = [U.quantize_fp8(f) for f in fs]
        feats, sc = [q for q, _ in qs], torch.cat([s for _, s in qs])
    else:
        feats, sc = [f.to(torch.bfloat16) for f in fs], None
    ref = _run(U.UnifiedFPN(), feats, input_scales=sc)
    for pl, pr, m2 in [(False, False, False), (True, False, True), (False, True, True)]:
        fpn = U.UnifiedFPN()
        fpn.set_schedule(programmatic_launch=pl, chain_priority=pr, merge_two_levels=m2)
        outs = _run(fpn, feats, input_scales=sc)
        assert fpn.device_status() == 0
        for a, b in zip(ref, outs):
            assert torch.equal(a, b), (pl, pr, m2)
        if m2 and not fp8:
            assert int(fpn.get_performance_breakdown(feats, input_scales=sc)[1][4].item()) == 7


@pytest.mark.parametrize("act,alpha", [("relu", 0.01), ("leaky_relu", 0.1), ("swish", 0.01)])
@pytest.mark.parametrize("mode", ["split", "fused", "fp32"])
def test_neck_activation(cuda_device, act, alpha, mode):
    """set_activation: every level's 3x3 output (and P6) activated in the epilogue, on the
    split and fused tensor-core schedules and the fp32 path, against the oracle neck."""
    import unified_fpn as U
    dtype = torch.float32 if mode == "fp32" else torch.bfloat16
    chans = (64, 128, 256, 256) if mode == "fp32" else O.R50_CHANNELS
    feats = O.make_features(2, chans, O.level_sizes(96, 160), seed=4, dist="normal")
    wts = O.make_weights(chans, seed=5, bias_scale=0.1)
    fpn = U.UnifiedFPN()
    fpn.set_schedule(fused_neck_kernel=mode == "fused")
    fpn.set_activation(act, alpha)
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    xin = [f.to(dtype).to(cuda_device) for f in feats]
    if dtype != torch.float32:
        xin = [_cl(x) for x in xin]
    outs = _run(fpn, xin)
    assert fpn.device_status() == 0
    if dtype == torch.float32:
        ref = O.fpn_neck(feats, wts, act=act, alpha=alpha)
    else:
        rw = O.NeckWeights([O.round_to(w, dtype) for w in wts.lat_w], wts.lat_b,
                           [O.round_to(w, dtype) for w in wts.out_w], wts.out_b)
        ref = O.fpn_neck([O.round_to(f, dtype) for f in feats], rw, act=act, alpha=alpha)
    _check(outs, ref, dtype)
    # back to the standard neck through the reference's string mapping (unknown -> none)
    fpn.set_kernel_config(activation="not-an-activation")
    plain = _run(fpn, xin)
    ref0 = O.fpn_neck(feats, wts) if dtype == torch.float32 else O.fpn_neck(
        [O.round_to(f, dtype) for f in feats], rw)
    _check(plain, ref0, dtype)


@pytest.mark.parametrize("case", [
    ("config 3 shard: R50 1024x1024, 8 images", O.R50_CHANNELS, (1024, 1024), 8, "normal"),
    ("config 4a: 128..1024 channels, 1344x1344, 8 images", O.SWIN_CHANNELS, (1344, 1344), 8, "normal"),
])
def test_neck_large_configs_against_oracle(cuda_device, case):
    """The per-GPU shards of the larger configurations: the whole batch through the engine,
    the first and last images against the oracle (fp32 on the same bf16-rounded inputs and
    weights), and each of those images alone gives bitwise its slice of the batch result."""
    import unified_fpn as U
    _, chans, (h, w), batch, dist = case
    sizes = O.level_sizes(h, w)
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(h + batch)
    xin = [_cl(torch.randn(batch, c, hh, ww, device=dev, generator=gen).to(torch.bfloat16))
           for c, (hh, ww) in zip(chans, sizes)]
    wts = O.make_weights(chans, seed=h, bias_scale=0.1)
    fpn = U.UnifiedFPN()
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    outs = [o.clone() for o in _run(fpn, xin)]
    assert fpn.device_status() == 0
    rw = O.NeckWeights([O.round_to(w_, torch.bfloat16) for w_ in wts.lat_w], wts.lat_b,
                       [O.round_to(w_, torch.bfloat16) for w_ in wts.out_w], wts.out_b)
    for n in (0, batch - 1):
        ref = O.fpn_neck([x[n:n + 1].float().cpu() for x in xin], rw)
        _check([o[n:n + 1] for o in outs], ref, torch.bfloat16)
        alone = _run(fpn, [x[n:n + 1].contiguous(memory_format=torch.channels_last) for x in xin])
        assert all(torch.equal(a, o[n:n + 1]) for a, o in zip(alone, outs))


def test_neck_config3_full_batch_large_offsets(cuda_device):
    """Config 3 at its full batch on one GPU: R50, 1024x1024, 64 images, bf16 NHWC.  The P2
    maps hold 2^30 elements (2 GiB), so every address computation must be 64-bit; the first
    and last images against the oracle, and the last image alone equals its slice bitwise."""
    import unified_fpn as U
    chans, sizes, batch = O.R50_CHANNELS, O.level_sizes(1024, 1024), 64
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(33)
    xin = [_cl(torch.randn(batch, c, h, w, device=dev, generator=gen).to(torch.bfloat16))
           for c, (h, w) in zip(chans, sizes)]
    wts = O.make_weights(chans, seed=34, bias_scale=0.1)
    fpn = U.UnifiedFPN()
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    outs = _run(fpn, xin)
    assert fpn.device_status() == 0
    rw = O.NeckWeights([O.round_to(w_, torch.bfloat16) for w_ in wts.lat_w], wts.lat_b,
                       [O.round_to(w_, torch.bfloat16) for w_ in wts.out_w], wts.out_b)
    for n in (0, batch - 1):
        ref = O.fpn_neck([x[n:n + 1].float().cpu() for x in xin], rw)
        _check([o[n:n + 1] for o in outs], ref, torch.bfloat16)
    last = [o[batch - 1:].clone() for o in outs]
    del outs
    alone = _run(fpn, [x[batch - 1:].contiguous(memory_format=torch.channels_last) for x in xin])
    assert all(torch.equal(a, b) for a, b in zip(alone, last))


# Maps whose widths are not multiples of 8 or 16 and whose heights are not multiples of 16:
# every 8 x 16 halo tile, 128-pixel lateral tile and coarse box meets a ragged edge or a
# seam inside the map.
RAGGED = [(52, 70), (26, 35), (13, 18), (7, 9)]


@pytest.mark.parametrize("opts", [
    {}, {"fused_neck_kernel": 1}, {"grouped_topdown": 1}, {"ksplit_p5": 2, "ksplit_p4": 2},
    {"grouped_topdown": 1, "ksplit_p5": 4, "ksplit_p4": 2, "ksplit_p3": 2}, {"merge_two_levels": 1},
    {"nsplit_p5": 2, "nsplit_p4": 2, "nsplit_p3": 2}, {"grouped_topdown": 1, "nsplit_p5": 2},
    {"nsplit_p5": 2, "ksplit_p4": 2, "nsplit_p3": 2}, {"p2_lateral_dynamic": 1},
    {"p2_lateral_dynamic": 1, "p2_lateral_ctas": 37}, {"grouped_laterals_pair": 1},
    {"grouped_laterals_pair": 1, "merge_two_levels": 1},
    {"grouped_laterals_pair": 0, "nsplit_p5": 2, "nsplit_p4": 2, "nsplit_p3": 2},
    {"conv3x3_dynamic": 1}, {"conv3x3_transpose": 0}, {"conv3x3_mixed": 0},
    {"conv3x3_p3": -1, "conv3x3_p4": -1, "conv3x3_p5": -1},
    {"conv3x3_p3": -1, "conv3x3_p4": -1, "conv3x3_p5": -1, "conv3x3_dynamic": 1},
    {"merge_units": -1}, {"conv3x3_ctas_p3": 40, "conv3x3_ctas_p2": 64, "conv3x3_ctas_p4": 9},
], ids=["split", "fused", "grouped_topdown", "ksplit", "topdown_ksplit", "merge_two_levels",
        "nsplit", "topdown_nsplit", "nsplit_ksplit", "p2_dynamic", "p2_dynamic_37ctas",
        "lateral_pairs", "lateral_pairs_two_level", "nsplit_single_cta", "conv_claims",
        "conv_plain_view", "conv_transposed_view", "conv_pairs_all_levels", "conv_pairs_all_levels_claims",
        "merge_warp_per_pixel", "conv_cta_caps"])
def test_neck_ragged_tile_seams(cuda_device, opts):
    """Every schedule option on ragged maps against the oracle (max-norm and per-element),
    bitwise deterministic, and each image alone equals its slice of the batch."""
    import unified_fpn as U
    host = O.make_features(2, O.R50_CHANNELS, RAGGED, seed=77, dist="normal")
    wts = O.make_weights(O.R50_CHANNELS, seed=78, bias_scale=0.1)
    fpn = U.UnifiedFPN()
    for k, v in opts.items():
        fpn.set_option(k, v)
        assert fpn.get_option(k) == v
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    xin = [_cl(f.to(torch.bfloat16).cuda()) for f in host]
    outs = [o.clone() for o in _run(fpn, xin)]
    assert fpn.device_status() == 0
    rw = O.NeckWeights([O.round_to(w, torch.bfloat16) for w in wts.lat_w], wts.lat_b,
                       [O.round_to(w, torch.bfloat16) for w in wts.out_w], wts.out_b)
    _check(outs, O.fpn_neck([O.round_to(f, torch.bfloat16) for f in host], rw), torch.bfloat16)
    again = _run(fpn, xin)
    assert all(torch.equal(a, b) for a, b in zip(outs, again))
    alone = _run(fpn, [_cl(x[1:2]) for x in xin])
    assert all(torch.equal(a, o[1:2]) for a, o in zip(alone, outs))
    assert fpn.device_status() == 0


@pytest.mark.parametrize("opts", [{"grouped_topdown": 1}, {"ksplit_p5": 4, "ksplit_p4": 2},
                                  {"grouped_topdown": 1, "ksplit_p5": 2, "ksplit_p4": 2, "ksplit_p3": 2},
                                  {"p2_lateral_dynamic": 1}, {"p2_lateral_ctas": 74},
                                  {"grouped_laterals_pair": 1}])
def test_grouped_launch_options_full_size(cuda_device, opts):
    """The grouped-lateral options at the R50 800x1216 batch-2 workload: the first image
    against the oracle, repeated launches bitwise equal (the split-K sum is order-free and the
    per-tile arrival counters reset themselves)."""
    import unified_fpn as U
    sizes = O.level_sizes(800, 1216)
    host = O.make_features(2, O.R50_CHANNELS, sizes, seed=91)
    wts = O.make_weights(O.R50_CHANNELS, seed=92, bias_scale=0.1)
    fpn = U.UnifiedFPN()
    for k, v in opts.items():
        fpn.set_option(k, v)
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    xin = [_cl(f.to(torch.bfloat16).cuda()) for f in host]
    outs = [o.clone() for o in _run(fpn, xin)]
    for _ in range(3):
        again = _run(fpn, xin)
        assert all(torch.equal(a, b) for a, b in zip(outs, again))
    assert fpn.device_status() == 0
    rw = O.NeckWeights([O.round_to(w, torch.bfloat16) for w in wts.lat_w], wts.lat_b,
                       [O.round_to(w, torch.bfloat16) for w in wts.out_w], wts.out_b)
    ref = O.fpn_neck([O.round_to(f[:1], torch.bfloat16) for f in host], rw)
    _check([o[:1] for o in outs], ref, torch.bfloat16)


@pytest.mark.parametrize("variant", [{"nsplit_p3": 2, "nsplit_p4": 2, "nsplit_p5": 2},
                                     {"grouped_laterals_pair": 1}], ids=["nsplit", "pairs"])
def test_grouped_lateral_variants_equal_whole_tiles_bitwise(cuda_device, variant):
    """Channel-half units (N = 128 MMAs over 128-row weight boxes) and the CTA-pair launch
    (M = 256 MMAs, each CTA streaming half of every weight k-block) accumulate every output
    element over the same K order as the single-CTA grouped launch: the neck is bitwise the
    same with and without them, at the R50 800x1216 batch-2 workload, and matches the
    oracle."""
    import unified_fpn as U
    sizes = O.level_sizes(800, 1216)
    host = O.make_features(2, O.R50_CHANNELS, sizes, seed=93)
    wts = O.make_weights(O.R50_CHANNELS, seed=94, bias_scale=0.1)
    xin = [_cl(f.to(torch.bfloat16).cuda()) for f in host]
    res = []
    for on in (0, 1):
        fpn = U.UnifiedFPN()
        fpn.set_option("grouped_laterals_pair", 0)  # the single-CTA grouped launch ...
        for k, v in (variant.items() if on else ()):
            fpn.set_option(k, v)                    # ... against the variant
        fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
        res.append([o.clone() for o in _run(fpn, xin)])
        assert fpn.device_status() == 0
    assert all(torch.equal(a, b) for a, b in zip(*res))
    rw = O.NeckWeights([O.round_to(w, torch.bfloat16) for w in wts.lat_w], wts.lat_b,
                       [O.round_to(w, torch.bfloat16) for w in wts.out_w], wts.out_b)
    ref = O.fpn_neck([O.round_to(f[:1], torch.bfloat16) for f in host], rw)
    _check([o[:1] for o in res[1]], ref, torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_conv3x3_tail_halves_bitwise_at_full_size(cuda_device, dtype):
    """At the R50 800x1216 batch-2 workload the merges run one warp per 8-pixel unit (the
    default; merge_units = -1: one warp per pixel) and the 3x3s tile the P2 / P3 / P4 maps
    with mixed tilings (the own view for whole 16-row tile rows, the transposed view for the
    rest: 950 / 248 / 70 tiles instead of 988 / 266 / 80; conv3x3_mixed = 0: the transposed
    views, 950 / 260 / 70), the P2 3x3 on single CTAs, whose last 62 of 950 tiles on 148 CTAs
    run as channel halves (conv3x3_tail_halves, the default).  On CTA pairs (conv3x3_p2 = -1)
    the P2 3x3 ends with 31 of 475 pair units on 74 pairs, run as channel halves.  The neck is bitwise the same with pairs, plain tiles,
    whole units and run-time item claims (conv3x3_dynamic), and matches the oracle."""
    import unified_fpn as U
    sizes = O.level_sizes(800, 1216)
    host = O.make_features(2, O.R50_CHANNELS, sizes, seed=95)
    wts = O.make_weights(O.R50_CHANNELS, seed=96, bias_scale=0.1)
    xin = [_cl(f.to(dtype).cuda()) for f in host]
    res = []
    for opts in ({}, {"conv3x3_tail_halves": 0}, {"conv3x3_p2": -1},
                 {"conv3x3_p2": -1, "conv3x3_tail_halves": 0},
                 {"conv3x3_transpose": 0},
                 {"conv3x3_p2": -1, "conv3x3_tail_halves": 0, "conv3x3_transpose": 0},
                 {"conv3x3_p2": -1, "conv3x3_dynamic": 1}, {"conv3x3_mixed": 0},
                 {"conv3x3_p2": -1, "conv3x3_mixed": 0}, {"merge_units": -1},
                 {"p2_lateral_ctas": 128}):
        fpn = U.UnifiedFPN()
        for k, v in opts.items():
            fpn.set_option(k, v)
            assert fpn.get_option(k) == v
        fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
        res.append([o.clone() for o in _run(fpn, xin)])
        assert fpn.device_status() == 0
    for r in res[1:]:
        assert all(torch.equal(a, b) for a, b in zip(res[0], r))
    rw = O.NeckWeights([O.round_to(w, dtype) for w in wts.lat_w], wts.lat_b,
                       [O.round_to(w, dtype) for w in wts.out_w], wts.out_b)
    ref = O.fpn_neck([O.round_to(f[:1], dtype) for f in host], rw)
    _check([o[:1] for o in res[0]], ref, dtype)


def test_options_set_before_the_first_forward_survive_configuration(cuda_device):
    """Geometry-dependent choices (tilings, the P2 lateral's form, merge blocks) are reset to
    the geometry's defaults when the engine configures its levels -- at the first forward and
    at every new geometry.  Values a caller set by name must survive both, and the forward
    with them must still match the oracle."""
    import unified_fpn as U
    chosen = {"p2_lateral_dynamic": 1, "merge_units": 4, "conv3x3_p3": 16, "lateral_tile_p2": 8,
              "conv3x3_ctas_p3": 50,
              "p2_lateral_ctas": 100}
    fpn = U.UnifiedFPN()
    for k, v in chosen.items():
        fpn.set_option(k, v)
    wts = O.make_weights(O.R50_CHANNELS, seed=99, bias_scale=0.1)
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    rw = O.NeckWeights([O.round_to(w, torch.bfloat16) for w in wts.lat_w], wts.lat_b,
                       [O.round_to(w, torch.bfloat16) for w in wts.out_w], wts.out_b)
    for sizes in (O.level_sizes(256, 384), RAGGED):  # first forward, then a new geometry
        host = O.make_features(2, O.R50_CHANNELS, sizes, seed=100, dist="normal")
        xin = [_cl(f.to(torch.bfloat16).cuda()) for f in host]
        outs = [o.clone() for o in _run(fpn, xin)]
        assert fpn.device_status() == 0
        assert {k: fpn.get_option(k) for k in chosen} == chosen
        _check(outs, O.fpn_neck([O.round_to(f, torch.bfloat16) for f in host], rw),
               torch.bfloat16)


def test_schedule_option_api_errors(cuda_device):
    import unified_fpn as U
    fpn = U.UnifiedFPN()
    assert fpn.get_option("grouped_topdown") in (0, 1)
    with pytest.raises(RuntimeError):
        fpn.set_option("no_such_option", 1)
    with pytest.raises(RuntimeError):
        fpn.set_option("ksplit_p5", 3)
    with pytest.raises(RuntimeError):
        fpn.set_option("nsplit_p4", 4)


def test_bounded_wait_runs_out_and_the_engine_recovers(cuda_device):
    """A device wait that runs out: on the fused schedule the P2 3x3 tiles wait for one more
    P2 lateral tile than exists, with a 5 ms limit.  The forward ends by itself within the
    limit (no trap, no hang), the status word names the dependency wait, the reset clears it
    together with the schedule counters, and the next forward matches the oracle again."""
    import time
    import unified_fpn as U
    from unified_fpn import _lib
    chans, sizes = O.R50_CHANNELS, O.level_sizes(160, 224)
    host = O.make_features(2, chans, sizes, seed=97)
    wts = O.make_weights(chans, seed=98, bias_scale=0.1)
    fpn = U.UnifiedFPN()
    fpn.set_schedule(fused_neck_kernel=True)
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    xin = [_cl(f.to(torch.bfloat16).cuda()) for f in host]
    rw = O.NeckWeights([O.round_to(w, torch.bfloat16) for w in wts.lat_w], wts.lat_b,
                       [O.round_to(w, torch.bfloat16) for w in wts.out_w], wts.out_b)
    ref = O.fpn_neck([O.round_to(f, torch.bfloat16) for f in host], rw)
    _check([o.clone() for o in _run(fpn, xin)], ref, torch.bfloat16)
    assert fpn.device_status() == 0

    fpn.set_option("test_stall_dependency_us", 5000)
    t0 = time.perf_counter()
    _run(fpn, xin)
    elapsed = time.perf_counter() - t0
    assert elapsed < 1.0, elapsed  # ended by itself, about 5 ms after the P2 3x3 tiles began
    assert fpn.device_status(reset=False) == _lib.DEV_TIMEOUT_DEPENDENCY
    assert fpn.device_status(reset=True) == _lib.DEV_TIMEOUT_DEPENDENCY
    assert fpn.device_status() == 0  # cleared

    fpn.set_option("test_stall_dependency_us", 0)
    for _ in range(2):  # the schedule counters start at zero again
        outs = [o.clone() for o in _run(fpn, xin)]
        assert fpn.device_status() == 0
        _check(outs, ref, torch.bfloat16)


def test_helpers_drop_in(cuda_device, tmp_path):
    """The reference package's helpers with its signatures and result keys
    (python/__init__.py:82-257) and UnifiedFPN.benchmark (fpn_pytorch.cpp:139-169)."""
    import json
    import unified_fpn as U
    sizes = O.level_sizes(256, 384)
    feats = [_cl(f.to(torch.bfloat16).cuda()) for f in O.make_features(2, O.R50_CHANNELS, sizes, seed=5)]
    fpn = U.UnifiedFPN()

    avg_ms, gbs, util = fpn.benchmark(feats, num_iterations=5)
    assert avg_ms > 0 and gbs > 0 and 0 < util < 1.5

    res = U.benchmark_fpn(feats, num_iterations=5, warmup_iterations=2, fpn=fpn)
    for key in ("avg_time_ms", "throughput_fps", "memory_bandwidth_gb_s", "compute_utilization",
                "memory_usage_mb", "detailed_metrics"):
        assert key in res, key
    assert res["avg_time_ms"] > 0 and res["throughput_fps"] == pytest.approx(1000.0 / res["avg_time_ms"])
    assert res["images_per_s"] == pytest.approx(2 * res["throughput_fps"])

    out = tmp_path / "fpn_profile.json"
    prof = U.profile_fpn(feats, str(out), fpn=fpn)
    saved = json.loads(out.read_text())
    for key in ("kernel_times_ms", "total_time_ms", "memory_bandwidth_gb_s", "compute_utilization",
                "peak_memory_mb", "num_kernel_launches"):
        assert key in saved and saved[key] == prof[key], key
    assert len(saved["kernel_times_ms"]) == 8 and min(saved["kernel_times_ms"]) >= 0
    assert saved["total_time_ms"] >= sum(saved["kernel_times_ms"]) * 0.99
    # utilisation is against the peaks the library reports (measured when available)
    pk = U.get_peaks()
    flops = sum(2.0 * 2 * h * w * 256 * (c + 9 * 256) for c, (h, w) in zip(O.R50_CHANNELS, sizes))
    assert saved["compute_utilization"] == pytest.approx(
        flops / (saved["total_time_ms"] * 1e-3) / (pk["tensor_tflops"] * 1e12), rel=1e-3)
    assert U.profile_fpn(feats, None, fpn=fpn)["num_kernel_launches"] == saved["num_kernel_launches"]

    info = U.get_device_info()
    for key in ("device_name", "compute_capability", "total_memory_gb", "multiprocessor_count",
                "max_threads_per_block", "max_threads_per_multiprocessor", "memory_clock_rate_mhz",
                "memory_bus_width_bits", "l2_cache_size_mb", "theoretical_bandwidth_gb_s"):
        assert key in info, key
    assert info["compute_capability"] == "10.0" and info["multiprocessor_count"] > 0
    assert U.check_installation() is True


def test_graph_cache_with_fresh_outputs_every_call(cuda_device):
    """The drop-in call fpn(feats) allocates new outputs each time (as the reference's binding
    did, fpn_pytorch.cpp:113-136).  Kept alive, every call has a new pointer set: each runs as
    direct launches (no capture, nothing evicted), bitwise what the graph replays give."""
    import unified_fpn as U
    feats = [_cl(f.to(torch.bfloat16).cuda()) for f in O.make_features(1, O.R50_CHANNELS, O.level_sizes(128, 192), seed=3)]
    fpn = U.UnifiedFPN()
    ref = _run(fpn, feats)  # kept alive: the allocator cannot hand its memory out again
    kept = [fpn(feats, return_p6=True) for _ in range(20)]
    torch.cuda.synchronize()
    st = fpn.graph_stats()
    assert st["captures"] == 0 and st["direct"] == 21, st
    for outs in kept:
        assert all(torch.equal(a, b) for a, b in zip(outs, ref))
    # a repeating pointer set: captured on its second use, replayed from then on
    out = [torch.empty_like(r) for r in ref]
    for _ in range(5):
        fpn(feats, return_p6=True, out=out)
    torch.cuda.synchronize()
    st2 = fpn.graph_stats()
    assert st2["captures"] == 1 and st2["replays"] == 3 and st2["direct"] == 22, st2
    assert all(torch.equal(a, b) for a, b in zip(out, ref))
    assert fpn.device_status() == 0


def test_autotune_moves_a_bad_lateral_choice_and_keeps_parity(cuda_device, tmp_path):
    """Whole-neck tuning (every knob timed inside the full forward): started from 128-pixel-wide
    P2 lateral tiles on a 40-pixel-wide map (3.2x padded work), the tuner picks another shape;
    the tuned forward matches the oracle; save/load re-applies every tuned knob."""
    import unified_fpn as U
    sizes = O.level_sizes(1024, 160)  # P2 256 x 40 ... P5 32 x 5
    host = O.make_features(1, O.R50_CHANNELS, sizes, seed=101)
    wts = O.make_weights(O.R50_CHANNELS, seed=102, bias_scale=0.1)
    xin = [_cl(f.to(torch.bfloat16).cuda()) for f in host]
    fpn = U.UnifiedFPN()
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    _run(fpn, xin)
    fpn.set_option("lateral_tile_p2", 128)
    report = fpn.autotune(xin, iterations=3)
    assert "lateral_tile_p2" in report and "tuned:" in report, report
    assert fpn.get_option("lateral_tile_p2") != 128, report
    outs = [o.clone() for o in _run(fpn, xin)]
    assert fpn.device_status() == 0
    rw = O.NeckWeights([O.round_to(w, torch.bfloat16) for w in wts.lat_w], wts.lat_b,
                       [O.round_to(w, torch.bfloat16) for w in wts.out_w], wts.out_b)
    _check(outs, O.fpn_neck([O.round_to(f, torch.bfloat16) for f in host], rw), torch.bfloat16)
    names = [f"lateral_tile_p{l}" for l in range(2, 6)] + [f"conv3x3_p{l}" for l in range(2, 6)] + \
            ["p2_lateral_pair", "grouped_topdown", "ksplit_p3", "ksplit_p4", "ksplit_p5", "merge_units",
             "merge_two_levels", "programmatic_launch"]
    tuned = {n: fpn.get_option(n) for n in names}
    path = tmp_path / "tune.txt"
    fpn.save_tuning(path)
    fpn2 = U.UnifiedFPN()
    fpn2.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    fpn2.load_tuning(path)
    again = _run(fpn2, xin)  # configures this geometry: the saved knobs apply
    assert {n: fpn2.get_option(n) for n in names} == tuned
    assert all(torch.equal(a, b) for a, b in zip(outs, again))


def test_autotune_e4m3_keeps_parity(cuda_device):
    import numpy as np
    import unified_fpn as U
    chans, sizes = O.R50_CHANNELS, O.level_sizes(128, 192)
    feats = O.make_features(2, chans, sizes, seed=111, dist="normal")
    wts = O.make_weights(chans, seed=112, bias_scale=0.1)
    qf, sc = zip(*[O.quantize_e4m3_tensor(f) for f in feats])
    qf = [torch.from_numpy(q) for q in qf]
    fpn = U.UnifiedFPN()
    fpn.initialize_weights(wts.lat_w, wts.lat_b, wts.out_w, wts.out_b)
    xin = [_cl(q.to(torch.float8_e4m3fn).cuda()) for q in qf]
    scales = [float(s) for s in sc]
    fpn(xin, return_p6=True, input_scales=scales)
    report = fpn.autotune(xin, iterations=2, input_scales=scales)
    assert "conv3x3_p2" in report and "fp8_two_pass_p2" in report, report
    outs = fpn(xin, return_p6=True, input_scales=scales)
    torch.cuda.synchronize()
    assert fpn.device_status() == 0
    ref = O.fpn_neck_e4m3(qf, [np.float32(s) for s in sc], O.quantize_neck_weights(wts))
    for o, r in zip(outs, ref):
        O.check_close(o.float().cpu(), r, "e4m3")


def test_lateral_tuner_feeds_the_engine(cuda_device):
    """fpn_auto_tune_lateral_conv (the reference's C entry point) tunes the lateral tile shape
    of one shape; an engine configuring a level of that shape afterwards uses it."""
    import unified_fpn as U
    from unified_fpn import _lib
    res = _lib.lib.fpn_auto_tune_lateral_conv(1, 512, 256, 160, 24)
    assert res, _lib.lib.ufpn_last_error()
    r = res.contents
    assert r.tile_w in (8, 16, 32, 64, 128) and r.tile_h * r.tile_w == 128
    assert r.time_ms > 0 and r.performance_gflops > 0
    sizes = [(320, 48), (160, 24), (80, 12), (40, 6)]  # P3 level: 1 x 512 x 160 x 24
    fpn = U.UnifiedFPN()
    _run(fpn, [_cl(torch.randn(1, c, h, w, device="cuda", dtype=torch.bfloat16))
               for c, (h, w) in zip(O.R50_CHANNELS, sizes)])
    assert fpn.get_option("lateral_tile_p3") == r.tile_w
    # the stream-taking form, fp16
    out = _lib.TuningResult()
    import ctypes
    assert _lib.lib.ufpn_autotune_lateral(_lib.DTYPE_F16, 2, 256, 50, 76,
                                          torch.cuda.current_stream().cuda_stream,
                                          ctypes.byref(out)) == 0
    assert out.tile_w in (8, 16, 32, 64, 128) and out.time_ms > 0
