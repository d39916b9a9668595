"""Backward pass (training) on the GPU against autograd through the CPU oracle.

The oracle's forward is the restated neck (oracle/fpn_oracle.py: conv2d laterals, the
bilinear whose formula is pinned to the reference's upsample tests, pad-1 3x3, P6 = P5[::2,
::2]); torch autograd through it gives the exact adjoints the library's backward kernels
compute.  Inputs and weights are rounded to the kernels' 16-bit dtype first and the oracle
runs in fp32, so the comparison measures the kernels' own rounding (16-bit gradient maps,
fp32 accumulation)."""
import pytest
import torch
import torch.nn.functional as F

from oracle import fpn_oracle as O

pytestmark = pytest.mark.gpu
TOL = 2e-2  # max |y - ref| / max |ref|, per tensor


def _cl(x):
    return x.contiguous(memory_format=torch.channels_last)


def _close(y, ref, kind="grad16", tol=TOL):
    """Both parity metrics (max-norm ratio <= tol, per-element bound of ``kind``)."""
    O.check_close(y.detach().float().cpu(), ref.detach().float(), kind, tol=tol)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 256, 20, 30), (1, 512, 25, 42), (1, 128, 33, 40), (2, 2048, 5, 7)])
def test_lateral_conv_backward(cuda_device, dtype, shape):
    import unified_fpn as U
    n, cin, h, w = shape
    g = torch.Generator().manual_seed(cin + h)
    x = torch.randn(n, cin, h, w, generator=g).to(dtype)
    wt = (torch.randn(256, cin, generator=g) * (2.0 / cin) ** 0.5).to(dtype)
    gy = torch.randn(n, 256, h, w, generator=g).to(dtype)
    gx, gw, gb = U.fpn_lateral_conv_backward(_cl(x.to(cuda_device)), wt.to(cuda_device), _cl(gy.to(cuda_device)))
    torch.cuda.synchronize()
    assert U.device_status() == 0
    xr = x.float().requires_grad_()
    wr = wt.float().requires_grad_()
    br = torch.zeros(256, requires_grad=True)
    O.lateral_conv(xr, wr, br).backward(gy.float())
    _close(gx, xr.grad)
    _close(gw, wr.grad)
    _close(gb, br.grad)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 20, 30), (1, 13, 17), (1, 50, 76)])
def test_conv3x3_backward(cuda_device, dtype, shape):
    import unified_fpn as U
    n, h, w = shape
    g = torch.Generator().manual_seed(h * 31 + w)
    x = torch.randn(n, 256, h, w, generator=g).to(dtype)
    w3 = (torch.randn(256, 256, 3, 3, generator=g) * 0.03).to(dtype)
    gy = torch.randn(n, 256, h, w, generator=g).to(dtype)
    gx, gw, gb = U.fpn_conv3x3_backward(_cl(x.to(cuda_device)), w3.to(cuda_device), _cl(gy.to(cuda_device)))
    torch.cuda.synchronize()
    assert U.device_status() == 0
    xr = x.float().requires_grad_()
    wr = w3.float().requires_grad_()
    br = torch.zeros(256, requires_grad=True)
    O.conv3x3(xr, wr, br).backward(gy.float())
    _close(gx, xr.grad)
    _close(gw, wr.grad)
    _close(gb, br.grad)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("sizes", [((2, 256, 25, 38), (50, 76)), ((1, 256, 84, 50), (167, 100)),
                                   ((1, 64, 7, 9), (13, 18)), ((1, 32, 5, 5), (5, 5)),
                                   ((1, 1024, 6, 10), (12, 20)),   # wide rows: narrow strips
                                   ((1, 32, 2, 3), (40, 50))])     # scale > 8: the gather kernel
def test_upsample_add_backward(cuda_device, dtype, sizes):
    import unified_fpn as U
    (n, c, hc, wc), (h, w) = sizes
    g = torch.Generator().manual_seed(hc * 7 + wc)
    gy = torch.randn(n, c, h, w, generator=g).to(dtype)
    base = torch.randn(n, c, hc, wc, generator=g).to(dtype)
    gc = U.fpn_upsample_add_backward(_cl(gy.to(cuda_device)), (hc, wc), base=_cl(base.to(cuda_device)))
    cr = torch.zeros(n, c, hc, wc, requires_grad=True)
    O.bilinear_upsample_t(cr, (h, w)).backward(gy.float())
    ref = cr.grad + base.float()
    _close(gc, ref, "f32" if dtype == torch.float32 else "grad16",
           1e-5 if dtype == torch.float32 else TOL)


def test_p6_backward(cuda_device):
    import unified_fpn as U
    g = torch.Generator().manual_seed(3)
    g5 = torch.randn(2, 256, 25, 38, generator=g).to(torch.bfloat16)
    g6 = torch.randn(2, 256, 13, 19, generator=g).to(torch.bfloat16)
    out = U.fpn_p6_backward(_cl(g6.to(cuda_device)), _cl(g5.to(cuda_device)))
    ref = g5.float().clone()
    ref[:, :, ::2, ::2] += g6.float()
    assert torch.equal(out.cpu().float(), ref.to(torch.bfloat16).float())


@pytest.mark.parametrize("dtype,chans,sizes,batch", [
    (torch.bfloat16, O.R50_CHANNELS, O.level_sizes(128, 160), 2),
    (torch.float16, O.R50_CHANNELS, O.level_sizes(128, 160), 2),
    # Swin-B channels, 1333x800-style sizes: non-2x top-down ratios (13->25->50->100 rows,
    # 21->42->84->167 columns), ragged tiles, odd P6
    (torch.float16, O.SWIN_CHANNELS, [(100, 167), (50, 84), (25, 42), (13, 21)], 1),
])
def test_neck_backward_matches_autograd(cuda_device, dtype, chans, sizes, batch):
    """Every input, weight and bias gradient of the whole neck (P6 included) against autograd
    through the oracle neck."""
    import unified_fpn as U
    fs = O.make_features(batch, chans, sizes, seed=21, dist="normal")
    wts = O.make_weights(chans, seed=22, bias_scale=0.1)
    neck = U.FPNNeck(chans).to(cuda_device)
    with torch.no_grad():
        for l in range(4):  # the module's fp32 master weights = the oracle's, rounded to dtype
            neck.lateral_w[l].copy_(wts.lat_w[l].to(dtype).float())
            neck.lateral_b[l].copy_(wts.lat_b[l])
            neck.output_w[l].copy_(wts.out_w[l].to(dtype).float())
            neck.output_b[l].copy_(wts.out_b[l])
    feats = [_cl(f.to(dtype).to(cuda_device)).requires_grad_() for f in fs]
    outs = neck(feats)
    g = torch.Generator().manual_seed(23)
    grads = [torch.randn(o.shape, generator=g).to(dtype) for o in outs]
    torch.autograd.backward(outs, [_cl(gg.to(cuda_device)) for gg in grads])
    torch.cuda.synchronize()
    assert U.device_status() == 0

    feats_r = [f.to(dtype).float().requires_grad_() for f in fs]
    lw = [w.to(dtype).float().requires_grad_() for w in wts.lat_w]
    lb = [b.clone().requires_grad_() for b in wts.lat_b]
    ow = [w.to(dtype).float().requires_grad_() for w in wts.out_w]
    ob = [b.clone().requires_grad_() for b in wts.out_b]
    outs_r = O.fpn_neck(feats_r, O.NeckWeights(lw, lb, ow, ob))  # P2..P6
    torch.autograd.backward(outs_r, [gg.float() for gg in grads])
    for o, r in zip(outs, outs_r):  # the forward agrees first
        _close(o, r)
    for f, r in zip(feats, feats_r):
        _close(f.grad, r.grad)
    for l in range(4):
        _close(neck.lateral_w[l].grad, lw[l].grad)
        _close(neck.lateral_b[l].grad, lb[l].grad)
        _close(neck.output_w[l].grad, ow[l].grad)
        _close(neck.output_b[l].grad, ob[l].grad)


def test_backward_is_deterministic(cuda_device):
    """No atomics: two backward passes give bitwise the same gradients."""
    import unified_fpn as U
    g = torch.Generator().manual_seed(5)
    x = _cl(torch.randn(2, 256, 40, 56, generator=g).to(torch.bfloat16).to(cuda_device))
    w3 = (torch.randn(256, 256, 3, 3, generator=g) * 0.03).to(cuda_device)
    gy = _cl(torch.randn(2, 256, 40, 56, generator=g).to(torch.bfloat16).to(cuda_device))
    a = U.fpn_conv3x3_backward(x, w3, gy)
    b = U.fpn_conv3x3_backward(x, w3, gy)
    for p, q in zip(a, b):
        assert torch.equal(p, q)
    up = [U.fpn_upsample_add_backward(gy, (20, 28)) for _ in range(2)]
    assert torch.equal(up[0], up[1])


@pytest.mark.parametrize("taps", [1, 9])
def test_bias_gradient_alone_and_with_weights(cuda_device, taps):
    """grad_b with grad_w (summed inside the weight-gradient launch) and grad_b alone (the
    column-sum kernels) both equal the sum of dY over its pixels."""
    import unified_fpn as U
    from unified_fpn import _lib
    g = torch.Generator().manual_seed(11 + taps)
    n, h, w = 2, 23, 37
    x = _cl(torch.randn(n, 256, h, w, generator=g).to(torch.bfloat16).to(cuda_device))
    gy = _cl(torch.randn(n, 256, h, w, generator=g).to(torch.bfloat16).to(cuda_device))
    ref = gy.float().sum(dim=(0, 2, 3)).cpu()
    if taps == 1:
        wt = (torch.randn(256, 256, generator=g) * 0.05).to(torch.bfloat16).to(cuda_device)
        _, _, gb_fused = U.fpn_lateral_conv_backward(x, wt, gy)
    else:
        wt = U.pack_conv3x3_weight((torch.randn(256, 256, 3, 3, generator=g) * 0.03).to(cuda_device),
                                   torch.bfloat16)
        _, _, gb_fused = U.fpn_conv3x3_backward(x, wt, gy)
    gb_alone = torch.zeros(256, device=cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    if taps == 1:
        rc = _lib.lib.ufpn_lateral_conv_backward(_lib.DTYPE_BF16, x.data_ptr(), wt.data_ptr(), gy.data_ptr(),
                                                 None, None, gb_alone.data_ptr(), n, 256, h, w, stream)
    else:
        rc = _lib.lib.ufpn_conv3x3_backward(_lib.DTYPE_BF16, x.data_ptr(), wt.data_ptr(), gy.data_ptr(),
                                            None, None, gb_alone.data_ptr(), n, h, w, stream)
    torch.cuda.synchronize()
    assert rc == 0 and U.device_status() == 0
    for gb in (gb_fused, gb_alone):
        assert O.rel_err(gb.cpu(), ref) < 1e-5


def test_graphed_training_step_matches_eager(cuda_device):
    """FPNNeck.make_graphed: forward and backward replayed as CUDA graphs give bitwise the
    outputs and gradients of the eager step, also after the weights change."""
    import unified_fpn as U
    sizes = O.level_sizes(128, 160)
    fs = O.make_features(2, O.R50_CHANNELS, sizes, seed=51, dist="normal")
    neck = U.FPNNeck(O.R50_CHANNELS).to(cuda_device)
    feats = [_cl(f.to(torch.bfloat16).to(cuda_device)).requires_grad_() for f in fs]
    g = torch.Generator().manual_seed(52)
    with torch.no_grad():
        shapes = [o.shape for o in neck([f.detach() for f in feats])]
    grads = [_cl(torch.randn(s, generator=g).to(torch.bfloat16).to(cuda_device)) for s in shapes]
    # (no eager autograd graph may be alive while the graphs are captured)
    run = neck.make_graphed([f.detach().clone().requires_grad_() for f in feats])
    for it in range(2):
        results = []
        for fn in (neck, run):
            for p in neck.parameters():
                p.grad = None
            for f in feats:
                f.grad = None
            outs = fn(feats)
            torch.autograd.backward(outs, grads)
            torch.cuda.synchronize()
            results.append([o.detach().clone() for o in outs] + [p.grad.clone() for p in neck.parameters()]
                           + [f.grad.clone() for f in feats])
        assert all(torch.equal(a, b) for a, b in zip(*results))
        with torch.no_grad():  # an optimiser step: the graphs read the weights in place
            for p in neck.parameters():
                p.mul_(0.5)
    assert U.device_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prepared_weights_and_their_backward_paths(cuda_device, dtype):
    """prepare_neck_weights (one launch, every layout) equals the separate conversions
    bitwise, and the backward entry points that take the prepared transposed / flipped weights
    give bitwise the gradients of the ones that derive them."""
    import unified_fpn as U
    g = torch.Generator().manual_seed(61)
    cins = (128, 512, 1024, 2048)
    lat = [(torch.randn(256, c, generator=g) * 0.05).to(cuda_device) for c in cins]
    conv = [(torch.randn(256, 256, 3, 3, generator=g) * 0.03).to(cuda_device) for _ in cins]
    lw, lw_t, packed, flipped = U.prepare_neck_weights(lat, conv, dtype)
    for l, c in enumerate(cins):
        assert torch.equal(lw[l], lat[l].to(dtype))
        ref_t = torch.zeros((c + 255) // 256 * 256, 256, dtype=dtype, device=cuda_device)
        ref_t[:c] = lat[l].to(dtype).t()
        assert torch.equal(lw_t[l], ref_t)
        assert torch.equal(packed[l], U.pack_conv3x3_weight(conv[l], dtype))
        assert torch.equal(flipped[l], packed[l].flip(1).permute(2, 1, 0))
    x = _cl(torch.randn(1, 512, 19, 27, generator=g).to(dtype).to(cuda_device))
    gy = _cl(torch.randn(1, 256, 19, 27, generator=g).to(dtype).to(cuda_device))
    a = U.fpn_lateral_conv_backward(x, lw[1], gy)
    b = U.fpn_lateral_conv_backward(x, lw[1], gy, weight_t=lw_t[1])
    assert all(torch.equal(p, q) for p, q in zip(a, b))
    m = _cl(torch.randn(1, 256, 19, 27, generator=g).to(dtype).to(cuda_device))
    a = U.fpn_conv3x3_backward(m, packed[0], gy)
    b = U.fpn_conv3x3_backward(m, packed[0], gy, weight_flipped=flipped[0])
    assert all(torch.equal(p, q) for p, q in zip(a, b))
    assert U.device_status() == 0


def test_training_step_full_size_properties(cuda_device):
    """R50 800x1216 batch 2 (the benchmark's size, beyond the oracle's reach at fp32 autograd):
    two eager steps give bitwise the same gradients, all finite; the graphed step gives them
    too; the bias gradients equal the pixel sums of the output gradients they come from (dP5's
    includes P6's through the P6 adjoint)."""
    import unified_fpn as U
    dev = torch.device(cuda_device)
    sizes = O.level_sizes(800, 1216)
    gen = torch.Generator(device=dev)
    gen.manual_seed(71)
    feats = [_cl(torch.randn(2, c, h, w, device=dev, generator=gen).clamp_min_(0).to(torch.bfloat16))
             .requires_grad_() for c, (h, w) in zip(O.R50_CHANNELS, sizes)]
    osz = list(sizes) + [((sizes[3][0] - 1) // 2 + 1, (sizes[3][1] - 1) // 2 + 1)]
    grads = [_cl(torch.randn(2, 256, h, w, device=dev, generator=gen).to(torch.bfloat16)) for h, w in osz]
    neck = U.FPNNeck(O.R50_CHANNELS).to(dev)

    def step(fn):
        for p in neck.parameters():
            p.grad = None
        for f in feats:
            f.grad = None
        torch.autograd.backward(fn(feats), grads)
        torch.cuda.synchronize()
        return [p.grad.clone() for p in neck.parameters()] + [f.grad.clone() for f in feats]

    a = step(neck)
    b = step(neck)
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    assert all(torch.isfinite(x).all() for x in a)
    # output-conv bias gradients: the sums of dP2..dP5 (dP5 with dP6 scattered in)
    ob = list(neck.output_b)
    for l in range(3):
        ref = grads[l].float().sum(dim=(0, 2, 3))
        assert O.rel_err(ob[l].grad.cpu(), ref.cpu()) < 1e-5
    ref5 = grads[3].float().sum(dim=(0, 2, 3)) + grads[4].float().sum(dim=(0, 2, 3))
    assert O.rel_err(ob[3].grad.cpu(), ref5.cpu()) < 1e-3  # (dP5 + dP6 rounded to bf16 once)
    run = neck.make_graphed([f.detach().clone().requires_grad_() for f in feats])
    c = step(run)
    assert all(torch.equal(x, y) for x, y in zip(a, c))
    assert U.device_status() == 0


def test_interleaved_steps_and_gradient_accumulation(cuda_device):
    """Each forward keeps its own workspace (merged maps, weight layouts) and the fp32 weight
    gradients are views of one buffer per backward: two forwards followed by their backwards in
    reverse order give bitwise the gradients of two separate steps, and accumulating both into
    .grad (no reset in between) gives their sum."""
    import unified_fpn as U
    dev = torch.device(cuda_device)
    sizes = O.level_sizes(96, 128)
    gen = torch.Generator(device=dev)
    gen.manual_seed(91)
    sets = [[_cl(torch.randn(2, c, h, w, device=dev, generator=gen).to(torch.bfloat16)).requires_grad_()
             for c, (h, w) in zip(O.R50_CHANNELS, sizes)] for _ in range(2)]
    osz = list(sizes) + [((sizes[3][0] - 1) // 2 + 1, (sizes[3][1] - 1) // 2 + 1)]
    grads = [[_cl(torch.randn(2, 256, h, w, device=dev, generator=gen).to(torch.bfloat16)) for h, w in osz]
             for _ in range(2)]
    neck = U.FPNNeck(O.R50_CHANNELS).to(dev)

    def reset():
        for p in neck.parameters():
            p.grad = None
        for s in sets:
            for f in s:
                f.grad = None

    alone = []
    for k in range(2):
        reset()
        torch.autograd.backward(neck(sets[k]), grads[k])
        alone.append([p.grad.clone() for p in neck.parameters()] + [f.grad.clone() for f in sets[k]])
    reset()
    outs = [neck(sets[0]), neck(sets[1])]
    torch.autograd.backward(outs[1], grads[1])
    second = [p.grad.clone() for p in neck.parameters()] + [f.grad.clone() for f in sets[1]]
    torch.autograd.backward(outs[0], grads[0])  # accumulates into the parameters' .grad
    torch.cuda.synchronize()
    assert all(torch.equal(x, y) for x, y in zip(second, alone[1]))
    assert all(torch.equal(f.grad, y) for f, y in zip(sets[0], alone[0][16:]))
    for p, a0, a1 in zip(neck.parameters(), alone[0][:16], alone[1][:16]):
        assert torch.equal(p.grad, a1 + a0)
    assert U.device_status() == 0


@pytest.mark.parametrize("h,w,batch", [(800, 1216, 2), (128, 160, 2), (640, 640, 4)])
def test_training_forward_equals_the_inference_forward(cuda_device, h, w, batch):
    """The training step's forward (FPNNeck: grouped raw laterals, both merges in one launch,
    the P2 lateral with the top-down add, single-CTA halo 3x3s) gives bitwise the outputs of
    UnifiedFPN's forward with the same fp32 weights: P2..P6."""
    import unified_fpn as U
    dev = torch.device(cuda_device)
    sizes = O.level_sizes(h, w)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    feats = [_cl(torch.randn(batch, c, hh, ww, device=dev, generator=gen).clamp_min_(0).to(torch.bfloat16))
             for c, (hh, ww) in zip(O.R50_CHANNELS, sizes)]
    neck = U.FPNNeck(O.R50_CHANNELS).to(dev)
    with torch.no_grad():
        for b in list(neck.lateral_b) + list(neck.output_b):
            b.normal_(0, 0.1, generator=gen)
        outs = neck(feats)
    fpn = U.UnifiedFPN(device=dev)
    fpn.initialize_weights([p.detach() for p in neck.lateral_w], [p.detach() for p in neck.lateral_b],
                           [p.detach() for p in neck.output_w], [p.detach() for p in neck.output_b])
    ref = fpn(feats, return_p6=True)
    torch.cuda.synchronize()
    assert len(outs) == len(ref) == 5
    for a, r in zip(outs, ref):
        assert a.shape == r.shape and torch.equal(a, r)
    assert U.device_status() == 0
