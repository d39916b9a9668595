"""CPU tests of the optional epilogue operations: the oracle's activations against the
formulas of the reference's activation_kernel and its unit test, and the library's host-side
BatchNorm folding against conv followed by the oracle's batch_norm (the reference's
batch_norm_kernel restated)."""
import pytest
import torch
import torch.nn.functional as F

from oracle import fpn_oracle as O


def test_oracle_activations_follow_the_reference_formulas():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, generator=g) * 4
    # tests/unit/test_fpn_kernels.cu:270-300: LeakyReLU with alpha 0.1, in > 0 ? in : alpha * in
    exp = torch.tensor([v if v > 0 else 0.1 * v for v in x.tolist()])
    assert torch.allclose(O.activation(x, "leaky_relu", 0.1), exp, atol=1e-6, rtol=0)
    assert torch.equal(O.activation(x, "relu"), torch.tensor([max(0.0, v) for v in x.tolist()]))
    assert torch.allclose(O.activation(x, "swish"), x * torch.sigmoid(x), atol=1e-6, rtol=1e-6)
    assert torch.equal(O.activation(x, None), x) and torch.equal(O.activation(x, "none"), x)
    with pytest.raises(ValueError):
        O.activation(x, "gelu")


@pytest.mark.parametrize("with_affine", [True, False])
def test_fold_batch_norm_equals_conv_then_batch_norm(with_affine):
    import unified_fpn as U
    g = torch.Generator().manual_seed(1)
    cout, cin = 32, 16
    w = torch.randn(cout, cin, 3, 3, generator=g) * 0.1
    b = torch.randn(cout, generator=g) if with_affine else None
    gamma = torch.rand(cout, generator=g) + 0.5 if with_affine else None
    beta = torch.randn(cout, generator=g) if with_affine else None
    mean = torch.randn(cout, generator=g)
    var = torch.rand(cout, generator=g) * 2 + 0.01
    x = torch.randn(2, cin, 9, 11, generator=g)
    wf, bf = U.fold_batch_norm(w, b, gamma, beta, mean, var, eps=1e-5)
    assert wf.shape == w.shape and bf.shape == (cout,)
    ref = O.batch_norm(F.conv2d(x.double(), w.double(), None if b is None else b.double(), padding=1),
                       None if gamma is None else gamma.double(), None if beta is None else beta.double(),
                       mean.double(), var.double(), 1e-5)
    got = F.conv2d(x.double(), wf.double(), bf.double(), padding=1)
    assert O.rel_err(got, ref) < 1e-6
    # the folded 1x1 lateral form ([Cout, Cin] weights) works the same way
    w1 = torch.randn(cout, cin, generator=g)
    wf1, bf1 = U.fold_batch_norm(w1, None, None, None, mean, var)
    ref1 = O.batch_norm(O.lateral_conv(x.double(), w1.double(), torch.zeros(cout, dtype=torch.float64)),
                        None, None, mean.double(), var.double())
    assert O.rel_err(O.lateral_conv(x.double(), wf1.double(), bf1.double()), ref1) < 1e-6


def test_fold_batch_norm_rejects_bad_parameters():
    import unified_fpn as U
    w = torch.randn(4, 3, 3, 3)
    with pytest.raises(U.UFPNError):
        U.fold_batch_norm(w, None, None, None, torch.zeros(4), -torch.ones(4))  # var + eps <= 0
    with pytest.raises(ValueError):
        U.fold_batch_norm(w, None, None, None, torch.zeros(3), torch.ones(3))


def test_training_entry_points_validate_on_the_host():
    """The training path rejects what it cannot run before any device work."""
    import unified_fpn as U
    feats = [torch.zeros(1, c, 4, 4, dtype=torch.bfloat16) for c in (256, 512, 1024, 2048)]
    w = [torch.zeros(256, c) for c in (256, 512, 1024, 2048)]
    b = [torch.zeros(256) for _ in range(4)]
    w3 = [torch.zeros(256, 256, 3, 3) for _ in range(4)]
    with pytest.raises(ValueError):  # CPU tensors
        U.fpn_neck_forward_train(feats, w, b, w3, b)
    with pytest.raises(ValueError):  # fp32 features
        U.fpn_neck_forward_train([f.float() for f in feats], w, b, w3, b)
    with pytest.raises(ValueError):  # three levels
        U.fpn_neck_forward_train(feats[:3], w, b, w3, b)
    with pytest.raises(ValueError):
        U.prepare_neck_weights(w, w3, torch.float32)


def test_batch_norm_identity_known_answer_of_the_reference_unit_test():
    """tests/unit/test_fpn_kernels.cu:185-240 (BatchNorm): weight 1, bias 0, mean 0, var 1,
    eps 1e-5 preserve the input within 1e-4 -- for the oracle's batch_norm and for a conv
    folded with those parameters."""
    import unified_fpn as U
    g = torch.Generator().manual_seed(9)
    x = torch.randn(2, 64, 8, 8, generator=g)
    ones, zeros = torch.ones(64), torch.zeros(64)
    assert (O.batch_norm(x, ones, zeros, zeros, ones, 1e-5) - x).abs().max() <= 1e-4
    w = torch.randn(64, 64, generator=g) * 0.1
    b = torch.randn(64, generator=g)
    wf, bf = U.fold_batch_norm(w, b, ones, zeros, zeros, ones, eps=1e-5)
    assert (wf - w).abs().max() <= 1e-4 * w.abs().max() and (bf - b).abs().max() <= 1e-4
