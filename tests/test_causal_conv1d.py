"""The direct depthwise causal 1D conv (``nvsubquadratic_b200.causal_conv1d``).

GPU: forward and gradients against the oracle restatement of the reference test's own
reference function (F.pad + depthwise F.conv1d + optional SiLU,
tests/ops/test_causal_conv1d_custom.py:62-68) at the reference test's shapes, with bias,
SiLU, bf16, long sequences that span several CTA segments and the longest filter; the
module form against the same reference; and the back-to-back composition.
CPU: argument checks of the C ABI and the module's construction errors (the reference's
construction tests, tests/modules/test_subq_ops_causal_conv1d.py:124-144).
Tolerances: rel-L2 <= 1e-5 (float32), <= 2e-2 (bf16).
"""

import pytest
import torch

from oracle.causal_conv1d import b2b_ref, causal_conv1d_ref
from tests.conftest import rel_l2

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2}

CASES = [
    # B, C, L, K, bias, activation, dtype
    (2, 16, 64, 3, False, "identity", torch.float32),   # reference test shapes
    (2, 36, 256, 3, True, "identity", torch.float32),
    (2, 64, 128, 7, False, "identity", torch.float32),
    (2, 36, 256, 3, False, "silu", torch.float32),
    (3, 24, 5000, 64, True, "silu", torch.float32),     # several 1024-sample segments, ragged tail
    (1, 8, 3000, 1024, True, "identity", torch.float32),  # the longest filter
    (2, 32, 4100, 4, True, "silu", torch.bfloat16),
    (1, 12, 1 << 16, 7, False, "identity", torch.bfloat16),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[f"C{c[1]}-L{c[2]}-K{c[3]}-{c[5]}-{c[6]}" for c in CASES])
def test_causal_conv1d_vs_oracle(case):
    from nvsubquadratic_b200.causal_conv1d import causal_conv1d

    B, C, L, K, with_bias, act, dt = case
    g = torch.Generator().manual_seed(L + K)
    x = torch.randn(B, C, L, generator=g).to(dt)
    w = torch.randn(C, K, generator=g) / K ** 0.5
    b = torch.randn(C, generator=g) if with_bias else None
    dy = torch.randn(B, C, L, generator=g).to(dt)
    xr, wr = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    br = b.clone().requires_grad_(True) if b is not None else None
    yr = causal_conv1d_ref(xr, wr, br, act)
    yr.backward(dy)
    xd, wd = x.cuda().requires_grad_(True), w.cuda().requires_grad_(True)
    bd = b.cuda().requires_grad_(True) if b is not None else None
    y = causal_conv1d(xd, wd, bd, act)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    tol = TOL[dt]
    assert y.dtype == dt and y.shape == (B, C, L)
    checks = [("y", yr, y), ("dx", xr.grad, xd.grad), ("dw", wr.grad, wd.grad)]
    if b is not None:
        checks.append(("db", br.grad, bd.grad))
    for name, a, bb in checks:
        e = rel_l2(a, bb)
        assert e <= tol, (name, e)


@pytest.mark.gpu
def test_causality_by_perturbation():
    from nvsubquadratic_b200.causal_conv1d import causal_conv1d

    g = torch.Generator().manual_seed(9)
    x = torch.randn(1, 8, 3000, generator=g).cuda()
    w = torch.randn(8, 33, generator=g).cuda()
    y0 = causal_conv1d(x, w)
    x2 = x.clone()
    x2[..., 1500:] += 1.0
    y1 = causal_conv1d(x2, w)
    assert torch.equal(y0[..., :1500], y1[..., :1500])
    assert (y0[..., 1500:] - y1[..., 1500:]).abs().max() > 0.1


@pytest.mark.gpu
def test_module_matches_reference_conv():
    """CausalConv1dB200 with a reference-shaped state dict (weight [C, 1, K], bias)."""
    from nvsubquadratic_b200.causal_conv1d import CausalConv1dB200

    torch.manual_seed(42)
    C, L, K = 36, 256, 3
    m = CausalConv1dB200(C, C, K, groups=C, bias=True, activation="silu").cuda()
    assert isinstance(m, torch.nn.Conv1d)
    x = torch.randn(2, C, L)
    xd = x.cuda().requires_grad_(True)
    m(xd).sum().backward()
    xr = x.clone().requires_grad_(True)
    wr = m.weight.detach().cpu().squeeze(1).clone().requires_grad_(True)
    br = m.bias.detach().cpu().clone().requires_grad_(True)
    causal_conv1d_ref(xr, wr, br, "silu").sum().backward()
    assert rel_l2(xr.grad, xd.grad) <= 1e-5
    assert rel_l2(wr.grad, m.weight.grad.squeeze(1)) <= 1e-5
    assert rel_l2(br.grad, m.bias.grad) <= 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("B,C,L,K", [(2, 16, 64, 3), (4, 32, 128, 4), (2, 16, 128, 8)])
def test_b2b_shape_and_composition(B, C, L, K):
    """The reference's shape contract (tests/ops/test_causal_conv1d_custom.py:124-133) and
    the composition against the oracle."""
    from nvsubquadratic_b200.causal_conv1d import b2b_causal_conv1d

    g = torch.Generator().manual_seed(42)
    x = torch.randn(B, 3 * C, L, generator=g)
    wp = torch.randn(3 * C, K, generator=g) / K
    wm = torch.randn(C, K, generator=g) / K
    sb = torch.randn(C, generator=g)
    y = b2b_causal_conv1d(x.cuda(), wp.cuda(), wm.cuda(), sb.cuda())
    assert y.shape == (B, C, L) and torch.isfinite(y).all()
    assert rel_l2(b2b_ref(x, wp, wm, sb), y) <= 1e-5


def test_abi_argument_checks():
    """Invalid requests are refused on the host before anything is launched."""
    from nvsubquadratic_b200 import _lib

    lib = _lib.load()
    p = 16  # never dereferenced: every call fails validation first
    assert lib.hyfft_causal_conv1d_forward(p, p, None, p, 1, 4, 32, 3, 2, 0, None) == _lib.HYFFT_ERR_INVALID  # act
    assert lib.hyfft_causal_conv1d_forward(p, p, None, p, 1, 4, 32, 0, 0, 0, None) == _lib.HYFFT_ERR_INVALID  # K
    assert lib.hyfft_causal_conv1d_forward(p, p, None, p, 1, 4, 32, 2048, 0, 0, None) == _lib.HYFFT_ERR_UNSUPPORTED
    assert lib.hyfft_causal_conv1d_forward(p, p, None, p, 1, 4, 32, 3, 0, 9, None) == _lib.HYFFT_ERR_INVALID  # dtype
    assert lib.hyfft_causal_conv1d_backward(p, p, None, None, p, p, None, 1, 4, 32, 3, 0, 0,
                                            None) == _lib.HYFFT_ERR_INVALID  # no dy


def test_module_construction_checks():
    from nvsubquadratic_b200.causal_conv1d import CausalConv1dB200, causal_conv1d

    with pytest.raises(ValueError, match="depthwise-only"):
        CausalConv1dB200(in_channels=16, out_channels=16, kernel_size=3, groups=4)
    with pytest.raises(ValueError, match="depthwise-only"):
        CausalConv1dB200(in_channels=16, out_channels=32, kernel_size=3, groups=16)
    with pytest.raises(ValueError, match="activation"):
        CausalConv1dB200(in_channels=16, out_channels=16, kernel_size=3, groups=16, activation="relu")
    assert isinstance(CausalConv1dB200(16, 16, 3, groups=16), torch.nn.Conv1d)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        causal_conv1d(torch.zeros(1, 4, 8), torch.zeros(4, 3))
