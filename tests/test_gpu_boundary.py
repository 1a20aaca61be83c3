"""GPU parity of circular (periodic) and mixed boundary conditions.

Against the reference's own outputs (tests/golden/boundary.pt from
nvsubquadratic/ops/circular_fftconv.py and ops/mixed_fftconv.py) and against the CPU
oracle on seeded inputs: op level (1D / 2D / 3D, bf16, per-sample kernels, the 1D
four-step length, the product-pass and full-spectrum variants) and the fused Hyena
mixer with periodic axes. Tolerances: rel-L2 <= 1e-5 (float32), <= 2e-2 (bf16).
"""

import math

import pytest
import torch

from oracle import fftconv as ofc
from oracle.hyena import hyena_forward
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def _run(fn, x, k, sc, dy):
    x = x.cuda().requires_grad_(True)
    k = k.cuda().requires_grad_(True)
    scg = sc.cuda().requires_grad_(True) if sc is not None else None
    y = fn(x, k, scg)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    return y, x.grad, k.grad, (scg.grad if scg is not None else None)


@pytest.mark.parametrize("idx", range(12))
def test_boundary_ops_vs_reference_golden(golden, idx):
    from nvsubquadratic_b200 import fftconv as b2

    cases = golden["boundary"]["cases"]
    if idx >= len(cases):
        pytest.skip("no such case")
    c = cases[idx]
    base = getattr(b2, c["fn"])
    fn = (lambda x, k, s: base(x, k, c["periodic"], s)) if c["periodic"] is not None else base
    y, dx, dk, ds = _run(fn, c["x"], c["k"], c["shortcut"], c["dy"])
    tol = TOL[c["x"].dtype]
    assert y.dtype == c["y"].dtype and tuple(y.shape) == tuple(c["y"].shape)
    for name, ref, got in (("y", c["y"], y), ("dx", c["dx"], dx), ("dk", c["dk"], dk)):
        assert rel_l2(ref, got) <= tol, (c["name"], name, rel_l2(ref, got))
    if ds is not None:
        assert rel_l2(c["dshortcut"], ds) <= tol, (c["name"], "dshortcut")


SHAPES = [
    # periodic, x shape, k shape, dtype
    ((True, True), (2, 16, 128, 128), (1, 16, 128, 128), torch.bfloat16),   # full-extent periodic 2D
    ((True,), (2, 4, 1 << 14), (1, 4, 1 << 14), torch.float32),               # four-step circular length
    ((True,), (3, 6, 256), (3, 6, 31), torch.float32),                        # per-sample kernels
    ((True, False, True), (2, 3, 16, 20, 32), (1, 3, 9, 39, 32), torch.float32),
    ((False, True), (2, 8, 48, 64), (1, 8, 95, 64), torch.bfloat16),
]


@pytest.mark.parametrize("case", SHAPES, ids=[f"{c[0]}-{c[1][2:]}" for c in SHAPES])
def test_boundary_ops_vs_oracle_seeded(case):
    from nvsubquadratic_b200 import fftconv as b2

    per, xs, ks, dt = case
    g = torch.Generator().manual_seed(1)
    x = torch.randn(xs, generator=g).to(dt)
    k = (torch.randn(ks, generator=g) / math.sqrt(math.prod(ks[2:]))).to(dt)
    sc = torch.randn(xs[1], generator=g).to(dt)
    dy = torch.randn(xs, generator=g).to(dt)
    xr, kr, sr = (t.clone().requires_grad_(True) for t in (x, k, sc))
    yr = ofc.fftconv_bhl(xr, kr, sr, periodic=per)
    yr.backward(dy)
    y, dx, dk, ds = _run(lambda a, b, c: b2.mixed_fftconv_nd(a, b, per, c), x, k, sc, dy)
    tol = TOL[dt]
    for name, a, b in (("y", yr, y), ("dx", xr.grad, dx), ("dk", kr.grad, dk), ("dD", sr.grad, ds)):
        assert rel_l2(a, b) <= tol, (name, rel_l2(a, b))


@pytest.mark.parametrize("env", ["HYFFT_DISABLE_PRODUCT_PASS", "HYFFT_FULL_KSPEC", "HYFFT_DISABLE_CL_PASS"])
def test_circular_pass_variants(env, monkeypatch):
    """The phase ramp is applied to every form of the filter spectrum the engine keeps
    (half spectrum for product passes, full spectrum for the elementwise product)."""
    monkeypatch.setenv(env, "1")
    test_boundary_ops_vs_oracle_seeded(((True, True), (2, 4, 64, 32), (1, 4, 33, 32), torch.float32))


@pytest.mark.parametrize("nd,per,S,K", [
    (2, (True, True), (64, 64), (64, 64)),
    (3, (True, True, False), (16, 16, 12), (16, 16, 23)),
    (1, (True,), (4096,), (4096,)),
])
def test_periodic_mixer_vs_oracle(nd, per, S, K):
    """The fused Hyena mixer with periodic axes of its long conv (CKConvND fft_padding
    "circular" / per-axis lists) against the oracle composition."""
    from nvsubquadratic_b200.hyena import hyena_fused

    g = torch.Generator().manual_seed(2)
    B, C, sk, dt = 2, 16, 3, torch.bfloat16
    qkv = torch.randn((B,) + S + (3 * C,), generator=g).to(dt)
    filt = torch.randn((1, C) + K, generator=g) / math.sqrt(math.prod(K))
    D = torch.randn(C, generator=g).to(dt)
    sw = ((torch.rand((3 * C, 1) + (sk,) * nd, generator=g) * 2 - 1) / sk ** (nd / 2)).to(dt)
    dy = torch.randn((B,) + S + (C,), generator=g).to(dt)
    kw = dict(gate1="silu", gate2="sigmoid", periodic=per)
    q, k, v = (t.clone().requires_grad_(True) for t in qkv.chunk(3, dim=-1))
    pr = [t.clone().requires_grad_(True) for t in (filt, D, sw)]
    yr = hyena_forward(q, k, v, *pr, None, **kw)
    yr.backward(dy)
    x = qkv.cuda().requires_grad_(True)
    pd = [t.cuda().requires_grad_(True) for t in (filt, D, sw)]
    y = hyena_fused(*x.chunk(3, dim=-1), *pd, None, **kw)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    ref = [yr, torch.cat([q.grad, k.grad, v.grad], dim=-1)] + [t.grad for t in pr]
    got = [y, x.grad] + [t.grad for t in pd]
    for name, a, b in zip(("y", "dqkv", "dfilt", "dD", "dsw"), ref, got):
        assert rel_l2(a, b) <= 2e-2, (name, rel_l2(a, b))


def test_periodic_axis_length_must_be_a_power_of_two():
    from nvsubquadratic_b200 import fftconv as b2

    x = torch.zeros(1, 2, 24, device="cuda")
    with pytest.raises(NotImplementedError, match="powers of two"):
        b2.circular_fftconv1d_fp32_bhl(x, torch.zeros(1, 2, 5, device="cuda"))
