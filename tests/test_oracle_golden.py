"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures come from ``tests/golden/make_golden.py`` (runs nvSubquadratic's own
``ops/fftconv.py``, ``Hyena.forward``/``CKConvND.forward`` and ``a2a_comms`` on
CPU). These tests need neither the reference tree nor a GPU.
"""

import pytest
import torch

from oracle import cp as ocp
from oracle import fftconv as ofc
from oracle.direct import direct_conv
from oracle.hyena import hyena_forward
from tests.conftest import rel_l2

OPS = {
    "causal_fftconv1d_fp32_bhl": (ofc.causal_fftconv1d_bhl, False),
    "fftconv1d_fp32_bhl": (ofc.fftconv1d_bhl, False),
    "fftconv2d_fp32_bhl": (ofc.fftconv2d_bhl, False),
    "fftconv3d_fp32_bhl": (ofc.fftconv3d_bhl, False),
    "causal_fftconv1d_fp32_bhl_w_reshape": (lambda x, k, s: ofc.fftconv_blh(x, k, s, causal=True), True),
    "fftconv1d_fp32_bhl_w_reshape": (lambda x, k, s: ofc.fftconv_blh(x, k, s), True),
    "fftconv2d_fp32_bhl_w_reshape": (lambda x, k, s: ofc.fftconv_blh(x, k, s), True),
    "fftconv3d_fp32_bhl_w_reshape": (lambda x, k, s: ofc.fftconv_blh(x, k, s), True),
}


def _tol(dtype):
    return 2e-6 if dtype == torch.float32 else 1e-2


def _op_cases(golden):
    return golden["ops"]["cases"]


@pytest.mark.parametrize("idx", range(26))
def test_oracle_ops_match_reference(golden, idx):
    cases = _op_cases(golden)
    if idx >= len(cases):
        pytest.skip("no such case")
    c = cases[idx]
    fn, _ = OPS[c["fn"]]
    x = c["x"].clone().requires_grad_(True)
    k = c["k"].clone().requires_grad_(True)
    sc = c["shortcut"].clone().requires_grad_(True) if c["shortcut"] is not None else None
    y = fn(x, k, sc)
    assert y.dtype == c["y"].dtype and y.shape == c["y"].shape
    y.backward(c["dy"])
    tol = _tol(c["x"].dtype)
    assert rel_l2(c["y"], y) <= tol, c["name"]
    assert rel_l2(c["dx"], x.grad) <= tol, c["name"]
    assert rel_l2(c["dk"], k.grad) <= tol, c["name"]
    if sc is not None:
        assert rel_l2(c["dshortcut"], sc.grad) <= tol, c["name"]


def test_oracle_matches_direct_convolution(golden):
    """Independent float64 spatial convolution (the reference tests' own method)."""
    n = 0
    for c in _op_cases(golden):
        if c["x"].dtype != torch.float32 or c["blh"] or c["name"] == "causal1d_alias":
            continue
        causal = c["fn"].startswith("causal")
        y = ofc.fftconv_bhl(c["x"], c["k"], None, causal=causal)
        ref = torch.from_numpy(direct_conv(c["x"].numpy(), c["k"].numpy(), causal=causal))
        assert rel_l2(ref, y) < 1e-5, c["name"]
        n += 1
    assert n >= 15


def test_causal_alias_case_differs_from_linear(golden):
    """K > L+1 with F = 2L wraps around in the reference; the oracle reproduces it."""
    c = next(c for c in _op_cases(golden) if c["name"] == "causal1d_alias")
    lin = torch.from_numpy(direct_conv(c["x"].numpy(), c["k"].numpy(), causal=True)).float()
    y = ofc.causal_fftconv1d_bhl(c["x"], c["k"])
    assert rel_l2(lin, y) > 1e-2
    assert rel_l2(c["y"] - (c["shortcut"].view(1, -1, 1) * c["x"]), y) < 1e-5


def test_shortcut_dtype_assert():
    x = torch.randn(2, 4, 16, dtype=torch.bfloat16)
    k = torch.randn(1, 4, 5, dtype=torch.bfloat16)
    with pytest.raises(AssertionError, match=r"shortcut\.dtype"):
        ofc.fftconv1d_bhl(x, k, torch.randn(4))


def test_kernel_too_long_assert():
    with pytest.raises(AssertionError):
        ofc.fftconv2d_bhl(torch.randn(1, 2, 8, 8), torch.randn(1, 2, 17, 3))


def _bhl_filter_from_blh(kernel_blh, causal):
    filt = kernel_blh
    if causal:  # ckconv_nd.py:1160-1164
        filt = filt[:, filt.shape[1] // 2:, :]
    return filt.movedim(-1, 1)


@pytest.mark.parametrize("idx", range(7))
def test_oracle_hyena_matches_reference(golden, idx):
    cases = golden["hyena"]["cases"]
    c = cases[idx]
    q, k, v = (c[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    kern = c["kernel_blh"].clone().requires_grad_(True)
    D = c["D"].clone().requires_grad_(True)
    sw = c["short_w"].clone().requires_grad_(True)
    sb = c["short_b"].clone().requires_grad_(True) if c["short_b"] is not None else None
    filt = _bhl_filter_from_blh(kern, c["causal"])
    y = hyena_forward(q, k, v, filt, D, sw, sb, causal=c["causal"], gate1=c["gate1"], gate2=c["gate2"])
    y.backward(c["dy"])
    tol = 2e-6 if c["q"].dtype == torch.float32 else 1.5e-2
    for name, got in (("y", y), ("dq", q.grad), ("dk", k.grad), ("dv", v.grad),
                      ("dkernel_blh", kern.grad), ("dD", D.grad), ("dshort_w", sw.grad)):
        assert rel_l2(c[name], got) <= tol, (c["name"], name, rel_l2(c[name], got))
    if sb is not None:
        assert rel_l2(c["dshort_b"], sb.grad) <= tol


def test_oracle_zigzag_orders(golden):
    for n, ref in golden["cp"]["zigzag"].items():
        assert ocp.zigzag_order(n) == ref
    for n, ref in golden["cp"]["inv_zigzag"].items():
        assert ocp.inverse_zigzag_order(n) == ref


@pytest.mark.parametrize("world", [2, 4])
def test_oracle_cp_matches_reference(golden, world):
    ranks = golden["cp"][f"world{world}"]
    for nd in (1, 2, 3):
        full = ranks[0][nd]["full"]
        locals_ = ocp.zigzag_split(full, world, dim=2)
        for r in range(world):
            assert torch.equal(locals_[r], ranks[r][nd]["local"])
        s2f = ocp.split_to_full(locals_, zigzag=True)
        s2f_nz = ocp.split_to_full(locals_, zigzag=False)
        f2s = ocp.full_to_split(s2f, zigzag=True)
        for r in range(world):
            assert torch.equal(s2f[r], ranks[r][nd]["s2f"])
            assert torch.equal(s2f_nz[r], ranks[r][nd]["s2f_nozigzag"])
            assert torch.equal(f2s[r], ranks[r][nd]["f2s"])
        assert torch.equal(ocp.zigzag_gather(locals_, dim=2), full)
        # channel block r of the natural-order sequence lives on rank r
        C = full.shape[1]
        d = C // world
        for r in range(world):
            assert torch.equal(s2f[r], full[:, r * d:(r + 1) * d])


@pytest.mark.parametrize("idx", range(12))
def test_oracle_boundary_ops_match_reference(golden, idx):
    """Circular and mixed boundary conditions (ops/circular_fftconv.py, ops/mixed_fftconv.py)."""
    cases = golden["boundary"]["cases"]
    if idx >= len(cases):
        pytest.skip("no such case")
    c = cases[idx]
    nd = c["x"].ndim - 2
    per = c["periodic"] if c["periodic"] is not None else (True,) * nd
    x = c["x"].clone().requires_grad_(True)
    k = c["k"].clone().requires_grad_(True)
    sc = c["shortcut"].clone().requires_grad_(True) if c["shortcut"] is not None else None
    y = ofc.fftconv_bhl(x, k, sc, periodic=per)
    y.backward(c["dy"])
    tol = _tol(c["x"].dtype)
    assert rel_l2(c["y"], y) <= tol, c["name"]
    assert rel_l2(c["dx"], x.grad) <= tol, c["name"]
    assert rel_l2(c["dk"], k.grad) <= tol, c["name"]
    if sc is not None:
        assert rel_l2(c["dshortcut"], sc.grad) <= tol, c["name"]


def test_oracle_circular_matches_direct_periodic_convolution():
    """Independent check of the circular restatement: float64 periodic spatial convolution
    with the "same" alignment (output t takes taps x[(t + (K - 1) // 2 - j) mod N])."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(1, 2, 8, 12, generator=g, dtype=torch.float64)
    k = torch.randn(1, 2, 4, 5, generator=g, dtype=torch.float64)
    y = ofc.fftconv_bhl(x, k, periodic=(True, True))
    ref = torch.zeros_like(x)
    N0, N1, K0, K1 = 8, 12, 4, 5
    s0, s1 = (K0 - 1) // 2, (K1 - 1) // 2
    for a in range(K0):
        for b in range(K1):
            ref += k[:, :, a, b, None, None] * torch.roll(x, shifts=(a - s0, b - s1), dims=(2, 3))
    assert rel_l2(ref, y) <= 1e-6
