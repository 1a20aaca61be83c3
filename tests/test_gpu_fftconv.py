"""GPU parity of the op-level long convolutions (the C-ABI through ctypes).

Checks, against the reference's golden vectors and against the CPU oracle on the
same seeded inputs: forward y and the gradients dx, dkernel, dshortcut.
Tolerance (north star): rel-L2 <= 1e-5 for float32 I/O, <= 2e-2 for bfloat16 I/O.
"""

import pytest
import torch

from oracle import fftconv as ofc
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 5e-3}


def _b2():
    from nvsubquadratic_b200 import fftconv as b2

    return b2


def _fn_map():
    b2 = _b2()
    return {
        "causal_fftconv1d_fp32_bhl": b2.causal_fftconv1d_fp32_bhl,
        "fftconv1d_fp32_bhl": b2.fftconv1d_fp32_bhl,
        "fftconv2d_fp32_bhl": b2.fftconv2d_fp32_bhl,
        "fftconv3d_fp32_bhl": b2.fftconv3d_fp32_bhl,
        "causal_fftconv1d_fp32_bhl_w_reshape": b2.causal_fftconv1d_fp32_bhl_w_reshape,
        "fftconv1d_fp32_bhl_w_reshape": b2.fftconv1d_fp32_bhl_w_reshape,
        "fftconv2d_fp32_bhl_w_reshape": b2.fftconv2d_fp32_bhl_w_reshape,
        "fftconv3d_fp32_bhl_w_reshape": b2.fftconv3d_fp32_bhl_w_reshape,
    }


def _run(fn, x, k, sc, dy):
    x = x.cuda().requires_grad_(True)
    k = k.cuda().requires_grad_(True)
    scg = sc.cuda().requires_grad_(True) if sc is not None else None
    y = fn(x, k, scg)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    return y, x.grad, k.grad, (scg.grad if scg is not None else None)


@pytest.mark.parametrize("idx", range(26))
def test_ops_vs_reference_golden(golden, idx):
    cases = golden["ops"]["cases"]
    if idx >= len(cases):
        pytest.skip("no such case")
    c = cases[idx]
    fn = _fn_map()[c["fn"]]
    y, dx, dk, ds = _run(fn, c["x"], c["k"], c["shortcut"], c["dy"])
    assert y.dtype == c["y"].dtype and tuple(y.shape) == tuple(c["y"].shape)
    tol = TOL[c["x"].dtype]
    assert rel_l2(c["y"], y) <= tol, (c["name"], "y", rel_l2(c["y"], y))
    assert rel_l2(c["dx"], dx) <= tol, (c["name"], "dx", rel_l2(c["dx"], dx))
    assert rel_l2(c["dk"], dk) <= tol, (c["name"], "dk", rel_l2(c["dk"], dk))
    if ds is not None:
        assert rel_l2(c["dshortcut"], ds) <= tol, (c["name"], "dshortcut")


SHAPES = [
    # (causal, x shape, k shape, dtype)
    (True, (2, 64, 4096), (1, 64, 4096), torch.float32),      # config 0 (reference CPU case)
    (True, (1, 8, 8192), (1, 8, 8192), torch.float32),        # four-step 1D (F = 16384)
    (True, (1, 4, 1 << 15), (1, 4, 1 << 15), torch.bfloat16),  # four-step 1D (F = 65536)
    (False, (2, 16, 64, 64), (1, 16, 15, 15), torch.float32),
    (False, (4, 8, 16, 16), (1, 8, 5, 5), torch.float32),
    (False, (3, 24, 14, 14), (1, 24, 27, 27), torch.bfloat16),  # ViT grid, double-grid kernel
    (False, (2, 4, 48, 40), (1, 4, 95, 79), torch.float32),
    (False, (1, 4, 16, 16, 16), (1, 4, 31, 31, 31), torch.float32),
    (False, (3, 2, 10, 12, 9), (1, 2, 7, 23, 9), torch.bfloat16),
    (False, (2, 8, 300), (1, 8, 77), torch.float32),
    # large-grid 2D kernels (F = 256 x 256, N <= 128)
    (False, (2, 6, 100, 120), (1, 6, 129, 150), torch.float32),
    (False, (3, 4, 128, 128), (1, 4, 128, 128), torch.bfloat16),
    (False, (1, 3, 128, 97), (1, 3, 255, 193), torch.float32),
]


@pytest.mark.parametrize("case", SHAPES, ids=[str(s[1]) for s in SHAPES])
def test_ops_vs_oracle_seeded(case):
    causal, xs, ks, dt = case
    g = torch.Generator().manual_seed(0)
    x = torch.randn(xs, generator=g).to(dt)
    k = (torch.randn(ks, generator=g) * 0.1).to(dt)
    sc = torch.randn(xs[1], generator=g).to(dt)
    dy = torch.randn(xs, generator=g).to(dt)

    xr, kr, sr = (t.clone().requires_grad_(True) for t in (x, k, sc))
    yr = ofc.fftconv_bhl(xr, kr, sr, causal=causal)
    yr.backward(dy)

    b2 = _b2()
    fn = b2.causal_fftconv1d_fp32_bhl if causal else b2.fftconv_nd
    y, dx, dk, ds = _run(fn, x, k, sc, dy)
    tol = TOL[dt]
    assert rel_l2(yr, y) <= tol, rel_l2(yr, y)
    assert rel_l2(xr.grad, dx) <= tol, rel_l2(xr.grad, dx)
    assert rel_l2(kr.grad, dk) <= tol, rel_l2(kr.grad, dk)
    assert rel_l2(sr.grad, ds) <= tol, rel_l2(sr.grad, ds)


@pytest.mark.parametrize("case", [SHAPES[3], SHAPES[1], SHAPES[8]], ids=["2d-64", "1d-four-step", "3d-ragged"])
def test_generic_pass_kernel_matches_oracle(case, monkeypatch):
    """With the channel-innermost two-level kernel switched off, the generic strided pass
    kernel (which keeps the real-I/O and four-step passes) runs the complex middle passes."""
    monkeypatch.setenv("HYFFT_DISABLE_CL_PASS", "1")
    test_ops_vs_oracle_seeded(case)


@pytest.mark.parametrize("case", [SHAPES[3], SHAPES[7]], ids=["2d-64", "3d-16"])
def test_unfused_backward_matches_oracle(case, monkeypatch):
    """The backward as separate passes plus the elementwise spectral kernel (the path taken
    when the merged backward product pass does not apply)."""
    monkeypatch.setenv("HYFFT_DISABLE_BWD_PASS", "1")
    test_ops_vs_oracle_seeded(case)


@pytest.mark.parametrize("case", [SHAPES[3], SHAPES[7]], ids=["2d-64", "3d-16"])
def test_full_filter_spectrum_matches_oracle(case, monkeypatch):
    """2D / 3D product passes normally read half of the (Hermitian) filter spectrum and mirror
    the rest; the full-spectrum form of the same passes matches too."""
    monkeypatch.setenv("HYFFT_FULL_KSPEC", "1")
    test_ops_vs_oracle_seeded(case)


def test_per_sample_kernel_and_odd_batch():
    g = torch.Generator().manual_seed(1)
    b2 = _b2()
    for xs, ks in (((3, 4, 20, 20), (3, 4, 9, 9)), ((5, 3, 17, 13), (1, 3, 33, 25))):
        x = torch.randn(xs, generator=g)
        k = torch.randn(ks, generator=g)
        dy = torch.randn(xs, generator=g)
        xr, kr = x.clone().requires_grad_(True), k.clone().requires_grad_(True)
        yr = ofc.fftconv_bhl(xr, kr)
        yr.backward(dy)
        y, dx, dk, _ = _run(b2.fftconv2d_fp32_bhl, x, k, None, dy)
        assert rel_l2(yr, y) < 1e-5
        assert rel_l2(xr.grad, dx) < 1e-5
        assert rel_l2(kr.grad, dk) < 1e-5


def test_causality_by_perturbation():
    """Output at i depends only on input[0..i] (reference tests/ops/test_fftconv.py:254-271,
    same shapes and bounds), plus a long-sequence variant with a relative bound."""
    b2 = _b2()
    torch.manual_seed(42)
    B, H, L, K = 1, 8, 64, 15
    x = torch.randn(B, H, L, device="cuda")
    k = torch.randn(1, H, K, device="cuda")
    y0 = b2.causal_fftconv1d_fp32_bhl(x, k)
    x2 = x.clone()
    x2[:, :, L // 2] += 1.0
    y1 = b2.causal_fftconv1d_fp32_bhl(x2, k)
    assert (y0[..., : L // 2] - y1[..., : L // 2]).abs().max().item() < 1e-5
    assert (y0[..., L // 2:] - y1[..., L // 2:]).abs().max().item() > 0.01

    g = torch.Generator().manual_seed(2)
    B, H, L = 2, 8, 1 << 14  # four-step path
    x = torch.randn(B, H, L, generator=g).cuda()
    k = torch.randn(1, H, L, generator=g).cuda()
    y0 = b2.causal_fftconv1d_fp32_bhl(x, k)
    x2 = x.clone()
    x2[..., L // 2:] += torch.randn(B, H, L - L // 2, generator=g).cuda()
    y1 = b2.causal_fftconv1d_fp32_bhl(x2, k)
    scale = y0.abs().max().item()
    assert (y0[..., : L // 2] - y1[..., : L // 2]).abs().max().item() < 1e-6 * scale * 8
    assert (y0[..., L // 2:] - y1[..., L // 2:]).abs().max().item() > 1e-2 * scale


def test_inputs_not_mutated_and_new_output():
    b2 = _b2()
    x = torch.randn(2, 4, 32, 32, device="cuda")
    k = torch.randn(1, 4, 7, 7, device="cuda")
    x0, k0 = x.clone(), k.clone()
    y = b2.fftconv2d_fp32_bhl(x, k)
    assert torch.equal(x, x0) and torch.equal(k, k0)
    assert y.data_ptr() != x.data_ptr()


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_large_grid_2d_matches_pass_chain_and_blh(dt, monkeypatch):
    """The fused large-grid 2D kernels agree with the multi-pass engine, and the
    channels-last entry agrees with the channels-first one."""
    b2 = _b2()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(3, 5, 112, 128, generator=g).to(dt)
    k = torch.randn(1, 5, 127, 101, generator=g) * 0.05
    sc = torch.randn(5, generator=g).to(dt)
    dy = torch.randn(3, 5, 112, 128, generator=g).to(dt)
    fused = _run(b2.fftconv2d_fp32_bhl, x, k, sc, dy)
    blh = _run(b2.fftconv2d_fp32_blh, x.permute(0, 2, 3, 1).contiguous(), k.permute(0, 2, 3, 1).contiguous(), sc,
               dy.permute(0, 2, 3, 1).contiguous())
    monkeypatch.setenv("HYFFT_DISABLE_BIG2D", "1")
    chain = _run(b2.fftconv2d_fp32_bhl, x, k, sc, dy)
    tol = TOL[dt]
    for a, b, c, name in zip(chain, fused, blh, ("y", "dx", "dk", "dshortcut")):
        assert rel_l2(a, b) <= tol, (name, rel_l2(a, b))
        c = c.permute(0, 3, 1, 2) if c.ndim == 4 else c
        assert rel_l2(b, c) <= tol, (name, "blh", rel_l2(b, c))


@pytest.mark.parametrize("causal,xs,ks,dt", [
    (True, (2, 8, 1000), (1, 8, 1000), torch.float32),       # one pass each way (F <= 4096)
    (True, (1, 4, 1 << 14), (1, 4, 1 << 14), torch.float32),  # four-step
    (False, (3, 6, 40, 36), (1, 6, 79, 35), torch.bfloat16),  # 2D
    (False, (2, 3, 12, 10, 9), (1, 3, 23, 19, 17), torch.float32),  # 3D
    (False, (3, 4, 300), (3, 4, 77), torch.float32),          # per-sample kernels
])
def test_product_pass_matches_unfused_chain(causal, xs, ks, dt, monkeypatch):
    """The merged forward/product/inverse pass gives the results of the separate passes."""
    b2 = _b2()
    g = torch.Generator().manual_seed(2)
    x = torch.randn(xs, generator=g).to(dt)
    k = torch.randn(ks, generator=g) * 0.05
    sc = torch.randn(xs[1], generator=g).to(dt)
    dy = torch.randn(xs, generator=g).to(dt)
    fn = b2.causal_fftconv1d_fp32_bhl if causal else b2.fftconv_nd
    fused = _run(fn, x, k, sc, dy)
    monkeypatch.setenv("HYFFT_DISABLE_PRODUCT_PASS", "1")
    plain = _run(fn, x, k, sc, dy)
    tol = TOL[dt]
    for a, b, name in zip(plain, fused, ("y", "dx", "dk", "dshortcut")):
        assert rel_l2(a, b) <= tol, (name, rel_l2(a, b))
