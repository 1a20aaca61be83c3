"""GPU parity at the benchmark configurations' own geometry.

The seeded parity tests elsewhere use small shapes; these cases run the shapes the
benchmark measures (or a channel / batch slice of them that the CPU oracle finishes in
seconds), so every path a bench line times is also checked against the oracle:

* cfg1 in full: B=32, C=768, 14x14 grid, 14x14 filter, 3x3 short conv, bf16 (the fused
  small-grid kernels, 24x24 transforms);
* cfg2's 128x128 grid with a 128x128 filter (the large-grid kernels, on the 192-point
  transforms they use for it and on 256-point ones) at B=2, C=32, mixer and op;
* cfg3's 64^3 volume with a full-extent 64^3 filter (F = 128^3, the channel-innermost
  passes and the 3x3x3 plane stencils) at B=2, C=8;
* cfg4's length: the causal op at L = 2^20 (F = 2^21, four-step passes) and the causal
  Hyena mixer at L = 2^20 with its 7-tap causal short conv, on a few channels;
* the channel-chunked engine (the path the context-parallel bench runs with a small
  workspace budget): op and mixer with HYFFT_WS_BUDGET_MB forcing several chunks.

Oracle: oracle/fftconv.py (nvsubquadratic/ops/fftconv.py restated) and oracle/hyena.py
(nvsubquadratic/modules/hyena_nd.py:497-583 restated), float32 FFTs on the CPU.
Tolerances (north star): rel-L2 <= 1e-5 for float32 I/O, <= 2e-2 for bf16 I/O with
float32 accumulation.
"""

import math

import pytest
import torch

from oracle import fftconv as ofc
from oracle.hyena import hyena_forward
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def _mixer_inputs(B, C, S, K, sk, dt, causal, seed=0):
    g = torch.Generator().manual_seed(seed)
    nd = len(S)
    qkv = torch.randn((B,) + S + (3 * C,), generator=g).to(dt)
    filt = torch.randn((1, C) + K, generator=g) / math.sqrt(math.prod(K))
    if causal:  # decaying causal filter as in the long-context configuration
        t = torch.arange(K[0], dtype=torch.float32)
        alpha = (torch.rand(C, 1, generator=g) * 4.5 + 0.5) / K[0]
        filt = filt * torch.exp(-alpha * t).view(1, C, K[0]) * math.sqrt(K[0] / 64)
    D = ((torch.rand(C, generator=g) * 2 - 1) / math.sqrt(C)).to(dt)
    sw = ((torch.rand((3 * C, 1) + (sk,) * nd, generator=g) * 2 - 1) / math.sqrt(sk ** nd)).to(dt)
    dy = torch.randn((B,) + S + (C,), generator=g).to(dt)
    return qkv, filt, D, sw, dy


def _check_mixer(B, C, S, K, sk, dt, causal=False, g1="identity", g2="identity"):
    from nvsubquadratic_b200.hyena import hyena_fused

    qkv, filt, D, sw, dy = _mixer_inputs(B, C, S, K, sk, dt, causal)
    kw = dict(causal=causal, gate1=g1, gate2=g2)
    # oracle on the CPU
    q, k, v = (t.clone().requires_grad_(True) for t in qkv.chunk(3, dim=-1))
    ins_r = [t.clone().requires_grad_(True) for t in (filt, D, sw)]
    yr = hyena_forward(q, k, v, *ins_r, None, **kw)
    yr.backward(dy)
    ref = [yr, torch.cat([q.grad, k.grad, v.grad], dim=-1)] + [t.grad for t in ins_r]
    # fused backend on the GPU, q, k, v as views of one projection output
    qkv_d = qkv.cuda().requires_grad_(True)
    ins_d = [t.cuda().requires_grad_(True) for t in (filt, D, sw)]
    y = hyena_fused(*qkv_d.chunk(3, dim=-1), *ins_d, None, **kw)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    got = [y, qkv_d.grad] + [t.grad for t in ins_d]
    tol = TOL[dt]
    for name, a, b in zip(("y", "dqkv", "dfilt", "dD", "dshort_w"), ref, got):
        e = rel_l2(a, b)
        assert e <= tol, (name, e)


def test_cfg1_full_size_vs_oracle():
    """cfg1 exactly as benchmarked: [32, 14, 14, 3*768] bf16 projection, 14x14 filter."""
    _check_mixer(32, 768, (14, 14), (14, 14), 3, torch.bfloat16)


@pytest.mark.parametrize("f256", [False, True], ids=["F192", "F256"])
def test_cfg2_grid_vs_oracle(f256, monkeypatch):
    """cfg2's 128x128 grid and 128x128 filter (large-grid kernels) at B=2, C=32, on the
    192-point transforms the library picks for it and on the 256-point ones."""
    if f256:
        monkeypatch.setenv("HYFFT_B2_F256", "1")
    _check_mixer(2, 32, (128, 128), (128, 128), 3, torch.bfloat16)


@pytest.mark.parametrize("f256", [False, True], ids=["F192", "F256"])
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_cfg2_grid_op_vs_oracle(dt, f256, monkeypatch):
    """The op-level 2D conv at cfg2's grid (forward, dx, dk, dshortcut) on both large-grid
    FFT lengths, odd batch and channel counts."""
    from nvsubquadratic_b200 import fftconv as b2

    if f256:
        monkeypatch.setenv("HYFFT_B2_F256", "1")
    g = torch.Generator().manual_seed(5)
    x = torch.randn(3, 5, 128, 128, generator=g).to(dt)
    k = torch.randn(1, 5, 128, 128, generator=g) / 128
    sc = torch.randn(5, generator=g).to(dt)
    dy = torch.randn(3, 5, 128, 128, generator=g).to(dt)
    xr, kr, sr = (t.clone().requires_grad_(True) for t in (x, k, sc))
    yr = ofc.fftconv_bhl(xr, kr, sr, causal=False)
    yr.backward(dy)
    xd, kd, sd = (t.cuda().requires_grad_(True) for t in (x, k, sc))
    y = b2.fftconv2d_fp32_bhl(xd, kd, sd)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    for name, a, b in (("y", yr, y), ("dx", xr.grad, xd.grad), ("dk", kr.grad, kd.grad), ("ds", sr.grad, sd.grad)):
        assert rel_l2(a, b) <= TOL[dt], (name, rel_l2(a, b))


def test_cfg3_volume_vs_oracle():
    """cfg3's 64^3 volume, full-extent 64^3 filter (F = 128^3), 3x3x3 short conv, at B=2, C=8."""
    _check_mixer(2, 8, (64, 64, 64), (64, 64, 64), 3, torch.bfloat16)


def test_cfg4_length_mixer_vs_oracle():
    """cfg4's sequence length with its causal 7-tap short conv (the local channel block of
    the context-parallel mixer runs exactly this), B=1, C=4."""
    _check_mixer(1, 4, (1 << 20,), (1 << 20,), 7, torch.bfloat16, causal=True)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_cfg4_length_causal_op_vs_oracle(dt):
    """The causal op at L = 2^20, K = L (F = 2^21 four-step passes), two channels."""
    from nvsubquadratic_b200.fftconv import causal_fftconv1d_fp32_bhl

    g = torch.Generator().manual_seed(3)
    B, H, L = 1, 2, 1 << 20
    x = torch.randn(B, H, L, generator=g).to(dt)
    t = torch.arange(L, dtype=torch.float32)
    alpha = (torch.rand(H, 1, generator=g) * 4.5 + 0.5) / L
    k = (torch.randn(1, H, L, generator=g) * torch.exp(-alpha * t) / 32).to(dt)
    sc = torch.randn(H, generator=g).to(dt)
    dy = torch.randn(B, H, L, generator=g).to(dt)
    xr, kr, sr = (u.clone().requires_grad_(True) for u in (x, k, sc))
    yr = ofc.fftconv_bhl(xr, kr, sr, causal=True)
    yr.backward(dy)
    xd, kd, sd = (u.cuda().requires_grad_(True) for u in (x, k, sc))
    y = causal_fftconv1d_fp32_bhl(xd, kd, sd)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    tol = TOL[dt]
    for name, a, b in (("y", yr, y), ("dx", xr.grad, xd.grad), ("dk", kr.grad, kd.grad), ("dD", sr.grad, sd.grad)):
        e = rel_l2(a, b)
        assert e <= tol, (name, e)


@pytest.mark.parametrize("C,L", [(16, 1 << 20), (64, 1 << 16), (24, 1 << 13)])
def test_long_passes_channel_runs_vs_oracle(C, L):
    """The long 1D passes with channel counts that fill every CTA's run of lines (one
    four-step multiplier per CTA: the store twiddles come from a per-CTA table) and with a
    ragged count (24: runs straddle rows, per-run twiddle factors), op and mixer."""
    from nvsubquadratic_b200.fftconv import causal_fftconv1d_fp32_bhl

    g = torch.Generator().manual_seed(5)
    x = torch.randn(1, C, L, generator=g)
    t = torch.arange(L, dtype=torch.float32)
    k = torch.randn(1, C, L, generator=g) * torch.exp(-(torch.rand(C, 1, generator=g) * 4.5 + 0.5) / L * t) / 32
    sc = torch.randn(C, generator=g)
    dy = torch.randn(1, C, L, generator=g)
    xr, kr, sr = (u.clone().requires_grad_(True) for u in (x, k, sc))
    yr = ofc.fftconv_bhl(xr, kr, sr, causal=True)
    yr.backward(dy)
    xd, kd, sd = (u.cuda().requires_grad_(True) for u in (x, k, sc))
    y = causal_fftconv1d_fp32_bhl(xd, kd, sd)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    for name, a, b in (("y", yr, y), ("dx", xr.grad, xd.grad), ("dk", kr.grad, kd.grad), ("dD", sr.grad, sd.grad)):
        assert rel_l2(a, b) <= 1e-5, (name, rel_l2(a, b))
    _check_mixer(1, C, (L,), (L,), 7, torch.bfloat16, causal=True, g1="silu")


@pytest.mark.parametrize("causal,xs,ks,dt", [
    # 1 MiB spectra per channel at F = 2^17: a 64 MiB budget holds 16 channels -> 16, 16, 8
    (True, (2, 40, 1 << 16), (1, 40, 1 << 16), torch.float32),
    # 128 KiB spectra per channel at F = 128^2: 128 channels per chunk -> 128, 32
    (False, (2, 160, 64, 64), (1, 160, 64, 64), torch.bfloat16),
])
def test_channel_chunked_op_vs_oracle(causal, xs, ks, dt, monkeypatch):
    """hyfft_conv_* with a workspace budget small enough to split the channels into
    several chunks (each chunk reuses the same spectrum buffers)."""
    from nvsubquadratic_b200 import fftconv as b2

    monkeypatch.setenv("HYFFT_WS_BUDGET_MB", "64")
    g = torch.Generator().manual_seed(4)
    x = torch.randn(xs, generator=g).to(dt)
    k = (torch.randn(ks, generator=g) / math.sqrt(math.prod(ks[2:]))).to(dt)
    sc = torch.randn(xs[1], generator=g).to(dt)
    dy = torch.randn(xs, generator=g).to(dt)
    xr, kr, sr = (u.clone().requires_grad_(True) for u in (x, k, sc))
    yr = ofc.fftconv_bhl(xr, kr, sr, causal=causal)
    yr.backward(dy)
    xd, kd, sd = (u.cuda().requires_grad_(True) for u in (x, k, sc))
    fn = b2.causal_fftconv1d_fp32_bhl if causal else b2.fftconv_nd
    y = fn(xd, kd, sd)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    tol = TOL[dt]
    for name, a, b in (("y", yr, y), ("dx", xr.grad, xd.grad), ("dk", kr.grad, kd.grad), ("dD", sr.grad, sd.grad)):
        e = rel_l2(a, b)
        assert e <= tol, (name, e)


@pytest.mark.parametrize("kh_cache", [True, False])
@pytest.mark.parametrize("B,C,S,K,sk,causal", [
    # F = 2^17, one pair: 4 MiB per channel -> chunks of 16 at a 64 MiB budget
    (1, 48, (1 << 16,), (1 << 16,), 7, True),
    # F = 64^3: 8 MiB per channel -> chunks of 8
    (2, 24, (32, 32, 32), (32, 32, 32), 3, False),
])
def test_channel_chunked_mixer_vs_oracle(B, C, S, K, sk, causal, kh_cache, monkeypatch):
    """hyfft_hyena_* on the general engine with several channel chunks: the backward reads
    each chunk's filter spectrum from the saved state, or (HYFFT_NO_KH_CACHE) recomputes it."""
    monkeypatch.setenv("HYFFT_WS_BUDGET_MB", "64")
    if not kh_cache:
        monkeypatch.setenv("HYFFT_NO_KH_CACHE", "1")
    _check_mixer(B, C, S, K, sk, torch.bfloat16, causal=causal, g1="silu", g2="sigmoid")


def test_cfg2_grid_tma_transposes_vs_oracle_and_fallback(monkeypatch):
    """cfg2's grid at 64 channels, where the channels-last <-> channel-major transposes
    around the large-grid kernels run on TMA (64 x 64 tiles): against the oracle, and
    against the shared-memory transpose kernel (pure data movement: y and the activation
    gradients agree bit for bit; the filter gradient is summed by atomics)."""
    from nvsubquadratic_b200.hyena import hyena_fused

    _check_mixer(2, 64, (128, 128), (128, 128), 3, torch.bfloat16)
    qkv, filt, D, sw, dy = _mixer_inputs(2, 64, (128, 128), (128, 128), 3, torch.bfloat16, False)
    outs = []
    for env in (None, "1"):
        if env:
            monkeypatch.setenv("HYFFT_DISABLE_TMA", env)
        x = qkv.cuda().requires_grad_(True)
        pd = [t.cuda().requires_grad_(True) for t in (filt, D, sw)]
        y = hyena_fused(*x.chunk(3, dim=-1), *pd, None)
        y.backward(dy.cuda())
        torch.cuda.synchronize()
        outs.append((y.detach(), x.grad, pd[0].grad))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert rel_l2(outs[1][2], outs[0][2]) <= 1e-6


def test_side_stream_matches_single_stream(monkeypatch):
    """The large-grid mixer with its filter transforms on the library's side stream gives
    the results of the single-stream order: y and the activation gradients bit for bit; the
    filter, D and short-conv weight gradients are sums of float atomics whose order differs
    from run to run, so they agree to 1e-4 (the short-conv weight sums cancel over 32 K
    positions)."""
    from nvsubquadratic_b200.hyena import hyena_fused

    qkv, filt, D, sw, dy = _mixer_inputs(2, 64, (128, 128), (128, 128), 3, torch.bfloat16, False, seed=3)
    outs = []
    for env in (None, "1"):
        if env:
            monkeypatch.setenv("HYFFT_NO_SIDE_STREAM", env)
        x = qkv.cuda().requires_grad_(True)
        pd = [t.cuda().requires_grad_(True) for t in (filt, D, sw)]
        y = hyena_fused(*x.chunk(3, dim=-1), *pd, None)
        y.backward(dy.cuda())
        torch.cuda.synchronize()
        outs.append((y.detach(), x.grad, pd[0].grad, pd[1].grad, pd[2].grad))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    for name, a, b in zip(("dfilt", "dD", "dshort_w"), outs[0][2:], outs[1][2:]):
        assert rel_l2(b, a) <= 1e-4, (name, rel_l2(b, a))
