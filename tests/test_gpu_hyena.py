"""GPU parity of the fused Hyena mixer (C-ABI hyfft_hyena_forward / _backward).

Compared with the reference Hyena.forward golden vectors and with the CPU oracle
composition on identical seeded inputs: y and the gradients of q, k, v, the
global filter, D and the short-conv weight / bias. rel-L2 <= 1e-5 (float32),
<= 2e-2 (bfloat16).
"""

import pytest
import torch

from oracle.hyena import hyena_forward
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def _fused():
    from nvsubquadratic_b200.hyena import hyena_fused

    return hyena_fused


def _grads_fused(q, k, v, filt, D, sw, sb, dy, **kw):
    ins = [t.cuda().requires_grad_(True) if t is not None else None for t in (q, k, v, filt, D, sw, sb)]
    y = _fused()(*ins, **kw)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    return y, [t.grad if t is not None else None for t in ins]


def _grads_oracle(q, k, v, filt, D, sw, sb, dy, **kw):
    ins = [t.clone().requires_grad_(True) if t is not None else None for t in (q, k, v, filt, D, sw, sb)]
    y = hyena_forward(*ins, **kw)
    y.backward(dy)
    return y, [t.grad if t is not None else None for t in ins]


@pytest.mark.parametrize("idx", range(7))
def test_hyena_vs_reference_golden(golden, idx):
    c = golden["hyena"]["cases"][idx]
    kern = c["kernel_blh"]
    if c["causal"]:
        kern = kern[:, kern.shape[1] // 2:, :]  # ckconv_nd.py:1160-1164
    filt = kern.movedim(-1, 1).contiguous()
    y, grads = _grads_fused(c["q"], c["k"], c["v"], filt, c["D"], c["short_w"], c["short_b"], c["dy"],
                            causal=c["causal"], gate1=c["gate1"], gate2=c["gate2"])
    tol = TOL[c["q"].dtype]
    dq, dk, dv, dfilt, dD, dsw, dsb = grads
    dkern = dfilt.movedim(1, -1)
    ref_dkern = c["dkernel_blh"]
    if c["causal"]:
        ref_dkern = ref_dkern[:, ref_dkern.shape[1] // 2:, :]
    checks = [("y", c["y"], y), ("dq", c["dq"], dq), ("dk", c["dk"], dk), ("dv", c["dv"], dv),
              ("dkernel", ref_dkern, dkern), ("dD", c["dD"], dD), ("dshort_w", c["dshort_w"], dsw)]
    if c["short_b"] is not None:
        checks.append(("dshort_b", c["dshort_b"], dsb))
    for name, ref, got in checks:
        assert rel_l2(ref, got) <= tol, (c["name"], name, rel_l2(ref, got))


CASES = [
    # nd, B, C, S, K, short_k, causal, gate1, gate2, dtype, bias, qkv_views
    (2, 4, 32, (14, 14), (14, 14), 3, False, "silu", "sigmoid", torch.bfloat16, False, True),
    (2, 4, 16, (14, 14), (27, 27), 3, False, "identity", "identity", torch.float32, False, True),
    (2, 2, 8, (32, 32), (32, 32), 3, False, "sigmoid", "sigmoid", torch.float32, True, False),
    (1, 2, 16, (1024,), (1024,), 7, True, "identity", "identity", torch.bfloat16, False, True),
    (1, 1, 8, (8192,), (8192,), 7, True, "sigmoid", "silu", torch.float32, False, False),
    (3, 2, 4, (8, 8, 8), (8, 8, 8), 3, False, "silu", "silu", torch.float32, False, True),
    # 3D 3x3x3 short conv on the plane-marching kernels (16-bit, channels a multiple of 8):
    # a channel tail block, ragged y / z tiles, bias, strided q/k/v views
    (3, 2, 72, (9, 13, 37), (9, 13, 37), 3, False, "silu", "sigmoid", torch.bfloat16, True, True),
    (3, 3, 16, (6, 5, 20), (11, 9, 39), 3, False, "identity", "identity", torch.bfloat16, False, False),
    # 2D 3x3 short conv on the same kernels as one x plane (ragged y / z tiles, channel tail)
    (2, 3, 72, (37, 45), (37, 45), 3, False, "sigmoid", "silu", torch.bfloat16, True, True),
    (2, 3, 8, (12, 10), (23, 19), 0, False, "identity", "sigmoid", torch.float32, False, False),
    # large-grid 2D kernels (F = 192 or 256 per axis)
    (2, 2, 8, (128, 128), (128, 128), 3, False, "silu", "sigmoid", torch.bfloat16, False, True),
    (2, 1, 4, (100, 90), (129, 120), 3, False, "identity", "sigmoid", torch.float32, True, False),
    # 2D grids whose rows march through the plane kernels (last axis >= 96): the transposed
    # stencil with the weight and bias gradients in one kernel, a channel tail block, a
    # ragged first axis, bias, strided q/k/v views
    (2, 2, 72, (45, 100), (45, 100), 3, False, "silu", "identity", torch.bfloat16, True, True),
    (2, 3, 16, (112, 128), (63, 63), 3, False, "sigmoid", "silu", torch.bfloat16, True, False),
]


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}d-{c[3]}-{c[9]}" for c in CASES])
def test_hyena_vs_oracle_seeded(case):
    nd, B, C, S, K, sk, causal, g1, g2, dt, bias, views = case
    g = torch.Generator().manual_seed(0)
    shape = (B,) + S + (C,)
    if views:
        qkv = torch.randn((B,) + S + (3 * C,), generator=g).to(dt)
        q, k, v = qkv.chunk(3, dim=-1)
    else:
        q, k, v = (torch.randn(shape, generator=g).to(dt) for _ in range(3))
    filt = torch.randn((1, C) + K, generator=g) * (1.0 / (torch.tensor(K).prod() ** 0.5))
    D = torch.randn(C, generator=g).to(dt)
    sw = ((torch.rand((3 * C, 1) + (sk,) * nd, generator=g) * 2 - 1) / sk ** (nd / 2)).to(dt) if sk else None
    sb = (0.1 * torch.randn(3 * C, generator=g)).to(dt) if (bias and sk) else None
    dy = torch.randn(shape, generator=g).to(dt)
    kw = dict(causal=causal, gate1=g1, gate2=g2)
    yr, gr = _grads_oracle(q, k, v, filt, D, sw, sb, dy, **kw)
    rest = [t.cuda().requires_grad_(True) if t is not None else None for t in (filt, D, sw, sb)]
    if views:
        # q, k, v as strided views into one [B, *S, 3C] device tensor (QKVSequenceMixer layout)
        qkv_d = qkv.cuda().requires_grad_(True)
        qc, kc, vc = qkv_d.chunk(3, dim=-1)
        assert qc.stride(-2) == 3 * C
        y = _fused()(qc, kc, vc, *rest, **kw)
        y.backward(dy.cuda())
        torch.cuda.synchronize()
        dq, dk, dv = qkv_d.grad.chunk(3, dim=-1)
    else:
        ins = [t.cuda().requires_grad_(True) for t in (q, k, v)]
        y = _fused()(*ins, *rest, **kw)
        y.backward(dy.cuda())
        torch.cuda.synchronize()
        dq, dk, dv = (t.grad for t in ins)
    got = [dq, dk, dv] + [t.grad if t is not None else None for t in rest]
    tol = TOL[dt]
    assert rel_l2(yr, y) <= tol, ("y", rel_l2(yr, y))
    for name, a, b in zip(("dq", "dk", "dv", "dfilt", "dD", "dsw", "dsb"), gr, got):
        if a is None:
            continue
        assert rel_l2(a, b) <= tol, (name, rel_l2(a, b))


FUSED_CASES = [
    # B, C, S, K, short_k, gate1, gate2, dtype, bias
    (32, 64, (14, 14), (14, 14), 3, "identity", "identity", torch.bfloat16, False),
    (17, 32, (14, 14), (28, 28), 0, "sigmoid", "silu", torch.bfloat16, False),
    (20, 16, (16, 16), (31, 31), 3, "silu", "sigmoid", torch.bfloat16, True),
    (6, 8, (8, 8), (15, 15), 3, "identity", "sigmoid", torch.bfloat16, False),
    (3, 16, (14, 14), (27, 27), 3, "silu", "sigmoid", torch.bfloat16, True),
    (5, 8, (16, 16), (31, 31), 0, "sigmoid", "silu", torch.float32, False),
    (2, 24, (8, 8), (15, 15), 3, "silu", "identity", torch.float32, True),
    # 24 = 3 * 8 point transforms (mixed radix) next to their power-of-two fallback
    (4, 16, (14, 14), (14, 14), 3, "silu", "sigmoid", torch.float32, True),
    (3, 8, (16, 16), (16, 16), 0, "identity", "silu", torch.float32, False),
    (5, 8, (14, 14), (13, 13), 3, "sigmoid", "identity", torch.bfloat16, False),
]


@pytest.mark.parametrize("case", FUSED_CASES, ids=[f"B{c[0]}-C{c[1]}-{c[2]}-{c[7]}" for c in FUSED_CASES])
def test_fused_path_matches_general_engine(case, monkeypatch):
    """The single-pass fused kernels and the multi-pass general engine agree."""
    B, C, S, K, sk, g1, g2, dt, bias = case
    g = torch.Generator().manual_seed(5)
    qkv = torch.randn((B,) + S + (3 * C,), generator=g).to(dt)
    filt = torch.randn((1, C) + K, generator=g) / (torch.tensor(K).prod() ** 0.5)
    D = torch.randn(C, generator=g).to(dt)
    sw = ((torch.rand((3 * C, 1, sk, sk), generator=g) * 2 - 1) / sk).to(dt) if sk else None
    sb = (0.1 * torch.randn(3 * C, generator=g)).to(dt) if (bias and sk) else None
    dy = torch.randn((B,) + S + (C,), generator=g).to(dt)
    outs = []
    # tensor-core Toeplitz kernels (bf16 grids <= 16x16, opt-in), default fused FFT kernels,
    # fused kernels on power-of-two transforms only, general multi-pass engine
    envs = ({"HYFFT_USE_TP": "1"}, {}, {"HYFFT_FUSED_POW2": "1"}, {"HYFFT_DISABLE_FUSED": "1"})
    for env in envs:
        for key in ("HYFFT_USE_TP", "HYFFT_FUSED_POW2", "HYFFT_DISABLE_FUSED"):
            if key in env:
                monkeypatch.setenv(key, env[key])
            else:
                monkeypatch.delenv(key, raising=False)
        qkv_d = qkv.cuda().requires_grad_(True)
        rest = [t.cuda().requires_grad_(True) if t is not None else None for t in (filt, D, sw, sb)]
        q, k, v = qkv_d.chunk(3, dim=-1)
        y = _fused()(q, k, v, *rest, gate1=g1, gate2=g2)
        y.backward(dy.cuda())
        torch.cuda.synchronize()
        outs.append([y, qkv_d.grad] + [t.grad if t is not None else None for t in rest])
    tol = 2e-2 if dt == torch.bfloat16 else 1e-5
    for variant in (0, 1, 2):
        for name, a, b in zip(("y", "dqkv", "dfilt", "dD", "dsw", "dsb"), outs[3], outs[variant]):
            if a is None:
                continue
            assert rel_l2(a, b) <= tol, (variant, name, rel_l2(a, b))


class _Kernel(torch.nn.Module):
    """Stand-in kernel generator with CKConvND's call shape: grid_lens -> ([1, *(2n-1), C], grid)."""

    def __init__(self, C, nd, n, gen):
        super().__init__()
        K = tuple(2 * s - 1 for s in n)
        self.w = torch.nn.Parameter(torch.randn((1,) + K + (C,), generator=gen) / (torch.tensor(K).prod() ** 0.5))

    def forward(self, grid_lens, conditioning=None):
        return self.w, None


class _RefLikeMixer(torch.nn.Module):
    """The attributes of a reference Hyena instance the b200 adapter reads."""

    def __init__(self, C, nd, n, short_conv, causal, gate1, gate2, gen):
        super().__init__()
        gc = torch.nn.Module()
        gc.fft_backend, gc.is_causal, gc.mask = "b200", causal, torch.nn.Identity()
        gc.kernel = _Kernel(C, nd, n, gen)
        gc.shortcut = torch.nn.Parameter(torch.randn(C, generator=gen))
        self.global_conv = gc
        self.short_conv = short_conv
        self.gate_nonlinear, self.gate_nonlinear_2 = gate1, gate2
        self.pixelhyena_norm = self.output_norm = torch.nn.Identity()
        self.q_norm = self.k_norm = None


@pytest.mark.parametrize("nd,causal", [(2, False), (1, True)])
def test_fused_adapter_runs_reference_module_parameters(nd, causal):
    """backend.FusedHyena on a reference-shaped Hyena instance == the oracle composition
    with that instance's parameters (kernel generated, causally cropped, channels moved)."""
    from nvsubquadratic_b200.backend import FusedHyena, ckconv_kernel

    g = torch.Generator().manual_seed(3)
    C = 16
    n = (12, 10) if nd == 2 else (256,)
    conv = (torch.nn.Conv2d(3 * C, 3 * C, 3, padding=1, groups=3 * C) if nd == 2 else
            torch.nn.Conv1d(3 * C, 3 * C, 4, padding=0, groups=3 * C))
    if nd == 1:
        conv.__class__ = type("CausalConv1D", (torch.nn.Conv1d,), {})
        conv.is_causal = True
    mixer = _RefLikeMixer(C, nd, n, conv, causal, torch.nn.SiLU(), torch.nn.Sigmoid(), g).cuda()
    shape = (2,) + n + (C,)
    q, k, v, dy = (torch.randn(shape, generator=g) for _ in range(4))
    adapter = FusedHyena(mixer)
    ins = [t.cuda().requires_grad_(True) for t in (q, k, v)]
    y = adapter(*ins)
    y.backward(dy.cuda())
    filt, D = ckconv_kernel(mixer.global_conv, list(n))
    ref_ins = [t.clone().requires_grad_(True) for t in (q, k, v)]
    yr = hyena_forward(*ref_ins, filt.detach().cpu(), D.detach().cpu(), conv.weight.detach().cpu(),
                       conv.bias.detach().cpu(), causal=causal, short_causal=causal, gate1="silu", gate2="sigmoid")
    yr.backward(dy)
    assert rel_l2(yr, y) <= 1e-5
    for a, b in zip(ref_ins, ins):
        assert rel_l2(a.grad, b.grad) <= 1e-5
    assert mixer.global_conv.kernel.w.grad is not None and conv.weight.grad is not None


def test_backend_apply_convolution_matches_oracle():
    from nvsubquadratic_b200 import backend
    from oracle.fftconv import fftconv_bhl

    g = torch.Generator().manual_seed(4)
    x = torch.randn(2, 8, 16, 12, generator=g)
    kern_blh = torch.randn(1, 31, 23, 8, generator=g) / 25
    D = torch.randn(8, generator=g)
    fns = backend.select_fftconv_fns(2, False)
    y_bhl = backend.apply_convolution(fns, x.cuda(), kern_blh.cuda(), D.cuda(), True)
    y_blh = backend.apply_convolution(fns, x.movedim(1, -1).contiguous().cuda(), kern_blh.cuda(), D.cuda(), False)
    ref = fftconv_bhl(x, kern_blh.movedim(-1, 1).contiguous(), D)
    assert rel_l2(ref, y_bhl) <= 1e-5
    assert rel_l2(ref.movedim(1, -1), y_blh) <= 1e-5
