"""Implicit filter generation (row f1): the SIREN kernel network and exponential window.

CPU: the oracle (oracle/siren.py) against the reference's own outputs
(tests/golden/siren.pt, made by tests/golden/make_golden.py from
nvsubquadratic/modules/kernels_nd.py SIRENKernelND and masks_nd.py ExponentialModulationND),
the module's parameter names against the reference's state dicts, and the C ABI's argument
checks. GPU: hyfft_siren_forward / _backward through SIRENKernelB200 and ckconv_filter
against the same golden vectors (kernel, masked kernel, every parameter gradient), both
output layouts, the causal half grid, and a larger grid against the oracle.
Tolerances: float32 end to end; rel-L2 <= 1e-5 for the kernels, <= 1e-4 for gradients
(sums over every grid point of products of sines of arguments up to ~2 pi omega_0).
"""

import math

import pytest
import torch

from oracle import siren as osr
from tests.conftest import rel_l2

KTOL, GTOL = 1e-5, 1e-4


def _params_from_state(state, num_layers):
    p = {"pe.weight": state["positional_embedding.linear.weight"], "out.weight": state["out_linear.weight"]}
    if "positional_embedding.linear.bias" in state:
        p["pe.bias"] = state["positional_embedding.linear.bias"]
        p["out.bias"] = state["out_linear.bias"]
    for i in range(num_layers - 1):
        p[f"hidden.{i}.weight"] = state[f"hidden_linears.{i}.weight"]
        if f"hidden_linears.{i}.bias" in state:
            p[f"hidden.{i}.bias"] = state[f"hidden_linears.{i}.bias"]
    return p


@pytest.mark.parametrize("idx", range(5))
def test_oracle_matches_reference_golden(golden, idx):
    c = golden["siren"]["cases"][idx]
    cfg = c["cfg"]
    p = {k: v.clone().requires_grad_(True) for k, v in _params_from_state(c["state"], cfg["num_layers"]).items()}
    k, grid = osr.siren_filter(p, c["seq_lens"], cfg["L_cache"])
    assert torch.equal(grid, c["grid"]), "coordinate grid"
    assert rel_l2(c["kernel"], k) <= 1e-6
    km, _ = osr.siren_filter(p, c["seq_lens"], cfg["L_cache"], c["mask_weight"])
    assert rel_l2(c["masked"], km) <= 1e-6
    km.backward(c["dk"])
    names = {"pe.weight": "positional_embedding.linear.weight", "pe.bias": "positional_embedding.linear.bias",
             "out.weight": "out_linear.weight", "out.bias": "out_linear.bias"}
    for key, t in p.items():
        ref_name = names.get(key) or key.replace("hidden.", "hidden_linears.")
        assert rel_l2(c["grads"][ref_name], t.grad) <= 1e-5, key


def test_module_state_dict_matches_reference_names(golden):
    from nvsubquadratic_b200.siren import SIRENKernelB200

    for c in golden["siren"]["cases"]:
        m = SIRENKernelB200(**c["cfg"])
        assert sorted(m.state_dict().keys()) == sorted(c["state"].keys())
        m.load_state_dict(c["state"])  # shapes agree


def test_init_bounds_follow_the_reference():
    from nvsubquadratic_b200.siren import SIRENKernelB200

    torch.manual_seed(0)
    m = SIRENKernelB200(out_dim=64, data_dim=2, mlp_hidden_dim=32, num_layers=3, embedding_dim=16, omega_0=10.0,
                        L_cache=14, use_bias=True)
    assert m.positional_embedding.linear.weight.abs().max() <= 2 * math.pi * 10.0 / 2
    assert m.hidden_linears[0].weight.abs().max() <= math.sqrt(6 / 16)
    assert m.out_linear.weight.abs().max() <= math.sqrt(6 / 32) / 14
    with pytest.raises(NotImplementedError):
        SIRENKernelB200(8, 1, 16, 2, 8, 1.0, 16, True, film_cfg=object())


def test_abi_argument_checks():
    import ctypes

    from nvsubquadratic_b200 import _lib

    lib = _lib.load()
    d = _lib.SirenDesc()
    d.ndim, d.embedding, d.hidden, d.num_hidden, d.channels, d.layout = 2, 16, 200, 1, 8, _lib.LAYOUT_BLH
    d.n[0] = d.n[1] = 5
    d.n[2] = 1
    p = 16  # never dereferenced: every call fails validation first
    assert lib.hyfft_siren_forward(ctypes.byref(d), p, p, None, p, None, p, None, None, p, p, 1 << 20,
                                   None) == _lib.HYFFT_ERR_UNSUPPORTED  # hidden > 128
    d.hidden, d.ndim = 16, 4
    assert lib.hyfft_siren_forward(ctypes.byref(d), p, p, None, p, None, p, None, None, p, p, 1 << 20,
                                   None) == _lib.HYFFT_ERR_INVALID
    d.ndim = 2
    assert lib.hyfft_siren_forward(ctypes.byref(d), p, p, None, p, None, p, None, None, p, p, 4,
                                   None) == _lib.HYFFT_ERR_WORKSPACE
    sv, ws = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.hyfft_siren_sizes(ctypes.byref(d), ctypes.byref(sv), ctypes.byref(ws)) == _lib.HYFFT_OK
    assert sv.value == ws.value == 4 * 25 * 16


def _gpu_module(c):
    from nvsubquadratic_b200.siren import SIRENKernelB200

    m = SIRENKernelB200(**c["cfg"]).cuda()
    m.load_state_dict(c["state"])
    return m


def _check_grads(c, m):
    for name, t in m.named_parameters():
        e = rel_l2(c["grads"][name], t.grad.cpu())
        assert e <= GTOL, (c["name"], name, e)


@pytest.mark.gpu
@pytest.mark.parametrize("idx", range(5))
def test_kernel_vs_reference_golden(golden, idx):
    c = golden["siren"]["cases"][idx]
    m = _gpu_module(c)
    k, grid = m(c["seq_lens"])
    torch.cuda.synchronize()
    assert torch.equal(grid.cpu(), c["grid"])
    assert rel_l2(c["kernel"], k.cpu()) <= KTOL


@pytest.mark.gpu
@pytest.mark.parametrize("layout", ["blh", "bhl"])
@pytest.mark.parametrize("idx", range(5))
def test_masked_kernel_and_grads_vs_reference_golden(golden, idx, layout):
    from nvsubquadratic_b200.siren import ckconv_filter

    c = golden["siren"]["cases"][idx]
    m = _gpu_module(c)
    km = ckconv_filter(m, c["mask_weight"].cuda(), c["seq_lens"], layout=layout)
    ref = c["masked"]
    dk = c["dk"]
    if layout == "bhl":  # [1, C, *S]
        perm = (0, ref.ndim - 1) + tuple(range(1, ref.ndim - 1))
        ref, dk = ref.permute(perm), dk.permute(perm)
    assert tuple(km.shape) == tuple(ref.shape)
    assert rel_l2(ref, km.detach().cpu()) <= KTOL
    km.backward(dk.contiguous().cuda())
    torch.cuda.synchronize()
    _check_grads(c, m)


@pytest.mark.gpu
def test_causal_half_grid_is_the_reference_crop(golden):
    """CKConvND's causal crop (ckconv_nd.py:1156-1164) taken as the generator's grid."""
    from nvsubquadratic_b200.siren import ckconv_filter

    c = golden["siren"]["cases"][0]  # 1D, 127 points
    m = _gpu_module(c)
    km = ckconv_filter(m, c["mask_weight"].cuda(), c["seq_lens"], causal=True, layout="blh")
    L = c["masked"].shape[1]
    assert rel_l2(c["masked"][:, L // 2:], km.detach().cpu()) <= KTOL


@pytest.mark.gpu
@pytest.mark.parametrize("C,D,H,NL,E,seq", [(768, 2, 64, 3, 64, (14, 14)), (96, 3, 32, 2, 32, (16, 16, 16)),
                                           (40, 1, 128, 2, 128, (2048,))])
def test_larger_grids_vs_oracle(C, D, H, NL, E, seq):
    """cfg1's channel count on its double grid, a 3D grid with several grid-stride rounds, the
    widest supported network on a long 1D grid: forward and gradients against the oracle."""
    from nvsubquadratic_b200.siren import SIRENKernelB200, ckconv_filter

    torch.manual_seed(7)
    m = SIRENKernelB200(out_dim=C, data_dim=D, mlp_hidden_dim=H, num_layers=NL, embedding_dim=E, omega_0=10.0,
                        L_cache=seq[0], use_bias=True)
    with torch.no_grad():
        for mod in [m.positional_embedding.linear, *m.hidden_linears, m.out_linear]:
            mod.bias.uniform_(-0.5, 0.5)
    mw = osr.mask_init(D, C)
    state = {k: v.clone() for k, v in m.state_dict().items()}
    p = {k: v.clone().requires_grad_(True) for k, v in _params_from_state(state, NL).items()}
    kr, _ = osr.siren_filter(p, seq, seq[0], mw)
    dk = torch.randn(kr.shape, generator=torch.Generator().manual_seed(8))
    kr.backward(dk)
    m = m.cuda()
    km = ckconv_filter(m, mw.cuda(), seq, layout="blh")
    assert rel_l2(kr, km.detach().cpu()) <= KTOL
    km.backward(dk.cuda())
    torch.cuda.synchronize()
    names = {"pe.weight": "positional_embedding.linear.weight", "pe.bias": "positional_embedding.linear.bias",
             "out.weight": "out_linear.weight", "out.bias": "out_linear.bias"}
    got = dict(m.named_parameters())
    for key, t in p.items():
        name = names.get(key) or key.replace("hidden.", "hidden_linears.")
        assert rel_l2(t.grad, got[name].grad.cpu()) <= GTOL, (key, rel_l2(t.grad, got[name].grad.cpu()))
