"""The whole sequence-mixer stack on the B200 backend (rows f1 and f2): QKVSequenceMixerB200
(nvsubquadratic/modules/sequence_mixer.py:129-296) around HyenaB200 whose filter comes from
SirenFilter (SIREN network + exponential window, ckconv_nd.py:1133-1164), forward and every
gradient against the CPU oracle composition (linear, oracle/siren.py, oracle/hyena.py,
linear). float32 end to end, rel-L2 <= 1e-4 (the SIREN parameter gradients sum products of
sines over the whole grid; the mixer alone is held to 1e-5 elsewhere)."""

import pytest
import torch

from oracle import siren as osr
from oracle.hyena import hyena_forward
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _oracle_params(m, NL):
    s = {k: v.detach().cpu().clone() for k, v in m.state_dict().items()}
    p = {"pe.weight": s["positional_embedding.linear.weight"], "pe.bias": s["positional_embedding.linear.bias"],
         "out.weight": s["out_linear.weight"], "out.bias": s["out_linear.bias"]}
    for i in range(NL - 1):
        p[f"hidden.{i}.weight"] = s[f"hidden_linears.{i}.weight"]
        p[f"hidden.{i}.bias"] = s[f"hidden_linears.{i}.bias"]
    return {k: v.requires_grad_(True) for k, v in p.items()}


@pytest.mark.parametrize("S,causal", [((8, 8), False), ((256,), True), ((6, 4, 4), False)])
def test_qkv_mixer_with_siren_filter_vs_oracle(S, causal):
    from nvsubquadratic_b200.hyena import HyenaB200
    from nvsubquadratic_b200.sequence_mixer import QKVSequenceMixerB200
    from nvsubquadratic_b200.siren import SIRENKernelB200, SirenFilter

    torch.manual_seed(11)
    B, C, nd, NL = 2, 16, len(S), 3
    siren = SIRENKernelB200(out_dim=C, data_dim=nd, mlp_hidden_dim=32, num_layers=NL, embedding_dim=16,
                            omega_0=10.0, L_cache=S[0], use_bias=True)
    with torch.no_grad():
        for mod in [siren.positional_embedding.linear, *siren.hidden_linears, siren.out_linear]:
            mod.bias.uniform_(-0.5, 0.5)
        siren.out_linear.weight.mul_(8.0)  # a filter of O(1) energy, so that the long conv matters
    mixer = HyenaB200(C, nd, SirenFilter(siren, causal=causal), short_kernel_size=3, gate1="silu", causal=causal)
    m = QKVSequenceMixerB200(C, mixer, qkv_bias=True, out_proj_bias=True)
    x = torch.randn((B,) + S + (C,))
    dy = torch.randn((B,) + S + (C,))
    # oracle on the CPU
    P = _oracle_params(siren, NL)
    Wi, bi, Wo, bo = (t.detach().clone().requires_grad_(True) for t in
                      (m.qkv_proj.weight, m.qkv_proj.bias, m.out_proj.weight, m.out_proj.bias))
    D = mixer.shortcut.detach().clone().requires_grad_(True)
    sw = mixer.short_weight.detach().clone().requires_grad_(True)
    xr = x.clone().requires_grad_(True)
    grid_lens = S
    filt, _ = osr.siren_filter(P, grid_lens, S[0], osr.mask_init(nd, C))
    if causal:
        filt = filt[:, filt.shape[1] // 2:]
    filt = filt.movedim(-1, 1)  # [1, C, *K]
    qkv = torch.nn.functional.linear(xr, Wi, bi)
    q, k, v = qkv.chunk(3, dim=-1)
    h = hyena_forward(q, k, v, filt, D, sw, None, causal=causal, gate1="silu")
    yr = torch.nn.functional.linear(h, Wo, bo)
    yr.backward(dy)
    # B200 stack
    m = m.cuda()
    xd = x.cuda().requires_grad_(True)
    y = m(xd)
    y.backward(dy.cuda())
    torch.cuda.synchronize()
    assert rel_l2(yr, y.detach().cpu()) <= TOL
    assert rel_l2(xr.grad, xd.grad.cpu()) <= TOL
    got = dict(m.named_parameters())
    for name, ref in (("qkv_proj.weight", Wi), ("qkv_proj.bias", bi), ("out_proj.weight", Wo),
                      ("out_proj.bias", bo), ("mixer.shortcut", D), ("mixer.short_weight", sw)):
        assert rel_l2(ref.grad, got[name].grad.cpu()) <= TOL, name
    names = {"pe.weight": "positional_embedding.linear.weight", "pe.bias": "positional_embedding.linear.bias",
             "out.weight": "out_linear.weight", "out.bias": "out_linear.bias"}
    for key, t in P.items():
        name = "mixer.kernel_fn.kernel." + (names.get(key) or key.replace("hidden.", "hidden_linears."))
        assert rel_l2(t.grad, got[name].grad.cpu()) <= TOL, (name, rel_l2(t.grad, got[name].grad.cpu()))
