"""Generate golden vectors by running the nvSubquadratic reference itself (CPU).

Run in the build container, where the read-only reference tree is mounted:

    python tests/golden/make_golden.py --ref /path/to/nvSubquadratic

It writes small ``*.pt`` fixtures next to this file. The fixtures are committed;
the reference is NOT needed at test time (it does not exist on the GPU box).

What is captured (all seeded, all CPU, float32 / bfloat16):

* ``ops.pt``: ``nvsubquadratic/ops/fftconv.py`` — ``causal_fftconv1d_fp32_bhl``,
  ``fftconv{1,2,3}d_fp32_bhl`` and the BLH ``*_w_reshape`` wrappers; forward
  outputs and autograd gradients w.r.t. x, kernel and shortcut for an upstream
  gradient ``dy``. Shapes mirror the reference's own op tests
  (``tests/ops/test_fftconv.py``) plus the edge cases K == L (causal),
  K == 2N-1, K > L+1 (causal aliasing at F = 2L), odd / non-square shapes and
  per-sample ``[B, H, *K]`` kernels.
* ``hyena.pt``: the reference ``Hyena.forward`` (``modules/hyena_nd.py``) driving
  the reference ``CKConvND.forward`` (``modules/ckconv_nd.py``) with a fixed
  kernel tensor in place of the SIREN generator (kernel generation is not on the
  hot path), identity norms, depthwise short conv, SiLU/Sigmoid/identity gates;
  1D causal, 2D and 3D; outputs and gradients for q, k, v, the kernel, the
  shortcut D and the short-conv weight.
* ``cp.pt``: zigzag index vectors (``parallel/a2a_comms.py``) and the outputs of
  ``all_to_all_single_fn`` / ``zigzag_split_across_group_ranks`` run on a real
  2-rank and 4-rank gloo group.

The module layer imports ``omegaconf`` at import time, which is absent here; a
stub providing the two names it touches while importing is installed first.
"""

from __future__ import annotations

import argparse
import os
import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def _install_omegaconf_stub() -> None:
    if "omegaconf" in sys.modules:
        return
    mod = types.ModuleType("omegaconf")

    class DictConfig(dict):
        pass

    class OmegaConf:
        @staticmethod
        def create(obj, flags=None):
            return DictConfig(obj)

        @staticmethod
        def to_container(obj, resolve=False):
            return dict(obj)

    mod.DictConfig = DictConfig
    mod.OmegaConf = OmegaConf
    sys.modules["omegaconf"] = mod


def _grad_case(fn, x, k, sc, dy):
    x = x.clone().requires_grad_(True)
    k = k.clone().requires_grad_(True)
    scg = sc.clone().requires_grad_(True) if sc is not None else None
    y = fn(x, k, scg)
    y.backward(dy)
    out = {"y": y.detach(), "dx": x.grad.detach(), "dk": k.grad.detach()}
    if scg is not None:
        out["dshortcut"] = scg.grad.detach()
    return out


def make_ops(ref) -> dict:
    F = ref
    cases = []
    # (name, fn_name, x_shape, k_shape, dtype, with_shortcut, blh)
    specs = [
        ("causal1d_a", "causal_fftconv1d_fp32_bhl", (2, 8, 64), (1, 8, 15), torch.float32, True, False),
        ("causal1d_b", "causal_fftconv1d_fp32_bhl", (1, 16, 128), (1, 16, 7), torch.float32, False, False),
        ("causal1d_KeqL", "causal_fftconv1d_fp32_bhl", (2, 4, 32), (1, 4, 32), torch.float32, True, False),
        ("causal1d_alias", "causal_fftconv1d_fp32_bhl", (2, 4, 16), (1, 4, 29), torch.float32, True, False),
        ("causal1d_odd", "causal_fftconv1d_fp32_bhl", (3, 5, 37), (1, 5, 37), torch.float32, True, False),
        ("causal1d_bf16", "causal_fftconv1d_fp32_bhl", (2, 8, 64), (1, 8, 64), torch.bfloat16, True, False),
        ("causal1d_persample", "causal_fftconv1d_fp32_bhl", (2, 4, 32), (2, 4, 32), torch.float32, True, False),
        ("causal1d_blh", "causal_fftconv1d_fp32_bhl_w_reshape", (2, 64, 16), (1, 7, 16), torch.float32, True, True),
        ("conv1d_a", "fftconv1d_fp32_bhl", (2, 16, 64), (1, 16, 7), torch.float32, True, False),
        ("conv1d_KeqL", "fftconv1d_fp32_bhl", (1, 8, 256), (1, 8, 256), torch.float32, True, False),
        ("conv1d_K2L", "fftconv1d_fp32_bhl", (2, 4, 32), (1, 4, 63), torch.float32, True, False),
        ("conv1d_even", "fftconv1d_fp32_bhl", (2, 4, 50), (1, 4, 20), torch.float32, False, False),
        ("conv1d_blh", "fftconv1d_fp32_bhl_w_reshape", (2, 64, 16), (1, 7, 16), torch.float32, True, True),
        ("conv2d_a", "fftconv2d_fp32_bhl", (2, 8, 32, 32), (1, 8, 7, 7), torch.float32, True, False),
        ("conv2d_b", "fftconv2d_fp32_bhl", (2, 4, 16, 16), (1, 4, 5, 5), torch.float32, False, False),
        ("conv2d_vit", "fftconv2d_fp32_bhl", (2, 3, 14, 14), (1, 3, 27, 27), torch.float32, True, False),
        ("conv2d_vit14", "fftconv2d_fp32_bhl", (2, 3, 14, 14), (1, 3, 14, 14), torch.float32, True, False),
        ("conv2d_odd", "fftconv2d_fp32_bhl", (1, 2, 12, 10), (1, 2, 23, 19), torch.float32, True, False),
        ("conv2d_rect", "fftconv2d_fp32_bhl", (2, 2, 9, 20), (1, 2, 4, 6), torch.float32, True, False),
        ("conv2d_bf16", "fftconv2d_fp32_bhl", (2, 4, 16, 16), (1, 4, 31, 31), torch.bfloat16, True, False),
        ("conv2d_persample", "fftconv2d_fp32_bhl", (2, 3, 8, 8), (2, 3, 15, 15), torch.float32, True, False),
        ("conv2d_blh", "fftconv2d_fp32_bhl_w_reshape", (2, 32, 32, 8), (1, 7, 7, 8), torch.float32, True, True),
        ("conv3d_a", "fftconv3d_fp32_bhl", (1, 2, 8, 8, 8), (1, 2, 5, 5, 5), torch.float32, True, False),
        ("conv3d_b", "fftconv3d_fp32_bhl", (2, 2, 6, 7, 5), (1, 2, 11, 13, 9), torch.float32, True, False),
        ("conv3d_bf16", "fftconv3d_fp32_bhl", (2, 2, 8, 8, 8), (1, 2, 15, 15, 15), torch.bfloat16, True, False),
        ("conv3d_blh", "fftconv3d_fp32_bhl_w_reshape", (1, 6, 6, 6, 4), (1, 3, 3, 3, 4), torch.float32, True, True),
    ]
    g = torch.Generator().manual_seed(0)
    for name, fn_name, xs, ks, dt, with_sc, blh in specs:
        fn = getattr(F, fn_name)
        x = torch.randn(xs, generator=g).to(dt)
        k = torch.randn(ks, generator=g).to(dt)
        H = xs[-1] if blh else xs[1]
        sc = torch.randn(H, generator=g).to(dt) if with_sc else None
        dy = torch.randn(xs, generator=g).to(dt)
        res = _grad_case(fn, x, k, sc, dy)
        case = {"name": name, "fn": fn_name, "blh": blh, "x": x, "k": k, "shortcut": sc, "dy": dy}
        case.update(res)
        cases.append(case)
    return {"cases": cases}


def make_boundary(circ, mixed) -> dict:
    """Circular (periodic) and mixed-boundary ops of the reference
    (nvsubquadratic/ops/circular_fftconv.py, nvsubquadratic/ops/mixed_fftconv.py)."""
    cases = []
    # (name, fn_name, periodic or None, x_shape, k_shape, dtype, with_shortcut)
    specs = [
        ("circ1d_a", "circular_fftconv1d_fp32_bhl", None, (2, 8, 64), (1, 8, 15), torch.float32, True),
        ("circ1d_even", "circular_fftconv1d_fp32_bhl", None, (2, 4, 32), (1, 4, 8), torch.float32, True),
        ("circ1d_KeqL", "circular_fftconv1d_fp32_bhl", None, (1, 4, 16), (1, 4, 16), torch.float32, False),
        ("circ2d_a", "circular_fftconv2d_fp32_bhl", None, (2, 4, 16, 32), (1, 4, 5, 7), torch.float32, True),
        ("circ2d_full", "circular_fftconv2d_fp32_bhl", None, (2, 3, 32, 32), (1, 3, 32, 32), torch.float32, True),
        ("circ2d_bf16", "circular_fftconv2d_fp32_bhl", None, (2, 4, 16, 16), (1, 4, 16, 16), torch.bfloat16, True),
        ("circ2d_persample", "circular_fftconv2d_fp32_bhl", None, (2, 3, 8, 8), (2, 3, 4, 6), torch.float32, True),
        ("circ3d_a", "circular_fftconv3d_fp32_bhl", None, (1, 2, 8, 16, 8), (1, 2, 3, 6, 8), torch.float32, True),
        ("mixed2d_xy", "mixed_fftconv2d_fp32_bhl", (True, False), (2, 4, 32, 20), (1, 4, 9, 39), torch.float32, True),
        ("mixed2d_yx", "mixed_fftconv2d_fp32_bhl", (False, True), (2, 4, 12, 32), (1, 4, 23, 32), torch.float32, True),
        ("mixed3d", "mixed_fftconv3d_fp32_bhl", (True, True, False), (1, 2, 16, 8, 6), (1, 2, 5, 8, 11),
         torch.float32, True),
        ("mixed3d_bf16", "mixed_fftconv3d_fp32_bhl", (False, True, True), (2, 2, 6, 16, 16), (1, 2, 11, 3, 16),
         torch.bfloat16, True),
    ]
    g = torch.Generator().manual_seed(5)
    for name, fn_name, per, xs, ks, dt, with_sc in specs:
        mod = mixed if fn_name.startswith("mixed") else circ
        base = getattr(mod, fn_name)
        fn = (lambda x, k, sc, _b=base, _p=per: _b(x, k, _p, sc)) if per is not None else base
        x = torch.randn(xs, generator=g).to(dt)
        k = (torch.randn(ks, generator=g) / (torch.tensor(ks[2:]).prod() ** 0.5)).to(dt)
        sc = torch.randn(xs[1], generator=g).to(dt) if with_sc else None
        dy = torch.randn(xs, generator=g).to(dt)
        res = _grad_case(fn, x, k, sc, dy)
        case = {"name": name, "fn": fn_name, "periodic": per, "x": x, "k": k, "shortcut": sc, "dy": dy}
        case.update(res)
        cases.append(case)
    return {"cases": cases}


class _FixedKernel(torch.nn.Module):
    """Stands in for SIRENKernelND: returns a stored channels-last kernel [1, *K, C]."""

    def __init__(self, kernel_blh: torch.Tensor):
        super().__init__()
        self.weight = torch.nn.Parameter(kernel_blh.clone())

    def forward(self, grid_lens, conditioning=None):
        return self.weight, None


def _make_ckconv(CKConvND, fftconv_mod, kernel_blh, shortcut, nd, causal):
    m = CKConvND.__new__(CKConvND)
    torch.nn.Module.__init__(m)
    m.data_dim = nd
    m.hidden_dim = kernel_blh.shape[-1]
    m.is_causal = causal
    m.grid_type = "double"
    m._periodic_per_axis = (False,) * nd
    m._is_tuple_mode = False
    m.kernel = _FixedKernel(kernel_blh)
    m.mask = torch.nn.Identity()
    m.shortcut = torch.nn.Parameter(shortcut.clone())
    if causal:
        m.fftconv_fn = fftconv_mod.causal_fftconv1d_fp32_bhl_w_reshape
        m.fftconv_fn_bhl_input = fftconv_mod.causal_fftconv1d_fp32_bhl
    else:
        name = {1: "fftconv1d", 2: "fftconv2d", 3: "fftconv3d"}[nd]
        m.fftconv_fn = getattr(fftconv_mod, name + "_fp32_bhl_w_reshape")
        m.fftconv_fn_bhl_input = getattr(fftconv_mod, name + "_fp32_bhl")
    return m


def make_hyena(Hyena, CKConvND, fftconv_mod) -> dict:
    specs = [
        # name, nd, B, C, S, short k, causal, gate1, gate2, dtype, short bias
        ("hyena2d_silu_sig_bf16", 2, 2, 4, (6, 6), 3, False, "silu", "sigmoid", torch.bfloat16, False),
        ("hyena2d_id_f32", 2, 2, 4, (7, 5), 3, False, "identity", "identity", torch.float32, False),
        ("hyena2d_sig_f32_bias", 2, 3, 2, (6, 6), 3, False, "sigmoid", "sigmoid", torch.float32, True),
        ("hyena1d_causal_f32", 1, 2, 4, (32,), 7, True, "sigmoid", "sigmoid", torch.float32, False),
        ("hyena1d_causal_bf16", 1, 1, 4, (48,), 7, True, "identity", "silu", torch.bfloat16, False),
        ("hyena3d_silu_f32", 3, 2, 2, (4, 5, 4), 3, False, "silu", "silu", torch.float32, False),
        ("hyena3d_id_bf16", 3, 2, 2, (4, 4, 4), 3, False, "identity", "identity", torch.bfloat16, False),
    ]
    acts = {"identity": torch.nn.Identity, "sigmoid": torch.nn.Sigmoid, "silu": torch.nn.SiLU}
    g = torch.Generator().manual_seed(1)
    out = []
    for name, nd, B, C, S, sk, causal, g1, g2, dt, sbias in specs:
        q = torch.randn((B,) + S + (C,), generator=g).to(dt)
        k = torch.randn((B,) + S + (C,), generator=g).to(dt)
        v = torch.randn((B,) + S + (C,), generator=g).to(dt)
        Kdims = tuple(2 * s - 1 for s in S)  # double grid (ckconv_nd.py:1143-1151)
        kern = (0.3 * torch.randn((1,) + Kdims + (C,), generator=g)).to(dt)
        D = torch.randn(C, generator=g).to(dt)
        ksz = (sk,) * nd
        sw = (torch.rand((3 * C, 1) + ksz, generator=g) * 2 - 1).div(sk ** (nd / 2)).to(dt)
        sb = (0.1 * torch.randn(3 * C, generator=g)).to(dt) if sbias else None
        dy = torch.randn((B,) + S + (C,), generator=g).to(dt)

        conv_cls = {1: torch.nn.Conv1d, 2: torch.nn.Conv2d, 3: torch.nn.Conv3d}[nd]
        if causal:
            short = torch.nn.Conv1d(3 * C, 3 * C, sk, groups=3 * C, padding=0, bias=sbias)
        else:
            short = conv_cls(3 * C, 3 * C, sk, groups=3 * C, padding=sk // 2, bias=sbias)
        short = short.to(dt)
        with torch.no_grad():
            short.weight.copy_(sw)
            if sbias:
                short.bias.copy_(sb)
        if causal:
            # left-pad causal short conv (modules/causal_conv1d.py:113-143)
            class _Causal(torch.nn.Conv1d):
                def forward(self, x):
                    return torch.nn.functional.conv1d(
                        torch.nn.functional.pad(x, (self.kernel_size[0] - 1, 0)),
                        self.weight, self.bias, groups=self.groups)
            c2 = _Causal(3 * C, 3 * C, sk, groups=3 * C, bias=sbias).to(dt)
            with torch.no_grad():
                c2.weight.copy_(sw)
                if sbias:
                    c2.bias.copy_(sb)
            short = c2

        ck = _make_ckconv(CKConvND, fftconv_mod, kern, D, nd, causal).to(dt)
        h = Hyena.__new__(Hyena)
        torch.nn.Module.__init__(h)
        h.global_conv = ck
        h.short_conv = short
        h.gate_nonlinear = acts[g1]()
        h.gate_nonlinear_2 = acts[g2]()
        h.pixelhyena_norm = torch.nn.Identity()
        h.output_norm = torch.nn.Identity()
        h.q_norm = None
        h.k_norm = None

        qq, kk, vv = (t.clone().requires_grad_(True) for t in (q, k, v))
        y = Hyena.forward(h, qq, kk, vv, None)
        y.backward(dy)
        out.append({
            "name": name, "nd": nd, "causal": causal, "gate1": g1, "gate2": g2, "short_k": sk,
            "q": q, "k": k, "v": v, "kernel_blh": kern, "D": D, "short_w": sw, "short_b": sb, "dy": dy,
            "y": y.detach(), "dq": qq.grad.detach(), "dk": kk.grad.detach(), "dv": vv.grad.detach(),
            "dkernel_blh": ck.kernel.weight.grad.detach(), "dD": ck.shortcut.grad.detach(),
            "dshort_w": short.weight.grad.detach(),
            "dshort_b": short.bias.grad.detach() if sbias else None,
        })
    return {"cases": out}


def _cp_worker(rank, world, port, ref_path, out_dir):
    sys.path.insert(0, ref_path)
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from nvsubquadratic.parallel import a2a_comms, utils as putils

    g = torch.Generator().manual_seed(7)
    res = {}
    for nd, shape in ((1, (2, 8, 32)), (2, (1, 8, 16, 3)), (3, (1, 4, 8, 2, 3))):
        full = torch.randn(shape, generator=g)
        local = putils.zigzag_split_across_group_ranks(full, dist.group.WORLD, seq_dim=2)
        s2f = a2a_comms.all_to_all_single_fn(dist.group.WORLD, "split_to_full", local, True)
        f2s = a2a_comms.all_to_all_single_fn(dist.group.WORLD, "full_to_split", s2f, True)
        s2f_nz = a2a_comms.all_to_all_single_fn(dist.group.WORLD, "split_to_full", local, False)
        res[nd] = {"full": full, "local": local, "s2f": s2f, "f2s": f2s, "s2f_nozigzag": s2f_nz}
    torch.save(res, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def make_cp(ref_path: str) -> dict:
    import torch.multiprocessing as mp
    from nvsubquadratic.parallel import a2a_comms

    out = {"zigzag": {}, "inv_zigzag": {}}
    for n in (2, 4, 6, 8, 16):
        out["zigzag"][n] = a2a_comms._get_zigzag_indices(n).tolist()
        out["inv_zigzag"][n] = a2a_comms._get_inverse_zigzag_indices(n).tolist()
    import tempfile

    ctx = mp.get_context("spawn")
    for world, port in ((2, 29611), (4, 29612)):
        with tempfile.TemporaryDirectory() as tmp:
            procs = [ctx.Process(target=_cp_worker, args=(r, world, port, ref_path, tmp)) for r in range(world)]
            for p in procs:
                p.start()
            for p in procs:
                p.join(timeout=180)
                assert p.exitcode == 0, f"cp worker failed with exit code {p.exitcode}"
            out[f"world{world}"] = [torch.load(os.path.join(tmp, f"rank{r}.pt")) for r in range(world)]
    return out


def make_siren(SIRENKernelND, ExponentialModulationND) -> dict:
    """The reference's implicit filter (nvsubquadratic/modules/kernels_nd.py SIRENKernelND, no
    FiLM) and exponential window (modules/masks_nd.py ExponentialModulationND) on seeded
    weights: kernel, masked kernel and the gradients of every SIREN parameter for a random
    upstream gradient of the masked kernel. Cases cover 1D / 2D / 3D grids, with and without
    biases, a grid extended past L_cache, and widths up to 64."""
    cases = []
    # (name, out_dim, data_dim, hidden, num_layers, emb, omega_0, L_cache, use_bias, seq_lens)
    specs = [
        ("siren1d", 16, 1, 32, 3, 16, 10.0, 64, True, (64,)),
        ("siren1d_ext", 8, 1, 16, 2, 8, 5.0, 32, True, (48,)),
        ("siren2d", 24, 2, 32, 3, 32, 10.0, 14, True, (14, 14)),
        ("siren2d_nobias", 12, 2, 64, 2, 32, 30.0, 8, False, (8, 6)),
        ("siren3d", 8, 3, 32, 3, 16, 10.0, 6, True, (6, 5, 4)),
    ]
    for i, (name, C, D, H, NL, E, w0, L, bias, seq) in enumerate(specs):
        torch.manual_seed(100 + i)
        m = SIRENKernelND(out_dim=C, data_dim=D, mlp_hidden_dim=H, num_layers=NL, embedding_dim=E, omega_0=w0,
                          L_cache=L, use_bias=bias)
        if bias:  # non-zero biases, so that they are exercised
            with torch.no_grad():
                for mod in [m.positional_embedding.linear, *m.hidden_linears, m.out_linear]:
                    mod.bias.uniform_(-0.5, 0.5)
        mask = ExponentialModulationND(data_dim=D, num_channels=C)
        k, grid = m(seq)
        km = mask(grid=grid, x=k)
        dk = torch.randn(km.shape, generator=torch.Generator().manual_seed(200 + i))
        km.backward(dk)
        cases.append(dict(
            name=name, cfg=dict(out_dim=C, data_dim=D, mlp_hidden_dim=H, num_layers=NL, embedding_dim=E,
                                omega_0=w0, L_cache=L, use_bias=bias), seq_lens=seq,
            state={kk: v.detach().clone() for kk, v in m.state_dict().items()},
            mask_weight=mask.weight.detach().clone(), kernel=k.detach(), masked=km.detach(), grid=grid.detach(),
            dk=dk, grads={kk: v.grad.detach().clone() for kk, v in m.named_parameters()}))
    return {"cases": cases}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the nvSubquadratic source tree (holds nvsubquadratic/)")
    ap.add_argument("--only", default="", help="comma-separated subset of ops,hyena,cp,boundary,siren to regenerate")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    _install_omegaconf_stub()
    torch.set_num_threads(4)
    from nvsubquadratic.ops import fftconv as ref_fftconv
    from nvsubquadratic.modules.ckconv_nd import CKConvND
    from nvsubquadratic.modules.hyena_nd import Hyena

    from nvsubquadratic.ops import circular_fftconv as ref_circ
    from nvsubquadratic.ops import mixed_fftconv as ref_mixed

    from nvsubquadratic.modules.kernels_nd import SIRENKernelND
    from nvsubquadratic.modules.masks_nd import ExponentialModulationND

    only = set(args.only.split(",")) if args.only else {"ops", "hyena", "cp", "boundary", "siren"}
    if "ops" in only:
        torch.save(make_ops(ref_fftconv), HERE / "ops.pt")
    if "hyena" in only:
        torch.save(make_hyena(Hyena, CKConvND, ref_fftconv), HERE / "hyena.pt")
    if "cp" in only:
        torch.save(make_cp(args.ref), HERE / "cp.pt")
    if "boundary" in only:
        torch.save(make_boundary(ref_circ, ref_mixed), HERE / "boundary.pt")
    if "siren" in only:
        torch.save(make_siren(SIRENKernelND, ExponentialModulationND), HERE / "siren.pt")
    for f in sorted(n + ".pt" for n in only):
        print(f, (HERE / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
