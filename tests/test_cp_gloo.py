"""Context-parallel redistribution on CPU gloo ranks (world 2 and 4).

Drives the product's collective choreography (``nvsubquadratic_b200.cp``: pack ->
``all_to_all_single`` -> unpack, autograd duals, zigzag helpers) on CPU processes, with
the device gather kernels swapped for a plain-torch restatement of the same
permutations (test-only), and checks the results against the reference's own
``all_to_all_single_fn`` outputs captured on a real gloo group
(``tests/golden/cp.pt``, ``tests/golden/make_golden.py``).
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tests.conftest import ROOT


def cpu_permute(x, op, B, l_rows, rest, G, C, P, zigzag, out):
    """Plain-torch restatement of the four channels-last permutations of hyfft_cp_permute_cl."""
    d = C // P
    h = l_rows // 2
    if op == 0:  # [B, l, *rest, G, C] -> [P, B, l, *rest, G, d]
        out.copy_(torch.stack([x[..., j * d:(j + 1) * d] for j in range(P)], dim=0))
    elif op == 1:  # recv [P, B, l, ...] -> [B, P*l, ...] natural order
        for r in range(P):
            if zigzag:
                out[:, r * h:(r + 1) * h] = x[r][:, :h]
                c2 = 2 * P - 1 - r
                out[:, c2 * h:(c2 + 1) * h] = x[r][:, h:]
            else:
                out[:, r * l_rows:(r + 1) * l_rows] = x[r]
    elif op == 2:  # [B, P*l, ...] -> [P, B, l, ...]
        for j in range(P):
            if zigzag:
                c2 = 2 * P - 1 - j
                out[j] = torch.cat([x[:, j * h:(j + 1) * h], x[:, c2 * h:(c2 + 1) * h]], dim=1)
            else:
                out[j] = x[:, j * l_rows:(j + 1) * l_rows]
    else:  # recv [P, B, l, ..., d] -> [B, l, ..., C]
        for r in range(P):
            out[..., r * d:(r + 1) * d] = x[r]
    return out


def cpu_permute_window(x, op, B, l_rows, rest, G, C, P, c_off, c_cnt, out):
    """Plain-torch restatement of hyfft_cp_permute_cl_window (the full-C side of the
    exchange for channels [j*C/P + c_off, j*C/P + c_off + c_cnt) of every rank block j)."""
    d = C // P
    if op == 0:  # [B, l, *rest, G, C] -> [P, B, l, *rest, G, c_cnt]
        out.copy_(torch.stack([x[..., j * d + c_off:j * d + c_off + c_cnt] for j in range(P)], dim=0))
    elif op == 3:  # [P, B, l, *rest, G, c_cnt] -> those channels of [B, l, *rest, G, C]
        for r in range(P):
            out[..., r * d + c_off:r * d + c_off + c_cnt] = x[r]
    else:
        raise ValueError(op)
    return out


def _worker(rank, world, port, result_dir):
    import sys

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    from nvsubquadratic_b200 import cp

    dist.init_process_group("gloo", rank=rank, world_size=world)
    cp._permute_impl = cpu_permute
    golden = torch.load(os.path.join(ROOT, "tests", "golden", "cp.pt"), weights_only=False)[f"world{world}"]
    group = dist.group.WORLD
    errors = []
    for nd in (1, 2, 3):
        ref = golden[rank][nd]
        local = cp.zigzag_split_across_group_ranks(ref["full"], group, seq_dim=2)
        if not torch.equal(local, ref["local"]):
            errors.append(f"zigzag split nd={nd}")
        s2f = cp.all_to_all_single_fn(group, "split_to_full", local, True)
        if not torch.equal(s2f, ref["s2f"]):
            errors.append(f"split_to_full nd={nd}")
        s2f_nz = cp.all_to_all_single_fn(group, "split_to_full", local, False)
        if not torch.equal(s2f_nz, ref["s2f_nozigzag"]):
            errors.append(f"split_to_full no-zigzag nd={nd}")
        f2s = cp.all_to_all_single_fn(group, "full_to_split", s2f, True)
        if not torch.equal(f2s, ref["f2s"]):
            errors.append(f"full_to_split nd={nd}")
        gathered = cp.zigzag_gather_from_group_ranks(local, group, seq_dim=2)
        if not torch.equal(gathered, ref["full"]):
            errors.append(f"zigzag gather nd={nd}")
        # autograd dual: d/dx <g, A2A(x)> = A2A^T(g)
        x = local.clone().requires_grad_(True)
        y = cp.AllToAllSingleFunction.apply(x, group, "split_to_full", True)
        g = torch.randn_like(y)
        (y * g).sum().backward()
        back = cp.all_to_all_single_fn(group, "full_to_split", g, True)
        if not torch.equal(x.grad, back):
            errors.append(f"autograd dual nd={nd}")
    # channels-last q/k/v path with 3 channel groups: seq->chan->seq round trip
    torch.manual_seed(rank)
    x = torch.randn(2, 8, 3, 3, 4 * world)  # [B, l, rest, G, C]
    y = cp.chan_to_seq(cp.seq_to_chan(x, group), group)
    if not torch.equal(x, y):
        errors.append("channels-last round trip")
    torch.save(errors, os.path.join(result_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_cp_collectives_match_reference(world, tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    for r in range(world):
        errors = torch.load(tmp_path / f"rank{r}.pt")
        assert errors == [], (r, errors)


def test_rank_failure_is_reported_not_hung(tmp_path):
    """A rank that raises before the collective must surface as a failure on the host side
    (process-group timeout), not hang the job (host-side fault injection, gloo, CPU)."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = sorted(p.exitcode for p in procs)
    assert all(c is not None for c in codes), "a rank hung"
    assert codes[-1] != 0, "the injected failure was not reported"


def _failing_worker(rank, world, port):
    import datetime
    import sys

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    from nvsubquadratic_b200 import cp

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    cp._permute_impl = cpu_permute
    if rank == 1:
        raise SystemExit(3)  # this rank dies before joining the collective
    x = torch.randn(1, 4, 8)
    cp.all_to_all_single_fn(dist.group.WORLD, "split_to_full", x, True)  # times out -> raises


def _oracle_local_forward(q, k, v, filt, D, sw, sb, cfg):
    """CPU stand-in for the fused mixer on one channel group (the oracle with autograd)."""
    from oracle.hyena import hyena_forward

    causal, short_k, short_causal, g1, g2 = cfg
    ins = [None if t is None else t.detach().clone().requires_grad_(True) for t in (q, k, v, filt, D, sw, sb)]
    with torch.enable_grad():
        y = hyena_forward(*ins, causal=causal, short_causal=short_causal, gate1=g1, gate2=g2)
    return y.detach(), (ins, y)


def _oracle_local_backward(state, dy, dq, dk, dv):
    ins, y = state
    grads = iter(torch.autograd.grad(y, [t for t in ins if t is not None], dy))
    g = [None if t is None else next(grads) for t in ins]
    dq.copy_(g[0])
    dk.copy_(g[1])
    dv.copy_(g[2])
    dsw = g[5].reshape(g[5].shape[0], -1) if g[5] is not None else None
    return g[3], g[4], dsw, g[6]


CP_MIXER_CASES = [
    # nd, B, C, S, causal, short_k, gate1, gate2
    (1, 2, 8, (32,), True, 7, "identity", "identity"),
    (2, 2, 8, (8, 6), False, 3, "silu", "sigmoid"),
    (1, 1, 8, (16,), False, 3, "sigmoid", "silu"),
]


def _mixer_worker(rank, world, port, result_dir):
    import sys

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    from nvsubquadratic_b200 import cp
    from nvsubquadratic_b200.hyena import ExplicitKernel, HyenaB200
    from oracle.hyena import hyena_forward

    dist.init_process_group("gloo", rank=rank, world_size=world)
    cp._permute_impl = cpu_permute
    cp._permute_window_impl = cpu_permute_window
    cp._local_forward = _oracle_local_forward
    cp._local_backward = _oracle_local_backward
    group = dist.group.WORLD
    out = []
    for nd, B, C, S, causal, sk, g1, g2 in CP_MIXER_CASES:
        gen = torch.Generator().manual_seed(7)
        q, k, v = (torch.randn((B,) + S + (C,), generator=gen, dtype=torch.float64) for _ in range(3))
        K = S if causal else tuple(2 * s - 1 for s in S)
        filt = torch.randn((1, C) + K, generator=gen, dtype=torch.float64) / (torch.tensor(K).prod() ** 0.5)
        dy = torch.randn((B,) + S + (C,), generator=gen, dtype=torch.float64)
        torch.manual_seed(7)  # identical module parameters on every rank
        mod = HyenaB200(C, nd, ExplicitKernel(filt), short_kernel_size=sk, gate1=g1, gate2=g2, causal=causal,
                        dtype=torch.float64)
        qf, kf, vf = (t.clone().requires_grad_(True) for t in (q, k, v))
        yf = hyena_forward(qf, kf, vf, mod.kernel_fn.weight, mod.shortcut, mod.short_weight, mod.short_bias,
                           causal=causal, gate1=g1, gate2=g2)
        yf.backward(dy)
        ref = [yf.detach(), qf.grad, kf.grad, vf.grad, mod.kernel_fn.weight.grad.clone(), mod.shortcut.grad.clone(),
               mod.short_weight.grad.clone()]
        mod.zero_grad()
        ql, kl, vl = (cp.zigzag_split_across_group_ranks(t, group, seq_dim=1).requires_grad_(True)
                      for t in (q, k, v))
        yl = mod(ql, kl, vl, cp_group=group)
        yl.backward(cp.zigzag_split_across_group_ranks(dy, group, seq_dim=1))
        got = [cp.zigzag_gather_from_group_ranks(t, group, seq_dim=1) for t in (yl.detach(), ql.grad, kl.grad, vl.grad)]
        for p in (mod.kernel_fn.weight, mod.shortcut, mod.short_weight):
            gsum = p.grad.clone()
            dist.all_reduce(gsum)  # each rank holds the gradient of its channel block
            got.append(gsum)
        out.append([float((a - b).norm() / a.norm()) for a, b in zip(ref, got)])
    torch.save(out, os.path.join(result_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_cp_mixer_choreography_matches_single_device(world, tmp_path):
    """hyena_context_parallel (zigzag split -> per channel group: seq->chan all-to-all ->
    local mixer -> chan->seq all-to-all, pipelined; and the backward duals) reproduces the
    single-device mixer and its gradients; the local mixer and the permutations are the
    CPU restatements here, the CUDA ones are covered by the GPU tests. With C = 8 every
    rank's block (4 or 2 channels) is exchanged in several groups."""
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_mixer_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    for r in range(world):
        errs = torch.load(tmp_path / f"rank{r}.pt")
        for case, e in zip(CP_MIXER_CASES, errs):
            assert max(e) < 1e-6, (r, case, e)  # the oracle's FFT runs in float32
