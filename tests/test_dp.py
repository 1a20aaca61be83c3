"""Batch (data-parallel) sharding with the gradient all-reduce (nvsubquadratic_b200.dp).

* CPU, gloo world 2: ``GradBucket`` packs parameter gradients into one flat buffer and
  one all-reduce sums them; the reduced views equal the sum of every rank's gradients,
  and ``batch_shard`` slices the batch evenly.
* GPU, 2 GPUs (NCCL, one process per GPU): the fused mixer on each rank's half of the
  batch, followed by the bucket all-reduce, gives the full-batch filter, D and short-conv
  gradients and the full-batch activations' gradients, compared with one device running
  the whole batch and with the CPU oracle. Shapes follow the 128x128 high-resolution
  configuration (large-grid 2D kernels) at a reduced channel count.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tests.conftest import ROOT, rel_l2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, result_dir):
    import sys

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist

    from nvsubquadratic_b200.dp import GradBucket, batch_shard

    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(7)
    full = torch.randn(4 * world, 3, generator=g)
    shard = batch_shard(full, rank, world)
    ok = torch.equal(shard, full[4 * rank:4 * (rank + 1)])
    params = [torch.nn.Parameter(torch.zeros(2, 3)), torch.nn.Parameter(torch.zeros(5)),
              torch.nn.Parameter(torch.zeros(1, 4, 2))]
    per_rank = [[torch.randn(p.shape, generator=g) for p in params] for _ in range(world)]
    for p, gr in zip(params, per_rank[rank]):
        p.grad = gr.clone()
    params[1].grad = None if rank == 1 else params[1].grad  # a missing gradient counts as zero
    bucket = GradBucket(params)
    bucket.reduce(dist.group.WORLD)
    for i, (p, got) in enumerate(zip(params, bucket.grads())):
        want = sum(per_rank[r][i] for r in range(world) if not (i == 1 and r == 1))
        ok = ok and got.shape == p.shape and torch.allclose(got, want, atol=1e-6)
    torch.save(bool(ok), os.path.join(result_dir, f"rank{rank}.pt"))
    dist.destroy_process_group()


def test_grad_bucket_allreduce_gloo(tmp_path):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(world):
        assert torch.load(tmp_path / f"rank{r}.pt")


def test_batch_shard_rejects_uneven_split():
    from nvsubquadratic_b200.dp import batch_shard

    with pytest.raises(ValueError):
        batch_shard(torch.zeros(5, 2), 0, 2)


DP_CASE = dict(B=4, C=8, S=(128, 128), K=(128, 128), sk=3, dt=torch.bfloat16)


def _dp_inputs():
    c = DP_CASE
    g = torch.Generator().manual_seed(21)
    qkv = torch.randn((c["B"],) + c["S"] + (3 * c["C"],), generator=g).to(c["dt"])
    filt = torch.randn((1, c["C"]) + c["K"], generator=g) / 128.0
    D = ((torch.rand(c["C"], generator=g) * 2 - 1) / c["C"] ** 0.5).to(c["dt"])
    sw = ((torch.rand((3 * c["C"], 1, c["sk"], c["sk"]), generator=g) * 2 - 1) / c["sk"]).to(c["dt"])
    dy = torch.randn((c["B"],) + c["S"] + (c["C"],), generator=g).to(c["dt"])
    return qkv, filt, D, sw, dy


def _nccl_worker(rank, world, port, result_dir):
    import datetime
    import sys

    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import torch.distributed as dist

    from nvsubquadratic_b200.dp import GradBucket, batch_shard
    from nvsubquadratic_b200.hyena import hyena_fused

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    qkv, filt, D, sw, dy = _dp_inputs()
    x = batch_shard(qkv, rank, world).contiguous().cuda().requires_grad_(True)
    params = [t.cuda().requires_grad_(True) for t in (filt, D, sw)]
    y = hyena_fused(*x.chunk(3, dim=-1), *params, None)
    y.backward(batch_shard(dy, rank, world).contiguous().cuda())
    bucket = GradBucket(params)
    bucket.reduce(dist.group.WORLD)
    out = {"y": y.detach().cpu(), "dqkv": x.grad.cpu(), "grads": [t.cpu() for t in bucket.grads()]}
    torch.save(out, os.path.join(result_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_batch_sharded_grads_match_full_batch(tmp_path):
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    shards = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    # every rank ends with the same (full-batch) parameter gradients
    for a, b in zip(shards[0]["grads"], shards[1]["grads"]):
        assert torch.equal(a, b)
    y = torch.cat([s["y"] for s in shards], dim=0)
    dqkv = torch.cat([s["dqkv"] for s in shards], dim=0)

    from nvsubquadratic_b200.hyena import hyena_fused
    from oracle.hyena import hyena_forward

    qkv, filt, D, sw, dy = _dp_inputs()
    # one device, whole batch
    x1 = qkv.cuda().requires_grad_(True)
    p1 = [t.cuda().requires_grad_(True) for t in (filt, D, sw)]
    y1 = hyena_fused(*x1.chunk(3, dim=-1), *p1, None)
    y1.backward(dy.cuda())
    torch.cuda.synchronize()
    # CPU oracle, whole batch
    q, k, v = (t.clone().requires_grad_(True) for t in qkv.chunk(3, dim=-1))
    pr = [t.clone().requires_grad_(True) for t in (filt, D, sw)]
    yr = hyena_forward(q, k, v, *pr, None)
    yr.backward(dy)
    dqkv_r = torch.cat([q.grad, k.grad, v.grad], dim=-1)
    tol = 2e-2
    # the same kernels on the same images: activations and their gradients agree exactly
    # up to float32 summation order
    assert rel_l2(y1, y) <= 1e-5 and rel_l2(x1.grad, dqkv) <= 1e-5
    for one, sharded, ref in zip(p1, shards[0]["grads"], pr):
        # the filter gradient is float32 on both sides (summation order differs); D and the
        # short-conv weights are bf16 parameters, so each rank's partial gradient is rounded
        # to bf16 before the float32 sum
        same = 1e-5 if one.dtype == torch.float32 else tol
        assert rel_l2(one.grad.float(), sharded) <= same
        assert rel_l2(ref.grad.float(), sharded) <= tol
    assert rel_l2(yr, y) <= tol and rel_l2(dqkv_r, dqkv) <= tol
