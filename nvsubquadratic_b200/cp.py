"""Context parallelism for the Hyena mixer: sequence <-> channel redistribution over NCCL.

Mirrors nvSubquadratic ``nvsubquadratic/parallel/a2a_comms.py`` (``all_to_all_single_fn``,
``AllToAllSingleFunction``, the zigzag chunk order) and ``nvsubquadratic/parallel/utils.py``
(``zigzag_split_across_group_ranks`` / ``zigzag_gather_from_group_ranks``), with the local
permutations done by one gather kernel each side (``libhyfft.so``) instead of
reshape/permute/contiguous/index_select copies, and the collective a single
``all_to_all_single`` on the caller's process group (NCCL over NVLink on B200).

The fused CP mixer (``hyena_context_parallel``) moves q, k, v from the sequence-sharded
layout (rank r holds zigzag chunks r and 2P-1-r of the first spatial axis) to a
channel-sharded layout with the full sequence, runs the single-device fused Hyena kernels
on the local channel block (short conv, gates, FFT long conv and D-skip all need the full
sequence per channel), and moves y back. Backward is the dual. That is 4 tensors of C
channels each way per pass (the reference moves 3C + 3C + C + C per pass), and it also
covers the causal case that the reference rejects under CP (ckconv_nd.py:1167-1169).

The exchange is pipelined over channel groups: every rank's channel block is cut into
groups, each group's seq->chan all-to-all is issued asynchronously on NCCL's stream as
soon as it is packed, the local mixer runs on group j while the all-to-alls of the next
groups (and the chan->seq all-to-all of the previous one) are in flight, and the results
are unpacked in place as their exchanges complete. q, k, v that are the three channel
chunks of one [B, l, 3C] projection are packed straight from it (no stacking copy).
"""

from __future__ import annotations

import ctypes
import math
import os

import torch
import torch.distributed as dist

from . import _lib

__all__ = [
    "all_to_all_single_fn",
    "AllToAllSingleFunction",
    "zigzag_split_across_group_ranks",
    "zigzag_gather_from_group_ranks",
    "SeqToChan",
    "ChanToSeq",
    "hyena_context_parallel",
]

PACK_SEQ_TO_CHAN, UNPACK_SEQ_TO_CHAN, PACK_CHAN_TO_SEQ, UNPACK_CHAN_TO_SEQ = 0, 1, 2, 3


# ---------------------------------------------------------------- permutation kernels
def _permute_cuda(x: torch.Tensor, op: int, B: int, l_rows: int, rest: int, G: int, C: int, P: int,
                  zigzag: bool, out: torch.Tensor) -> torch.Tensor:
    dev = _lib.require_cuda(x, out)
    rc = _lib.load().hyfft_cp_permute_cl(x.data_ptr(), out.data_ptr(), op, B, l_rows, rest, G, C, P,
                                         1 if zigzag else 0, x.element_size(), _lib.stream_ptr(dev))
    _lib.check(rc, "hyfft_cp_permute_cl")
    return out


# Swappable so that host-side tests can drive the collective choreography on CPU gloo
# ranks with reference permutations; the product path is the CUDA kernel.
_permute_impl = _permute_cuda


def _permute_window_cuda(x: torch.Tensor, op: int, B: int, l_rows: int, rest: int, G: int, C: int, P: int,
                         c_off: int, c_cnt: int, out: torch.Tensor) -> torch.Tensor:
    dev = _lib.require_cuda(x, out)
    rc = _lib.load().hyfft_cp_permute_cl_window(x.data_ptr(), out.data_ptr(), op, B, l_rows, rest, G, C, P, c_off,
                                                c_cnt, x.element_size(), _lib.stream_ptr(dev))
    _lib.check(rc, "hyfft_cp_permute_cl_window")
    return out


_permute_window_impl = _permute_window_cuda


def _collective(send: torch.Tensor, group) -> torch.Tensor:
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv


def seq_to_chan(x: torch.Tensor, group, zigzag: bool = True) -> torch.Tensor:
    """[B, l, *rest, G, C] (this rank's zigzag sequence chunks) -> [B, P*l, *rest, G, C/P]
    (full sequence in natural order, channel block ``rank``)."""
    P = group.size()
    B, l = x.shape[0], x.shape[1]
    G, C = x.shape[-2], x.shape[-1]
    rest = 1
    for s in x.shape[2:-2]:
        rest *= s
    assert C % P == 0, f"channels {C} not divisible by the CP size {P}"
    if zigzag and l % 2 != 0:
        raise ValueError(f"Spatial dimension length {l * P} is not divisible by num_chunks {2 * P}")
    d = C // P
    x = x.contiguous()
    send = torch.empty((P,) + tuple(x.shape[:-1]) + (d,), dtype=x.dtype, device=x.device)
    _permute_impl(x, PACK_SEQ_TO_CHAN, B, l, rest, G, C, P, zigzag, send)
    recv = _collective(send, group)
    out = torch.empty((B, P * l) + tuple(x.shape[2:-1]) + (d,), dtype=x.dtype, device=x.device)
    return _permute_impl(recv, UNPACK_SEQ_TO_CHAN, B, l, rest, G, C, P, zigzag, out)


def chan_to_seq(y: torch.Tensor, group, zigzag: bool = True) -> torch.Tensor:
    """[B, L, *rest, G, d] (full sequence, channel block ``rank``) -> [B, L/P, *rest, G, P*d]."""
    P = group.size()
    B, L = y.shape[0], y.shape[1]
    G, d = y.shape[-2], y.shape[-1]
    rest = 1
    for s in y.shape[2:-2]:
        rest *= s
    assert L % P == 0
    l = L // P
    if zigzag and l % 2 != 0:
        raise ValueError(f"Spatial dimension length {L} is not divisible by num_chunks {2 * P}")
    C = d * P
    y = y.contiguous()
    send = torch.empty((P, B, l) + tuple(y.shape[2:]), dtype=y.dtype, device=y.device)
    _permute_impl(y, PACK_CHAN_TO_SEQ, B, l, rest, G, C, P, zigzag, send)
    recv = _collective(send, group)
    out = torch.empty((B, l) + tuple(y.shape[2:-1]) + (C,), dtype=y.dtype, device=y.device)
    return _permute_impl(recv, UNPACK_CHAN_TO_SEQ, B, l, rest, G, C, P, zigzag, out)


class SeqToChan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, zigzag):
        ctx.group, ctx.zigzag = group, zigzag
        return seq_to_chan(x.detach(), group, zigzag)

    @staticmethod
    def backward(ctx, g):
        return chan_to_seq(g, ctx.group, ctx.zigzag), None, None


class ChanToSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, group, zigzag):
        ctx.group, ctx.zigzag = group, zigzag
        return chan_to_seq(y.detach(), group, zigzag)

    @staticmethod
    def backward(ctx, g):
        return seq_to_chan(g, ctx.group, ctx.zigzag), None, None


# ---------------------------------------------------------------- reference-shaped API (BHL)
def all_to_all_single_fn(group, type: str, input: torch.Tensor, with_zigzag_splitting: bool = True) -> torch.Tensor:
    """a2a_comms.py:125-285: ``split_to_full`` [B, C, l, *rest] -> [B, C/P, P*l, *rest];
    ``full_to_split`` the inverse. 1D/2D/3D (input rank 3..5)."""
    if input.ndim not in (3, 4, 5):
        raise ValueError(
            f"Unsupported input tensor dimension: {input.ndim}. Expected 3D (1D), 4D (2D), or 5D (3D) tensors.")
    # channels-last view of the BHL tensor: [B, seq, *rest, 1, C]
    x = input.movedim(1, -1).unsqueeze(-2)
    if type == "split_to_full":
        out = seq_to_chan(x, group, with_zigzag_splitting)
    elif type == "full_to_split":
        out = chan_to_seq(x, group, with_zigzag_splitting)
    else:
        raise ValueError(f"Unknown type {type}")
    return out.squeeze(-2).movedim(-1, 1).contiguous()


class AllToAllSingleFunction(torch.autograd.Function):
    """a2a_comms.py:288-380: differentiable redistribution; backward is the dual direction."""

    @staticmethod
    def forward(ctx, input_tensor, group, type, with_zigzag_splitting):
        ctx.group, ctx.type, ctx.zz = group, type, with_zigzag_splitting
        return all_to_all_single_fn(group, type, input_tensor.detach(), with_zigzag_splitting)

    @staticmethod
    def backward(ctx, grad_output):
        other = "full_to_split" if ctx.type == "split_to_full" else "split_to_full"
        return all_to_all_single_fn(ctx.group, other, grad_output, ctx.zz), None, None, None


def zigzag_split_across_group_ranks(data: torch.Tensor, group, seq_dim: int = 0) -> torch.Tensor:
    """parallel/utils.py:122-160: rank r keeps chunks r and 2P-1-r of 2P along ``seq_dim``."""
    P = dist.get_world_size(group)
    if P == 1:
        return data
    r = dist.get_rank(group)
    chunks = torch.chunk(data, 2 * P, dim=seq_dim)
    return torch.cat([chunks[r], chunks[2 * P - 1 - r]], dim=seq_dim).contiguous()


def zigzag_gather_from_group_ranks(data: torch.Tensor, group, seq_dim: int = 0) -> torch.Tensor:
    """parallel/utils.py:163-206 (autograd-aware all-gather, then reorder the chunks)."""
    P = dist.get_world_size(group)
    if P == 1:
        return data
    from torch.distributed.nn.functional import all_gather

    parts = all_gather(data.contiguous(), group=group)
    seq = [None] * (2 * P)
    for r, part in enumerate(parts):
        a, b = torch.split(part, part.size(seq_dim) // 2, dim=seq_dim)
        seq[r], seq[2 * P - 1 - r] = a, b
    return torch.cat(seq, dim=seq_dim)


# ---------------------------------------------------------------- fused CP mixer
def _channel_block(t: torch.Tensor | None, dim: int, r: int, d: int, groups: int = 1, C: int = 0):
    if t is None:
        return None
    if groups == 1:
        return t.narrow(dim, r * d, d)
    return torch.cat([t.narrow(dim, g * C + r * d, d) for g in range(groups)], dim=dim)


def _fused_local(*args, **kwargs):
    from .hyena import hyena_fused

    return hyena_fused(*args, **kwargs)


def _local_forward_cuda(q, k, v, filt, D, sw, sb, cfg):
    """The single-device fused mixer on one channel group: (y, state for the backward)."""
    from .hyena import _params32, forward_call

    filt32, D32, sw32, sb32 = _params32(filt, D, sw, sb, q.shape[-1])
    y, st = forward_call(q, k, v, filt32, D32, sw32, sb32, cfg)
    return y, (q, k, v, filt32, D32, sw32, sb32, st)


def _local_backward_cuda(state, dy, dq, dk, dv):
    """Gradients of one channel group: dq, dk, dv written in place (the chunks of one
    [B, L, *rest, 3, dg] buffer); returns float32 dfilt, dD, dshort_w [3dg, taps], dshort_b."""
    from .hyena import backward_call

    q, k, v, filt32, D32, sw32, sb32, st = state
    return backward_call(q, k, v, filt32, D32, sw32, sb32, st, dy, dq, dk, dv)


# The single-device mixer run on each channel group. Swappable so that host-side tests can
# drive the CP choreography on CPU gloo ranks; the product path is the CUDA one.
_local_forward = _local_forward_cuda
_local_backward = _local_backward_cuda


def cp_channel_groups(d: int) -> int:
    """Channel groups the local block of ``d`` channels is exchanged in: the largest divisor
    of d not above HYFFT_CP_GROUPS (default 4), so that each group's all-to-all overlaps
    the mixer on another group."""
    want = int(os.environ.get("HYFFT_CP_GROUPS", "4"))
    g = max(1, min(want, d))
    while d % g:
        g -= 1
    return g


def _group_params(filt_r, D_r, sw, sb, r, d, C, j, dg):
    """Channel group j (dg channels) of rank r's block: filter, D and the q/k/v rows of the
    short-conv weight and bias."""
    sl = slice(j * dg, (j + 1) * dg)
    rows = lambda t: None if t is None else torch.cat(  # noqa: E731
        [t[g * C + r * d + j * dg:g * C + r * d + (j + 1) * dg] for g in range(3)], dim=0)
    return filt_r[:, sl], D_r[sl], rows(sw), rows(sb)


class _ContextParallelMixer(torch.autograd.Function):
    """Pipelined CP Hyena: input x5 [B, l, *rest, 3, C] (q, k, v as 3 channel groups of this
    rank's zigzag sequence chunks); output y [B, l, *rest, C]."""

    @staticmethod
    def forward(ctx, x5, filt, D, sw, sb, meta):
        group, zigzag, cfg = meta
        P, r = group.size(), group.rank()
        B, l, C = x5.shape[0], x5.shape[1], x5.shape[-1]
        rest_shape = tuple(x5.shape[2:-2])
        rest = math.prod(rest_shape)
        d = C // P
        NG = cp_channel_groups(d)
        dg = d // NG
        L = P * l
        x5 = x5.contiguous()
        full_filt = filt.shape[1] == C and d != C
        filt_r = filt[:, r * d:(r + 1) * d] if full_filt else filt
        D_r = D[r * d:(r + 1) * d].to(x5.dtype)
        # every group's seq -> chan exchange is packed and put in flight first
        works, recvs, keep = [], [], []
        for j in range(NG):
            send = torch.empty((P, B, l) + rest_shape + (3, dg), dtype=x5.dtype, device=x5.device)
            _permute_window_impl(x5, PACK_SEQ_TO_CHAN, B, l, rest, 3, C, P, j * dg, dg, send)
            recv = torch.empty_like(send)
            works.append(dist.all_to_all_single(recv, send, group=group, async_op=True))
            recvs.append(recv)
            keep.append(send)
        y = torch.empty((B, l) + rest_shape + (C,), dtype=x5.dtype, device=x5.device)
        states, back = [], []
        for j in range(NG):
            works[j].wait()
            loc = torch.empty((B, L) + rest_shape + (3, dg), dtype=x5.dtype, device=x5.device)
            _permute_impl(recvs[j], UNPACK_SEQ_TO_CHAN, B, l, rest, 3, dg * P, P, zigzag, loc)
            q, k, v = loc.unbind(dim=-2)
            f_j, D_j, sw_j, sb_j = _group_params(filt_r, D_r, sw, sb, r, d, C, j, dg)
            y_loc, st = _local_forward(q, k, v, f_j, D_j, sw_j, sb_j, cfg)
            states.append(st)
            send = torch.empty((P, B, l) + rest_shape + (1, dg), dtype=x5.dtype, device=x5.device)
            _permute_impl(y_loc.unsqueeze(-2), PACK_CHAN_TO_SEQ, B, l, rest, 1, dg * P, P, zigzag, send)
            recv = torch.empty_like(send)
            back.append((dist.all_to_all_single(recv, send, group=group, async_op=True), recv))
            keep.append(send)
        y5 = y.unsqueeze(-2)
        for j, (w, recv) in enumerate(back):
            w.wait()
            _permute_window_impl(recv, UNPACK_CHAN_TO_SEQ, B, l, rest, 1, C, P, j * dg, dg, y5)
        ctx.meta = (group, zigzag, P, r, B, l, C, rest_shape, rest, d, NG, dg, full_filt)
        ctx.states = states
        ctx.shapes = (filt.shape, filt.dtype, D.shape, D.dtype, x5.dtype,
                      None if sw is None else (sw.shape, sw.dtype), None if sb is None else (sb.shape, sb.dtype))
        return y

    @staticmethod
    def backward(ctx, dy):
        group, zigzag, P, r, B, l, C, rest_shape, rest, d, NG, dg, full_filt = ctx.meta
        (fshape, fdt, Dshape, Ddt, xdt, swinfo, sbinfo) = ctx.shapes
        dev = dy.device
        L = P * l
        dy5 = dy.to(xdt).contiguous().unsqueeze(-2)  # [B, l, *rest, 1, C]
        works, recvs, keep = [], [], []
        for j in range(NG):
            send = torch.empty((P, B, l) + rest_shape + (1, dg), dtype=xdt, device=dev)
            _permute_window_impl(dy5, PACK_SEQ_TO_CHAN, B, l, rest, 1, C, P, j * dg, dg, send)
            recv = torch.empty_like(send)
            works.append(dist.all_to_all_single(recv, send, group=group, async_op=True))
            recvs.append(recv)
            keep.append(send)
        dx5 = torch.empty((B, l) + rest_shape + (3, C), dtype=xdt, device=dev)
        dfilt_r = torch.empty((fshape[0], d) + tuple(fshape[2:]), dtype=torch.float32, device=dev)
        dD_r = torch.empty(d, dtype=torch.float32, device=dev)
        dsw = torch.zeros((3 * C, math.prod(swinfo[0][2:])), dtype=torch.float32, device=dev) if swinfo else None
        dsb = torch.zeros(3 * C, dtype=torch.float32, device=dev) if sbinfo else None
        back = []
        for j in range(NG):
            works[j].wait()
            dyl = torch.empty((B, L) + rest_shape + (1, dg), dtype=xdt, device=dev)
            _permute_impl(recvs[j], UNPACK_SEQ_TO_CHAN, B, l, rest, 1, dg * P, P, zigzag, dyl)
            dqkv = torch.empty((B, L) + rest_shape + (3, dg), dtype=xdt, device=dev)
            dq, dk, dv = dqkv.unbind(dim=-2)
            df, dD_j, dsw_j, dsb_j = _local_backward(ctx.states[j], dyl.squeeze(-2), dq, dk, dv)
            ctx.states[j] = None  # release the group's saved state as soon as it is used
            dfilt_r[:, j * dg:(j + 1) * dg] = df
            dD_r[j * dg:(j + 1) * dg] = dD_j
            for g in range(3):
                c0 = g * C + r * d + j * dg
                if dsw is not None:
                    dsw[c0:c0 + dg] = dsw_j[g * dg:(g + 1) * dg]
                if dsb is not None:
                    dsb[c0:c0 + dg] = dsb_j[g * dg:(g + 1) * dg]
            send = torch.empty((P, B, l) + rest_shape + (3, dg), dtype=xdt, device=dev)
            _permute_impl(dqkv, PACK_CHAN_TO_SEQ, B, l, rest, 3, dg * P, P, zigzag, send)
            recv = torch.empty_like(send)
            back.append((dist.all_to_all_single(recv, send, group=group, async_op=True), recv))
            keep.append(send)
        for j, (w, recv) in enumerate(back):
            w.wait()
            _permute_window_impl(recv, UNPACK_CHAN_TO_SEQ, B, l, rest, 3, C, P, j * dg, dg, dx5)
        if full_filt:
            dfilt = torch.zeros(fshape, dtype=fdt, device=dev)
            dfilt[:, r * d:(r + 1) * d] = dfilt_r
        else:
            dfilt = dfilt_r.to(fdt)
        # D entered the mixer rounded to the activation dtype; its gradient is rounded the same way
        dD = torch.zeros(Dshape, dtype=Ddt, device=dev)
        dD[r * d:(r + 1) * d] = dD_r.to(xdt).to(Ddt)
        dsw = dsw.reshape(swinfo[0]).to(swinfo[1]) if dsw is not None else None
        dsb = dsb.to(sbinfo[1]) if dsb is not None else None
        return dx5, dfilt, dD, dsw, dsb, None


def hyena_context_parallel(module, query, key, value, filt, group, zigzag: bool = True):
    """CP forward of ``HyenaB200``: q, k, v ``[B, l, *rest, C]`` hold this rank's zigzag
    sequence chunks; returns y in the same layout. ``filt`` is the full ``[1, C, *K]``
    filter or this rank's channel block ``[1, C/P, *K]``."""
    from .hyena import _packed_base

    P = group.size()
    C = query.shape[-1]
    assert C % P == 0, f"hidden_dim {C} must be divisible by the CP size {P}"
    assert query.shape == key.shape == value.shape, "query, key and value must have the same shape"
    base = _packed_base(query, key, value) if torch.is_grad_enabled() else None
    if base is not None:  # the [B, l, *rest, 3C] projection itself, viewed as 3 channel groups
        x5 = base.view(tuple(query.shape[:-1]) + (3, C))
    else:
        x5 = torch.stack([query, key, value], dim=-2)
    short_k = tuple(module.short_weight.shape[2:]) if module.short_weight is not None else ()
    per = getattr(module, "periodic", None)
    if per is not None and any(per):
        raise NotImplementedError("context parallelism with periodic (circular) axes is not supported")
    cfg = (bool(module.causal), short_k, bool(module.short_causal), module.gate1, module.gate2)
    return _ContextParallelMixer.apply(x5, filt, module.shortcut, module.short_weight, module.short_bias,
                                       (group, zigzag, cfg))
