"""Context parallelism for the Hyena mixer: sequence <-> channel redistribution over NCCL.

Mirrors nvSubquadratic ``nvsubquadratic/parallel/a2a_comms.py`` (``all_to_all_single_fn``,
``AllToAllSingleFunction``, the zigzag chunk order) and ``nvsubquadratic/parallel/utils.py``
(``zigzag_split_across_group_ranks`` / ``zigzag_gather_from_group_ranks``), with the local
permutations done by one gather kernel each side (``libhyfft.so``) instead of
reshape/permute/contiguous/index_select copies, and the collective a single
``all_to_all_single`` on the caller's process group (NCCL over NVLink on B200).

The fused CP mixer (``hyena_context_parallel``) moves q, k, v from the sequence-sharded
layout (rank r holds zigzag chunks r and 2P-1-r of the first spatial axis) to a
channel-sharded layout with the full sequence (one all-to-all for all three, as G = 3
channel groups), runs the single-device fused Hyena kernels on the local channel block
(short conv, gates, FFT long conv and D-skip all need the full sequence per channel), and
moves y back (one all-to-all). Backward is the dual. That is 4 tensors of C channels each
way per pass (the reference moves 3C + 3C + C + C per pass), and it also covers the causal
case that the reference rejects under CP (ckconv_nd.py:1167-1169).
"""

from __future__ import annotations

import ctypes

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


# The single-device mixer run on the local channel block. Swappable so that host-side
# tests can drive the CP choreography on CPU gloo ranks; the product path is the CUDA one.
_local_mixer = _fused_local


def hyena_context_parallel(module, query, key, value, filt, group, zigzag: bool = True):
    """CP forward of ``HyenaB200``: q, k, v ``[B, l, *rest, C]`` hold this rank's zigzag
    sequence chunks; returns y in the same layout."""
    P, r = group.size(), group.rank()
    C = query.shape[-1]
    assert C % P == 0, f"hidden_dim {C} must be divisible by the CP size {P}"
    d = C // P
    qkv = torch.stack([query, key, value], dim=-2)                     # [B, l, *rest, 3, C]
    loc = SeqToChan.apply(qkv, group, zigzag)                          # [B, L, *rest, 3, d]
    q, k, v = loc.unbind(dim=-2)                                       # channel-last views, pos stride 3d
    # the full filter [1, C, *K], or this rank's channel block [1, C/P, *K] already
    filt_r = filt if filt.shape[1] == d and d != C else _channel_block(filt, 1, r, d)
    D_r = _channel_block(module.shortcut, 0, r, d).to(query.dtype)
    sw_r = _channel_block(module.short_weight, 0, r, d, groups=3, C=C)
    sb_r = _channel_block(module.short_bias, 0, r, d, groups=3, C=C)
    y_loc = _local_mixer(q, k, v, filt_r, D_r, sw_r, sb_r, causal=module.causal, short_causal=module.short_causal,
                         gate1=module.gate1, gate2=module.gate2)       # [B, L, *rest, d]
    y = ChanToSeq.apply(y_loc.unsqueeze(-2), group, zigzag)            # [B, l, *rest, 1, C]
    return y.squeeze(-2)
