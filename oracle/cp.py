"""CPU oracle: context-parallel redistribution — TEST INFRASTRUCTURE ONLY.

Restates, as single-process index arithmetic over a list of per-rank tensors,

* the zigzag chunk order ``[0, 2P-1, 1, 2P-2, ...]`` and its inverse
  (nvSubquadratic ``nvsubquadratic/parallel/a2a_comms.py:86-122``),
* ``zigzag_split_across_group_ranks`` / ``zigzag_gather_from_group_ranks``
  (``nvsubquadratic/parallel/utils.py:122-206``): rank r holds chunks
  ``r`` and ``2P-1-r`` of ``2P`` equal chunks along the sequence axis,
* ``all_to_all_single_fn`` (``a2a_comms.py:125-285``):
  ``split_to_full`` turns rank-local ``[B, C, L/P, ...]`` (zigzag layout) into
  ``[B, C/P, L, ...]`` (natural order, channel block r on rank r);
  ``full_to_split`` is its inverse.
"""

from __future__ import annotations

import torch


def zigzag_order(n_chunks: int) -> list[int]:
    """a2a_comms.py:86-101: chunk order [0, n-1, 1, n-2, ...]."""
    half = (n_chunks + 1) // 2
    first = list(range(half))
    second = list(range(n_chunks - 1, half - 1, -1))
    out = [0] * n_chunks
    out[0::2] = first
    out[1::2] = second
    return out


def inverse_zigzag_order(n_chunks: int) -> list[int]:
    """a2a_comms.py:104-122 (argsort of the even-n zigzag order)."""
    half = n_chunks // 2
    first = list(range(half))
    second = list(range(n_chunks - 1, half - 1, -1))
    order = [0] * n_chunks
    order[0::2] = first
    order[1::2] = second
    inv = [0] * n_chunks
    for pos, chunk in enumerate(order):
        inv[chunk] = pos
    return inv


def zigzag_split(full: torch.Tensor, P: int, dim: int) -> list[torch.Tensor]:
    """parallel/utils.py:122-160: rank r gets chunks r and 2P-1-r."""
    if P == 1:
        return [full]
    chunks = torch.chunk(full, 2 * P, dim=dim)
    return [torch.cat([chunks[r], chunks[2 * P - 1 - r]], dim=dim).contiguous() for r in range(P)]


def zigzag_gather(parts: list[torch.Tensor], dim: int) -> torch.Tensor:
    """parallel/utils.py:163-206."""
    P = len(parts)
    if P == 1:
        return parts[0]
    seq: list[torch.Tensor | None] = [None] * (2 * P)
    for r, part in enumerate(parts):
        a, b = torch.split(part, part.size(dim) // 2, dim=dim)
        seq[r] = a
        seq[2 * P - 1 - r] = b
    return torch.cat(seq, dim=dim)


def split_to_full(per_rank: list[torch.Tensor], zigzag: bool = True) -> list[torch.Tensor]:
    """a2a_comms.py:171-226 for every rank at once."""
    P = len(per_rank)
    B, C = per_rank[0].shape[:2]
    assert C % P == 0
    d = C // P
    outs = []
    for j in range(P):
        got = torch.cat([x[:, j * d:(j + 1) * d] for x in per_rank], dim=2)
        if zigzag:
            L = got.shape[2]
            n = 2 * P
            if L % n != 0:
                raise ValueError(f"Spatial dimension length {L} is not divisible by num_chunks {n}")
            inv = torch.tensor(inverse_zigzag_order(n))
            rest = list(got.shape[3:])
            got = got.reshape([B, d, n, L // n] + rest).index_select(2, inv).reshape([B, d, L] + rest)
        outs.append(got.contiguous())
    return outs


def full_to_split(per_rank: list[torch.Tensor], zigzag: bool = True) -> list[torch.Tensor]:
    """a2a_comms.py:228-282 for every rank at once."""
    P = len(per_rank)
    prepared = []
    for x in per_rank:
        B, d, L = x.shape[:3]
        rest = list(x.shape[3:])
        if zigzag:
            n = 2 * P
            if L % n != 0:
                raise ValueError(f"Spatial dimension length {L} is not divisible by num_chunks {n}")
            zz = torch.tensor(zigzag_order(n))
            x = x.reshape([B, d, n, L // n] + rest).index_select(2, zz).reshape([B, d, L] + rest)
        prepared.append(torch.chunk(x, P, dim=2))
    return [torch.cat([prepared[r][j] for r in range(P)], dim=1).contiguous() for j in range(P)]
