"""CPU oracle: zero-padded linear FFT convolution — TEST INFRASTRUCTURE ONLY.

Restates the algorithm of nvSubquadratic ``nvsubquadratic/ops/fftconv.py`` as a
single N-D routine (the reference spells it out four times, once per rank and
causality):

* cast ``x`` and ``kernel`` to float32            (fftconv.py:568-569, :680-681)
* per-axis FFT length
    causal 1D   F = min(L + K, 2L)                 (fftconv.py:580)
    non-causal  F_d = min(N_d + (K_d + 1)//2, 2N_d) (fftconv.py:627, :699-702, :773-777)
* ``rfftn`` of x and of the kernel at that size, pointwise product,
  ``irfftn``                                        (fftconv.py:582-593, :705-725, :781-805)
* crop: causal keeps ``[0, L)``; non-causal keeps ``[K_d//2, K_d//2 + N_d)``
                                                    (fftconv.py:593, :648-650, :714-725, :791-805)
* round to ``x.dtype``, then add ``shortcut ⊙ x`` in ``x.dtype``
                                                    (fftconv.py:595-599, :727-731, :807-811)

Error behaviour mirrors the reference asserts (``AssertionError`` on a bad
kernel rank, leading kernel dim not in {1, B}, ``K > 2N``, channel mismatch,
shortcut dtype/shape mismatch).

Everything is written with differentiable torch ops on the CPU, so
``torch.autograd`` gives the reference's backward (the reference has no custom
backward on this path: gradients come from autograd through ``torch.fft``).
"""

from __future__ import annotations

import torch

__all__ = [
    "fft_sizes",
    "crop_starts",
    "fftconv_bhl",
    "fftconv_blh",
    "causal_fftconv1d_bhl",
    "fftconv1d_bhl",
    "fftconv2d_bhl",
    "fftconv3d_bhl",
]


def fft_sizes(spatial: tuple[int, ...], kshape: tuple[int, ...], causal: bool) -> tuple[int, ...]:
    """FFT length per axis chosen by the reference (fftconv.py:580, :627, :699-702, :773-777)."""
    if causal:
        assert len(spatial) == 1, "causal convolution is 1D only"
        (L,), (K,) = spatial, kshape
        return (min(L + K, 2 * L),)
    return tuple(min(n + (k + 1) // 2, 2 * n) for n, k in zip(spatial, kshape))


def crop_starts(kshape: tuple[int, ...], causal: bool) -> tuple[int, ...]:
    """First kept index of the inverse FFT per axis (fftconv.py:593, :648, :714-715, :791-793)."""
    if causal:
        return (0,)
    return tuple(k // 2 for k in kshape)


def fftconv_bhl(
    x: torch.Tensor,
    kernel: torch.Tensor,
    shortcut: torch.Tensor | None = None,
    causal: bool = False,
    periodic: tuple[bool, ...] | None = None,
) -> torch.Tensor:
    """Generic N-D (N = x.ndim - 2) FFT conv, BHL layout: zero-padded linear on every axis,
    or per-axis circular where ``periodic[d]`` is set (mixed_fftconv.py:295-342 recipe: FFT
    length N_d, no crop, output rolled by -((K_d - 1) // 2); circular_fftconv.py:374-396).

    x: ``[B, H, *S]`` any float dtype; kernel: ``[1|B, H, *K]``;
    shortcut: ``[H]`` of ``x.dtype`` or None. Returns ``[B, H, *S]`` in ``x.dtype``.
    """
    nd = x.ndim - 2
    assert nd in (1, 2, 3), f"Unsupported input rank {x.ndim}"
    assert kernel.ndim == x.ndim, f"Unexpected kernel shape: {kernel.shape}."
    B, H = x.shape[:2]
    assert kernel.shape[0] in (1, B), (
        f"Leading dimension must be 1 or batch_size ({B}). Got kernel.shape={kernel.shape}."
    )
    spatial = tuple(x.shape[2:])
    kshape = tuple(kernel.shape[2:])
    per = tuple(bool(p) for p in periodic) if periodic is not None else (False,) * nd
    assert len(per) == nd, f"periodic must have length {nd}"
    for d, (n, k) in enumerate(zip(spatial, kshape)):
        if per[d]:
            assert not causal and k <= n, f"K must be <= N on periodic axis {d}: K={k}, N={n}."
        else:
            assert k <= 2 * n, f"Kernel size must be at most 2 * input size. Got {k} for size {n}."
    if nd > 1:
        assert kernel.shape[1] == H, "Input and kernel must have the same number of channels (H)."

    sizes = list(fft_sizes(spatial, kshape, causal))
    starts = list(crop_starts(kshape, causal))
    shifts = [0] * nd
    for d in range(nd):
        if per[d]:
            sizes[d], starts[d], shifts[d] = spatial[d], 0, -((kshape[d] - 1) // 2)
    dims = tuple(range(2, 2 + nd))

    xs = torch.fft.rfftn(x.to(torch.float32), s=sizes, dim=dims)
    ks = torch.fft.rfftn(kernel.to(torch.float32), s=sizes, dim=dims)
    full = torch.fft.irfftn(xs * ks, s=sizes, dim=dims)
    if any(shifts):
        full = torch.roll(full, shifts=tuple(shifts), dims=dims)
    window = tuple(slice(c, c + n) for c, n in zip(starts, spatial))
    y = full[(slice(None), slice(None)) + window].to(x.dtype)

    if shortcut is not None:
        assert shortcut.dtype == x.dtype, f"shortcut.dtype ({shortcut.dtype}) must match x.dtype ({x.dtype})"
        assert tuple(shortcut.shape) == (H,)
        y = y + shortcut.view((1, H) + (1,) * nd) * x
    return y


def fftconv_blh(
    x: torch.Tensor,
    kernel: torch.Tensor,
    shortcut: torch.Tensor | None = None,
    causal: bool = False,
) -> torch.Tensor:
    """Channels-last ``[B, *S, H]`` form (the reference's ``*_blh`` / ``*_w_reshape``, fftconv.py:163-538)."""
    y = fftconv_bhl(x.movedim(-1, 1), kernel.movedim(-1, 1), shortcut, causal)
    return y.movedim(1, -1)


def causal_fftconv1d_bhl(x, kernel, shortcut=None):
    """fftconv.py:546-600."""
    assert x.ndim == 3
    return fftconv_bhl(x, kernel, shortcut, causal=True)


def fftconv1d_bhl(x, kernel, shortcut=None):
    """fftconv.py:603-659."""
    assert x.ndim == 3
    return fftconv_bhl(x, kernel, shortcut, causal=False)


def fftconv2d_bhl(x, kernel, shortcut=None):
    """fftconv.py:662-733."""
    assert x.ndim == 4
    return fftconv_bhl(x, kernel, shortcut, causal=False)


def fftconv3d_bhl(x, kernel, shortcut=None):
    """fftconv.py:736-812."""
    assert x.ndim == 5
    return fftconv_bhl(x, kernel, shortcut, causal=False)
