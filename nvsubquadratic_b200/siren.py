"""Implicit filter generation on the B200 backend: the SIREN kernel network and its
exponential window, forward and backward in ``libhyfft.so`` (``hyfft_siren_forward`` /
``hyfft_siren_backward``), with no CPU fallback.

``SIRENKernelB200`` mirrors nvSubquadratic ``SIRENKernelND``
(``nvsubquadratic/modules/kernels_nd.py:876-1199``; positional embedding ``:647-874``): the
same constructor arguments, initialisation and parameter names (``positional_embedding.linear``,
``hidden_linears.{i}``, ``out_linear``), so a reference state dict loads unchanged, and
``forward(seq_lens) -> (kernel [1, *S, C], grid [1, *S, D])`` over the reference's grid
(``2 * seq_len - 1`` points per axis, sliced from ``linspace(-1, 1, 2 * L_cache - 1)``).
FiLM conditioning is not covered (``NotImplementedError``).

``ckconv_filter`` is what ``CKConvND.forward`` (``modules/ckconv_nd.py:1133-1164``) builds
before the convolution — kernel, ``ExponentialModulationND`` window (``modules/masks_nd.py:229-255``),
causal crop to the second half of the grid — in one generator call that evaluates only the
kept points and writes the filter straight in the mixer's channel-major ``[1, C, *S]``
layout (or the reference's ``[1, *S, C]``).
"""

from __future__ import annotations

import ctypes
import math
from typing import Sequence

import torch

from . import _lib

__all__ = ["SIRENKernelB200", "siren_generate", "ckconv_filter"]


def _per_axis(L_cache, data_dim: int) -> tuple[int, ...]:
    if isinstance(L_cache, int):
        return (L_cache,) * data_dim
    L = tuple(int(v) for v in L_cache)
    if len(L) != data_dim:
        raise ValueError(f"L_cache has {len(L)} entries for data_dim={data_dim}")
    return L


def grid_axis(seq_len: int, L: int, device=None) -> torch.Tensor:
    """The reference's coordinates of one axis: the central 2 * seq_len - 1 points of
    linspace(-1, 1, 2 L - 1), or, past the cache, of the grid extended with the same step
    (kernels_nd.py:754-797 and :843-857)."""
    if seq_len <= L:
        full = torch.linspace(-1.0, 1.0, 2 * L - 1, dtype=torch.float32, device=device)
        return full[L - seq_len:L - seq_len + 2 * seq_len - 1]
    m = 1.0 + (1.0 / (L - 1)) * (seq_len - L)
    return torch.linspace(-m, m, 2 * seq_len - 1, dtype=torch.float32, device=device)


class _SirenFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, coords, n, mask_w, layout, pe_w, pe_b, out_w, out_b, n_hidden, *hidden):
        dev = _lib.require_cuda(coords, pe_w, out_w)
        hws, hbs = hidden[:n_hidden], hidden[n_hidden:]
        D = len(n)
        E, H, C = pe_w.shape[0], out_w.shape[1], out_w.shape[0]
        desc = _lib.SirenDesc()
        desc.ndim = D
        for a in range(3):
            desc.n[a] = n[a] if a < D else 1
        desc.embedding, desc.hidden, desc.num_hidden, desc.channels = E, H, n_hidden, C
        desc.layout = _lib.LAYOUT_BLH if layout == "blh" else _lib.LAYOUT_BHL
        f32 = [t.detach().to(torch.float32).contiguous() if t is not None else None
               for t in (pe_w, pe_b, out_w, out_b, mask_w)]
        hw = torch.cat([w.detach().to(torch.float32).reshape(-1) for w in hws])
        hb = torch.cat([b.detach().to(torch.float32).reshape(-1) for b in hbs]) if hbs else None
        lib = _lib.load()
        sv, wsz = ctypes.c_size_t(), ctypes.c_size_t()
        _lib.check(lib.hyfft_siren_sizes(ctypes.byref(desc), ctypes.byref(sv), ctypes.byref(wsz)), "hyfft_siren_sizes")
        G = math.prod(n)
        kernel = torch.empty((G, C) if layout == "blh" else (C, G), dtype=torch.float32, device=dev)
        saved = torch.empty(sv.value // 4, dtype=torch.float32, device=dev)
        rc = lib.hyfft_siren_forward(ctypes.byref(desc), coords.data_ptr(), f32[0].data_ptr(), _lib.ptr(f32[1]),
                                     hw.data_ptr(), _lib.ptr(hb), f32[2].data_ptr(), _lib.ptr(f32[3]), _lib.ptr(f32[4]),
                                     kernel.data_ptr(), saved.data_ptr(), sv.value, _lib.stream_ptr(dev))
        _lib.check(rc, "hyfft_siren_forward")
        ctx.desc, ctx.wsz, ctx.n_hidden = desc, wsz.value, n_hidden
        ctx.shapes = [w.shape for w in hws]
        ctx.dtypes = [t.dtype if t is not None else None for t in (pe_w, pe_b, out_w, out_b)] + [w.dtype for w in hidden]
        ctx.save_for_backward(coords, saved, hw, hb if hb is not None else torch.empty(0, device=dev),
                              *[t if t is not None else torch.empty(0, device=dev) for t in f32])
        ctx.has = (pe_b is not None, hb is not None, out_b is not None, mask_w is not None)
        return kernel

    @staticmethod
    def backward(ctx, dk):
        coords, saved, hw, hb, pe_w, pe_b, out_w, out_b, mask_w = ctx.saved_tensors
        has_pe_b, has_hb, has_out_b, has_mask = ctx.has
        dev = dk.device
        dkc = dk.to(torch.float32).contiguous()
        d_pe_w, d_out_w, d_hw = torch.empty_like(pe_w), torch.empty_like(out_w), torch.empty_like(hw)
        d_pe_b = torch.empty_like(pe_b) if has_pe_b else None
        d_out_b = torch.empty_like(out_b) if has_out_b else None
        d_hb = torch.empty_like(hb) if has_hb else None
        ws = torch.empty(ctx.wsz // 4, dtype=torch.float32, device=dev)
        rc = _lib.load().hyfft_siren_backward(
            ctypes.byref(ctx.desc), coords.data_ptr(), pe_w.data_ptr(), _lib.ptr(pe_b if has_pe_b else None),
            hw.data_ptr(), _lib.ptr(hb if has_hb else None), out_w.data_ptr(), _lib.ptr(mask_w if has_mask else None),
            dkc.data_ptr(), saved.data_ptr(), d_pe_w.data_ptr(), _lib.ptr(d_pe_b), d_hw.data_ptr(), _lib.ptr(d_hb),
            d_out_w.data_ptr(), _lib.ptr(d_out_b), ws.data_ptr(), ctx.wsz, _lib.stream_ptr(dev))
        _lib.check(rc, "hyfft_siren_backward")
        # split the concatenated hidden-layer gradients back into the layers
        gw, off = [], 0
        for shp in ctx.shapes:
            k = shp[0] * shp[1]
            gw.append(d_hw[off:off + k].view(shp))
            off += k
        gb = list(d_hb.view(ctx.n_hidden, -1).unbind(0)) if has_hb else []
        dts = ctx.dtypes
        cast = lambda g, dt: g.to(dt) if (g is not None and dt is not None) else g  # noqa: E731
        grads_hidden = [cast(g, dt) for g, dt in zip(gw + gb, dts[4:])]
        return (None, None, None, None, cast(d_pe_w, dts[0]), cast(d_pe_b, dts[1]), cast(d_out_w, dts[2]),
                cast(d_out_b, dts[3]), None, *grads_hidden)


def siren_generate(module: "SIRENKernelB200", axes: Sequence[torch.Tensor], mask_weight: torch.Tensor | None = None,
                   layout: str = "blh") -> torch.Tensor:
    """The masked filter over the grid spanned by the per-axis coordinate vectors ``axes``:
    ``[G, C]`` (layout "blh") or ``[C, G]`` ("bhl"), G = prod(len(axis))."""
    coords = torch.cat([a.to(torch.float32).reshape(-1) for a in axes]).contiguous()
    n = tuple(int(a.numel()) for a in axes)
    lin = module.positional_embedding.linear
    hid = list(module.hidden_linears)
    hidden = [l.weight for l in hid] + ([l.bias for l in hid] if hid[0].bias is not None else [])
    return _SirenFunction.apply(coords, n, mask_weight, layout, lin.weight, lin.bias, module.out_linear.weight,
                                module.out_linear.bias, len(hid), *hidden)


class _PositionalEmbedding(torch.nn.Module):
    """Parameter holder with the reference's names (``positional_embedding.linear``)."""

    def __init__(self, data_dim: int, embedding_dim: int, omega_0: float, use_bias: bool):
        super().__init__()
        self.linear = torch.nn.Linear(data_dim, embedding_dim, bias=use_bias)
        with torch.no_grad():  # first-layer SIREN bound 2 pi w0 / d (kernels_nd.py:570-609)
            bound = 2.0 * math.pi * omega_0 / data_dim
            self.linear.weight.uniform_(-bound, bound)
            if use_bias:
                self.linear.bias.zero_()


class SIRENKernelB200(torch.nn.Module):
    """B200 counterpart of ``SIRENKernelND`` (kernels_nd.py:876-1199) without FiLM."""

    def __init__(self, out_dim: int, data_dim: int, mlp_hidden_dim: int, num_layers: int, embedding_dim: int,
                 omega_0: float, L_cache: int | Sequence[int], use_bias: bool, hidden_omega_0: float = 1.0,
                 film_cfg=None, film_after_pos_embed: bool = False):
        super().__init__()
        if film_cfg is not None or film_after_pos_embed:
            raise NotImplementedError("FiLM-conditioned SIREN kernels are not covered by the B200 backend")
        if num_layers < 2:
            raise ValueError("num_layers must be >= 2 (embedding plus at least one hidden layer)")
        self.out_dim, self.data_dim, self.mlp_hidden_dim, self.num_layers = out_dim, data_dim, mlp_hidden_dim, num_layers
        self.embedding_dim, self.omega_0, self.hidden_omega_0 = embedding_dim, float(omega_0), float(hidden_omega_0)
        self.L_cache = L_cache
        self.L_cache_per_axis = _per_axis(L_cache, data_dim)
        self.positional_embedding = _PositionalEmbedding(data_dim, embedding_dim, omega_0, use_bias)
        dims = [embedding_dim] + [mlp_hidden_dim] * (num_layers - 1)
        self.hidden_linears = torch.nn.ModuleList(
            torch.nn.Linear(dims[i], dims[i + 1], bias=use_bias) for i in range(num_layers - 1))
        self.out_linear = torch.nn.Linear(mlp_hidden_dim, out_dim, bias=use_bias)
        with torch.no_grad():  # hidden / readout bound sqrt(6 / d) (the frequency cancels), zero bias
            for lin in list(self.hidden_linears) + [self.out_linear]:
                bound = math.sqrt(6.0 / lin.in_features)
                lin.weight.uniform_(-bound, bound)
                if lin.bias is not None:
                    lin.bias.zero_()
            self.out_linear.weight.mul_(math.sqrt(1.0 / math.prod(self.L_cache_per_axis)))  # Wang init

    def axes(self, seq_lens: Sequence[int], device=None) -> list[torch.Tensor]:
        assert len(seq_lens) == self.data_dim, f"seq_lens must be of length {self.data_dim}"
        return [grid_axis(int(s), L, device) for s, L in zip(seq_lens, self.L_cache_per_axis)]

    def forward(self, seq_lens: Sequence[int], conditioning: torch.Tensor | None = None):
        if conditioning is not None:
            raise NotImplementedError("FiLM conditioning is not covered by the B200 backend")
        dev = self.out_linear.weight.device
        ax = self.axes(seq_lens, dev)
        grid = torch.stack(torch.meshgrid(*ax, indexing="ij"), dim=-1).unsqueeze(0)
        k = siren_generate(self, ax)
        return k.view((1,) + tuple(a.numel() for a in ax) + (self.out_dim,)), grid


def ckconv_filter(kernel: SIRENKernelB200, mask_weight: torch.Tensor | None, grid_lens: Sequence[int],
                  causal: bool = False, layout: str = "bhl") -> torch.Tensor:
    """The filter CKConvND convolves with (ckconv_nd.py:1150-1164): SIREN kernel on the grid,
    exponential window (decay rates ``mask_weight`` [D, C], or None), and for causal 1D the
    second half of the grid only. ``layout`` "bhl" gives the mixer's ``[1, C, *S]``, "blh"
    the reference's ``[1, *S, C]``."""
    ax = kernel.axes(grid_lens, kernel.out_linear.weight.device)
    if causal:
        assert len(ax) == 1, "causal filters are 1D"
        ax = [ax[0][ax[0].numel() // 2:]]
    k = siren_generate(kernel, ax, mask_weight, layout)
    S = tuple(a.numel() for a in ax)
    return k.view((1, kernel.out_dim) + S) if layout == "bhl" else k.view((1,) + S + (kernel.out_dim,))


class SirenFilter(torch.nn.Module):
    """The implicit filter of a CKConvND (ckconv_nd.py:1133-1164) as the ``kernel_fn`` of
    ``HyenaB200``: ``spatial_dims -> [1, C, *K]`` from the SIREN network on the double grid
    (K = 2 N - 1 per axis), the exponential window (``mask.weight`` [D, C], the reference's
    ``ExponentialModulationND`` default decay ramp unless given) and, causal, the second half of
    the grid (K = N)."""

    def __init__(self, kernel: SIRENKernelB200, causal: bool = False, mask_weight: torch.Tensor | None = None,
                 use_mask: bool = True):
        super().__init__()
        self.kernel = kernel
        self.causal = causal
        if use_mask:
            if mask_weight is None:  # masks_nd.py:197-201: linspace(2.3, 13.81, C) / D on every axis
                ramp = torch.linspace(2.3, 13.81, kernel.out_dim) / kernel.data_dim
                mask_weight = torch.stack([ramp] * kernel.data_dim, dim=0)
            self.mask = torch.nn.Module()
            self.mask.register_buffer("weight", mask_weight.to(torch.float32).clone())
        else:
            self.mask = None

    def forward(self, spatial_dims, **_):
        mw = self.mask.weight if self.mask is not None else None
        return ckconv_filter(self.kernel, mw, tuple(int(s) for s in spatial_dims), causal=self.causal, layout="bhl")
