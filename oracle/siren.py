"""CPU oracle: SIREN implicit filter with exponential modulation — TEST INFRASTRUCTURE ONLY.

Restates the implicit-filter generator of nvSubquadratic in plain float32 torch:

* coordinate grid: per axis ``linspace(-m, m, 2 * L_cache - 1)``, centrally sliced to
  ``2 * seq_len - 1`` points (``modules/kernels_nd.py:754-771`` and ``:843-857``); with
  ``seq_len <= L_cache`` the limit m is 1;
* positional embedding ``h0 = sin(W0 x + b0)`` computed in float32
  (``modules/kernels_nd.py:859-871``);
* hidden layers ``h = sin(W_i h + b_i)`` (``modules/kernels_nd.py:1185-1196``, no FiLM);
* readout ``k = W_out h + b_out`` (``modules/kernels_nd.py:1197``);
* exponential modulation ``k[p, c] *= prod_d exp(-|x_d(p)| * |w[d, c]|)``
  (``modules/masks_nd.py:229-255``).

Parameter names and shapes follow the reference modules so a state dict moves across.
"""

from __future__ import annotations

import math

import torch


def grid_axes(seq_lens, L_cache):
    """Per-axis coordinate vectors of the sliced grid (float32), reference order."""
    L_cache = (L_cache,) * len(seq_lens) if isinstance(L_cache, int) else tuple(L_cache)
    axes = []
    for sl, L in zip(seq_lens, L_cache):
        if sl <= L:
            full = torch.linspace(-1.0, 1.0, 2 * L - 1, dtype=torch.float32)
            off = L - sl
        else:  # extended cache: same step 1 / (L - 1), limit grown to cover seq_len
            m = 1.0 + (1.0 / (L - 1)) * (sl - L)
            full = torch.linspace(-m, m, 2 * sl - 1, dtype=torch.float32)
            off = 0
        axes.append(full[off:off + 2 * sl - 1].contiguous())
    return axes


def siren_filter(params: dict, seq_lens, L_cache, mask_weight: torch.Tensor | None = None):
    """params: ``pe.weight`` [E, D], ``pe.bias`` [E] | None, ``hidden.{i}.weight`` / ``.bias``,
    ``out.weight`` [C, H], ``out.bias`` [C] | None. Returns (kernel [1, *S, C], grid [1, *S, D])."""
    axes = grid_axes(seq_lens, L_cache)
    grid = torch.stack(torch.meshgrid(*axes, indexing="ij"), dim=-1).unsqueeze(0)
    h = torch.sin(torch.nn.functional.linear(grid, params["pe.weight"], params.get("pe.bias")))
    i = 0
    while f"hidden.{i}.weight" in params:
        h = torch.sin(torch.nn.functional.linear(h, params[f"hidden.{i}.weight"], params.get(f"hidden.{i}.bias")))
        i += 1
    k = torch.nn.functional.linear(h, params["out.weight"], params.get("out.bias"))
    if mask_weight is not None:
        decay = torch.exp(-grid.unsqueeze(-1).abs() * mask_weight.abs()).prod(dim=-2)
        k = k * decay
    return k, grid


def init_params(out_dim: int, data_dim: int, hidden: int, num_layers: int, emb: int, omega_0: float,
                L_cache, use_bias: bool, gen: torch.Generator | None = None) -> dict:
    """SIREN initialisation (``modules/kernels_nd.py:570-609``): first layer U(+-2 pi w0 / d), later
    layers U(+-sqrt(6 / d)) (the hidden frequency cancels out of the bound), zero biases; the
    readout Wang-scaled by sqrt(1 / prod(L_cache))."""
    L_cache = (L_cache,) * data_dim if isinstance(L_cache, int) else tuple(L_cache)

    def u(shape, bound):
        return (torch.rand(shape, generator=gen) * 2 - 1) * bound

    p = {"pe.weight": u((emb, data_dim), 2 * math.pi * omega_0 / data_dim)}
    dims = [emb] + [hidden] * (num_layers - 1)
    for i in range(num_layers - 1):
        p[f"hidden.{i}.weight"] = u((dims[i + 1], dims[i]), math.sqrt(6.0 / dims[i]))
    p["out.weight"] = u((out_dim, hidden), math.sqrt(6.0 / hidden)) * math.sqrt(1.0 / math.prod(L_cache))
    if use_bias:
        p["pe.bias"] = torch.zeros(emb)
        for i in range(num_layers - 1):
            p[f"hidden.{i}.bias"] = torch.zeros(dims[i + 1])
        p["out.bias"] = torch.zeros(out_dim)
    return p


def mask_init(data_dim: int, channels: int, fast: float = 13.81, slow: float = 2.3) -> torch.Tensor:
    """Decay rates of ExponentialModulationND (``modules/masks_nd.py:197-201``): [D, C]."""
    ramp = torch.linspace(slow, fast, channels) / data_dim
    return torch.stack([ramp] * data_dim, dim=0)
