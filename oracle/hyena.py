"""CPU oracle: the Hyena mixer composition — TEST INFRASTRUCTURE ONLY.

Restates ``Hyena.forward`` (nvSubquadratic ``nvsubquadratic/modules/hyena_nd.py:432-583``)
for the configuration the fused backend accelerates: identity QK/PixelHyena/
output norms, identity / sigmoid / SiLU gates, no context parallelism (the CP
redistribution is restated separately in ``oracle/cp.py``).

Order of operations (hyena_nd.py line numbers):

1. channels-last ``[B, *S, C]`` -> channels-first                    (:498-500)
2. ``cat([q, k, v], dim=1)`` -> depthwise short conv on 3C channels  (:505-516)
   * "same" padding (``torch.nn.Conv{1,2,3}d(padding=k//2)`` and
     ``DistributedDepthwiseConv*d`` non-causal, distributed_depthwise_conv_nd.py:240-253)
   * causal 1D: left pad ``K-1`` (distributed_depthwise_conv_nd.py:229-239,
     causal_conv1d.py:113-143)
3. split back into q, k, v                                          (:523-527)
4. gate 1: ``z = q * gate1(k)``                                     (:546)
5. global conv ``h = fftconv(z, filt) + D * z`` (CKConvND -> ops/fftconv.py) (:563)
6. gate 2: ``y = h * gate2(v)`` (gate2 defaults to gate1)            (:570, :274-278)
7. channels-first -> channels-last                                   (:583)

Every tensor op runs in the activation dtype exactly as the reference module
does when its parameters share that dtype (each elementwise op rounds to the
activation dtype; the FFT conv computes in float32 and rounds once).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .fftconv import fftconv_bhl

GATES = ("identity", "sigmoid", "silu")


def gate_fn(name: str, t: torch.Tensor) -> torch.Tensor:
    if name == "identity":
        return t
    if name == "sigmoid":
        return torch.sigmoid(t)
    if name == "silu":
        return F.silu(t)
    raise ValueError(f"unknown gate {name!r}")


def depthwise_short_conv(
    x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, causal: bool
) -> torch.Tensor:
    """Depthwise cross-correlation; ``weight`` is ``[C, 1, *k]``.

    Non-causal pads like ``padding="same"`` (left ``(k-1)//2``, right the rest);
    causal (1D only) pads ``k-1`` on the left.
    """
    nd = x.ndim - 2
    C = x.shape[1]
    ks = weight.shape[2:]
    pads: list[int] = []
    for k in reversed(ks):  # F.pad takes the last axis first
        if causal:
            pads += [k - 1, 0]
        else:
            left = (k - 1) // 2
            pads += [left, k - 1 - left]
    xp = F.pad(x, pads)
    conv = {1: F.conv1d, 2: F.conv2d, 3: F.conv3d}[nd]
    w = weight.to(x.dtype)
    b = bias.to(x.dtype) if bias is not None else None
    return conv(xp, w, b, groups=C)


def hyena_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    filt: torch.Tensor,
    D: torch.Tensor | None,
    short_w: torch.Tensor | None = None,
    short_b: torch.Tensor | None = None,
    *,
    causal: bool = False,
    short_causal: bool | None = None,
    gate1: str = "identity",
    gate2: str | None = None,
    periodic: tuple[bool, ...] | None = None,
) -> torch.Tensor:
    """q, k, v: ``[B, *S, C]``; filt: ``[1|B, C, *K]`` (the BHL kernel CKConvND hands to
    the op, ckconv_nd.py:1055-1062); D: ``[C]`` in the activation dtype or None;
    short_w: ``[3C, 1, *k]``; returns ``[B, *S, C]``."""
    if short_causal is None:
        short_causal = causal
    if gate2 is None:
        gate2 = gate1
    C = q.shape[-1]
    qb, kb, vb = (t.movedim(-1, 1) for t in (q, k, v))
    if short_w is not None:
        x = torch.cat([qb, kb, vb], dim=1)
        x = depthwise_short_conv(x, short_w, short_b, short_causal)
        qb, kb, vb = (t.contiguous() for t in x.split(C, dim=1))
    z = qb * gate_fn(gate1, kb)
    h = fftconv_bhl(z, filt, D, causal=causal, periodic=periodic)
    y = h * gate_fn(gate2, vb)
    return y.movedim(1, -1)
