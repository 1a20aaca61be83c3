"""CPU oracle: direct depthwise causal 1D convolution — TEST INFRASTRUCTURE ONLY.

Restates the reference function the reference's own tests pin the direct causal conv
op against (nvSubquadratic ``tests/ops/test_causal_conv1d_custom.py:62-68``): left-pad
the sequence by K - 1, depthwise ``F.conv1d`` with weight ``[C, 1, K]`` and bias, then
optionally SiLU. The op it checks is ``nvsubquadratic/ops/causal_conv1d_custom.py:81-98``.

``b2b_ref`` composes two such convolutions with Hyena's gate order
(``nvsubquadratic/modules/hyena_nd.py:505-570``): q, k, v = split(proj_conv(x)),
z = q * k, h = mixer_conv(z) + skip_bias * z, y = h * v (the reference pins only the
output shape of its fused b2b kernel, tests/ops/test_causal_conv1d_custom.py:115-133).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def causal_conv1d_ref(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                      activation: str = "identity") -> torch.Tensor:
    K = weight.shape[-1]
    xp = F.pad(x, (K - 1, 0))
    y = F.conv1d(xp, weight.to(x.dtype).unsqueeze(1), bias.to(x.dtype) if bias is not None else None,
                 groups=weight.shape[0])
    return F.silu(y) if activation == "silu" else y


def b2b_ref(x: torch.Tensor, weight_proj: torch.Tensor, weight_mixer: torch.Tensor,
            skip_bias: torch.Tensor) -> torch.Tensor:
    C = x.shape[1] // 3
    q, k, v = causal_conv1d_ref(x, weight_proj).split(C, dim=1)
    z = q * k
    h = causal_conv1d_ref(z, weight_mixer) + skip_bias.to(z.dtype).view(1, C, 1) * z
    return h * v
