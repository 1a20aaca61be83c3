"""QKV sequence mixer on the B200 backend: the reference's ``QKVSequenceMixer``
(``nvsubquadratic/modules/sequence_mixer.py:129-296``) with the projections kept as
``torch.nn.Linear`` (cuBLAS GEMMs) and the mixer reading q, k, v as strided views of the one
``[B, *S, 3C]`` projection output: the fused Hyena kernels take the batch / position strides
of that buffer, and write dq, dk, dv into one ``[B, *S, 3C]`` gradient buffer with the same
strides, so neither the split after ``qkv_proj`` nor the concatenation of the gradients
before its backward copies anything. Same parameter names (``qkv_proj``, ``mixer``,
``out_proj``) and initialiser hooks as the reference.
"""

from __future__ import annotations

from typing import Callable

import torch

__all__ = ["QKVSequenceMixerB200"]


class QKVSequenceMixerB200(torch.nn.Module):
    def __init__(self, hidden_dim: int, mixer: torch.nn.Module, qkv_bias: bool = False, out_proj_bias: bool = False,
                 init_method_in: Callable | None = None, init_method_out: Callable | None = None):
        super().__init__()
        self.mixer = mixer
        self.qkv_proj = torch.nn.Linear(hidden_dim, 3 * hidden_dim, bias=qkv_bias)
        self.out_proj = torch.nn.Linear(hidden_dim, hidden_dim, bias=out_proj_bias)
        for lin, init in ((self.qkv_proj, init_method_in), (self.out_proj, init_method_out)):
            if init is not None:
                init(hidden_dim)(lin.weight.data)
                if lin.bias is not None:
                    torch.nn.init.zeros_(lin.bias)

    def forward(self, x: torch.Tensor, cp_group=None, **mixer_kwargs) -> torch.Tensor:
        """x ``[B, *S, C]`` -> ``[B, *S, C]``."""
        qkv = self.qkv_proj(x)
        C = qkv.shape[-1] // 3
        q, k, v = qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]  # views, no copy
        return self.out_proj(self.mixer(q, k, v, cp_group, **mixer_kwargs))
