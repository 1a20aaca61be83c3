"""Direct (non-FFT) depthwise causal 1D convolution on the B200 backend.

Mirrors nvSubquadratic ``nvsubquadratic/ops/causal_conv1d_custom.py`` (``causal_conv1d``,
``b2b_causal_conv1d``, lines 81-121) and ``nvsubquadratic/modules/subq_ops_causal_conv1d.py``
(``SubqOpsCausalConv1d``, lines 36-83): same names, argument meaning and constructor
error types; the computation runs in ``libhyfft.so`` (``hyfft_causal_conv1d_forward`` /
``_backward``), with no CPU fallback.

    causal_conv1d(x [B, C, L], weight [C, K], bias [C] | None, activation) -> [B, C, L]
    y = act(F.conv1d(F.pad(x, (K - 1, 0)), weight[:, None], bias, groups=C))

``b2b_causal_conv1d`` (projection conv, pre-gate, mixer conv with skip, post-gate) is a
composition of two direct convolutions with Hyena's gate order
(nvsubquadratic/modules/hyena_nd.py:505-570): q, k, v = split(proj_conv(x)),
z = q * k, h = mixer_conv(z) + skip_bias * z, y = h * v. The reference binds an external
kernel there and pins only the output shape [B, C, L]
(tests/ops/test_causal_conv1d_custom.py:115-133).
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["causal_conv1d", "b2b_causal_conv1d", "CausalConv1dB200"]

_ACT = {"identity": 0, "silu": 1}


def _check(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, activation: str):
    if activation not in _ACT:
        raise ValueError(f"unknown activation {activation!r}: use 'identity' or 'silu'")
    assert x.ndim == 3, f"x must be [B, C, L]; got {tuple(x.shape)}"
    assert weight.ndim == 2 and weight.shape[0] == x.shape[1], (
        f"weight must be [C, K] with C = {x.shape[1]}; got {tuple(weight.shape)}")
    if bias is not None:
        assert tuple(bias.shape) == (x.shape[1],), f"bias must be [C]; got {tuple(bias.shape)}"
    if x.dtype not in _lib.DTYPE_CODE:
        raise NotImplementedError(f"dtype {x.dtype} is not supported (float32, bfloat16, float16)")


class _CausalConv1dFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, activation):
        dev = _lib.require_cuda(x, weight, bias)
        x = x.contiguous()
        B, C, L = x.shape
        K = weight.shape[1]
        w32 = weight.detach().to(torch.float32).contiguous()
        b32 = bias.detach().to(torch.float32).contiguous() if bias is not None else None
        y = torch.empty_like(x)
        rc = _lib.load().hyfft_causal_conv1d_forward(x.data_ptr(), w32.data_ptr(), _lib.ptr(b32), y.data_ptr(), B, C,
                                                     L, K, _ACT[activation], _lib.DTYPE_CODE[x.dtype],
                                                     _lib.stream_ptr(dev))
        _lib.check(rc, "hyfft_causal_conv1d_forward")
        ctx.save_for_backward(x, w32, b32)
        ctx.act = _ACT[activation]
        ctx.dtypes = (weight.dtype, bias.dtype if bias is not None else None)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w32, b32 = ctx.saved_tensors
        B, C, L = x.shape
        K = w32.shape[1]
        dyc = dy.to(x.dtype).contiguous()
        dx = torch.empty_like(x)
        dw = torch.empty_like(w32)
        db = torch.empty_like(b32) if b32 is not None else None
        rc = _lib.load().hyfft_causal_conv1d_backward(x.data_ptr(), w32.data_ptr(), _lib.ptr(b32), dyc.data_ptr(),
                                                      dx.data_ptr(), dw.data_ptr(), _lib.ptr(db), B, C, L, K, ctx.act,
                                                      _lib.DTYPE_CODE[x.dtype], _lib.stream_ptr(x.device))
        _lib.check(rc, "hyfft_causal_conv1d_backward")
        wdt, bdt = ctx.dtypes
        return dx, dw.to(wdt), (db.to(bdt) if db is not None else None), None


def causal_conv1d(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                  activation: str = "identity") -> torch.Tensor:
    """Depthwise causal 1D conv (causal_conv1d_custom.py:81-98): x ``[B, C, L]``, weight
    ``[C, K]``, bias ``[C]`` or None, activation ``"identity"`` or ``"silu"``; returns
    ``[B, C, L]`` in x's dtype."""
    _check(x, weight, bias, activation)
    return _CausalConv1dFunction.apply(x, weight, bias, activation)


def b2b_causal_conv1d(x: torch.Tensor, weight_proj: torch.Tensor, weight_mixer: torch.Tensor,
                      skip_bias: torch.Tensor) -> torch.Tensor:
    """Back-to-back causal conv (causal_conv1d_custom.py:101-121): x ``[B, 3C, L]``,
    weight_proj ``[3C, K]``, weight_mixer ``[C, K]``, skip_bias ``[C]`` -> ``[B, C, L]``."""
    assert x.ndim == 3 and x.shape[1] % 3 == 0, f"x must be [B, 3C, L]; got {tuple(x.shape)}"
    C = x.shape[1] // 3
    assert weight_proj.ndim == 2 and weight_proj.shape[0] == 3 * C, "weight_proj must be [3C, K]"
    assert weight_mixer.ndim == 2 and weight_mixer.shape[0] == C, "weight_mixer must be [C, K]"
    assert tuple(skip_bias.shape) == (C,), "skip_bias must be [C]"
    proj = causal_conv1d(x, weight_proj)
    q, k, v = proj.split(C, dim=1)
    z = q * k
    h = causal_conv1d(z, weight_mixer) + skip_bias.to(z.dtype).view(1, C, 1) * z
    return h * v


class CausalConv1dB200(torch.nn.Conv1d):
    """Depthwise causal 1D conv module, the B200 counterpart of ``SubqOpsCausalConv1d``
    (subq_ops_causal_conv1d.py:36-83): a ``torch.nn.Conv1d`` subclass (so Hyena's short-conv
    type check passes) with weight ``[C, 1, K]``, optional bias and activation."""

    def __init__(self, in_channels: int, out_channels: int, kernel_size: int, *, groups: int, bias: bool = False,
                 activation: str = "identity") -> None:
        # the reference's construction tests match on "depthwise-only" and "activation"
        # (tests/modules/test_subq_ops_causal_conv1d.py:124-138)
        if not (groups == in_channels == out_channels):
            raise ValueError(f"CausalConv1dB200 is depthwise-only (groups, in_channels and out_channels equal); "
                             f"got groups={groups}, in_channels={in_channels}, out_channels={out_channels}")
        if activation not in _ACT:
            raise ValueError(f"unknown activation {activation!r}: use 'identity' or 'silu'")
        super().__init__(in_channels=in_channels, out_channels=out_channels, kernel_size=kernel_size, groups=groups,
                         bias=bias, padding=0)
        self.activation = activation

    def forward(self, input: torch.Tensor) -> torch.Tensor:  # type: ignore[override]
        return causal_conv1d(input, self.weight.squeeze(1), self.bias, self.activation)
