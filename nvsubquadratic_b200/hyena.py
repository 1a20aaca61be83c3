"""Fused Hyena mixer on the B200 backend.

Mirrors ``Hyena.forward(query, key, value, cp_group=None, **mixer_kwargs)``
(nvSubquadratic ``nvsubquadratic/modules/hyena_nd.py:432-583``) for the
configuration this backend fuses: identity QK / PixelHyena / output norms,
identity / sigmoid / SiLU gates, an optional depthwise short conv on
``cat([q, k, v])`` ("same" padding, or causal left padding for 1D), and the
CKConvND global conv with its D-skip. Tensors enter and leave channels-last
``[B, *S, C]``; q, k, v may be strided views into one ``[B, *S, 3C]`` projection
output (as ``QKVSequenceMixer`` produces them, sequence_mixer.py:290-291) and
are read in place, without the reference's transpose / cat / split copies.

    z = q' * gate1(k')            (q', k', v') = short_conv(q, k, v)
    h = conv(z, filt) + D * z     (the CKConvND global conv)
    y = h * gate2(v')

Forward and backward are ``libhyfft.so`` calls on the current CUDA stream.
"""

from __future__ import annotations

import ctypes
import math
import os
from typing import Callable

import torch

from . import _lib

__all__ = ["hyena_fused", "HyenaB200", "ExplicitKernel", "gate_name"]


def gate_name(g) -> str:
    """Map a gate spec (string or nn.Module instance / class) to identity / sigmoid / silu."""
    if g is None:
        return "identity"
    if isinstance(g, str):
        name = g.lower()
    else:
        cls = g if isinstance(g, type) else type(g)
        name = {"Identity": "identity", "Sigmoid": "sigmoid", "SiLU": "silu"}.get(cls.__name__, "")
    if name not in _lib.GATE_CODE:
        raise NotImplementedError(f"gate {g!r} is not fused by the b200 backend (identity / sigmoid / silu only)")
    return name


def _pos_strides(t: torch.Tensor) -> tuple[int, int] | None:
    """(batch_stride, position_stride) if t is [B, *S, C] with unit channel stride and a
    uniform stride over the flattened positions; else None."""
    if t.stride(-1) != 1:
        return None
    S = t.shape[1:-1]
    ps = t.stride(-2) if len(S) else 1
    expect = ps
    for d in range(len(S) - 1, -1, -1):
        if S[d] > 1 and t.stride(1 + d) != expect:
            return None
        expect *= S[d]
    return t.stride(0), ps


def _hyena_desc(B, C, spatial, kshape, causal, short_k, short_causal, short_bias, g1, g2, dtype,
                in_strides, out_strides, periodic=0) -> _lib.HyenaDesc:
    d = _lib.HyenaDesc()
    d.periodic = periodic
    d.ndim = len(spatial)
    d.batch = B
    d.channels = C
    for i in range(3):
        d.n[i] = spatial[i] if i < len(spatial) else 1
        d.k[i] = kshape[i] if i < len(kshape) else 1
        d.short_k[i] = (short_k[i] if i < len(short_k) else 1) if short_k else 0
    d.causal = 1 if causal else 0
    d.short_causal = 1 if short_causal else 0
    d.short_bias = 1 if short_bias else 0
    d.gate1 = _lib.GATE_CODE[g1]
    d.gate2 = _lib.GATE_CODE[g2]
    d.dtype = _lib.DTYPE_CODE[dtype]
    d.in_batch_stride, d.in_pos_stride = in_strides
    d.out_batch_stride, d.out_pos_stride = out_strides
    return d


def _sizes(desc) -> tuple[int, int, int]:
    f, b, s = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    _lib.check(_lib.load().hyfft_hyena_workspace_size(ctypes.byref(desc), ctypes.byref(f), ctypes.byref(b),
                                                       ctypes.byref(s)), "hyfft_hyena_workspace_size")
    return f.value, b.value, s.value


_PLANS: dict = {}
# the library's switches that change which kernels (and so which workspace sizes) a plan uses
_PLAN_SWITCHES = ("HYFFT_USE_TP", "HYFFT_DISABLE_TP", "HYFFT_DISABLE_FUSED", "HYFFT_FUSED_POW2", "HYFFT_NO_KH_CACHE",
                  "HYFFT_WS_BUDGET_MB", "HYFFT_DISABLE_BIG2D", "HYFFT_B2_F256")


def _plan(*args):
    """(descriptor, (fwd, bwd, saved) workspace bytes) for one problem, built once per
    shape (and per setting of the library's HYFFT_* switches, which pick its kernels):
    the per-step host cost of a call is then a dictionary lookup."""
    key = args + tuple(os.environ.get(k) for k in _PLAN_SWITCHES)
    hit = _PLANS.get(key)
    if hit is None:
        desc = _hyena_desc(*args)
        hit = (desc, _sizes(desc))
        if len(_PLANS) >= 256:
            _PLANS.clear()
        _PLANS[key] = hit
    return hit


def _packed_views(q, k, v) -> bool:
    """True if q, k, v are the three channel chunks of one contiguous [B, *S, 3C] tensor."""
    C = q.shape[-1]
    if not (q.shape == k.shape == v.shape) or q.dtype != k.dtype or q.dtype != v.dtype:
        return False
    es = q.element_size()
    if k.data_ptr() != q.data_ptr() + C * es or v.data_ptr() != q.data_ptr() + 2 * C * es:
        return False
    want, acc = [1], 3 * C  # strides of a contiguous [B, *S, 3C] tensor
    for n in reversed(q.shape[:-1]):
        want.append(acc)
        acc *= n
    want = tuple(reversed(want))
    return all(all(n == 1 or st == w for n, st, w in zip(t.shape, t.stride(), want)) for t in (q, k, v))


def _packed_base(q, k, v):
    """The [B, *S, 3C] tensor whose channel chunks q, k, v are (a view of their common base
    over the same memory), or None. Autograd on it hands the fused backward's one gradient
    buffer straight to the projection, without re-assembling three chunk gradients."""
    base = q._base
    if base is None or k._base is not base or v._base is not base or not _packed_views(q, k, v):
        return None
    shape = tuple(q.shape[:-1]) + (3 * q.shape[-1],)
    if not base.is_contiguous() or base.data_ptr() != q.data_ptr() or base.numel() != math.prod(shape):
        return None
    return base if tuple(base.shape) == shape else base.view(shape)


def _chunks(qkv):
    C = qkv.shape[-1] // 3
    return qkv[..., :C], qkv[..., C:2 * C], qkv[..., 2 * C:]


def _params32(filt, D, short_w, short_b, C):
    """float32 contiguous copies of the parameters the library reads (no copy when they
    already are); short_w flattened to [3C, taps]."""
    filt32 = filt.detach().to(torch.float32).contiguous()
    D32 = D.detach().to(torch.float32).contiguous()
    sw32 = short_w.detach().to(torch.float32).reshape(3 * C, -1).contiguous() if short_w is not None else None
    sb32 = short_b.detach().to(torch.float32).contiguous() if short_b is not None else None
    return filt32, D32, sw32, sb32


def forward_call(q, k, v, filt32, D32, sw32, sb32, cfg):
    """One ``hyfft_hyena_forward`` on q, k, v ``[B, *S, C]`` (contiguous, or the three
    channel chunks of one packed ``[B, *S, 3C]`` tensor). Returns ``(y, state)``; the
    state (descriptor, saved buffer, backward workspace size) feeds ``backward_call``."""
    dev = q.device
    causal, short_k, short_causal, g1, g2 = cfg[:5]
    periodic = cfg[5] if len(cfg) > 5 else 0  # bit mask of circular axes
    B, C = q.shape[0], q.shape[-1]
    y = torch.empty(q.shape, dtype=q.dtype, device=dev)
    desc, (wf, wb, sv) = _plan(B, C, tuple(q.shape[1:-1]), tuple(filt32.shape[2:]), causal, short_k, short_causal,
                               sb32 is not None, g1, g2, q.dtype, _pos_strides(q), _pos_strides(y), periodic)
    ws = _lib.workspace(wf, dev)
    saved = _lib.workspace(sv, dev)
    rc = _lib.load().hyfft_hyena_forward(ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                         filt32.data_ptr(), D32.data_ptr(), _lib.ptr(sw32), _lib.ptr(sb32),
                                         y.data_ptr(), saved.data_ptr(), ws.data_ptr(), ws.numel(),
                                         _lib.stream_ptr(dev))
    _lib.check(rc, "hyfft_hyena_forward")
    return y, (desc, saved, wb)


def backward_call(q, k, v, filt32, D32, sw32, sb32, state, dy, dq, dk, dv):
    """One ``hyfft_hyena_backward``: dq, dk, dv are written with q's strides (one packed
    buffer for packed views); returns float32 (dfilt, dD, dshort_w [3C, taps], dshort_b)."""
    desc, saved, wb = state
    dev = q.device
    ws = _lib.workspace(wb, dev)
    dfilt = torch.empty_like(filt32)
    dD = torch.empty_like(D32)
    dsw = torch.empty_like(sw32) if sw32 is not None else None
    dsb = torch.empty_like(sb32) if sb32 is not None else None
    rc = _lib.load().hyfft_hyena_backward(ctypes.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                          filt32.data_ptr(), D32.data_ptr(), _lib.ptr(sw32), _lib.ptr(sb32),
                                          dy.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                                          dfilt.data_ptr(), dD.data_ptr(), _lib.ptr(dsw), _lib.ptr(dsb),
                                          saved.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(rc, "hyfft_hyena_backward")
    return dfilt, dD, dsw, dsb


def _in_place_views(q, k, v):
    """q, k, v as the library reads them: in place when contiguous or the three chunks of
    one packed projection (their gradients then share that layout); else contiguous copies."""
    strides = _pos_strides(q)
    dense = (math.prod(q.shape[1:]), q.shape[-1])
    if strides is None or _pos_strides(k) != strides or _pos_strides(v) != strides or (
            strides != dense and not _packed_views(q, k, v)):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    return q, k, v


def _grad_buffers(q):
    """dq, dk, dv with q's layout: separate tensors for contiguous q, else three chunks of
    one packed [B, *S, 3C] buffer (returned as the fourth value)."""
    shape, C, dev = q.shape, q.shape[-1], q.device
    if q.is_contiguous():
        dq, dk, dv = (torch.empty(shape, dtype=q.dtype, device=dev) for _ in range(3))
        return dq, dk, dv, None
    dqkv = torch.empty(tuple(shape[:-1]) + (3 * C,), dtype=q.dtype, device=dev)
    dq, dk, dv = _chunks(dqkv)
    return dq, dk, dv, dqkv


class _HyenaFunction(torch.autograd.Function):
    """Fused Hyena on q, k, v (PACKED False) or on their packed [B, *S, 3C] projection
    (PACKED True: one input, one gradient)."""

    @staticmethod
    def forward(ctx, packed, *args):
        if packed:
            qkv, filt, D, short_w, short_b, cfg = args
            q, k, v = _chunks(qkv)
        else:
            q, k, v, filt, D, short_w, short_b, cfg = args
        _lib.require_cuda(q, k, v, filt, D, short_w, short_b)
        q, k, v = _in_place_views(q, k, v)
        ctx.packed = packed
        filt32, D32, sw32, sb32 = _params32(filt, D, short_w, short_b, q.shape[-1])
        y, state = forward_call(q, k, v, filt32, D32, sw32, sb32, cfg)
        ctx.save_for_backward(q, k, v, filt32, D32, sw32, sb32, state[1])
        ctx.state = (state[0], state[2])
        ctx.dtypes = (filt.dtype, D.dtype, short_w.dtype if short_w is not None else None,
                      short_b.dtype if short_b is not None else None)
        ctx.sw_shape = short_w.shape if short_w is not None else None
        return y

    @staticmethod
    def backward(ctx, dy):
        q, k, v, filt32, D32, sw32, sb32, saved = ctx.saved_tensors
        desc, wb = ctx.state
        dyc = dy.to(q.dtype).contiguous()
        dq, dk, dv, dqkv = _grad_buffers(q)
        dfilt, dD, dsw, dsb = backward_call(q, k, v, filt32, D32, sw32, sb32, (desc, saved, wb), dyc, dq, dk, dv)
        fdt, Ddt, swdt, sbdt = ctx.dtypes
        dfilt = dfilt.to(fdt)
        dD = dD.to(Ddt)
        if dsw is not None:
            dsw = dsw.reshape(ctx.sw_shape).to(swdt)
        if dsb is not None:
            dsb = dsb.to(sbdt)
        if ctx.packed:
            if dqkv is None:
                dqkv = torch.cat((dq, dk, dv), dim=-1)
            return None, dqkv, dfilt, dD, dsw, dsb, None
        return None, dq, dk, dv, dfilt, dD, dsw, dsb, None


def hyena_fused(q, k, v, filt, D, short_w=None, short_b=None, *, causal=False, short_causal=None,
                gate1="identity", gate2=None, periodic=None):
    """Functional fused Hyena. q, k, v ``[B, *S, C]``; filt ``[1, C, *K]`` (BHL, any float
    dtype, computed in float32); D ``[C]``; short_w ``[3C, 1, *k]`` or ``[3C, *k]``; short_b
    ``[3C]`` or None; periodic: per-axis circular flags of the long conv (CKConvND's
    fft_padding "circular" / per-axis list) or None (zero padding). Returns ``[B, *S, C]``
    in q's dtype."""
    nd = q.ndim - 2
    assert nd in (1, 2, 3), f"unsupported rank {q.ndim}"
    assert q.shape == k.shape == v.shape, "query, key and value must have the same shape"
    C = q.shape[-1]
    assert filt.ndim == nd + 2 and filt.shape[0] == 1 and filt.shape[1] == C, (
        f"filter must be [1, C, *K]; got {tuple(filt.shape)}")
    assert tuple(D.shape) == (C,)
    per = tuple(bool(x) for x in periodic) if periodic is not None else (False,) * nd
    assert len(per) == nd, f"periodic must have length {nd} (data_dim), got length {len(per)}"
    for ax, (n, kk) in enumerate(zip(q.shape[1:-1], filt.shape[2:])):
        if per[ax]:
            assert kk <= n, f"K must be <= N on periodic axis {ax}: K={kk}, N={n}."
        else:
            assert kk <= 2 * n, f"Kernel size must be less than or equal to 2 * input size. Got {kk} for size {n}."
    g1 = gate_name(gate1)
    g2 = gate_name(gate2) if gate2 is not None else g1
    short_k = ()
    if short_w is not None:
        short_k = tuple(short_w.shape[-nd:])
        assert short_w.shape[0] == 3 * C and short_w.numel() == 3 * C * int(torch.tensor(short_k).prod())
    if short_causal is None:
        short_causal = causal
    if causal:
        L, K = q.shape[1], filt.shape[2]
        assert nd == 1, "causal Hyena is 1D only"
        assert K <= L + 1, "causal filter longer than L+1 is not supported by the fused path"
    cfg = (bool(causal), short_k, bool(short_causal), g1, g2, sum(1 << ax for ax, p_ in enumerate(per) if p_))
    base = _packed_base(q, k, v) if torch.is_grad_enabled() else None
    if base is not None:
        return _HyenaFunction.apply(True, base, filt, D, short_w, short_b, cfg)
    return _HyenaFunction.apply(False, q, k, v, filt, D, short_w, short_b, cfg)


class ExplicitKernel(torch.nn.Module):
    """A stored filter ``[1, C, *K]`` (stands in for the implicit SIREN generator, which is
    not part of this backend); ``forward(spatial_dims)`` returns it."""

    def __init__(self, filt: torch.Tensor):
        super().__init__()
        self.weight = torch.nn.Parameter(filt.detach().clone())

    def forward(self, spatial_dims=None, **kwargs):
        return self.weight


class HyenaB200(torch.nn.Module):
    """Fused replacement for ``Hyena`` (hyena_nd.py:126) with identity norms.

    Args:
        hidden_dim: C.
        data_dim: spatial rank 1..3.
        kernel_fn: module / callable ``(spatial_dims, **mixer_kwargs) -> [1, C, *K]`` float filter
            (the global conv kernel after masking and causal crop, BHL).
        short_kernel_size: depthwise short conv size on cat([q, k, v]) (None: no short conv).
        gate1 / gate2: "identity" | "sigmoid" | "silu" (or the matching nn.Module); gate2
            defaults to gate1 (hyena_nd.py:274-278).
        causal: causal 1D global conv (short conv is causal too unless short_causal=False).
        short_bias: learnable bias on the short conv.
        periodic: per-axis circular flags of the global conv (None: zero padding on every axis).
    """

    def __init__(self, hidden_dim: int, data_dim: int, kernel_fn: Callable, *, short_kernel_size: int | None = 3,
                 gate1="identity", gate2=None, causal: bool = False, short_causal: bool | None = None,
                 short_bias: bool = False, periodic=None, dtype=torch.float32, device=None):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.periodic = tuple(bool(x) for x in periodic) if periodic is not None else None
        self.data_dim = data_dim
        self.kernel_fn = kernel_fn
        self.gate1 = gate_name(gate1)
        self.gate2 = gate_name(gate2) if gate2 is not None else self.gate1
        self.causal = causal
        self.short_causal = causal if short_causal is None else short_causal
        C3 = 3 * hidden_dim
        # D-skip, init U(+-1/sqrt(C)) as CKConvND.shortcut (ckconv_nd.py:792-794)
        bound = hidden_dim ** -0.5
        self.shortcut = torch.nn.Parameter(torch.empty(hidden_dim, dtype=dtype, device=device).uniform_(-bound, bound))
        if short_kernel_size:
            ks = (short_kernel_size,) * data_dim
            fan = short_kernel_size ** data_dim
            b = fan ** -0.5  # nn.ConvNd default for groups=C: U(+-1/sqrt(fan_in))
            self.short_weight = torch.nn.Parameter(
                torch.empty((C3, 1) + ks, dtype=dtype, device=device).uniform_(-b, b))
            self.short_bias = (torch.nn.Parameter(torch.empty(C3, dtype=dtype, device=device).uniform_(-b, b))
                               if short_bias else None)
        else:
            self.short_weight = None
            self.short_bias = None

    def forward(self, query, key, value, cp_group=None, **mixer_kwargs):
        spatial = tuple(query.shape[1:-1])
        filt = self.kernel_fn(spatial, **mixer_kwargs)
        if cp_group is not None and cp_group.size() > 1:
            from .cp import hyena_context_parallel

            return hyena_context_parallel(self, query, key, value, filt, cp_group)
        return hyena_fused(query, key, value, filt, self.shortcut.to(query.dtype), self.short_weight,
                           self.short_bias, causal=self.causal, short_causal=self.short_causal,
                           gate1=self.gate1, gate2=self.gate2, periodic=self.periodic)
