"""Op-level long convolutions on the B200 backend.

Same names, arguments, return values and errors as nvSubquadratic's
``nvsubquadratic/ops/fftconv.py`` (the ``torch_fft`` backend), so a
``CKConvND`` function table can point at these instead:

* ``causal_fftconv1d_fp32_bhl``  (fftconv.py:546-600)
* ``fftconv1d_fp32_bhl``         (fftconv.py:603-659)
* ``fftconv2d_fp32_bhl``         (fftconv.py:662-733)
* ``fftconv3d_fp32_bhl``         (fftconv.py:736-812)
* ``*_fp32_blh`` channels-last natives (fftconv.py:163-446) and the
  ``*_fp32_bhl_w_reshape`` channels-last wrappers (fftconv.py:449-538)

Contract: ``fn(x, kernel, shortcut=None) -> y`` with x ``[B, H, *S]`` (BHL) or
``[B, *S, H]`` (BLH) of any float dtype, kernel ``[1|B, H, *K]`` / ``[1|B, *K, H]``,
``K <= 2N`` per axis, shortcut ``[H]`` of x's dtype. The convolution is computed
in float32 and rounded to x's dtype once, then ``shortcut * x`` is added in
x's dtype. Inputs are not modified; ``y`` is a new tensor. Backward is the
exact adjoint (dx, dkernel, dshortcut), computed by the same CUDA engine.

Everything runs in ``libhyfft.so`` on the caller's current CUDA stream; a
CPU tensor raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

__all__ = [
    "causal_fftconv1d_fp32_bhl",
    "causal_fftconv1d_fp32_bhl_w_reshape",
    "causal_fftconv1d_fp32_blh",
    "fftconv1d_fp32_bhl",
    "fftconv1d_fp32_bhl_w_reshape",
    "fftconv1d_fp32_blh",
    "fftconv2d_fp32_bhl",
    "fftconv2d_fp32_bhl_w_reshape",
    "fftconv2d_fp32_blh",
    "fftconv3d_fp32_bhl",
    "fftconv3d_fp32_bhl_w_reshape",
    "fftconv3d_fp32_blh",
    "fftconv_nd",
    "mixed_fftconv_nd",
    "circular_fftconv1d_fp32_bhl",
    "circular_fftconv2d_fp32_bhl",
    "circular_fftconv3d_fp32_bhl",
    "circular_fftconv1d_fp32_bhl_w_reshape",
    "circular_fftconv2d_fp32_bhl_w_reshape",
    "circular_fftconv3d_fp32_bhl_w_reshape",
    "mixed_fftconv1d_fp32_bhl",
    "mixed_fftconv2d_fp32_bhl",
    "mixed_fftconv3d_fp32_bhl",
    "mixed_fftconv1d_fp32_bhl_w_reshape",
    "mixed_fftconv2d_fp32_bhl_w_reshape",
    "mixed_fftconv3d_fp32_bhl_w_reshape",
]


def _conv_desc(B, H, spatial, kshape, kB, causal, dtype, layout, periodic=0) -> _lib.ConvDesc:
    d = _lib.ConvDesc()
    d.periodic = periodic
    d.ndim = len(spatial)
    d.batch = B
    d.channels = H
    for i in range(3):
        d.n[i] = spatial[i] if i < len(spatial) else 1
        d.k[i] = kshape[i] if i < len(kshape) else 1
    d.kernel_batch = kB
    d.causal = 1 if causal else 0
    d.dtype = _lib.DTYPE_CODE[dtype]
    d.layout = layout
    return d


def _workspace_sizes(desc: _lib.ConvDesc) -> tuple[int, int]:
    f = ctypes.c_size_t()
    b = ctypes.c_size_t()
    _lib.check(_lib.load().hyfft_conv_workspace_size(ctypes.byref(desc), ctypes.byref(f), ctypes.byref(b)),
               "hyfft_conv_workspace_size")
    return f.value, b.value


_PLANS: dict = {}
# the library's switches that change the conv plan (and so its workspace sizes)
_PLAN_SWITCHES = ("HYFFT_WS_BUDGET_MB", "HYFFT_DISABLE_BIG2D", "HYFFT_B2_F256")


def _plan(*args):
    """(descriptor, (forward, backward) workspace bytes) for one problem, built once per
    shape: the per-call host cost is then a dictionary lookup."""
    key = args + tuple(os.environ.get(k) for k in _PLAN_SWITCHES)
    hit = _PLANS.get(key)
    if hit is None:
        desc = _conv_desc(*args)
        hit = (desc, _workspace_sizes(desc))
        if len(_PLANS) >= 256:
            _PLANS.clear()
        _PLANS[key] = hit
    return hit


class _FFTConvFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, kernel, shortcut, causal, layout, periodic=0):
        dev = _lib.require_cuda(x, kernel, shortcut)
        lib = _lib.load()
        nd = x.ndim - 2
        if layout == _lib.LAYOUT_BHL:
            B, H = x.shape[0], x.shape[1]
            spatial = tuple(x.shape[2:])
            kshape = tuple(kernel.shape[2:])
        else:
            B, H = x.shape[0], x.shape[-1]
            spatial = tuple(x.shape[1:-1])
            kshape = tuple(kernel.shape[1:-1])
        kB = kernel.shape[0]
        xc = x.contiguous()
        kf = kernel.detach().to(torch.float32).contiguous()
        sc = shortcut.detach().contiguous() if shortcut is not None else None
        desc, (wf, wb) = _plan(B, H, spatial, kshape, kB, causal, x.dtype, layout, periodic)
        ctx.wb = wb
        ws = _lib.workspace(wf, dev)
        y = torch.empty_like(xc)
        rc = lib.hyfft_conv_forward(ctypes.byref(desc), xc.data_ptr(), kf.data_ptr(), _lib.ptr(sc), y.data_ptr(),
                                    ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
        _lib.check(rc, "hyfft_conv_forward")
        ctx.save_for_backward(xc, kf, sc)
        ctx.desc = desc
        ctx.kernel_dtype = kernel.dtype
        ctx.has_shortcut = shortcut is not None
        ctx.shortcut_dtype = shortcut.dtype if shortcut is not None else None
        ctx.nd = nd
        return y

    @staticmethod
    def backward(ctx, dy):
        xc, kf, sc = ctx.saved_tensors
        dev = xc.device
        lib = _lib.load()
        desc = ctx.desc
        ws = _lib.workspace(ctx.wb, dev)
        dyc = dy.to(xc.dtype).contiguous()
        need_x, need_k, need_s = ctx.needs_input_grad[0], ctx.needs_input_grad[1], ctx.needs_input_grad[2]
        dx = torch.empty_like(xc) if need_x else None
        dk = torch.empty_like(kf) if need_k else None
        ds = torch.empty(sc.shape, dtype=torch.float32, device=dev) if (ctx.has_shortcut and need_s) else None
        rc = lib.hyfft_conv_backward(ctypes.byref(desc), xc.data_ptr(), kf.data_ptr(), _lib.ptr(sc), dyc.data_ptr(),
                                     _lib.ptr(dx), _lib.ptr(dk), _lib.ptr(ds), ws.data_ptr(), ws.numel(),
                                     _lib.stream_ptr(dev))
        _lib.check(rc, "hyfft_conv_backward")
        if dk is not None and ctx.kernel_dtype != torch.float32:
            dk = dk.to(ctx.kernel_dtype)
        if ds is not None and ctx.shortcut_dtype != torch.float32:
            ds = ds.to(ctx.shortcut_dtype)
        return dx, dk, ds, None, None, None


def _check_common(x, kernel, shortcut, nd, layout, periodic=()):
    assert x.ndim == nd + 2, f"Unexpected input shape: {tuple(x.shape)}."
    assert kernel.ndim == nd + 2, f"Unexpected kernel shape: {kernel.shape}."
    B = x.shape[0]
    assert kernel.shape[0] in (1, B), (
        f"Leading dimension must be 1 or batch_size ({B}). Got kernel.shape={kernel.shape}."
    )
    if layout == _lib.LAYOUT_BHL:
        H, spatial, kshape, kH = x.shape[1], x.shape[2:], kernel.shape[2:], kernel.shape[1]
    else:
        H, spatial, kshape, kH = x.shape[-1], x.shape[1:-1], kernel.shape[1:-1], kernel.shape[-1]
    for d, (n, k) in enumerate(zip(spatial, kshape)):
        if d < len(periodic) and periodic[d]:
            assert k <= n, f"K must be <= N on periodic axis {d}: K={k}, N={n}."
        else:
            assert k <= 2 * n, f"Kernel size must be less than or equal to 2 * input size. Got {k} for size {n}."
    assert kH == H, "Input and kernel must have the same number of channels (H)."
    if shortcut is not None:
        assert shortcut.dtype == x.dtype, f"shortcut.dtype ({shortcut.dtype}) must match x.dtype ({x.dtype})"
        assert tuple(shortcut.shape) == (H,)
    assert x.dtype in _lib.DTYPE_CODE, f"unsupported dtype {x.dtype}"


def _causal_alias_kernel(kernel: torch.Tensor, L: int, layout: int) -> torch.Tensor:
    """Centred kernel of length 2L-1 equal to what the reference computes for a causal
    kernel with K >= L + 2 at its FFT length F = 2L (fftconv.py:580), where taps
    j >= L + 1 wrap around to negative lags j - 2L."""
    ax = 2 if layout == _lib.LAYOUT_BHL else 1
    K = kernel.shape[ax]
    kp = torch.nn.functional.pad(kernel, _pad_spec(kernel.ndim, ax, 2 * L - K))
    neg = kp.narrow(ax, L + 1, L - 1)
    pos = kp.narrow(ax, 0, L)
    return torch.cat([neg, pos], dim=ax)


def _pad_spec(ndim: int, ax: int, right: int) -> list[int]:
    spec: list[int] = []
    for d in range(ndim - 1, -1, -1):
        spec += [0, right] if d == ax else [0, 0]
    return spec


def fftconv_nd(x, kernel, shortcut=None, *, causal: bool = False, layout: int = _lib.LAYOUT_BHL):
    """Generic entry: 1D/2D/3D, BHL or BLH, causal (1D) or centred."""
    nd = x.ndim - 2
    _check_common(x, kernel, shortcut, nd, layout)
    if causal:
        assert nd == 1, "causal convolution is 1D only"
        ax = 2 if layout == _lib.LAYOUT_BHL else 1
        L, K = x.shape[ax], kernel.shape[ax]
        if K >= L + 2:
            kernel = _causal_alias_kernel(kernel, L, layout)
            causal = False
    return _FFTConvFunction.apply(x, kernel, shortcut, causal, layout, 0)


# ---------------------------------------------------------------- BHL
def causal_fftconv1d_fp32_bhl(x, kernel, shortcut=None):
    """Causal 1D conv, x ``[B, H, L]``, kernel ``[1|B, H, K]`` (fftconv.py:546-600)."""
    return fftconv_nd(x, kernel, shortcut, causal=True, layout=_lib.LAYOUT_BHL)


def fftconv1d_fp32_bhl(x, kernel, shortcut=None):
    """Centred 1D conv, crop at K//2 (fftconv.py:603-659)."""
    return fftconv_nd(x, kernel, shortcut, causal=False, layout=_lib.LAYOUT_BHL)


def fftconv2d_fp32_bhl(x, kernel, shortcut=None):
    """Centred 2D conv, x ``[B, H, X, Y]``, kernel ``[1|B, H, Kx, Ky]`` (fftconv.py:662-733)."""
    return fftconv_nd(x, kernel, shortcut, causal=False, layout=_lib.LAYOUT_BHL)


def fftconv3d_fp32_bhl(x, kernel, shortcut=None):
    """Centred 3D conv (fftconv.py:736-812)."""
    return fftconv_nd(x, kernel, shortcut, causal=False, layout=_lib.LAYOUT_BHL)


# ---------------------------------------------------------------- BLH (channels-last, no transpose copies)
def causal_fftconv1d_fp32_blh(x, kernel, shortcut=None):
    """x ``[B, L, H]``, kernel ``[1|B, K, H]`` (fftconv.py:163-219)."""
    return fftconv_nd(x, kernel, shortcut, causal=True, layout=_lib.LAYOUT_BLH)


def fftconv1d_fp32_blh(x, kernel, shortcut=None):
    """fftconv.py:222-277."""
    return fftconv_nd(x, kernel, shortcut, causal=False, layout=_lib.LAYOUT_BLH)


def fftconv2d_fp32_blh(x, kernel, shortcut=None):
    """fftconv.py:280-349."""
    return fftconv_nd(x, kernel, shortcut, causal=False, layout=_lib.LAYOUT_BLH)


def fftconv3d_fp32_blh(x, kernel, shortcut=None):
    """fftconv.py:352-446."""
    return fftconv_nd(x, kernel, shortcut, causal=False, layout=_lib.LAYOUT_BLH)


# The reference's *_w_reshape wrappers transpose BLH -> BHL and back because torch.fft
# is faster on contiguous axes (fftconv.py:449-538). The CUDA engine reads channels-last
# directly, so the same names map to the BLH natives.
causal_fftconv1d_fp32_bhl_w_reshape = causal_fftconv1d_fp32_blh
fftconv1d_fp32_bhl_w_reshape = fftconv1d_fp32_blh
fftconv2d_fp32_bhl_w_reshape = fftconv2d_fp32_blh
fftconv3d_fp32_bhl_w_reshape = fftconv3d_fp32_blh


# ---------------------------------------------------------------- circular and mixed boundaries
def _normalize_periodic(periodic, data_dim: int) -> tuple[bool, ...]:
    """Per-axis periodic flags as a tuple of bools of length data_dim (mixed_fftconv.py:420-442)."""
    t = tuple(bool(p) for p in periodic)
    assert len(t) == data_dim, f"periodic must have length {data_dim} (data_dim), got length {len(t)}"
    return t


def _mask(periodic: tuple[bool, ...]) -> int:
    return sum(1 << d for d, p in enumerate(periodic) if p)


def mixed_fftconv_nd(x, kernel, periodic, shortcut=None, *, layout: int = _lib.LAYOUT_BHL):
    """Per-axis boundary conditions: periodic axes are circular (FFT length N, output
    aligned by (K - 1) // 2, K <= N), the others zero-padded "same" (crop at K // 2);
    ops/mixed_fftconv.py:504-623. Periodic axis lengths must be powers of two here."""
    nd = x.ndim - 2
    per = _normalize_periodic(periodic, nd)
    _check_common(x, kernel, shortcut, nd, layout, per)
    return _FFTConvFunction.apply(x, kernel, shortcut, False, layout, _mask(per))


def _circular(nd):
    def fn(x, kernel, shortcut=None, use_phase_shift: bool = True):
        # use_phase_shift picks how the reference applies the alignment (phase ramp or roll);
        # both give the same result, and the library always uses the phase ramp
        return mixed_fftconv_nd(x, kernel, (True,) * nd, shortcut, layout=_lib.LAYOUT_BHL)

    return fn


def _circular_blh(nd):
    def fn(x, kernel, shortcut=None, use_phase_shift: bool = True):
        return mixed_fftconv_nd(x, kernel, (True,) * nd, shortcut, layout=_lib.LAYOUT_BLH)

    return fn


circular_fftconv1d_fp32_bhl = _circular(1)
circular_fftconv1d_fp32_bhl.__doc__ = "Circular 1D conv, x [B, H, L], kernel [1|B, H, K<=L] (circular_fftconv.py:310-403)."
circular_fftconv2d_fp32_bhl = _circular(2)
circular_fftconv2d_fp32_bhl.__doc__ = "Circular 2D conv (circular_fftconv.py:406-483)."
circular_fftconv3d_fp32_bhl = _circular(3)
circular_fftconv3d_fp32_bhl.__doc__ = "Circular 3D conv (circular_fftconv.py:486-582)."
# channels-last forms (the reference transposes to BHL, circular_fftconv.py:585-660; read in place here)
circular_fftconv1d_fp32_bhl_w_reshape = _circular_blh(1)
circular_fftconv2d_fp32_bhl_w_reshape = _circular_blh(2)
circular_fftconv3d_fp32_bhl_w_reshape = _circular_blh(3)


def _mixed(nd, layout):
    def fn(x, kernel, periodic, shortcut=None, use_phase_shift: bool = True):
        return mixed_fftconv_nd(x, kernel, periodic, shortcut, layout=layout)

    return fn


mixed_fftconv1d_fp32_bhl = _mixed(1, _lib.LAYOUT_BHL)
mixed_fftconv2d_fp32_bhl = _mixed(2, _lib.LAYOUT_BHL)
mixed_fftconv3d_fp32_bhl = _mixed(3, _lib.LAYOUT_BHL)
mixed_fftconv1d_fp32_bhl_w_reshape = _mixed(1, _lib.LAYOUT_BLH)
mixed_fftconv2d_fp32_bhl_w_reshape = _mixed(2, _lib.LAYOUT_BLH)
mixed_fftconv3d_fp32_bhl_w_reshape = _mixed(3, _lib.LAYOUT_BLH)
for _f, _n in ((mixed_fftconv1d_fp32_bhl, "mixed_fftconv.py:631-660"), (mixed_fftconv2d_fp32_bhl, "mixed_fftconv.py:663-697"),
               (mixed_fftconv3d_fp32_bhl, "mixed_fftconv.py:700-723")):
    _f.__doc__ = f"Mixed boundary conditions, periodic = per-axis flags ({_n})."
