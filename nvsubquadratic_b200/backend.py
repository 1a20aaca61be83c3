"""``fft_backend="b200"``: the backend slot of CKConvND and the fused Hyena mixer.

What a maintainer wires into the reference (nvSubquadratic) to select this backend,
restated as plain functions so that they can be called from ``CKConvND.__init__`` /
``apply_convolution`` and tested without the module layer:

* ``BACKENDS`` / ``check_fft_backend``: the allow-list assert of ckconv_nd.py:628-630,
  extended by ``"b200"``.
* ``validate_ckconv_config``: the constructor constraints of ckconv_nd.py:640-724 for
  this backend (zero, circular or per-axis mixed padding; causal is 1D and zero-padded;
  data_dim 1..3).
* ``select_fftconv_fns``: the binding of ``fftconv_fn`` (BLH) and
  ``fftconv_fn_bhl_input`` (BHL) of ckconv_nd.py:796-871.
* ``apply_convolution``: ckconv_nd.py:1006-1062 (the kernel arrives channels-last and
  is moved to channels-first for the BHL entry).
* ``ckconv_kernel``: the kernel CKConvND.forward hands to the op (ckconv_nd.py:1143-1188:
  generator, mask, causal crop, context-parallel channel slice), as ``[1|B, C, *K]``.
* ``fused_mixer_config``: whether a reference ``Hyena`` instance can run on the fused
  mixer (identity norms, identity / sigmoid / SiLU gates, a depthwise short conv the
  fused kernels cover, a ``"b200"`` global conv), hyena_nd.py:256-302, :432-583.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from . import fftconv as _ops
from .hyena import gate_name

__all__ = [
    "FFT_BACKEND",
    "BACKENDS",
    "check_fft_backend",
    "validate_ckconv_config",
    "select_fftconv_fns",
    "resolve_periodic",
    "apply_convolution",
    "ckconv_kernel",
    "fused_mixer_config",
    "FusedHyena",
]

FFT_BACKEND = "b200"
BACKENDS = ("torch_fft", "subq_ops", FFT_BACKEND)

# effective padding -> data_dim -> (fftconv_fn [BLH input], fftconv_fn_bhl_input [BHL input])
FFT_FUNCTIONS = {
    "zero": {
        1: (_ops.fftconv1d_fp32_bhl_w_reshape, _ops.fftconv1d_fp32_bhl),
        2: (_ops.fftconv2d_fp32_bhl_w_reshape, _ops.fftconv2d_fp32_bhl),
        3: (_ops.fftconv3d_fp32_bhl_w_reshape, _ops.fftconv3d_fp32_bhl),
    },
    "causal": {
        1: (_ops.causal_fftconv1d_fp32_bhl_w_reshape, _ops.causal_fftconv1d_fp32_bhl),
    },
    "circular": {
        1: (_ops.circular_fftconv1d_fp32_bhl_w_reshape, _ops.circular_fftconv1d_fp32_bhl),
        2: (_ops.circular_fftconv2d_fp32_bhl_w_reshape, _ops.circular_fftconv2d_fp32_bhl),
        3: (_ops.circular_fftconv3d_fp32_bhl_w_reshape, _ops.circular_fftconv3d_fp32_bhl),
    },
}
# per-axis padding lists (ckconv_nd.py:832-850): the mixed ops with ``periodic`` bound
MIXED_FFT_FUNCTIONS = {
    1: (_ops.mixed_fftconv1d_fp32_bhl_w_reshape, _ops.mixed_fftconv1d_fp32_bhl),
    2: (_ops.mixed_fftconv2d_fp32_bhl_w_reshape, _ops.mixed_fftconv2d_fp32_bhl),
    3: (_ops.mixed_fftconv3d_fp32_bhl_w_reshape, _ops.mixed_fftconv3d_fp32_bhl),
}


def _is_tuple_mode(fft_padding) -> bool:
    return isinstance(fft_padding, Sequence) and not isinstance(fft_padding, (str, bytes))


def resolve_periodic(fft_padding, data_dim: int) -> tuple[bool, ...]:
    """Per-axis periodic flags of a CKConvND ``fft_padding`` ("zero", "circular" or a
    per-axis list of them)."""
    if _is_tuple_mode(fft_padding):
        modes = tuple(fft_padding)
        if len(modes) != data_dim:
            raise ValueError(f"fft_padding has {len(modes)} entries for data_dim={data_dim}.")
        for m in modes:
            if m not in ("zero", "circular"):
                raise ValueError(f"Unknown fft_padding mode {m!r}: use 'zero' or 'circular'.")
        return tuple(m == "circular" for m in modes)
    if fft_padding not in ("zero", "circular"):
        raise ValueError(f"Unknown fft_padding mode {fft_padding!r}: use 'zero' or 'circular'.")
    return (fft_padding == "circular",) * data_dim


def check_fft_backend(fft_backend: str) -> None:
    """ckconv_nd.py:628-630 with ``"b200"`` added to the allow-list."""
    assert fft_backend in BACKENDS, (
        f"Invalid fft_backend: {fft_backend!r}. Must be 'torch_fft', 'subq_ops' or 'b200'.")


def validate_ckconv_config(data_dim: int, fft_padding, grid_type, is_causal: bool = False,
                           use_chunked_fftconv: bool = False, fft_backend: str = FFT_BACKEND) -> None:
    """Constructor checks of CKConvND for ``fft_backend="b200"``.

    Raises the reference's exception types with its messages where the check is the
    reference's own (grid type, causal rank, circular constraints), and the
    backend-specific ones in the style of the ``subq_ops`` block (ckconv_nd.py:700-724).
    ``use_chunked_fftconv`` is accepted: the engine chunks channels by itself.
    """
    check_fft_backend(fft_backend)
    tuple_mode = isinstance(fft_padding, Sequence) and not isinstance(fft_padding, (str, bytes))
    if tuple_mode:
        if grid_type is not None:
            raise ValueError(
                "grid_type must be None (or omitted) when fft_padding is a per-axis list of mode strings. "
                f"Got grid_type={grid_type!r}, fft_padding={fft_padding!r}.")
    else:
        assert grid_type in ["double", "single"], (
            f"Invalid grid type: {grid_type}. Must be 'double' or 'single' when fft_padding is a single mode string.")
    if is_causal:
        assert data_dim == 1, f"Causal CKConvND only supports 1D inputs. Got {data_dim}D."
        if tuple_mode:
            raise ValueError(
                "is_causal=True is not supported with a per-axis fft_padding list. Use fft_padding='zero' "
                f"(single-mode string) for 1D causal. Got fft_padding={fft_padding!r}.")
        if fft_padding == "circular":
            raise ValueError(
                f"is_causal=True is incompatible with periodic FFT padding. Got fft_padding={fft_padding!r}.")
    if not tuple_mode and fft_padding == "circular":
        assert grid_type == "single", (
            "fft_padding='circular' requires grid_type='single' (kernel size equals input size).")
    if fft_backend != FFT_BACKEND:
        return
    assert data_dim in (1, 2, 3), f"fft_backend='b200' only supports data_dim in (1, 2, 3). Got data_dim={data_dim}."
    resolve_periodic(fft_padding, data_dim)  # zero / circular per axis (lengths checked per call)
    del use_chunked_fftconv


def _bind_periodic(op_fn, periodic):
    def _wrapped(x, kernel, shortcut):
        return op_fn(x, kernel, periodic, shortcut)

    return _wrapped


def select_fftconv_fns(data_dim: int, is_causal: bool, fft_padding="zero"):
    """(fftconv_fn, fftconv_fn_bhl_input) for this backend (ckconv_nd.py:796-871): causal,
    zero-padded or circular ops for a single padding mode, the mixed ops with the per-axis
    flags bound for a per-axis list."""
    if _is_tuple_mode(fft_padding) and not is_causal:
        per = resolve_periodic(fft_padding, data_dim)
        try:
            fn_blh, fn_bhl = MIXED_FFT_FUNCTIONS[data_dim]
        except KeyError:
            raise ValueError(f"Mixed-BC FFT conv not implemented for data_dim={data_dim}. "
                             f"Valid: {sorted(MIXED_FFT_FUNCTIONS)}") from None
        return _bind_periodic(fn_blh, per), _bind_periodic(fn_bhl, per)
    mode = "causal" if is_causal else ("circular" if fft_padding == "circular" else "zero")
    table = FFT_FUNCTIONS[mode]
    try:
        return table[data_dim]
    except KeyError:
        raise ValueError(
            f"Unsupported configuration: fft_padding='{mode}', data_dim={data_dim}. "
            f"Valid dimensions: {sorted(table)}") from None


def apply_convolution(fns, x: torch.Tensor, conv_kernel: torch.Tensor, shortcut: torch.Tensor,
                      is_bhl_input: bool) -> torch.Tensor:
    """ckconv_nd.py:1006-1062. ``conv_kernel`` is channels-last ``[1|B, *K, C]``."""
    fn_blh, fn_bhl = fns
    if is_bhl_input:
        return fn_bhl(x, conv_kernel.movedim(-1, 1), shortcut)
    return fn_blh(x, conv_kernel, shortcut)


def ckconv_kernel(global_conv, spatial_dims, cp_group=None, **mixer_kwargs):
    """The BHL kernel ``[1|B, C, *K]`` and shortcut ``[C]`` a reference ``CKConvND``
    would hand to its op for inputs of ``spatial_dims`` (ckconv_nd.py:1143-1188).

    ``global_conv`` is duck-typed: ``kernel``, ``mask``, ``is_causal``, ``shortcut``,
    ``grid_type`` and ``_periodic_per_axis`` as CKConvND defines them: a single grid on
    every axis for ``grid_type == "single"``, per axis on the periodic axes when
    ``grid_type`` is None (per-axis padding, ckconv_nd.py:406-440, :1143-1148)."""
    grid_type = getattr(global_conv, "grid_type", "double")
    per = getattr(global_conv, "_periodic_per_axis", None) or (False,) * len(spatial_dims)
    single = tuple(per) if grid_type is None else (grid_type == "single",) * len(spatial_dims)
    grid_lens = [(n + 1) // 2 if s else n for n, s in zip(spatial_dims, single)]
    conv_kernel, grid = global_conv.kernel(grid_lens, conditioning=mixer_kwargs.get("conditioning"))
    if not isinstance(global_conv.mask, torch.nn.Identity):
        conv_kernel = global_conv.mask(grid=grid, x=conv_kernel)
    if global_conv.is_causal:
        conv_kernel = conv_kernel[..., conv_kernel.shape[-2] // 2:, :]
    shortcut = global_conv.shortcut
    if cp_group is not None and cp_group.size() > 1:
        if global_conv.is_causal:
            raise ValueError("Causal CKConvND has not been verified to work with context parallelism.")
        d = conv_kernel.shape[-1] // cp_group.size()
        lo = cp_group.rank() * d
        conv_kernel = conv_kernel[..., lo:lo + d]
        shortcut = shortcut[lo:lo + d]
    return conv_kernel.movedim(-1, 1), shortcut


def _short_conv_spec(sc):
    """(kernel extents, causal, weight_fn, bias_fn) of a reference short conv the fused
    kernels cover, else None. weight_fn() -> [3C, 1, *k]; bias_fn() -> [3C] or None."""
    name = type(sc).__name__
    if name.startswith("DistributedDepthwiseConv"):
        # weights [num_groups, *k] shared by group_dim consecutive channels
        # (distributed_depthwise_conv_nd.py:150-164, :316-328, :452-465)
        ks = tuple(sc.weight.shape[1:])
        causal = bool(getattr(sc, "causal", False))
        if causal and len(ks) != 1:
            return None
        rep = int(getattr(sc, "group_dim", 1))

        def weight_fn():
            w = sc.weight.repeat_interleave(rep, dim=0) if rep > 1 else sc.weight
            return w.unsqueeze(1)

        def bias_fn():
            b = sc.bias
            return None if b is None else (b.repeat_interleave(rep, dim=0) if rep > 1 else b)

        return ks, causal, weight_fn, bias_fn
    if not isinstance(sc, (torch.nn.Conv1d, torch.nn.Conv2d, torch.nn.Conv3d)):
        return None
    w = sc.weight
    if sc.groups != w.shape[0] or w.shape[1] != 1 or sc.in_channels != sc.out_channels:
        return None  # not depthwise
    if any(s != 1 for s in sc.dilation) or any(s != 1 for s in sc.stride):
        return None
    ks = tuple(w.shape[2:])
    if name == "CausalConv1D":  # pads in forward (causal_conv1d.py:113-143)
        causal = bool(sc.is_causal)
        if not causal and any(k % 2 == 0 for k in ks):
            return None
    else:
        causal = False
        pad = sc.padding
        if sc.padding_mode != "zeros":
            return None
        if pad != "same" and not all(k % 2 == 1 and p == k // 2 for p, k in zip(pad, ks)):
            return None  # only centred ("same") short convs
    return ks, causal, (lambda: sc.weight), (lambda: sc.bias)


def fused_mixer_config(mixer) -> dict | None:
    """The fused-mixer settings for a reference ``Hyena`` instance, or None when the
    instance needs the unfused composition (a norm that is not Identity, another gate,
    a short conv the fused kernels do not cover, or a global conv on another backend).

    Returned keys: ``gate1``, ``gate2``, ``causal``, ``short_k`` (tuple or None),
    ``short_causal``, ``short_weight`` / ``short_bias`` (callables returning the
    ``[3C, 1, *k]`` weight and the ``[3C]`` bias or None)."""
    gc = getattr(mixer, "global_conv", None)
    if gc is None or getattr(gc, "fft_backend", None) != FFT_BACKEND:
        return None
    for name in ("pixelhyena_norm", "output_norm", "q_norm", "k_norm"):
        m = getattr(mixer, name, None)
        if m is not None and not isinstance(m, torch.nn.Identity):
            return None
    try:
        g1 = gate_name(mixer.gate_nonlinear)
        g2 = gate_name(mixer.gate_nonlinear_2)
    except NotImplementedError:
        return None
    per = tuple(getattr(gc, "_periodic_per_axis", None) or ())
    cfg = dict(gate1=g1, gate2=g2, causal=bool(gc.is_causal), short_k=None, short_causal=bool(gc.is_causal),
               short_weight=lambda: None, short_bias=lambda: None, periodic=per if any(per) else None)
    sc = mixer.short_conv
    if isinstance(sc, torch.nn.Identity):
        return cfg
    spec = _short_conv_spec(sc)
    if spec is None:
        return None
    cfg["short_k"], cfg["short_causal"], cfg["short_weight"], cfg["short_bias"] = spec
    return cfg


class FusedHyena(torch.nn.Module):
    """Runs a reference ``Hyena`` instance (same parameters, same call signature
    ``forward(query, key, value, cp_group=None, **mixer_kwargs)``, hyena_nd.py:432) on the
    fused kernels; raises ``NotImplementedError`` for instances ``fused_mixer_config``
    rejects. Under context parallelism the inputs hold this rank's zigzag chunks of the
    first spatial axis, as in the reference."""

    def __init__(self, mixer):
        super().__init__()
        cfg = fused_mixer_config(mixer)
        if cfg is None:
            raise NotImplementedError("this Hyena configuration is not covered by the fused b200 mixer")
        self.mixer = mixer
        self._cfg = cfg
        self.gate1, self.gate2 = cfg["gate1"], cfg["gate2"]
        self.causal, self.short_causal = cfg["causal"], cfg["short_causal"]
        self.periodic = cfg["periodic"]

    @property
    def shortcut(self):
        return self.mixer.global_conv.shortcut

    @property
    def short_weight(self):
        return self._cfg["short_weight"]()

    @property
    def short_bias(self):
        return self._cfg["short_bias"]()

    def forward(self, query, key, value, cp_group=None, **mixer_kwargs):
        from .hyena import hyena_fused

        spatial = list(query.shape[1:-1])
        cp = cp_group is not None and cp_group.size() > 1
        if cp:
            spatial[0] *= cp_group.size()  # the kernel covers the full sequence
        filt, _ = ckconv_kernel(self.mixer.global_conv, spatial, None, **mixer_kwargs)
        if cp:
            from .cp import hyena_context_parallel

            return hyena_context_parallel(self, query, key, value, filt, cp_group)
        return hyena_fused(query, key, value, filt, self.shortcut.to(query.dtype), self.short_weight,
                           self.short_bias, causal=self.causal, short_causal=self.short_causal,
                           gate1=self.gate1, gate2=self.gate2, periodic=self.periodic)
