"""CPU tests of the ``fft_backend="b200"`` selection logic (no kernels run).

Mirrors the reference's constructor-rejection tests for a CUDA backend
(tests/modules/test_ckconv_nd_subq.py:215-271) for the checks this backend keeps, and
checks which reference ``Hyena`` configurations the fused mixer accepts.
"""

import pytest
import torch

from nvsubquadratic_b200 import backend, fftconv


def test_accepts_supported_configs():
    backend.validate_ckconv_config(1, "zero", "double", is_causal=True)
    backend.validate_ckconv_config(1, "zero", "double", is_causal=False)  # non-causal 1D is wired here
    backend.validate_ckconv_config(2, "zero", "double")
    backend.validate_ckconv_config(3, "zero", "double", use_chunked_fftconv=True)
    backend.validate_ckconv_config(2, "circular", "single", fft_backend="torch_fft")  # other backends untouched


def test_rejects_invalid_backend():
    with pytest.raises(AssertionError, match="Invalid fft_backend"):
        backend.validate_ckconv_config(2, "zero", "double", fft_backend="not_a_backend")


def test_accepts_circular_and_per_axis_padding():
    backend.validate_ckconv_config(2, "circular", "single")
    backend.validate_ckconv_config(3, ["circular", "circular", "zero"], None)
    assert backend.resolve_periodic(["zero", "circular"], 2) == (False, True)
    assert backend.resolve_periodic("circular", 3) == (True, True, True)
    with pytest.raises(ValueError, match="Unknown fft_padding"):
        backend.validate_ckconv_config(2, ["zero", "reflect"], None)
    with pytest.raises(AssertionError, match="requires grid_type='single'"):
        backend.validate_ckconv_config(2, "circular", "double")
    with pytest.raises(ValueError, match="incompatible with periodic"):
        backend.validate_ckconv_config(1, "circular", "single", is_causal=True)


def test_rejects_causal_with_2d():
    with pytest.raises(AssertionError, match="Causal CKConvND only supports 1D"):
        backend.validate_ckconv_config(2, "zero", "double", is_causal=True)


def test_rejects_per_axis_padding_misuse():
    with pytest.raises(ValueError, match="not supported with a per-axis"):
        backend.validate_ckconv_config(1, ["zero"], None, is_causal=True)
    with pytest.raises(ValueError, match="grid_type must be None"):
        backend.validate_ckconv_config(2, ["zero", "circular"], "double")


def test_rejects_data_dim_4_and_bad_grid():
    with pytest.raises(AssertionError, match=r"only supports data_dim in \(1, 2, 3\)"):
        backend.validate_ckconv_config(4, "zero", "double")
    with pytest.raises(AssertionError, match="Invalid grid type"):
        backend.validate_ckconv_config(2, "zero", "triple")


def test_function_binding():
    assert backend.select_fftconv_fns(1, True) == (fftconv.causal_fftconv1d_fp32_bhl_w_reshape,
                                                   fftconv.causal_fftconv1d_fp32_bhl)
    for nd in (1, 2, 3):
        blh, bhl = backend.select_fftconv_fns(nd, False)
        assert bhl is getattr(fftconv, f"fftconv{nd}d_fp32_bhl")
        assert blh is getattr(fftconv, f"fftconv{nd}d_fp32_bhl_w_reshape")
    with pytest.raises(ValueError, match="Valid dimensions"):
        backend.select_fftconv_fns(2, True)
    for nd in (1, 2, 3):
        blh, bhl = backend.select_fftconv_fns(nd, False, "circular")
        assert bhl is getattr(fftconv, f"circular_fftconv{nd}d_fp32_bhl")
    blh, bhl = backend.select_fftconv_fns(2, False, ["circular", "zero"])
    assert callable(blh) and callable(bhl)


class _GlobalConv(torch.nn.Module):
    def __init__(self, C, is_causal=False, fft_backend="b200"):
        super().__init__()
        self.fft_backend = fft_backend
        self.is_causal = is_causal
        self.mask = torch.nn.Identity()
        self.shortcut = torch.nn.Parameter(torch.randn(C))


class _Mixer(torch.nn.Module):
    def __init__(self, C, nd=2, short_conv=None, gate=torch.nn.SiLU(), gate2=None, **gc):
        super().__init__()
        self.global_conv = _GlobalConv(C, **gc)
        self.short_conv = short_conv if short_conv is not None else torch.nn.Identity()
        self.gate_nonlinear = gate
        self.gate_nonlinear_2 = gate2 if gate2 is not None else gate
        self.pixelhyena_norm = torch.nn.Identity()
        self.output_norm = torch.nn.Identity()
        self.q_norm = None
        self.k_norm = None


def test_fused_mixer_config_accepts_and_rejects():
    C = 8
    conv = torch.nn.Conv2d(3 * C, 3 * C, 3, padding=1, groups=3 * C, bias=True)
    cfg = backend.fused_mixer_config(_Mixer(C, short_conv=conv, gate2=torch.nn.Sigmoid()))
    assert cfg["gate1"] == "silu" and cfg["gate2"] == "sigmoid" and cfg["short_k"] == (3, 3)
    assert not cfg["short_causal"] and cfg["short_bias"]() is conv.bias
    conv_same = torch.nn.Conv2d(3 * C, 3 * C, 3, padding="same", groups=3 * C, bias=False)
    assert backend.fused_mixer_config(_Mixer(C, short_conv=conv_same))["short_bias"]() is None
    assert backend.fused_mixer_config(_Mixer(C))["short_k"] is None
    # rejections: another backend, a norm, another gate, a non-depthwise conv, even "same" with padding 0
    assert backend.fused_mixer_config(_Mixer(C, fft_backend="torch_fft")) is None
    m = _Mixer(C)
    m.output_norm = torch.nn.LayerNorm(C)
    assert backend.fused_mixer_config(m) is None
    assert backend.fused_mixer_config(_Mixer(C, gate=torch.nn.GELU())) is None
    assert backend.fused_mixer_config(_Mixer(C, short_conv=torch.nn.Conv2d(3 * C, 3 * C, 3, padding=1))) is None
    assert backend.fused_mixer_config(
        _Mixer(C, short_conv=torch.nn.Conv2d(3 * C, 3 * C, 3, padding=0, groups=3 * C))) is None
    with pytest.raises(NotImplementedError):
        backend.FusedHyena(_Mixer(C, gate=torch.nn.GELU()))


def test_ckconv_kernel_causal_crop_and_cp_slice():
    C, L = 4, 6

    class Gen(torch.nn.Module):
        def forward(self, grid_lens, conditioning=None):
            n = grid_lens[0]
            k = torch.arange(C * (2 * n - 1), dtype=torch.float32).reshape(1, 2 * n - 1, C)
            return k, None

    gc = _GlobalConv(C, is_causal=True)
    gc.kernel = Gen()
    filt, D = backend.ckconv_kernel(gc, [L])
    full, _ = Gen()([L])
    assert torch.equal(filt, full[:, (2 * L - 1) // 2:, :].movedim(-1, 1))
    assert D is gc.shortcut

    class G2:
        def size(self):
            return 2

        def rank(self):
            return 1

    gc.is_causal = False
    filt, D = backend.ckconv_kernel(gc, [L], G2())
    assert torch.equal(filt, full[..., 2:4].movedim(-1, 1)) and torch.equal(D, gc.shortcut[2:4])
