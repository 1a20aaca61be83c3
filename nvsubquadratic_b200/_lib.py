"""ctypes binding of ``libhyfft.so`` (the C ABI declared in ``include/hyfft.h``).

This is the Python-side equivalent of the FFI a maintainer would add to
nvSubquadratic for the new backend. There is no CPU fallback: if the shared
library is missing or the tensors are not on a CUDA device, calls raise.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
_LIB_PATH = _PKG / "libhyfft.so"

HYFFT_OK = 0
HYFFT_ERR_INVALID = 1
HYFFT_ERR_UNSUPPORTED = 2
HYFFT_ERR_WORKSPACE = 3
HYFFT_ERR_CUDA = 4

F32, BF16, F16 = 0, 1, 2
LAYOUT_BHL, LAYOUT_BLH = 0, 1
GATE_IDENTITY, GATE_SIGMOID, GATE_SILU = 0, 1, 2

DTYPE_CODE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}
GATE_CODE = {"identity": GATE_IDENTITY, "sigmoid": GATE_SIGMOID, "silu": GATE_SILU}


class ConvDesc(ctypes.Structure):
    _fields_ = [
        ("ndim", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("channels", ctypes.c_int32),
        ("n", ctypes.c_int32 * 3),
        ("k", ctypes.c_int32 * 3),
        ("kernel_batch", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("layout", ctypes.c_int32),
        ("periodic", ctypes.c_int32),
    ]


class HyenaDesc(ctypes.Structure):
    _fields_ = [
        ("ndim", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("channels", ctypes.c_int32),
        ("n", ctypes.c_int32 * 3),
        ("k", ctypes.c_int32 * 3),
        ("causal", ctypes.c_int32),
        ("short_k", ctypes.c_int32 * 3),
        ("short_causal", ctypes.c_int32),
        ("short_bias", ctypes.c_int32),
        ("gate1", ctypes.c_int32),
        ("gate2", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("in_batch_stride", ctypes.c_int64),
        ("in_pos_stride", ctypes.c_int64),
        ("out_batch_stride", ctypes.c_int64),
        ("out_pos_stride", ctypes.c_int64),
        ("periodic", ctypes.c_int32),
    ]


_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32

# name -> argtypes (restype is int unless listed in _STR_FUNCS)
class SirenDesc(ctypes.Structure):
    _fields_ = [
        ("ndim", ctypes.c_int32),
        ("n", ctypes.c_int32 * 3),
        ("embedding", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("num_hidden", ctypes.c_int32),
        ("channels", ctypes.c_int32),
        ("layout", ctypes.c_int32),
    ]


SIGNATURES = {
    "hyfft_conv_workspace_size": [ctypes.POINTER(ConvDesc), ctypes.POINTER(_sz), ctypes.POINTER(_sz)],
    "hyfft_conv_forward": [ctypes.POINTER(ConvDesc), _vp, _vp, _vp, _vp, _vp, _sz, _vp],
    "hyfft_conv_forward_static_scratch": [ctypes.POINTER(ConvDesc), _vp, _vp, _vp, _vp, _vp],
    "hyfft_conv_backward": [ctypes.POINTER(ConvDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp],
    "hyfft_hyena_workspace_size": [ctypes.POINTER(HyenaDesc), ctypes.POINTER(_sz), ctypes.POINTER(_sz),
                                   ctypes.POINTER(_sz)],
    "hyfft_hyena_forward": [ctypes.POINTER(HyenaDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp],
    "hyfft_hyena_backward": [ctypes.POINTER(HyenaDesc), _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                             _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp],
    "hyfft_cp_pack_split_to_full": [_vp, _vp, _i64, _i64, _i64, _i64, _i32, _i32, _vp],
    "hyfft_cp_unpack_split_to_full": [_vp, _vp, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _vp],
    "hyfft_cp_pack_full_to_split": [_vp, _vp, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _vp],
    "hyfft_cp_unpack_full_to_split": [_vp, _vp, _i64, _i64, _i64, _i64, _i32, _i32, _vp],
    "hyfft_cp_permute_cl": [_vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i32, _i32, _i32, _vp],
    "hyfft_cp_permute_cl_window": [_vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _i32, _i64, _i64, _i32, _vp],
    "hyfft_causal_conv1d_forward": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp],
    "hyfft_causal_conv1d_backward": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp],
    "hyfft_siren_sizes": [ctypes.POINTER(SirenDesc), ctypes.POINTER(_sz), ctypes.POINTER(_sz)],
    "hyfft_siren_forward": [ctypes.POINTER(SirenDesc)] + [_vp] * 10 + [_sz, _vp],
    "hyfft_siren_backward": [ctypes.POINTER(SirenDesc)] + [_vp] * 16 + [_sz, _vp],
    "hyfft_last_error": [],
    "hyfft_version": [],
    "hyfft_launch_count": [],
}
_STR_FUNCS = {"hyfft_last_error", "hyfft_version"}

_lib = None
_lock = threading.Lock()


def library_path() -> Path:
    return Path(os.environ.get("HYFFT_LIBRARY", str(_LIB_PATH)))


def load() -> ctypes.CDLL:
    """Load libhyfft.so once; raise ImportError if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise ImportError(
                f"{path} not found: build the CUDA backend first "
                "(python -m nvsubquadratic_b200.build). There is no CPU fallback."
            )
        lib = ctypes.CDLL(str(path))
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_char_p if name in _STR_FUNCS else ctypes.c_int
        lib.hyfft_launch_count.restype = ctypes.c_longlong
        _lib = lib
        return lib


class HyfftError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc == HYFFT_OK:
        return
    msg = load().hyfft_last_error().decode(errors="replace")
    if rc == HYFFT_ERR_INVALID:
        raise AssertionError(f"{what}: {msg}")
    if rc == HYFFT_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise HyfftError(f"{what} failed (status {rc}): {msg}")


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "the b200 FFT-conv backend runs on CUDA tensors only (got a tensor on "
                f"{t.device}); there is no CPU fallback"
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    if dev is None:
        raise RuntimeError("no CUDA tensor given")
    return dev


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def launch_count() -> int:
    """Kernels launched through libhyfft.so by this process so far."""
    return int(load().hyfft_launch_count())
