"""GPU tests of hyfft_conv_forward_static_scratch, the forward conv that runs on the
library's fixed device scratch instead of a caller workspace.

Each case calls it twice in a row through the C ABI and compares both outputs with
hyfft_conv_forward (caller workspace) on the same inputs, then once more on fresh
inputs; some cases are large enough to be split into several channel chunks (one of
them a 128 x 128 grid that the workspace entry point runs on its large-grid kernels),
and one is too large for the scratch and must be refused before anything runs. The file is
collected last and also passes alone in a fresh process.
"""

import ctypes

import pytest
import torch

from nvsubquadratic_b200 import _lib
from nvsubquadratic_b200.fftconv import _conv_desc, _workspace_sizes
from tests.conftest import rel_l2

pytestmark = pytest.mark.gpu

BHL, BLH = 0, 1
SCRATCH_MAX = 32 << 20

CASES = [
    # B, H, spatial, kernel, kernel_batch, causal, dtype, layout, shortcut
    (2, 8, (4096,), (4096,), 1, True, torch.float32, BHL, True),
    (3, 16, (32, 24), (63, 47), 1, False, torch.bfloat16, BHL, True),
    (2, 8, (8, 8, 8), (15, 15, 15), 2, False, torch.float32, BLH, False),
    # 2 MiB of spectra per channel: 24 channels run as chunks of 15 and 9
    (2, 24, (65536,), (65536,), 1, False, torch.float32, BHL, True),
    # shapes the workspace entry point sends to its large-grid 2D kernels (F = 256 x 256,
    # N <= 128, shared kernel); here they run the pass chain: 1 MiB of spectra per
    # channel, so 4 channels fit one chunk and 64 channels run as chunks of 31, 31, 2
    (2, 4, (128, 128), (128, 128), 1, False, torch.bfloat16, BLH, True),
    (2, 64, (128, 128), (128, 128), 1, False, torch.float32, BHL, True),
]


def _inputs(case, seed):
    B, H, S, K, kB, causal, dt, layout, with_skip = case
    g = torch.Generator().manual_seed(seed)
    xs = (B, H) + S if layout == BHL else (B,) + S + (H,)
    ks = (kB, H) + K if layout == BHL else (kB,) + K + (H,)
    x = torch.randn(xs, generator=g).to(dt).cuda()
    k = (torch.randn(ks, generator=g) / (torch.tensor(K).prod() ** 0.5)).cuda()
    skip = torch.randn(H, generator=g).to(dt).cuda() if with_skip else None
    return x, k, skip


def _with_workspace(desc, x, k, skip):
    lib = _lib.load()
    wf, _ = _workspace_sizes(desc)
    ws = _lib.workspace(wf, x.device)
    y = torch.empty_like(x)
    rc = lib.hyfft_conv_forward(ctypes.byref(desc), x.data_ptr(), k.data_ptr(), _lib.ptr(skip), y.data_ptr(),
                                ws.data_ptr(), ws.numel(), _lib.stream_ptr(x.device))
    _lib.check(rc, "hyfft_conv_forward")
    return y


def _static(desc, x, k, skip):
    lib = _lib.load()
    y = torch.empty_like(x)
    rc = lib.hyfft_conv_forward_static_scratch(ctypes.byref(desc), x.data_ptr(), k.data_ptr(), _lib.ptr(skip),
                                               y.data_ptr(), _lib.stream_ptr(x.device))
    _lib.check(rc, "hyfft_conv_forward_static_scratch")
    return y


@pytest.mark.parametrize("case", CASES, ids=[f"{len(c[2])}d-{c[2][0]}-H{c[1]}-{c[6]}" for c in CASES])
def test_static_scratch_matches_workspace_entry_point(case):
    B, H, S, K, kB, causal, dt, layout, _ = case
    desc = _conv_desc(B, H, S, K, kB, causal, dt, layout)
    tol = 1e-5 if dt == torch.float32 else 2e-2
    x, k, skip = _inputs(case, 0)
    ref = _with_workspace(desc, x, k, skip)
    first = _static(desc, x, k, skip)
    second = _static(desc, x, k, skip)
    torch.cuda.synchronize()
    assert rel_l2(ref, first) <= tol
    assert rel_l2(ref, second) <= tol
    # fresh inputs: nothing carried over from the previous calls' scratch contents
    x2, k2, skip2 = _inputs(case, 1)
    ref2 = _with_workspace(desc, x2, k2, skip2)
    third = _static(desc, x2, k2, skip2)
    torch.cuda.synchronize()
    assert rel_l2(ref2, third) <= tol


def test_static_scratch_refuses_problems_beyond_its_size():
    # one channel of a 2^21-point non-causal conv needs 2 x 32 MiB of spectra
    n = 1 << 21
    desc = _conv_desc(1, 1, (n,), (n,), 1, False, torch.float32, BHL)
    x = torch.zeros(16, device="cuda")
    lib = _lib.load()
    rc = lib.hyfft_conv_forward_static_scratch(ctypes.byref(desc), x.data_ptr(), x.data_ptr(), None, x.data_ptr(),
                                               _lib.stream_ptr(x.device))
    assert rc == 3  # HYFFT_ERR_WORKSPACE
    msg = lib.hyfft_last_error().decode()
    assert "static scratch holds" in msg and str(SCRATCH_MAX) in msg
    torch.cuda.synchronize()
    assert torch.count_nonzero(x) == 0
