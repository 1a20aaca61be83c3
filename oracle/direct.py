"""Independent float64 direct (spatial) convolution — TEST INFRASTRUCTURE ONLY.

Used to check the FFT restatement in ``oracle/fftconv.py`` on tiny shapes,
the same known-answer method the reference's own tests use (spatial depthwise
conv with a flipped kernel, ``tests/ops/test_fftconv.py:68-99``): a linear
convolution ``y[n] = sum_m x[m] k[n + c - m]`` with ``c = K//2`` per axis for the
"same" (non-causal) form and ``c = 0`` for the causal form.

Pure numpy loops over kernel taps; only for small inputs.
"""

from __future__ import annotations

import itertools

import numpy as np


def direct_conv(x: np.ndarray, kernel: np.ndarray, causal: bool = False) -> np.ndarray:
    """x: [B, H, *S]; kernel: [1|B, H, *K]; returns float64 [B, H, *S]."""
    x = np.asarray(x, dtype=np.float64)
    kernel = np.asarray(kernel, dtype=np.float64)
    nd = x.ndim - 2
    S = x.shape[2:]
    K = kernel.shape[2:]
    c = (0,) * nd if causal else tuple(k // 2 for k in K)
    y = np.zeros_like(x)
    kb = np.broadcast_to(kernel, (x.shape[0], x.shape[1]) + K)
    for tap in itertools.product(*[range(k) for k in K]):
        # y[n] += k[tap] * x[n + c - tap]
        shift = tuple(ci - ti for ci, ti in zip(c, tap))
        src, dst = [], []
        ok = True
        for s, n in zip(shift, S):
            lo = max(0, -s)
            hi = min(n, n - s)
            if hi <= lo:
                ok = False
                break
            dst.append(slice(lo, hi))
            src.append(slice(lo + s, hi + s))
        if not ok:
            continue
        w = kb[(slice(None), slice(None)) + tap]
        w = w.reshape(w.shape + (1,) * nd)
        y[(slice(None), slice(None)) + tuple(dst)] += w * x[(slice(None), slice(None)) + tuple(src)]
    return y
