"""Tolerances used by the GPU parity tests.

Quantised linear outputs (GEMV / GEMM, fp32 accumulation) must be within 1e-2
relative of the oracle's dequantise-then-matmul: the relative L2 error and the
max abs error normalised by max |y_ref| are both <= 1e-2.
"""

import numpy as np

LINEAR_RTOL = 1e-2
SALIENCE_RTOL = 1e-3


def assert_linear_close(y, y_ref, rtol=LINEAR_RTOL, what=""):
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    assert y.shape == y_ref.shape, (y.shape, y_ref.shape)
    scale = max(np.abs(y_ref).max(), 1e-30)
    l2 = np.linalg.norm(y - y_ref) / max(np.linalg.norm(y_ref), 1e-30)
    mx = np.abs(y - y_ref).max() / scale
    assert l2 <= rtol and mx <= rtol, f"{what}: rel L2 {l2:.3e}, max/maxref {mx:.3e}"
    return l2, mx
