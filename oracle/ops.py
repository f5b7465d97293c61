"""Per-op CPU restatements of the reference C engine's math (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Each function names the
reference code it restates.  Dot products are accumulated in float64 so the
oracle is at least as accurate as the reference's fp32 accumulation; the parity
bar for fp32-accumulated GPU outputs is relative L2 <= 1e-3.
"""
from __future__ import annotations

import numpy as np

from . import formats as F


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def gemv(w_raw: np.ndarray, qt: int, x: np.ndarray, n_rows: int, n_cols: int) -> np.ndarray:
    """out[b][r] = sum_k W[r][k] * x[b][k] with W decoded exactly (float64 accumulate).

    The math every *_matmul_omp / *_batch_matmul of the reference computes where it is
    correct (quant_kernels_omp.c:135-734, cengine_batch_instr.c:68-534): x [B][K],
    out [B][N] (cengine_batch_instr.c:251)."""
    w = F.dequantize(qt, w_raw, n_rows * n_cols).reshape(n_rows, n_cols).astype(np.float64)
    xb = np.asarray(x, np.float64).reshape(-1, n_cols)
    return (xb @ w.T).astype(np.float32)
