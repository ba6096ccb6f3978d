"""Seeded synthetic inputs of the five benchmark configurations (test helper).

Each generator draws from ``np.random.default_rng(seed)`` (seed 0 by default)
in the order the configuration text gives: X, then weights, then noise, then
masks. ``n`` may be smaller than the configuration's row count (a slice with
the same shape per row and the same distributions); everything is float32.

  c1  20,000 x 20 N(0,1); y = sin x0 + x1 x2 + 0.5 x3^2 + sum_{4..9} 0.2 x_j + N(0, 0.1^2)
  c2  100,000 x 50 N(0,1), the last 10 columns replaced by integers(0, 8);
      logit = 0.8 x0 - 0.5 x1 + x2 x3 + 0.3 sum_{4..14} x_j; y ~ Bernoulli(sigmoid(logit))
  c3  1,000,000 x 100: 80 N(0,1) columns, 20 lognormal(0,1) columns;
      y = sum_{j<20} w_j x_j + 0.5 x20 x21 + N(0, 0.5^2), w ~ N(0,1) (from the NaN-free
      values), then 5% of the entries of every column set to NaN
  c4  10,000,000 x 200: within each block of 10 columns X = sqrt(0.7) Z + sqrt(0.3) z_block
      (pairwise correlation 0.3); y = sum_{j<50} w_j tanh x_j + sum_{k<10} x_{2k} x_{2k+1} + N(0,1)
  c5  5,000,000 x 128 N(0,1) with 30% exact zeros per column; 10 classes,
      s_c = X W_c + 0.2 x_c x_{c+10}, W_c ~ N(0, 0.3^2); y = argmax_c(s_c + Gumbel)
"""

from __future__ import annotations

import numpy as np

ROWS = {"c1": 20_000, "c2": 100_000, "c3": 1_000_000, "c4": 10_000_000, "c5": 5_000_000}
COLS = {"c1": 20, "c2": 50, "c3": 100, "c4": 200, "c5": 128}


def make(cfg: str, n: int | None = None, seed: int = 0, classes: int = 10):
    """(X (n, F) float32, y (n,) float32) of configuration ``cfg``."""
    n = ROWS[cfg] if n is None else int(n)
    F = COLS[cfg]
    rng = np.random.default_rng(seed)
    f32 = np.float32
    if cfg == "c1":
        X = rng.standard_normal((n, F), dtype=f32)
        y = (np.sin(X[:, 0]) + X[:, 1] * X[:, 2] + f32(0.5) * X[:, 3] ** 2
             + f32(0.2) * X[:, 4:10].sum(axis=1, dtype=f32))
        y = y + f32(0.1) * rng.standard_normal(n, dtype=f32)
    elif cfg == "c2":
        X = rng.standard_normal((n, F), dtype=f32)
        X[:, F - 10:] = rng.integers(0, 8, size=(n, 10)).astype(f32)
        logit = (f32(0.8) * X[:, 0] - f32(0.5) * X[:, 1] + X[:, 2] * X[:, 3]
                 + f32(0.3) * X[:, 4:15].sum(axis=1, dtype=f32))
        p = 1.0 / (1.0 + np.exp(-logit.astype(np.float64)))
        y = (rng.random(n) < p).astype(f32)
    elif cfg == "c3":
        X = np.empty((n, F), f32)
        X[:, :80] = rng.standard_normal((n, 80), dtype=f32)
        X[:, 80:] = rng.lognormal(0.0, 1.0, size=(n, 20)).astype(f32)
        w = rng.standard_normal(20, dtype=f32)
        y = X[:, :20] @ w + f32(0.5) * X[:, 20] * X[:, 21]
        y = y + f32(0.5) * rng.standard_normal(n, dtype=f32)
        X[rng.random((n, F)) < 0.05] = np.nan
    elif cfg == "c4":
        X = rng.standard_normal((n, F), dtype=f32)
        X *= f32(np.sqrt(0.7))
        zb = rng.standard_normal((n, F // 10), dtype=f32) * f32(np.sqrt(0.3))
        X.reshape(n, F // 10, 10)[...] += zb[:, :, None]
        del zb
        w = rng.standard_normal(50, dtype=f32)
        y = np.tanh(X[:, :50]) @ w
        for k in range(10):
            y += X[:, 2 * k] * X[:, 2 * k + 1]
        y = y + rng.standard_normal(n, dtype=f32)
    elif cfg == "c5":
        X = rng.standard_normal((n, F), dtype=f32)
        X[rng.random((n, F)) < 0.3] = 0.0
        W = rng.standard_normal((F, classes), dtype=f32) * f32(0.3)
        s = X @ W + f32(0.2) * X[:, :classes] * X[:, 10:10 + classes]
        gumbel = -np.log(-np.log(rng.random((n, classes)).clip(1e-12, 1 - 1e-7))).astype(f32)
        y = np.argmax(s + gumbel, axis=1).astype(f32)
    else:
        raise ValueError(cfg)
    return np.ascontiguousarray(X), np.ascontiguousarray(y, dtype=f32)
