"""Oracle restatement of the quantile binner (test infrastructure only).

Restates ``Binner`` of yabt/binning.py:12-129 (numpy branch). The quantile
edges are computed here with an explicit sort + 'linear' (Hyndman-Fan type 7)
interpolation written out operation by operation, so that the exact float
arithmetic the CUDA binning kernel must reproduce is visible in one place.
``tests/test_oracle.py`` pins this restatement against ``np.quantile`` and the
golden vectors produced by the reference itself.

Arithmetic of one quantile q = k/256 on a sorted float32 column s of length m
(numpy ``_quantile`` with method='linear'):
    v   = (m - 1) * q                        float64, exact (q is dyadic)
    lo  = floor(v); hi = lo + 1; if v >= m-1: lo = hi = m-1
    t   = v - lo                             float64
    d   = s[hi] - s[lo]                      float32 subtraction
    out = s[lo] + float64(d) * t             if t <  0.5
          s[hi] - float64(d) * (1 - t)       if t >= 0.5
    edge = float32(out)
Edges are then de-duplicated (sorted unique), yabt/binning.py:60.
"""

from __future__ import annotations

import numpy as np

MAX_BINS = 256
QUANTILE_SAMPLE = 200_000  # yabt/binning.py:36-38


def quantile_sorted(s: np.ndarray, q: np.ndarray) -> np.ndarray:
    """Linear-interpolated quantiles of an already sorted float32 column.

    Returns float64 values (before the float32 cast), numpy's arithmetic."""
    m = s.shape[0]
    v = (m - 1) * q.astype(np.float64)
    lo = np.floor(v)
    top = v >= m - 1
    # numpy marks an index at/after the last element as -1 (the last element)
    # and takes the interpolation weight against that -1, i.e. t = v + 1.
    lo = np.where(top, -1.0, lo)
    t = v - lo
    lo_i = np.where(top, m - 1, lo).astype(np.int64)
    hi_i = np.where(top, m - 1, lo_i + 1).astype(np.int64)
    a = s[lo_i]
    b = s[hi_i]
    d = (b - a).astype(np.float32)            # float32 subtraction
    low = a.astype(np.float64) + d.astype(np.float64) * t
    high = b.astype(np.float64) - d.astype(np.float64) * (1.0 - t)
    return np.where(t >= 0.5, high, low)


def nanmedian_f32(col: np.ndarray) -> np.float32:
    """np.nanmedian of a float32 column: mean of the two middle order
    statistics computed as float32(a + b) / 2 (yabt/binning.py:32-33)."""
    c = col[~np.isnan(col)]
    m = c.shape[0]
    if m == 0:
        return np.float32(np.nan)
    # the middle order statistics (a partial sort places them as a full sort would)
    if m % 2 == 1:
        return np.float32(np.partition(c, m // 2)[m // 2])
    c = np.partition(c, [m // 2 - 1, m // 2])
    s = np.float32(c[m // 2 - 1]) + np.float32(c[m // 2])
    return np.float32(s / np.float32(2.0))


class Binner:
    """Restates yabt/binning.py:12-129 (numpy path of ``fit``)."""

    def __init__(self, max_bins: int = MAX_BINS):
        if not 2 <= max_bins <= 256:
            raise ValueError("max_bins must be in [2, 256]")
        self.max_bins = max_bins
        self.edges_: list[np.ndarray] | None = None
        self.medians_: np.ndarray | None = None
        self.scales_: np.ndarray | None = None

    @staticmethod
    def sample_rows(n: int) -> np.ndarray | None:
        """Row subsample for quantile estimation, yabt/binning.py:36-40."""
        if n > QUANTILE_SAMPLE:
            return np.random.default_rng(0).choice(n, QUANTILE_SAMPLE, replace=False)
        return None

    def fit(self, X: np.ndarray) -> "Binner":
        X = np.asarray(X, dtype=np.float32)
        n, F = X.shape
        med = np.array([nanmedian_f32(np.ascontiguousarray(X[:, f])) for f in range(F)], dtype=np.float32)
        self.medians_ = np.where(np.isnan(med), np.float32(0.0), med).astype(np.float32)
        idx = self.sample_rows(n)
        Xq = X if idx is None else X[idx]
        qpts = np.arange(1, self.max_bins, dtype=np.float64) / self.max_bins
        edges, scales = [], np.empty(F, dtype=np.float32)
        for f in range(F):
            col = Xq[:, f]
            col = col[~np.isnan(col)]
            if col.size == 0:
                col = np.zeros(1, dtype=np.float32)
            s = np.sort(col)
            e = quantile_sorted(s, qpts).astype(np.float32)
            edges.append(np.unique(e))
            q25, q75 = quantile_sorted(s, np.array([0.25, 0.75]))
            sc = float(q75 - q25)
            if sc == 0.0:
                sc = float(col.std()) or 1.0
            scales[f] = sc
        self.edges_ = edges
        self.scales_ = scales
        return self

    def impute(self, X: np.ndarray) -> np.ndarray:
        """yabt/binning.py:121-124."""
        Xi = np.array(X, dtype=np.float32)          # one copy
        np.copyto(Xi, self.medians_[None, :], where=np.isnan(Xi))
        return Xi

    def transform(self, X: np.ndarray) -> np.ndarray:
        """bin(x) = #{edges < x} as uint8 (yabt/binning.py:97-112)."""
        X = np.asarray(X, dtype=np.float32)
        n, F = X.shape
        out = np.empty((n, F), dtype=np.uint8)
        from concurrent.futures import ThreadPoolExecutor
        import os
        with ThreadPoolExecutor(max(1, min(16, os.cpu_count() or 1))) as pool:
            for r0 in range(0, n, 1 << 16):       # row blocks: contiguous columns within a block
                XiT = np.ascontiguousarray(self.impute(X[r0:r0 + (1 << 16)]).T)
                ob = np.empty(XiT.shape, np.uint8)

                def one(f):                        # searchsorted releases the GIL
                    ob[f] = np.searchsorted(self.edges_[f], XiT[f], side="left")
                list(pool.map(one, range(F)))
                out[r0:r0 + (1 << 16)] = ob.T
        return out

    def edge_value(self, f: int, b: int) -> float:
        """Raw threshold equivalent to ``bin <= b`` (yabt/binning.py:126-129)."""
        e = self.edges_[f]
        return float(e[min(b, len(e) - 1)])
