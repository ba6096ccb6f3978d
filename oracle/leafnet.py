"""Oracle restatement of ridge-linear neural leaves (test infrastructure only).

Restates ``fit_leaf_networks`` with ``leaf_net_hidden == 0``
(yabt/neural_leaves.py:131-184), ``_select_features`` (:21-39) and
``_fit_linear`` (:42-90). The per-leaf normal equations are accumulated in
float64 in row order (torch CPU ``index_add_`` is sequential) and solved with
a float64 LU solve, as the reference does.

Parity notes:
* ``Xs.mean`` / ``Xs.std`` are computed in float64 and rounded to float32
  (torch's float32 reduction order is ISA specific);
* the split-feature ranking breaks count ties by ascending feature id, which is
  what torch's CPU ``argsort(descending=True)`` does on the ascending output of
  ``unique`` (observed, not documented);
* the gradient-correlation padding score is computed in float64.
"""

from __future__ import annotations

import numpy as np

from .grow import LEAF, OTree

f32 = np.float32


def column_stats(X: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Column mean and unbiased std (float64 accumulation, float32 result)."""
    n, F = X.shape
    mu = np.empty(F, np.float64)
    var = np.empty(F, np.float64)
    for f0 in range(0, F, 16):                # column blocks bound the float64 copies
        X64 = X[:, f0:f0 + 16].astype(np.float64)
        mu[f0:f0 + 16] = X64.mean(axis=0)
        var[f0:f0 + 16] = ((X64 - mu[f0:f0 + 16]) ** 2).sum(axis=0) / max(n - 1, 1)
    return mu.astype(np.float32), np.sqrt(var).astype(np.float32)


def select_features(tree: OTree, Xraw: np.ndarray, grad: np.ndarray, k: int,
                    col_mean: np.ndarray | None = None,
                    col_std: np.ndarray | None = None) -> np.ndarray:
    """yabt/neural_leaves.py:21-39."""
    F = Xraw.shape[1]
    k = min(k, F)
    fs = tree.feature[tree.feature >= 0]
    if fs.size:
        vals, counts = np.unique(fs, return_counts=True)
        order = np.lexsort((vals, -counts))       # count desc, feature asc
        used = vals[order][:k]
    else:
        used = np.empty(0, np.int64)
    if used.size >= k:
        return used.astype(np.int64)
    if col_mean is None or col_std is None:
        col_mean, col_std = column_stats(Xraw)
    g64 = grad.astype(np.float64)
    score = np.abs(Xraw.astype(np.float64).T @ g64 - col_mean.astype(np.float64) * g64.sum())
    score = score / np.maximum(col_std.astype(np.float64), 1e-6)
    score = score.astype(np.float32)
    score[used] = -np.inf
    extra = np.argsort(-score, kind="stable")[: k - used.size]
    return np.concatenate([used, extra]).astype(np.int64)


def fit_linear(Xn: np.ndarray, grad: np.ndarray, hess: np.ndarray, leaf: np.ndarray,
               eligible: np.ndarray, n_nodes: int, lam: float):
    """yabt/neural_leaves.py:42-90. Returns (W (nodes,K) f32, db (nodes,) f32,
    M (nodes,K+1,K+1) f64, b (nodes,K+1) f64)."""
    K = Xn.shape[1]
    W = np.zeros((n_nodes, K), np.float32)
    db = np.zeros(n_nodes, np.float32)
    X1 = np.concatenate([Xn.astype(np.float64), np.ones((Xn.shape[0], 1))], axis=1)
    g = grad.astype(np.float64)
    h = hess.astype(np.float64)
    Xh = X1 * h[:, None]
    M = np.zeros((n_nodes, K + 1, K + 1))
    bv = np.zeros((n_nodes, K + 1))
    if Xn.shape[0] <= 200_000:
        # sequential float64 sums in row order, as torch's CPU index_add_
        np.add.at(M, leaf, X1[:, :, None] * Xh[:, None, :])
        np.add.at(bv, leaf, -(X1 * g[:, None]))
    else:
        # large inputs (CPU baseline timing): per-leaf BLAS products; float64
        # rounding order differs from the sequential sums only in the last bits
        order = np.argsort(leaf, kind="stable")
        ls = leaf[order]
        bounds = np.flatnonzero(np.diff(ls)) + 1
        for seg in np.split(np.arange(ls.size), bounds):
            if seg.size == 0:
                continue
            rows = order[seg]
            l = ls[seg[0]]
            M[l] = X1[rows].T @ Xh[rows]
            bv[l] = -(X1[rows] * g[rows, None]).sum(axis=0)
    elig = np.nonzero(eligible)[0]
    if elig.size == 0:
        return W, db, M, bv
    reg = np.eye(K + 1) * lam
    reg[K, K] = 1e-8
    theta = np.linalg.solve(M[elig] + reg, bv[elig][..., None])[..., 0].astype(np.float32)
    W[elig] = theta[:, :K]
    db[elig] = theta[:, K]
    return W, db, M, bv


def fit_leaf_networks(tree: OTree, Xraw: np.ndarray, y: np.ndarray, margin: np.ndarray,
                      loss, params, leaf_idx: np.ndarray,
                      col_mean: np.ndarray | None = None,
                      col_std: np.ndarray | None = None) -> OTree:
    """yabt/neural_leaves.py:131-184 (linear leaves). ``params`` needs
    leaf_net_features, leaf_net_min_samples, leaf_net_l2, learning_rate."""
    grad, hess = loss.grad_hess((margin + tree.value[leaf_idx]).astype(np.float32), y)
    feats = select_features(tree, Xraw, grad, params.leaf_net_features, col_mean, col_std)
    if feats.size == 0:
        return tree
    Xs = Xraw[:, feats]
    if col_mean is None or col_std is None:
        mu, sd = column_stats(Xs)
    else:
        mu, sd = col_mean[feats], col_std[feats]
    sd = np.maximum(sd, f32(1e-6))
    Xn = ((Xs - mu) / sd).astype(np.float32)
    n_nodes = tree.value.shape[0]
    counts = np.bincount(leaf_idx, minlength=n_nodes).astype(np.float32)
    eligible = (tree.feature == LEAF) & (counts >= params.leaf_net_min_samples)
    if not eligible.any():
        return tree
    lr = params.learning_rate
    K = feats.size
    lo = np.full((n_nodes, K), np.inf, np.float32)
    hi = np.full((n_nodes, K), -np.inf, np.float32)
    np.minimum.at(lo, leaf_idx, Xs)
    np.maximum.at(hi, leaf_idx, Xs)
    W, db, _, _ = fit_linear(Xn, grad, hess, leaf_idx, eligible, n_nodes, params.leaf_net_l2)
    lr32 = f32(lr)
    value = (tree.value + lr32 * (db - (W * (mu / sd)).sum(axis=1, dtype=np.float32))).astype(np.float32)
    linear = ((lr32 * W) / sd).astype(np.float32)
    return OTree(feature=tree.feature, threshold=tree.threshold, left=tree.left,
                 right=tree.right, value=value, depth=tree.depth, gate_scale=tree.gate_scale,
                 leaf_net_feats=feats, leaf_net_linear=linear, leaf_net_lo=lo, leaf_net_hi=hi,
                 split_bin=tree.split_bin, extras=dict(tree.extras, W=W, db=db, mu=mu, sd=sd))
