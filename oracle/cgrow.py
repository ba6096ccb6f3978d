"""ctypes binding of the reference's OpenMP C grower (test infrastructure only).

``oracle/_ref/libcgrow.so`` is compiled from the reference's own
yabt/_cgrow/grow.c by ``oracle/Makefile``. This module marshals arguments the
way the reference's wrapper does (yabt/grow_c.py:336-456 for ``cgrow``,
yabt/grow_c.py:303-333 for ``capply``) and is used for the timed CPU
baseline of ``bench.py`` (and the reference arm, ``--impl reference``).
"""

from __future__ import annotations

import ctypes
import os
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libcgrow.so")
_lib = None


def available() -> bool:
    return os.path.exists(LIB)


def load():
    global _lib
    if _lib is None:
        if not available():
            raise RuntimeError(f"{LIB} missing: run `make -C oracle` where the reference source exists")
        _lib = ctypes.CDLL(LIB)
        vp = ctypes.c_void_p
        _lib.cgrow.restype = ctypes.c_int
        _lib.cgrow.argtypes = [vp, vp, vp, vp, vp, ctypes.c_float, ctypes.c_int, vp, vp, vp, vp,
                               ctypes.c_int, vp, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                               ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                               ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                               vp, vp, vp, vp, vp, vp]
        _lib.capply.restype = None
        _lib.capply.argtypes = [vp, vp, vp, vp, vp, ctypes.c_int64, ctypes.c_int, ctypes.c_int, vp]
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def grow(binned_fm: np.ndarray, grad: np.ndarray, hess: np.ndarray, nbins: np.ndarray,
         max_leaves: int, max_depth: int, lam=1.0, gamma=0.0, mcw=1e-3, msl=20, lr=0.1,
         imat: np.ndarray | None = None, ib: float = 0.5, threads: int = 0,
         fmask: np.ndarray | None = None):
    """One leaf-wise tree with the reference C grower. binned_fm is (F, n) uint8.
    Returns (feature, thr_bin, left, right, value, depth) arrays."""
    lib = load()
    F, n = binned_fm.shape
    m = 2 * max_leaves + 1
    outs = [np.empty(m, np.int64) for _ in range(4)] + [np.empty(m, np.float32), np.empty(m, np.int64)]
    z64, z32 = np.zeros(1, np.int64), np.zeros(1, np.int32)
    fmask = np.ones(F, np.uint8) if fmask is None else np.ascontiguousarray(fmask, np.uint8)
    im = np.ascontiguousarray(imat, np.float32) if imat is not None else np.zeros((1, 1), np.float32)
    k = lib.cgrow(_p(binned_fm), _p(grad), _p(hess), _p(fmask), _p(im), float(ib), int(imat is not None),
                  _p(z64), _p(z32), _p(z32), _p(z32), 0, _p(nbins), n, F, 256, float(lam), float(gamma),
                  float(mcw), int(msl), float(lr), int(max_leaves), int(max_depth), int(threads),
                  *[_p(o) for o in outs])
    return [o[:k] for o in outs]


def apply(X: np.ndarray, feature, threshold, left, right, threads: int = 0) -> np.ndarray:
    lib = load()
    n, F = X.shape
    out = np.empty(n, np.int64)
    lib.capply(_p(X), _p(np.ascontiguousarray(feature, np.int64)), _p(np.ascontiguousarray(threshold, np.float32)),
               _p(np.ascontiguousarray(left, np.int64)), _p(np.ascontiguousarray(right, np.int64)),
               n, F, int(threads), _p(out))
    return out


def boosting_step_seconds(binned_fm, X, y, margin, edges, max_leaves, max_depth, lr, threads,
                          leaf_nets: bool = True, detector=None, col_stats=None):
    """Time one CPU boosting iteration of the reference path on the given rows:
    squared-loss gradients, the interaction matrix (yabt/boosting.py:339,410-412:
    steering is on for n >= 2000; ``detector`` is an oracle.boost.InteractionDetector
    kept across iterations, or None to steer nothing), the C grower
    (yabt/grow_c.py:336), the C apply (yabt/grow_c.py:303), ridge-linear leaf
    models (oracle restatement of yabt/neural_leaves.py:131-184), the detector's
    update with the tree's path pairs (yabt/boosting.py:508-509) and the margin
    update. Returns (seconds, new_margin)."""
    from .grow import OTree
    from .leafnet import fit_leaf_networks
    from .boost import MSELoss

    class P:
        leaf_net_features, leaf_net_min_samples, leaf_net_l2, learning_rate = 8, 50, 1.0, lr

    nbins = np.array([min(len(e) + 1, 256) for e in edges], np.int32)
    t0 = time.perf_counter()
    g = (margin - y).astype(np.float32)
    h = np.ones_like(g)
    imat = detector.normalized() if detector is not None else None
    feat, tb, left, right, value, depth = grow(binned_fm, g, h, nbins, max_leaves, max_depth, lr=lr,
                                               threads=threads, imat=imat)
    thr = np.array([edges[f][min(b, len(edges[f]) - 1)] if f >= 0 else 0.0
                    for f, b in zip(feat, tb)], np.float32)
    leaf = apply(X, feat, thr, left, right, threads)
    tree = OTree(feat, thr, left, right, value, int(depth.max()) + 1, np.ones(len(feat), np.float32))
    if leaf_nets:
        cm, cs = col_stats if col_stats is not None else (None, None)
        tree = fit_leaf_networks(tree, X, y, margin, MSELoss(), P(), leaf, cm, cs)
    if detector is not None:
        detector.update(tree.path_feature_pairs())
    contrib = tree.value[leaf]
    if tree.leaf_net_feats is not None:
        contrib = contrib + tree.net_contribution(X, leaf)
    new_margin = (margin + contrib).astype(np.float32)
    return time.perf_counter() - t0, new_margin
