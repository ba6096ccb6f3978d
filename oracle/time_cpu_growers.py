"""Times the reference's two CPU tree growers on one host (measurement only).

    python oracle/time_cpu_growers.py [REFERENCE_ROOT] [ROWS]

The reference's Numba grower (yabt/grow_numba.py:398, single-threaded: its
kernels are ``njit`` without ``parallel``) is Python source that cannot travel
to the GPU box, so it is timed where the reference is importable, beside the
reference's OpenMP C grower (yabt/_cgrow/grow.c, built by oracle/Makefile into
oracle/_ref) at 1 thread, at the reference's default cap of 8
(yabt/grow_c.py:283-302) and at every core of this host. Input: the C4
distributions (tests/config_data.py, correlated blocks of 10 columns) on ROWS
rows (default 500,000) x 200 features, binned by the oracle binner (the
reference's numpy path), 255 leaves, max depth 10, squared loss, interaction
steering from the trees grown so far. Each grower runs 4 boosting iterations
(the tree's values update the margin); the reported time is the median of
iterations 2-4 of the grower call alone. Prints one JSON line per grower.
Numba's compile cache goes to oracle/_ref/numba_cache (git-ignored).
"""

from __future__ import annotations

import json
import os
import statistics
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def main(ref: str = "/root/reference", rows: int = 500_000) -> None:
    os.environ.setdefault("NUMBA_CACHE_DIR", os.path.join(HERE, "_ref", "numba_cache"))
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import numpy as np
    import config_data
    from oracle import cgrow
    from oracle.binning import Binner
    from oracle.boost import InteractionDetector
    from oracle.grow import OTree

    X, y = config_data.make("c4", rows)
    F = X.shape[1]
    b = Binner().fit(X)
    bins = b.transform(X)
    bins_fm = np.ascontiguousarray(bins.T)
    nbins = np.array([min(len(e) + 1, 256) for e in b.edges_], np.int32)
    leaves, depth, lr = 255, 10, 0.1

    def leaf_of(feat, tb, left, right):
        t = OTree(feat, np.zeros(len(feat), np.float32), left, right, np.zeros(len(feat), np.float32),
                  64, np.ones(len(feat), np.float32), split_bin=tb)
        return t, t.apply_bins(bins)

    def run(name, grow_fn, threads):
        margin = np.full(rows, float(y.mean()), np.float32)
        det = InteractionDetector(F)
        times = []
        for it in range(4):
            g = (margin - y).astype(np.float32)
            h = np.ones_like(g)
            imat = det.normalized()
            t0 = time.perf_counter()
            feat, tb, left, right, value = grow_fn(g, h, imat)
            times.append(time.perf_counter() - t0)
            tree, leaf = leaf_of(feat, tb, left, right)
            det.update(tree.path_feature_pairs())
            margin = (margin + value[leaf]).astype(np.float32)
        per = statistics.median(times[1:])
        print(json.dumps({"grower": name, "threads": threads, "rows": rows, "features": F, "leaves": leaves,
                          "s_per_tree": per, "ns_per_row": per / rows * 1e9,
                          "bin_reads_per_s": rows * F * 2 / per,      # ~2 n F bin reads per leaf-wise tree
                          "host_cpu_count": os.cpu_count()}), flush=True)

    def c_grower(threads):
        def fn(g, h, imat):
            feat, tb, left, right, value, _ = cgrow.grow(bins_fm, g, h, nbins, leaves, depth, lr=lr,
                                                         imat=imat, threads=threads)
            return feat, tb, left, right, value
        return fn

    if os.path.exists(os.path.join(ref, "yabt", "grow_numba.py")):
        sys.path.insert(0, ref)
        import torch
        from yabt.grow_numba import grow_tree_numba
        from yabt.tree import TreeParams

        class RefBinner:                 # the attributes grow_tree_numba reads
            edges_ = b.edges_
            scales_ = torch.from_numpy(b.scales_)

            @staticmethod
            def edge_value(f, k):
                return b.edge_value(f, k)

        tp = TreeParams(max_leaves=leaves, max_depth=depth, learning_rate=lr)
        bt = torch.from_numpy(bins)

        def numba_fn(g, h, imat):
            t = grow_tree_numba(bt, torch.from_numpy(g), torch.from_numpy(h), RefBinner, tp,
                                interaction_matrix=torch.from_numpy(imat), interaction_boost=0.5)
            feat = t.feature.numpy()
            tb = np.array([int(np.searchsorted(b.edges_[f], thr, side="left")) if f >= 0 else -1
                           for f, thr in zip(feat, t.threshold.numpy())], np.int64)
            return feat, tb, t.left.numpy(), t.right.numpy(), t.value.numpy()
        numba_fn(np.zeros(rows, np.float32) + 0.5, np.ones(rows, np.float32), np.zeros((F, F), np.float32))
        run("numba (reference yabt/grow_numba.py)", numba_fn, 1)
    cores = os.cpu_count() or 1
    for th in sorted({1, min(8, cores), cores}):
        run("openmp C (reference yabt/_cgrow/grow.c)", c_grower(th), th)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference",
         int(sys.argv[2]) if len(sys.argv) > 2 else 500_000)
