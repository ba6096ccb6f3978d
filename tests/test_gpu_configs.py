"""Parity on the benchmark configurations' own data (GPU tests).

Inputs are the five configurations' seeded generators (``config_data.make``:
``np.random.default_rng(0)``, the configuration text's shapes, distributions
and draw order; C4 and C5 as row slices of the same distributions), and the
benchmark's own C4 input (``bench.make_data``), so the trees that
``bench.py`` times are trees of a data set compared here. Each case fits the
CUDA booster and the CPU oracle booster on the same matrix and requires:

* bins, edges and medians bit-exact (the reference's numpy binning path);
* the root histogram's per-bin row counts bit-exact;
* every compared tree's features, thresholds and children bit-exact, and the
  leaf of every training row (``Tree.apply`` on the imputed matrix) equal to
  the oracle's;
* leaf values within 1e-5 relative to the gradient magnitudes summed along
  their histograms' path from the root (the north-star bound on histogram
  sums: the oracle adds float32 row by row and subtracts float32 histograms,
  the device sums exactly) and predictions within 1e-4 relative.
"""

import os
import sys

import numpy as np
import pytest
import torch

from oracle.boost import Booster as OBooster, BoostParams as OBP, LogLoss as OLog, MSELoss as OMSE

sys.path.insert(0, os.path.dirname(__file__))
import config_data  # noqa: E402

pytestmark = pytest.mark.gpu


def _fit(X, y, loss, trees, **kw):
    from yabt_b200 import Booster, BoostParams, LogLoss, MSELoss
    okw = {k: v for k, v in kw.items() if k in OBP.__dataclass_fields__}
    ob = OBooster(OBP(n_estimators=trees, **okw), OMSE() if loss == "mse" else OLog())
    ob.fit(X, y, record=True)
    gb = Booster(BoostParams(n_estimators=trees, **kw), MSELoss() if loss == "mse" else LogLoss())
    gb.fit(X, y)
    torch.cuda.synchronize()
    return ob, gb


def _check_binning(X, ob, gb):
    np.testing.assert_array_equal(gb.binner.medians_, ob.binner.medians_)
    for f in range(X.shape[1]):
        np.testing.assert_array_equal(gb.binner.edges_[f].numpy(), ob.binner.edges_[f], err_msg=f"edges f={f}")
    bins = ob.binner.transform(X)
    np.testing.assert_array_equal(gb.binner.transform(X).cpu().numpy(), bins)
    return bins


def _check_root_counts(bins, gb):
    got = gb.grower_.root_counts().cpu().numpy()
    want = np.stack([np.bincount(bins[:, f], minlength=256) for f in range(bins.shape[1])])
    np.testing.assert_array_equal(got, want)


def _value_tolerance(rec, tree, lr, lam=1.0):
    """Per-node bound on a leaf value's difference from the oracle's.

    The oracle restates the reference's arithmetic: float32 histograms added
    row by row, and every larger child's histogram the float32 difference
    parent - smaller child, so a node's bin sums carry the rounding of every
    histogram on its path from the root. The device sums exactly and rounds
    once. The bound is the north-star tolerance for histogram sums, 1e-5
    relative to the magnitudes summed, taken along that path (sum over the
    node's ancestors a and itself of sum_{rows in a} |g|), carried through
    v = -lr G / (H + lambda)."""
    nodes = tree.value.size
    leaf = rec["leaf"]
    s = np.bincount(leaf, weights=np.abs(rec["g"].astype(np.float64)), minlength=nodes)
    hsum = np.bincount(leaf, weights=rec["h"].astype(np.float64), minlength=nodes)
    parent = np.full(nodes, -1, np.int64)
    inner = np.nonzero(tree.feature >= 0)[0]
    parent[tree.left[inner]] = inner
    parent[tree.right[inner]] = inner
    for v in range(nodes - 1, 0, -1):          # children are created after their parent
        if parent[v] >= 0:
            s[parent[v]] += s[v]
    path = s.copy()
    for v in range(1, nodes):
        if parent[v] >= 0:
            path[v] += path[parent[v]]
    return 1e-5 * lr * path / (hsum + lam) + 1e-6


def _check_trees(X, ob, gb, trees):
    from yabt_b200.predict import apply_tree
    Xi = torch.from_numpy(ob.binner.impute(X)).cuda()
    lr = ob.p.learning_rate
    for t in range(trees):
        gt, ot = gb.trees[t], ob.trees[t]
        for k in ("feature", "threshold", "left", "right"):
            np.testing.assert_array_equal(getattr(gt, k).cpu().numpy(), getattr(ot, k), err_msg=f"tree {t} {k}")
        gv = gt.value.cpu().numpy()
        tol = _value_tolerance(ob.records[t], ot, lr) + 1e-5 * np.abs(ot.value)
        bad = np.abs(gv.astype(np.float64) - ot.value) > tol
        assert not bad.any(), (f"tree {t} values: nodes {np.nonzero(bad)[0][:8]}, got {gv[bad][:8]}, "
                               f"want {ot.value[bad][:8]}, tolerance {tol[bad][:8]}")
        np.testing.assert_array_equal(apply_tree(gt, Xi).cpu().numpy(), ob.records[t]["leaf"],
                                      err_msg=f"tree {t} leaf of every row")
        if ot.leaf_net_feats is not None:
            np.testing.assert_array_equal(gt.leaf_net_feats.cpu().numpy(), ot.leaf_net_feats)
            leaf = ot.feature == -1
            np.testing.assert_array_equal(gt.leaf_net_lo.cpu().numpy()[leaf], ot.leaf_net_lo[leaf])
            np.testing.assert_array_equal(gt.leaf_net_hi.cpu().numpy()[leaf], ot.leaf_net_hi[leaf])
            np.testing.assert_allclose(gt.leaf_net_linear.cpu().numpy()[leaf], ot.leaf_net_linear[leaf],
                                       rtol=1e-4, atol=1e-6, err_msg=f"tree {t} leaf models")


def _check_predictions(X, ob, gb):
    po = ob.predict_margin(X)
    np.testing.assert_allclose(gb.predict_margin(X), po, rtol=1e-4, atol=1e-4 * max(1.0, float(np.abs(po).mean())))


def test_c1_full():
    """C1 (20,000 x 20, squared loss, 31 leaves, lr 0.1, neural leaves,
    interaction steering): the first 30 of its 200 trees."""
    X, y = config_data.make("c1")
    ob, gb = _fit(X, y, "mse", 30, max_leaves=31, learning_rate=0.1)
    bins = _check_binning(X, ob, gb)
    _check_root_counts(bins, gb)
    _check_trees(X, ob, gb, 30)
    _check_predictions(X, ob, gb)


def test_c2_full():
    """C2 (100,000 x 50 with ten integer columns, log-loss, 63 leaves, lr 0.05):
    the first 10 of its 300 trees."""
    X, y = config_data.make("c2")
    ob, gb = _fit(X, y, "logloss", 10, max_leaves=63, learning_rate=0.05)
    bins = _check_binning(X, ob, gb)
    _check_root_counts(bins, gb)
    _check_trees(X, ob, gb, 10)
    _check_predictions(X, ob, gb)


def test_c3_full():
    """C3 (1,000,000 x 100, 20 lognormal columns, 5% NaN, 127 leaves, leaf models
    on the top 8 features): the first 3 of its 500 trees."""
    X, y = config_data.make("c3")
    ob, gb = _fit(X, y, "mse", 3, max_leaves=127, learning_rate=0.1)
    bins = _check_binning(X, ob, gb)
    _check_root_counts(bins, gb)
    _check_trees(X, ob, gb, 3)
    _check_predictions(X, ob, gb)


def test_c4_slice():
    """C4's distributions (correlated blocks of 10 columns, 255 leaves, max depth
    10) on 2,000,000 of its 10,000,000 rows: the first tree."""
    X, y = config_data.make("c4", 2_000_000)
    ob, gb = _fit(X, y, "mse", 1, max_leaves=255, max_depth=10, learning_rate=0.1)
    bins = _check_binning(X, ob, gb)
    _check_root_counts(bins, gb)
    _check_trees(X, ob, gb, 1)
    _check_predictions(X, ob, gb)


def test_bench_c4_data():
    """The benchmark's own C4 generator (bench.make_data, seeded on the device)
    at 2,000,000 rows: the first tree, as bench.py grows it."""
    sys.path.insert(0, os.path.dirname(os.path.dirname(__file__)))
    import bench
    Xd, yd = bench.make_data("c4", 2_000_000, 200, torch.device("cuda"), seed=1000)
    X, y = Xd.cpu().numpy(), yd.cpu().numpy()
    del Xd, yd
    ob, gb = _fit(X, y, "mse", 1, max_leaves=255, max_depth=10, learning_rate=0.1)
    bins = _check_binning(X, ob, gb)
    _check_root_counts(bins, gb)
    _check_trees(X, ob, gb, 1)
    _check_predictions(X, ob, gb)


def test_c5_slice_one_vs_rest():
    """C5's distributions (30% exact zeros per column, 63 leaves, log-loss per
    class) on 200,000 rows and 3 classes: every class's booster equals the
    oracle booster of that class for 5 rounds."""
    from yabt_b200.multiclass import MulticlassBooster
    from yabt_b200.boosting import BoostParams
    X, y = config_data.make("c5", 200_000, classes=3)
    mc = MulticlassBooster(BoostParams(n_estimators=5, max_leaves=63, learning_rate=0.1)).fit(X, y)
    torch.cuda.synchronize()
    assert list(mc.classes_) == [0.0, 1.0, 2.0]
    for c, gb in zip(mc.classes_, mc.boosters_):
        yc = (y == c).astype(np.float32)
        ob = OBooster(OBP(n_estimators=5, max_leaves=63, learning_rate=0.1), OLog()).fit(X, yc, record=True)
        if c == 0:
            bins = _check_binning(X, ob, gb)
            _check_root_counts(bins, gb)
        _check_trees(X, ob, gb, 5)
        _check_predictions(X, ob, gb)


def _chain(n=30000, F=12, seed=3, chain=10):
    """A nested target whose trees grow a long chain (about `chain` levels),
    far past the device-side level loop's first level."""
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, F)).astype(np.float32)
    X[:, chain:][rng.random(size=(n, F - chain)) < 0.02] = np.nan
    on = np.ones(n, dtype=bool)
    y = np.zeros(n, dtype=np.float32)
    for k in range(chain):
        on &= X[:, k] > -0.3
        y += 2.0 * on
    return X, y + 0.01 * rng.normal(size=n).astype(np.float32)


def test_deep_trees_in_level_loop():
    """Trees whose deeper levels run in the device-side level loop (31 leaves,
    the default depth limit of 64, trees about ten levels deep), with leaf
    models and interaction steering, against the oracle booster."""
    X, y = _chain()
    ob, gb = _fit(X, y, "mse", 6, max_leaves=31, learning_rate=0.3, min_samples_leaf=5, levelwise=True)
    first = gb.grower_.level_loop_start()
    assert first > 0
    depth = []
    for t in ob.trees:
        d, st = 0, [(0, 0)]
        while st:
            i, k = st.pop()
            d = max(d, k)
            if t.left[i] >= 0:
                st += [(int(t.left[i]), k + 1), (int(t.right[i]), k + 1)]
        depth.append(d)
    assert max(depth) > first, depth
    bins = _check_binning(X, ob, gb)
    _check_root_counts(bins, gb)
    _check_trees(X, ob, gb, 6)
    _check_predictions(X, ob, gb)
