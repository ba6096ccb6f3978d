"""The CPU oracle pinned against golden vectors produced by the reference.

These run without a GPU. They establish that ``oracle/`` restates the
reference's GPU tree-growth path exactly (tree structure bit-exact, float
leaf values within a few ulp where the reference sums in an ISA-specific
order), so that the CUDA tests can use the oracle as their checker.
"""
import os
import sys

import numpy as np
import pytest

from oracle.binning import Binner, nanmedian_f32, quantile_sorted
from oracle.boost import Booster, BoostParams, InteractionDetector, LogLoss, MSELoss
from oracle.grow import OTree, TreeParams, grow_levelwise, scatter_hist, split_scan
from oracle.leafnet import fit_leaf_networks

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_golden import _data  # noqa: E402  (seeded input generator shared with the fixtures)


def test_quantile_matches_numpy():
    rng = np.random.default_rng(5)
    q = np.arange(1, 256) / 256
    for m in (1, 2, 3, 7, 255, 256, 257, 1000, 4097):
        col = (rng.standard_cauchy(m) * 3).astype(np.float32)
        col[: m // 5] = 0.0
        s = np.sort(col)
        np.testing.assert_array_equal(quantile_sorted(s, q), np.quantile(col, q))
        np.testing.assert_array_equal(quantile_sorted(s, np.array([0.25, 0.75])),
                                      np.quantile(col, [0.25, 0.75]))


def test_nanmedian_matches_numpy():
    rng = np.random.default_rng(6)
    for m in (1, 2, 5, 600, 601, 2000):
        col = rng.normal(size=m).astype(np.float32)
        col[rng.random(m) < 0.1] = np.nan
        if np.isnan(col).all():
            continue
        assert nanmedian_f32(col) == np.nanmedian(col)


def test_binner_matches_reference(golden):
    z = golden("binning")
    cases = z["cases"]
    for i in range(int(z["ncases"])):
        seed, n, F, nanf = cases[i]
        if f"c{i}_X" in z:
            X = z[f"c{i}_X"]
        else:
            X, _ = _data(int(seed), int(n), int(F), float(nanf))
        b = Binner(256).fit(X)
        np.testing.assert_array_equal(b.medians_, z[f"c{i}_medians"])
        np.testing.assert_array_equal(b.scales_, z[f"c{i}_scales"])
        np.testing.assert_array_equal(np.array([len(e) for e in b.edges_]), z[f"c{i}_nedges"])
        np.testing.assert_array_equal(np.concatenate(b.edges_), z[f"c{i}_edges"])
        np.testing.assert_array_equal(b.transform(X), z[f"c{i}_bins"])


def test_bin_split_equivalence():
    """bin(x) <= b  <=>  x <= edge_value(f, b) (reference tests/test_splits.py:58-68)."""
    rng = np.random.default_rng(1)
    X = rng.normal(size=(1000, 3)).astype(np.float32)
    b = Binner(16).fit(X)
    bins = b.transform(X)
    for f in range(3):
        for k in range(len(b.edges_[f])):
            assert ((bins[:, f] <= k) == (X[:, f] <= b.edge_value(f, k))).all()


@pytest.mark.parametrize("case", range(4))
def test_levelwise_grower_matches_reference(golden, case):
    z = golden("grow")
    X = z[f"g{case}_X"]
    leaves, depth, msl = (int(v) for v in z[f"g{case}_params"])
    b = Binner().fit(X)
    imat = z[f"g{case}_imat"]
    fm = z[f"g{case}_fmask"]
    tree, leaf, _ = grow_levelwise(b.transform(X), z[f"g{case}_g"], z[f"g{case}_h"], b.edges_,
                                   b.scales_, TreeParams(max_leaves=leaves, max_depth=depth,
                                                         min_samples_leaf=msl),
                                   fm if fm.size else None, imat if imat.size else None, 0.5)
    for k in ("feature", "threshold", "left", "right", "gate_scale"):
        np.testing.assert_array_equal(getattr(tree, k), z[f"g{case}_{k}"], err_msg=k)
    assert tree.depth == int(z[f"g{case}_depth"])
    # leaf values: the reference's Gtot is a float32 sum in an ISA-specific order
    np.testing.assert_allclose(tree.value, z[f"g{case}_value"], rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(leaf, z[f"g{case}_leaf"])
    # training-row leaf == apply(raw X) (the bin/threshold equivalence)
    np.testing.assert_array_equal(tree.apply(b.impute(X)), leaf)


@pytest.mark.parametrize("case", range(4))
def test_bestfirst_grower_matches_reference(golden, case):
    """The best-first (heap) grower, yabt/tree.py:206-360, against the reference run."""
    from oracle.grow import grow_bestfirst
    z = golden("bestfirst")
    X = z[f"b{case}_X"]
    leaves, depth, msl = (int(v) for v in z[f"b{case}_params"])
    b = Binner().fit(X)
    imat = z[f"b{case}_imat"]
    fm = z[f"b{case}_fmask"]
    tree, leaf = grow_bestfirst(b.transform(X), z[f"b{case}_g"], z[f"b{case}_h"], b.edges_, b.scales_,
                                TreeParams(max_leaves=leaves, max_depth=depth, min_samples_leaf=msl),
                                fm if fm.size else None, imat if imat.size else None, 0.5)
    for k in ("feature", "threshold", "left", "right", "gate_scale"):
        np.testing.assert_array_equal(getattr(tree, k), z[f"b{case}_{k}"], err_msg=k)
    np.testing.assert_allclose(tree.value, z[f"b{case}_value"], rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(leaf, z[f"b{case}_leaf"])
    np.testing.assert_array_equal(tree.apply(b.impute(X)), leaf)


def test_leaf_networks_match_reference(golden):
    z = golden("leafnet")

    class P:
        leaf_net_features, leaf_net_min_samples, leaf_net_l2, learning_rate = 8, 50, 1.0, 0.1

    for i in range(2):
        X, y = z[f"l{i}_X"], z[f"l{i}_y"]
        Xraw = Binner().fit(X).impute(X)
        t = OTree(*(z[f"l{i}_tree_{k}"] for k in ("feature", "threshold", "left", "right", "value")),
                  int(z[f"l{i}_tree_depth"]), np.ones(len(z[f"l{i}_tree_value"]), np.float32))
        t2 = fit_leaf_networks(t, Xraw, y, z[f"l{i}_margin"], MSELoss(), P(), z[f"l{i}_leaf"])
        np.testing.assert_array_equal(t2.leaf_net_feats, z[f"l{i}_feats"])
        np.testing.assert_array_equal(t2.leaf_net_lo, z[f"l{i}_lo"])
        np.testing.assert_array_equal(t2.leaf_net_hi, z[f"l{i}_hi"])
        np.testing.assert_allclose(t2.leaf_net_linear, z[f"l{i}_linear"], rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(t2.value, z[f"l{i}_value"], rtol=1e-5, atol=1e-6)


def test_boosting_matches_reference(golden):
    z = golden("boost")
    bm = Booster(BoostParams(n_estimators=12, max_leaves=15, learning_rate=0.1, levelwise=True), MSELoss())
    bm.fit(z["mse_X"], z["mse_y"])
    for t in range(3):
        np.testing.assert_array_equal(bm.trees[t].feature, z[f"mse_t{t}_feature"])
    np.testing.assert_allclose(bm.predict_margin(z["mse_X"]), z["mse_pred"], rtol=1e-4, atol=1e-5)
    bl = Booster(BoostParams(n_estimators=10, max_leaves=15, learning_rate=0.2, levelwise=True), LogLoss())
    bl.fit(z["log_X"], z["log_y"])
    np.testing.assert_allclose(bl.predict_margin(z["log_X"]), z["log_pred"], rtol=1e-4, atol=1e-5)


def test_scatter_hist_matches_reference(golden):
    z = golden("hist")
    w = z["w"]
    got = scatter_hist(z["binned"], z["slot"], z["g"] * w, z["h"] * w, w, 5)
    np.testing.assert_array_equal(got, z["hist"])


def test_split_scan_brute_force():
    """Known answer (reference tests/test_splits.py:9-44)."""
    rng = np.random.default_rng(42)
    n, F = 500, 6
    binned = rng.integers(0, 30, size=(n, F)).astype(np.uint8)
    g = rng.normal(size=n).astype(np.float32)
    h = rng.uniform(0.1, 1.0, size=n).astype(np.float32)
    hist = scatter_hist(binned, np.zeros(n, np.int64), g, h, None, 1)
    idx, gain, _ = split_scan(hist, 1.0, 0.0, 0.0, 1)
    best = (-np.inf, -1, -1)
    G, H = g.astype(np.float64).sum(), h.astype(np.float64).sum()
    for f in range(F):
        for b in range(255):
            m = binned[:, f] <= b
            if m.sum() < 1 or (~m).sum() < 1:
                continue
            GL, HL = g[m].astype(np.float64).sum(), h[m].astype(np.float64).sum()
            v = 0.5 * (GL ** 2 / (HL + 1) + (G - GL) ** 2 / (H - HL + 1) - G ** 2 / (H + 1))
            if v > best[0]:
                best = (v, f, b)
    assert (int(idx[0]) // 256, int(idx[0]) % 256) == best[1:]
    assert gain[0] == pytest.approx(best[0], rel=1e-3)


def test_interaction_detector_normalisation():
    """reference tests/test_interaction_aware.py:58-77."""
    d = InteractionDetector(5)
    for _ in range(10):
        d.update([(0, 1), (0, 1), (2, 3)])
    m = d.normalized()
    assert m.max() == pytest.approx(1.0) and m[0, 1] == pytest.approx(1.0) and m[2, 3] == 0.0
    d2 = InteractionDetector(6)
    d2.update([(0, 1), (2, 3), (4, 5)])
    assert d2.normalized().max() == 0.0


@pytest.mark.parametrize("case", range(4))
def test_multitask_grower_matches_reference(golden, case):
    """The multi-task grower, yabt/multitask.py:60-150, against the reference run."""
    from oracle.multitask import grow_multitask
    z = golden("multitask")
    X, g = z[f"m{case}_X"], z[f"m{case}_g"]
    leaves, depth, msl = (int(v) for v in z[f"m{case}_params"])
    fm = z[f"m{case}_fmask"]
    b = Binner().fit(X)
    feat, thr, left, right, value, _, leaf = grow_multitask(
        b.transform(X), g, np.ones_like(g), b.edges_,
        TreeParams(max_leaves=leaves, max_depth=depth, min_samples_leaf=msl), fm if fm.size else None)
    np.testing.assert_array_equal(feat, z[f"m{case}_feature"])
    np.testing.assert_array_equal(left, z[f"m{case}_left"])
    np.testing.assert_array_equal(right, z[f"m{case}_right"])
    np.testing.assert_array_equal(thr, z[f"m{case}_threshold"])
    np.testing.assert_allclose(value, z[f"m{case}_value"], rtol=1e-6, atol=1e-7)
    np.testing.assert_array_equal(leaf, z[f"m{case}_leaf"])
