"""CUDA best-first growth on the GPU.

* The heap grower, yabt/tree.py:206-360, against the CPU oracle restatement
  (oracle.grow.grow_bestfirst, itself pinned to the reference's own runs in
  tests/golden/bestfirst.npz).
* The C / Numba grower's arithmetic (grow_tree_c) against the reference's own
  C grower, yabt/_cgrow/grow.c, compiled from its source into oracle/_ref."""
import numpy as np
import pytest
import torch

from oracle.binning import Binner as OBinner
from oracle.grow import TreeParams as OTP, grow_bestfirst

pytestmark = pytest.mark.gpu


def _run(X, g, h, leaves, depth, msl, imat=None, fmask=None):
    from yabt_b200.grower import grow_tree
    from yabt_b200.tree import TreeParams
    b = OBinner().fit(X)
    binned = b.transform(X)
    ot, oleaf = grow_bestfirst(binned, g, h, b.edges_, b.scales_,
                               OTP(max_leaves=leaves, max_depth=depth, min_samples_leaf=msl), fmask, imat, 0.5)
    im = torch.from_numpy(imat).cuda() if imat is not None else None
    fm = torch.from_numpy(fmask).cuda() if fmask is not None else None
    gtree, gleaf = grow_tree(torch.from_numpy(binned).cuda(), torch.from_numpy(g).cuda(), torch.from_numpy(h).cuda(),
                             b, TreeParams(max_leaves=leaves, max_depth=depth, min_samples_leaf=msl), fm, im, 0.5,
                             return_leaf=True)
    return ot, oleaf, gtree, gleaf.cpu().numpy()


def _check(ot, oleaf, gtree, gleaf):
    for k in ("feature", "left", "right", "threshold", "gate_scale"):
        np.testing.assert_array_equal(getattr(gtree, k).cpu().numpy(), getattr(ot, k), err_msg=k)
    assert gtree.depth == ot.depth
    np.testing.assert_allclose(gtree.value.cpu().numpy(), ot.value, rtol=1e-5, atol=1e-7)
    np.testing.assert_array_equal(gleaf, oleaf)


def _dyadic(seed, n, F):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, F)).astype(np.float32)
    X[rng.random(size=X.shape) < 0.01] = np.nan
    g = (rng.integers(-512, 512, size=n) / 256.0).astype(np.float32)
    h = (rng.integers(1, 64, size=n) / 256.0).astype(np.float32)
    return X, g, h


@pytest.mark.parametrize("seed,n,F,leaves,depth", [(0, 3000, 8, 15, 64), (1, 20000, 20, 8, 64),
                                                   (2, 5000, 70, 12, 3), (3, 1500, 10, 63, 10),
                                                   (4, 257, 3, 15, 64), (5, 31, 1, 7, 64),
                                                   (6, 9000, 33, 2, 64), (7, 4000, 5, 4, 1)])
def test_bestfirst_dyadic_exact(seed, n, F, leaves, depth):
    """Dyadic gradients: every sum is exact, so the GPU tree equals the oracle's
    (structure, node numbering, thresholds, leaf of every row)."""
    X, g, h = _dyadic(seed, n, F)
    _check(*_run(X, g, h, leaves, depth, 5 if n < 2000 else 20))


def test_bestfirst_unit_hessian():
    rng = np.random.default_rng(8)
    n, F = 40000, 65
    X = rng.normal(size=(n, F)).astype(np.float32)
    g = (rng.integers(-1000, 1000, size=n) / 128.0).astype(np.float32)
    _check(*_run(X, g, np.ones(n, np.float32), 15, 64, 20))


def test_bestfirst_interaction_and_mask():
    """Path-max interaction boost (selection only) and a feature mask."""
    X, g, h = _dyadic(9, 6000, 12)
    rng = np.random.default_rng(9)
    imat = rng.random(size=(12, 12)).astype(np.float32)
    fmask = (rng.random(12) < 0.7).astype(np.uint8)
    fmask[0] = 1
    _check(*_run(X, g, h, 14, 6, 20, imat, fmask.astype(bool)))


def test_bestfirst_single_leaf():
    """No split possible or allowed: one leaf holding every row."""
    X, g, h = _dyadic(10, 500, 4)
    for leaves, depth in ((1, 64), (8, 0)):
        ot, oleaf, gt, gl = _run(X, g, h, leaves, depth, 5)
        assert gt.feature.numel() == 1
        _check(ot, oleaf, gt, gl)


@pytest.mark.parametrize("case", range(4))
def test_bestfirst_matches_golden(golden, case):
    """The reference's own best-first runs (continuous gradients): structure,
    thresholds and leaves must match; values within float32 rounding."""
    z = golden("bestfirst")
    leaves, depth, msl = (int(v) for v in z[f"b{case}_params"])
    imat = z[f"b{case}_imat"]
    fm = z[f"b{case}_fmask"]
    ot, oleaf, gt, gl = _run(z[f"b{case}_X"], z[f"b{case}_g"], z[f"b{case}_h"], leaves, depth, msl,
                             imat if imat.size else None, fm if fm.size else None)
    _check(ot, oleaf, gt, gl)
    for k in ("feature", "left", "right", "threshold"):
        np.testing.assert_array_equal(getattr(gt, k).cpu().numpy(), z[f"b{case}_{k}"], err_msg=k)
    np.testing.assert_array_equal(gl, z[f"b{case}_leaf"])


def test_booster_auto_uses_bestfirst_below_16_leaves():
    """levelwise="auto" with max_leaves < 16 grows best-first (yabt/boosting.py:420):
    the booster's trees equal the oracle booster's under the same rule."""
    from oracle.boost import Booster as OBooster, BoostParams as OBP, MSELoss as OMSE
    from yabt_b200 import Booster, BoostParams, MSELoss
    rng = np.random.default_rng(11)
    n, F = 6000, 10
    X = rng.normal(size=(n, F)).astype(np.float32)
    y = (np.sin(X[:, 0] * 2) + X[:, 1] * (X[:, 2] > 0) + 0.1 * rng.normal(size=n)).astype(np.float32)
    ob = OBooster(OBP(n_estimators=4, max_leaves=6, learning_rate=0.3), OMSE()).fit(X, y)
    gb = Booster(BoostParams(n_estimators=4, max_leaves=6, learning_rate=0.3), MSELoss()).fit(X, y)
    for t in range(4):
        np.testing.assert_array_equal(gb.trees[t].feature.cpu().numpy(), ob.trees[t].feature, err_msg=f"tree {t}")
        np.testing.assert_array_equal(gb.trees[t].left.cpu().numpy(), ob.trees[t].left, err_msg=f"tree {t}")
    np.testing.assert_allclose(gb.predict_margin(X), ob.predict_margin(X), rtol=1e-4, atol=1e-4)


def _cgrow_pair(seed, n, F, leaves, depth, msl, imat=None, fmask=None, unit_h=False, gamma=0.0):
    from oracle import cgrow
    from yabt_b200.grower import grow_tree_c
    from yabt_b200.tree import TreeParams
    if not cgrow.available():
        pytest.skip("oracle/_ref/libcgrow.so not built")
    X, g, h = _dyadic(seed, n, F)
    if unit_h:
        h = np.ones(n, np.float32)
    b = OBinner().fit(X)
    binned = b.transform(X)
    nbins = np.array([min(len(e) + 1, 256) for e in b.edges_], np.int32)
    ref = cgrow.grow(np.ascontiguousarray(binned.T), g, h, nbins, leaves, depth, lam=1.0, gamma=gamma, mcw=1e-3,
                     msl=msl, lr=0.1, imat=imat, ib=0.5, fmask=fmask)
    tp = TreeParams(max_leaves=leaves, max_depth=depth, min_samples_leaf=msl, gamma=gamma)
    gt, gl = grow_tree_c(torch.from_numpy(binned).cuda(), torch.from_numpy(g).cuda(), torch.from_numpy(h).cuda(),
                         b, tp, torch.from_numpy(fmask.astype(bool)).cuda() if fmask is not None else None,
                         torch.from_numpy(imat).cuda() if imat is not None else None, 0.5, return_leaf=True)
    return b, binned, ref, gt, gl.cpu().numpy()


def _check_cgrow(b, binned, ref, gt, gl):
    feat, thr_bin, left, right, value, depth = ref
    np.testing.assert_array_equal(gt.feature.cpu().numpy(), feat, err_msg="feature")
    np.testing.assert_array_equal(gt.left.cpu().numpy(), left, err_msg="left")
    np.testing.assert_array_equal(gt.right.cpu().numpy(), right, err_msg="right")
    np.testing.assert_array_equal(gt.value.cpu().numpy(), value, err_msg="value")   # float64 math on exact sums
    thr = np.array([b.edges_[f][min(int(t), len(b.edges_[f]) - 1)] if f >= 0 else 0.0
                    for f, t in zip(feat, thr_bin)], np.float32)
    np.testing.assert_array_equal(gt.threshold.cpu().numpy(), thr, err_msg="threshold")
    assert gt.depth == int(depth.max()) + 1
    # the leaf of every row: the C grower's tree routed on the bins
    node = np.zeros(binned.shape[0], np.int64)
    for _ in range(int(depth.max()) + 1):
        f = feat[node]
        inner = f >= 0
        go_left = binned[np.arange(len(node)), np.where(inner, f, 0)] <= thr_bin[node]
        node = np.where(inner, np.where(go_left, left[node], right[node]), node)
    np.testing.assert_array_equal(gl, node)


@pytest.mark.parametrize("seed,n,F,leaves,depth", [(20, 3000, 8, 15, 64), (21, 20000, 20, 31, 64),
                                                   (22, 5000, 70, 12, 3), (23, 1500, 10, 63, 10),
                                                   (24, 257, 3, 15, 64), (25, 9000, 33, 2, 64)])
def test_c_grower_math_matches_reference_cgrow(seed, n, F, leaves, depth):
    """grow_tree_c on the GPU equals the reference's own C grower bit for bit
    (dyadic gradients: the C grower's float32 histogram bins are exact)."""
    _check_cgrow(*_cgrow_pair(seed, n, F, leaves, depth, 5 if n < 2000 else 20))


def test_c_grower_math_unit_hessian_and_gamma():
    _check_cgrow(*_cgrow_pair(26, 30000, 65, 31, 64, 20, unit_h=True, gamma=0.25))


def test_c_grower_math_interaction_and_mask():
    rng = np.random.default_rng(27)
    imat = rng.random(size=(12, 12)).astype(np.float32)
    fmask = (rng.random(12) < 0.7).astype(np.uint8)
    fmask[0] = 1
    _check_cgrow(*_cgrow_pair(27, 6000, 12, 14, 6, 20, imat, fmask))
