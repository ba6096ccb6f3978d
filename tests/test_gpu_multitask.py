"""Multi-task trees on the GPU (yabt/multitask.py:60-251): the grower against
the CPU oracle (oracle.multitask, pinned to the reference's runs in
tests/golden/multitask.npz) and the reference's own outputs; the estimator
against the reference's predictions."""

import numpy as np
import pytest
import torch

from oracle.binning import Binner as OBinner
from oracle.grow import TreeParams as OTP
from oracle.multitask import grow_multitask

pytestmark = pytest.mark.gpu


def _pair(X, g, leaves, depth, msl, fmask=None):
    from yabt_b200.boosting import BoostParams
    from yabt_b200.multitask import grow_multitask_tree
    b = OBinner().fit(X)
    binned = b.transform(X)
    ref = grow_multitask(binned, g, np.ones_like(g), b.edges_,
                         OTP(max_leaves=leaves, max_depth=depth, min_samples_leaf=msl), fmask)
    p = BoostParams(max_leaves=leaves, max_depth=depth, min_samples_leaf=msl, learning_rate=0.1)
    fm = torch.from_numpy(fmask).cuda() if fmask is not None else None
    tree, leaf = grow_multitask_tree(torch.from_numpy(binned).cuda(), torch.from_numpy(g).cuda(),
                                     torch.ones(g.shape, device="cuda"), b, p, fm, return_leaf=True)
    return ref, tree, leaf.cpu().numpy()


def _check(ref, tree, leaf, exact_values):
    feat, thr, left, right, value, depth, oleaf = ref
    np.testing.assert_array_equal(tree.feature.cpu().numpy(), feat, err_msg="feature")
    np.testing.assert_array_equal(tree.left.cpu().numpy(), left, err_msg="left")
    np.testing.assert_array_equal(tree.right.cpu().numpy(), right, err_msg="right")
    np.testing.assert_array_equal(tree.threshold.cpu().numpy(), thr, err_msg="threshold")
    assert tree.depth == depth
    if exact_values:
        np.testing.assert_array_equal(tree.value.cpu().numpy(), value)
    else:
        np.testing.assert_allclose(tree.value.cpu().numpy(), value, rtol=1e-5, atol=1e-7)
    np.testing.assert_array_equal(leaf, oleaf)


@pytest.mark.parametrize("seed,n,F,T,leaves,depth", [(0, 3000, 8, 2, 15, 64), (1, 20000, 20, 3, 31, 64),
                                                     (2, 5000, 40, 1, 12, 3), (3, 1500, 10, 8, 63, 10),
                                                     (4, 400, 3, 5, 15, 64), (5, 9000, 33, 4, 2, 64)])
def test_multitask_dyadic_exact(seed, n, F, T, leaves, depth):
    """Dyadic gradients: every sum is exact, so the GPU tree and its per-task
    values equal the oracle's bit for bit."""
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, F)).astype(np.float32)
    X[rng.random(size=X.shape) < 0.01] = np.nan
    g = (rng.integers(-512, 512, size=(n, T)) / 256.0).astype(np.float32)
    _check(*_pair(X, g, leaves, depth, 5 if n < 2000 else 20), exact_values=True)


def test_multitask_feature_mask():
    rng = np.random.default_rng(6)
    X = rng.normal(size=(6000, 12)).astype(np.float32)
    g = (rng.integers(-512, 512, size=(6000, 3)) / 256.0).astype(np.float32)
    fmask = rng.random(12) < 0.6
    fmask[0] = True
    _check(*_pair(X, g, 20, 64, 20, fmask), exact_values=True)


@pytest.mark.parametrize("case", range(4))
def test_multitask_matches_golden(golden, case):
    """The reference's own multi-task trees (continuous gradients)."""
    z = golden("multitask")
    leaves, depth, msl = (int(v) for v in z[f"m{case}_params"])
    fm = z[f"m{case}_fmask"]
    ref, tree, leaf = _pair(z[f"m{case}_X"], z[f"m{case}_g"], leaves, depth, msl, fm if fm.size else None)
    _check(ref, tree, leaf, exact_values=False)
    for k in ("feature", "left", "right", "threshold"):
        np.testing.assert_array_equal(getattr(tree, k).cpu().numpy(), z[f"m{case}_{k}"], err_msg=k)
    np.testing.assert_allclose(tree.value.cpu().numpy(), z[f"m{case}_value"], rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(leaf, z[f"m{case}_leaf"])


def test_multitask_estimator_matches_reference(golden):
    from yabt_b200 import YABTMultiTaskRegressor
    z = golden("multitask")
    est = YABTMultiTaskRegressor(n_estimators=8, max_leaves=15, learning_rate=0.2).fit(z["est_X"], z["est_Y"])
    np.testing.assert_array_equal(est.booster_.trees[0].feature.cpu().numpy(), z["est_feature0"])
    np.testing.assert_allclose(est.predict(z["est_X"]), z["est_pred"], rtol=1e-4, atol=1e-4)


def test_multitask_sampling_and_eval_set():
    """Row subsampling and feature masks (the single-task draw order), eval_set
    with early stopping, a 1-D target."""
    from yabt_b200 import YABTMultiTaskRegressor
    rng = np.random.default_rng(8)
    X = rng.normal(size=(5000, 9)).astype(np.float32)
    Y = np.stack([X[:, 0] + X[:, 1] * X[:, 2], np.sin(X[:, 3])], axis=1).astype(np.float32)
    est = YABTMultiTaskRegressor(n_estimators=30, max_leaves=15, subsample=0.7, colsample=0.8,
                                 early_stopping_rounds=5).fit(X[:4000], Y[:4000], eval_set=(X[4000:], Y[4000:]))
    pred = est.predict(X[4000:])
    r2 = 1 - ((Y[4000:] - pred) ** 2).mean(axis=0) / Y[4000:].var(axis=0)
    assert pred.shape == (1000, 2) and (r2 > 0.5).all()
    one = YABTMultiTaskRegressor(n_estimators=5, max_leaves=7).fit(X, Y[:, 0])
    assert one.predict(X[:10]).shape == (10,)
