"""CUDA binning, neural leaves and the boosting loop vs the CPU oracle (GPU tests)."""
import os
import sys

import numpy as np
import pytest
import torch

from oracle.binning import Binner as OBinner
from oracle.boost import Booster as OBooster, BoostParams as OBP, LogLoss as OLog, MSELoss as OMSE
from oracle.grow import OTree
from oracle.leafnet import column_stats, fit_leaf_networks as o_fit_leaf_networks

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_golden import _data  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("seed,n,F,nanf", [(0, 3000, 7, 0.0), (1, 1001, 5, 0.05), (2, 210_000, 3, 0.02),
                                           (3, 599, 4, 0.0), (4, 1, 2, 0.0), (5, 65537, 70, 0.01)])
def test_binner_bit_exact(seed, n, F, nanf):
    from yabt_b200.binning import Binner
    X, _ = _data(seed, n, F, nanf)
    if seed == 0:
        X[:, 4] = 1.5
        X[:, 5] = np.nan
    ob = OBinner().fit(X)
    gb = Binner().fit(X)
    np.testing.assert_array_equal(gb.medians_, ob.medians_)
    for f in range(F):
        np.testing.assert_array_equal(gb.edges_[f].numpy(), ob.edges_[f], err_msg=f"edges f={f}")
    np.testing.assert_allclose(gb.scales_.numpy(), ob.scales_, rtol=1e-6)
    np.testing.assert_array_equal(gb.transform(X).cpu().numpy(), ob.transform(X))


def test_binner_golden(golden):
    from yabt_b200.binning import Binner
    z = golden("binning")
    for i in range(int(z["ncases"])):
        seed, n, F, nanf = z["cases"][i]
        X = z[f"c{i}_X"] if f"c{i}_X" in z else _data(int(seed), int(n), int(F), float(nanf))[0]
        gb = Binner().fit(X)
        np.testing.assert_array_equal(np.concatenate([e.numpy() for e in gb.edges_]), z[f"c{i}_edges"])
        np.testing.assert_array_equal(gb.medians_, z[f"c{i}_medians"])
        np.testing.assert_array_equal(gb.transform(X).cpu().numpy(), z[f"c{i}_bins"])


def _fit_pair(X, y, loss, n_trees, **kw):
    from yabt_b200 import Booster, BoostParams, LogLoss, MSELoss
    okw = {k: v for k, v in kw.items() if k in OBP.__dataclass_fields__}
    ob = OBooster(OBP(n_estimators=n_trees, **okw), OMSE() if loss == "mse" else OLog())
    ob.fit(X, y, record=True)
    gb = Booster(BoostParams(n_estimators=n_trees, **kw), MSELoss() if loss == "mse" else LogLoss())
    gb.fit(X, y)
    return ob, gb


@pytest.mark.parametrize("loss,n", [("mse", 6000), ("logloss", 6000), ("mse", 1_300_000)])
def test_first_tree_with_leaf_nets_matches_oracle(loss, n):
    """One full boosting iteration (grad -> tree -> leaf nets -> margin) vs the
    oracle; at 1.3M rows each fp64 Gram partial holds 4,096 rows (8,192 rows per
    leaf and more span several partials)."""
    X, y = _data(40, n, 10, 0.02)
    if loss == "logloss":
        y = (y > np.median(y)).astype(np.float32)
    ob, gb = _fit_pair(X, y, loss, 1, max_leaves=31)
    ot, gt = ob.trees[0], gb.trees[0]
    np.testing.assert_array_equal(gt.feature.cpu().numpy(), ot.feature)
    np.testing.assert_array_equal(gt.threshold.cpu().numpy(), ot.threshold)
    np.testing.assert_array_equal(gt.left.cpu().numpy(), ot.left)
    np.testing.assert_allclose(gt.value.cpu().numpy(), ot.value, rtol=1e-5, atol=1e-6)
    assert (gt.leaf_net_feats is None) == (ot.leaf_net_feats is None)
    if ot.leaf_net_feats is not None:
        np.testing.assert_array_equal(gt.leaf_net_feats.cpu().numpy(), ot.leaf_net_feats)
        leaf = ot.feature == -1
        np.testing.assert_array_equal(gt.leaf_net_lo.cpu().numpy()[leaf], ot.leaf_net_lo[leaf])
        np.testing.assert_array_equal(gt.leaf_net_hi.cpu().numpy()[leaf], ot.leaf_net_hi[leaf])
        np.testing.assert_allclose(gt.leaf_net_linear.cpu().numpy()[leaf], ot.leaf_net_linear[leaf],
                                   rtol=1e-4, atol=1e-6)
    pm = gb.predict_margin(X)
    np.testing.assert_allclose(pm, ob.predict_margin(X), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(gb._margin_train.cpu().numpy(), ob.margin_, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("loss,n,F,leaves,trees", [("mse", 20000, 20, 31, 12), ("logloss", 8000, 15, 63, 8)])
def test_boosting_matches_oracle(loss, n, F, leaves, trees):
    """Several trees with interaction steering on (n >= 2000): every tree's
    structure matches the oracle's and predictions agree within 1e-4."""
    X, y = _data(41, n, F, 0.0)
    if loss == "logloss":
        y = (y > np.median(y)).astype(np.float32)
    ob, gb = _fit_pair(X, y, loss, trees, max_leaves=leaves, learning_rate=0.1)
    for t in range(trees):
        np.testing.assert_array_equal(gb.trees[t].feature.cpu().numpy(), ob.trees[t].feature, err_msg=f"tree {t}")
    np.testing.assert_allclose(gb.predict_margin(X), ob.predict_margin(X), rtol=1e-4, atol=1e-4)


def test_reference_golden_predictions(golden):
    """Booster fits on the reference's golden inputs reproduce its predictions."""
    from yabt_b200 import Booster, BoostParams, LogLoss, MSELoss
    z = golden("boost")
    bm = Booster(BoostParams(n_estimators=12, max_leaves=15, learning_rate=0.1, levelwise=True), MSELoss()).fit(z["mse_X"], z["mse_y"])
    for t in range(3):
        np.testing.assert_array_equal(bm.trees[t].feature.cpu().numpy(), z[f"mse_t{t}_feature"])
    np.testing.assert_allclose(bm.predict_margin(z["mse_X"]), z["mse_pred"], rtol=1e-4, atol=1e-4)
    bl = Booster(BoostParams(n_estimators=10, max_leaves=15, learning_rate=0.2, levelwise=True), LogLoss()).fit(z["log_X"], z["log_y"])
    np.testing.assert_allclose(bl.predict_margin(z["log_X"]), z["log_pred"], rtol=1e-4, atol=1e-4)


def test_sklearn_estimators_golden(golden):
    from yabt_b200 import YABTClassifier, YABTRegressor
    z = golden("boost")
    clf = YABTClassifier(n_estimators=6, max_leaves=15, levelwise=True, seed=0).fit(z["mc_X"], z["mc_y"])
    np.testing.assert_allclose(clf.predict_proba(z["mc_X"]), z["mc_proba"], rtol=1e-4, atol=1e-5)
    reg = YABTRegressor(n_estimators=20).fit(z["mse_X"], z["mse_y"])
    r = z["mse_y"] - reg.predict(z["mse_X"])
    assert 1 - r.var() / z["mse_y"].var() > 0.8


def test_apply_equals_training_leaf():
    """Tree.apply on the imputed raw matrix equals the grower's final leaf of
    every training row (the bin / threshold equivalence)."""
    from yabt_b200 import Booster, BoostParams, MSELoss
    X, y = _data(42, 5000, 9, 0.03)
    b = Booster(BoostParams(n_estimators=3, max_leaves=63), MSELoss()).fit(X, y)
    Xi = torch.from_numpy(b.binner.impute(X)).cuda()
    from yabt_b200.predict import apply_tree
    leaf = apply_tree(b.trees[-1], Xi)
    ob = OBinner().fit(X)
    t = b.trees[-1]
    ot = OTree(t.feature.cpu().numpy(), t.threshold.cpu().numpy(), t.left.cpu().numpy(), t.right.cpu().numpy(),
               t.value.cpu().numpy(), t.depth, t.gate_scale.cpu().numpy())
    np.testing.assert_array_equal(leaf.cpu().numpy(), ot.apply(ob.impute(X)))


def test_predict_on_zero_rows():
    """Every estimator predicts an empty matrix as an empty result (the
    reference's numpy / torch prediction path does)."""
    from yabt_b200 import YABTClassifier, YABTMultiTaskRegressor, YABTRegressor
    X, y = _data(11, 2000, 6, 0.02)
    X0 = X[:0]
    reg = YABTRegressor(n_estimators=3, max_leaves=15).fit(X, y)
    assert reg.predict(X0).shape == (0,)
    clf = YABTClassifier(n_estimators=3, max_leaves=15).fit(X, (y > np.median(y)).astype(int))
    assert clf.predict(X0).shape == (0,)
    assert clf.predict_proba(X0).shape == (0, 2)
    yc = np.digitize(y, np.quantile(y, [1 / 3, 2 / 3]))
    mc = YABTClassifier(n_estimators=3, max_leaves=15).fit(X, yc)
    assert mc.predict(X0).shape == (0,)
    assert mc.predict_proba(X0).shape == (0, 3)
    mt = YABTMultiTaskRegressor(n_estimators=3, max_leaves=15).fit(X, np.stack([y, -y], axis=1))
    assert mt.predict(X0).shape == (0, 2)
    assert tuple(reg.booster_.binner.transform(X0).shape) == (0, 6)
