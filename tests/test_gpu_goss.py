"""GOSS (yabt/adaptive_features.py:61-110 via yabt/boosting.py:371-396) on the
GPU against the oracle booster: both draw the rows with torch's device sort and
a device generator seeded once per fit (the reference's own draw), grow on the
sampled rows with reweighted grad / hess, and route every row through the tree
for the leaf models and the margin update."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _data(n=6000, F=10, seed=31):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, F)).astype(np.float32)
    X[rng.random(size=X.shape) < 0.02] = np.nan
    z = np.nan_to_num(X)
    y = (np.sin(z[:, 0]) + z[:, 1] * z[:, 2] + 0.3 * z[:, 3] + 0.1 * rng.normal(size=n)).astype(np.float32)
    return X, y


@pytest.mark.parametrize("loss", ["mse", "logloss"])
@pytest.mark.parametrize("levelwise", [True, "auto"])
def test_goss_matches_oracle(loss, levelwise):
    from oracle.boost import Booster as OBooster, BoostParams as OBP, LogLoss as OLog, MSELoss as OMSE
    from yabt_b200 import Booster, BoostParams, LogLoss, MSELoss
    X, y = _data()
    if loss == "logloss":
        y = (y > np.median(y)).astype(np.float32)
    kw = dict(n_estimators=4, max_leaves=15, learning_rate=0.2, goss_enabled=True, goss_ratio=0.6,
              seed=5, neural_leaves=False, levelwise=levelwise)
    ob = OBooster(OBP(**kw, goss_device="cuda"), OMSE() if loss == "mse" else OLog()).fit(X, y)
    gb = Booster(BoostParams(**kw), MSELoss() if loss == "mse" else LogLoss()).fit(X, y)
    for t in range(4):
        for k in ("feature", "left", "right", "threshold"):
            np.testing.assert_array_equal(getattr(gb.trees[t], k).cpu().numpy(), getattr(ob.trees[t], k),
                                          err_msg=f"tree {t} {k}")
        np.testing.assert_allclose(gb.trees[t].value.cpu().numpy(), ob.trees[t].value, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(gb.predict_margin(X), ob.predict_margin(X), rtol=1e-4, atol=1e-4)


def test_goss_with_leaf_models():
    """Leaf models fit on every row (the tree saw the sample): first tree exact,
    predictions within the north-star tolerance."""
    from oracle.boost import Booster as OBooster, BoostParams as OBP, MSELoss as OMSE
    from yabt_b200 import Booster, BoostParams, MSELoss
    X, y = _data(seed=32)
    kw = dict(n_estimators=3, max_leaves=31, learning_rate=0.2, goss_enabled=True, goss_ratio=0.7, seed=6,
              leaf_net_min_samples=40)
    ob = OBooster(OBP(**kw, goss_device="cuda"), OMSE()).fit(X, y)
    gb = Booster(BoostParams(**kw), MSELoss()).fit(X, y)
    np.testing.assert_array_equal(gb.trees[0].feature.cpu().numpy(), ob.trees[0].feature)
    np.testing.assert_allclose(gb.predict_margin(X), ob.predict_margin(X), rtol=1e-4, atol=1e-4)


def test_goss_ratio_one_keeps_the_top_rows_only():
    """ratio 1.0: keep = n, top = max(1, round(0)) = 1, so 1 top row plus n - 1
    drawn rows weighted (n - 1) / (n - 1) = 1; the tree sees every row."""
    from yabt_b200.sampling import goss_sample
    import torch
    g = torch.randn(1000, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(0)
    rows, w = goss_sample(g, 1.0, gen)
    assert rows.numel() == 1000 and torch.unique(rows).numel() == 1000
    assert w is not None and bool(torch.all(w == 1.0))
