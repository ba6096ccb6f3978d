"""One-vs-rest multiclass (yabt/multiclass.py:9-48) on the GPU: the class
boosters run interleaved on their own CUDA streams; every class's model must
equal, bit for bit, an independent binary booster fitted alone on the default
stream (the binary booster itself is checked against the oracle in
test_gpu_pipeline.py)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _data(n=4000, F=9, classes=4, seed=11):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, F)).astype(np.float32)
    X[rng.random(size=X.shape) < 0.02] = np.nan
    z = np.nan_to_num(X)
    W = rng.normal(scale=0.8, size=(F, classes))
    s = z @ W + 0.3 * z[:, :classes] * z[:, 1:classes + 1]
    y = np.argmax(s + rng.gumbel(size=s.shape), axis=1).astype(np.float32)
    return X, y


def _params():
    from yabt_b200.boosting import BoostParams
    return BoostParams(n_estimators=6, max_leaves=12, max_depth=5, learning_rate=0.2, neural_leaves=True,
                       leaf_net_min_samples=40, min_samples_leaf=10)


def test_streams_match_independent_boosters():
    from yabt_b200.boosting import Booster, LogLoss
    from yabt_b200.multiclass import MulticlassBooster
    X, y = _data()
    mc = MulticlassBooster(_params()).fit(X, y)
    assert list(mc.classes_) == [0.0, 1.0, 2.0, 3.0]
    for c, bm in zip(mc.classes_, mc.boosters_):
        b = Booster(_params(), LogLoss()).fit(X, (y == c).astype(np.float32))
        assert len(b.trees) == len(bm.trees)
        for ta, tb in zip(bm.trees, b.trees):
            for k in ("feature", "threshold", "left", "right", "value"):
                np.testing.assert_array_equal(getattr(ta, k).cpu().numpy(), getattr(tb, k).cpu().numpy(),
                                              err_msg=f"class {c} {k}")
        np.testing.assert_array_equal(bm.predict_margin(X[:500]), b.predict_margin(X[:500]))
    p = mc.predict_proba(X[:500])
    np.testing.assert_allclose(p.sum(axis=1), 1.0, rtol=1e-6)
    assert (mc.predict(X) == y).mean() > 0.5          # four classes: chance is ~0.25


def test_classifier_estimator_multiclass():
    from yabt_b200 import YABTClassifier
    X, y = _data(n=3000, classes=3, seed=12)
    est = YABTClassifier(n_estimators=5, max_leaves=8, learning_rate=0.3).fit(X, y)
    proba = est.predict_proba(X[:200])
    assert proba.shape == (200, 3)
    assert set(np.unique(est.predict(X[:200]))) <= {0.0, 1.0, 2.0}
