"""The device-side level loop (GPU tests).

A level-wise tree whose depth limit lies far beyond the depth its leaf budget
lets it reach (the reference's default max_depth with a small max_leaves)
would queue many levels that only find the tree complete. The grower instead
launches the levels below ``level_loop_start()`` as usual and then one CUDA
graph whose conditional WHILE node repeats a level's kernels while the tree
is active (the reference's host ``while`` over levels, yabt/tree.py:484-625).
These tests fit the same data with the loop on and off: every tree, leaf
value and prediction must be the same bits, the loop must have run (levels
counted on the device), and the host must have launched fewer kernels. The
loop-on fits are also the path every other GPU test of level-wise trees now
takes, where they are compared with the oracle.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _data(n=30000, F=12, seed=3, classify=False, chain=10):
    """A nested target: y steps up by 2 each time x_0, x_1, ... x_{chain-1} all
    stay above -0.3. Rows that leave the chain share one target value, so their
    nodes have no split with positive gain, and the trees grow a long chain
    (depth about `chain`) instead of a balanced tree."""
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, F)).astype(np.float32)
    X[:, chain:][rng.random(size=(n, F - chain)) < 0.02] = np.nan
    on = np.ones(n, dtype=bool)
    y = np.zeros(n, dtype=np.float32)
    for k in range(chain):
        on &= X[:, k] > -0.3
        y += 2.0 * on
    if classify:
        y = (y >= 6.0).astype(np.float32)
    return X, y


def _fit(params, X, y, loss, loop):
    import torch
    from yabt_b200 import _lib
    from yabt_b200.boosting import Booster
    lib = _lib.load()
    b = Booster(params, loss)
    b._level_loop = loop
    torch.cuda.synchronize()
    _lib.check(lib.yabt_launch_count_device_reset(_lib.stream_ptr()), "reset")
    h0 = int(lib.yabt_launch_count())
    b.fit(X, y)
    torch.cuda.synchronize()
    return b, int(lib.yabt_launch_count()) - h0, int(lib.yabt_launch_count_device())


def _same(a, b, X):
    assert len(a.trees) == len(b.trees)
    for t, (ta, tb) in enumerate(zip(a.trees, b.trees)):
        for k in ("feature", "threshold", "left", "right", "value"):
            np.testing.assert_array_equal(getattr(ta, k).cpu().numpy(), getattr(tb, k).cpu().numpy(),
                                          err_msg=f"tree {t} {k}")
    np.testing.assert_array_equal(a.predict_margin(X), b.predict_margin(X))


CASES = [
    # (loss, max_leaves, max_depth, neural, subsample, colsample, trees reach past the loop's start)
    ("mse", 31, 64, False, 1.0, 1.0, True),
    ("logloss", 63, 64, False, 1.0, 1.0, True),
    ("mse", 31, 9, False, 1.0, 1.0, True),      # the depth limit stops the trees inside the loop
    ("mse", 31, 64, True, 1.0, 1.0, False),     # neural leaves
    ("mse", 24, 64, False, 0.7, 0.6, False),    # row sample (root row list) and feature masks
]


@pytest.mark.parametrize("loss_name,leaves,depth,neural,subsample,colsample,deep", CASES)
def test_loop_matches_host_levels(loss_name, leaves, depth, neural, subsample, colsample, deep):
    from yabt_b200.boosting import BoostParams, LogLoss, MSELoss
    X, y = _data(classify=loss_name == "logloss")
    params = BoostParams(n_estimators=6, max_leaves=leaves, max_depth=depth, learning_rate=0.3,
                         neural_leaves=neural, leaf_net_min_samples=60, min_samples_leaf=5,
                         subsample=subsample, colsample=colsample, levelwise=True)
    loss = (lambda: LogLoss()) if loss_name == "logloss" else (lambda: MSELoss())
    on, host_on, dev_on = _fit(params, X, y, loss(), True)
    off, host_off, dev_off = _fit(params, X, y, loss(), False)
    L = on.grower_.level_loop_start()
    assert L > 0
    _same(on, off, X[:3000])
    assert dev_off == 0
    assert host_on < host_off
    if deep:
        # trees split nodes inside the loop: the loop ran passes, and a tree
        # reached below the loop's first level (to max_depth when it binds)
        assert dev_on >= 7, dev_on
        reach = max(_depth(t) for t in on.trees)
        assert reach > L
        assert reach <= depth


def _depth(tree) -> int:
    left, right = tree.left.cpu().numpy(), tree.right.cpu().numpy()
    depth, stack = 0, [(0, 0)]
    while stack:
        i, d = stack.pop()
        depth = max(depth, d)
        if left[i] >= 0:
            stack += [(int(left[i]), d + 1), (int(right[i]), d + 1)]
    return depth


def test_loop_start_rules():
    from yabt_b200.grower import Grower
    g = Grower(1000, 8, 31, 64, False, "cuda")
    assert g.level_loop_start() == -1               # a new grower waits on the host (its own stop rule)
    g.set_level_wait(False)
    assert g.level_loop_start() == 6                # 2^5 >= max_pairs = 30
    g.set_level_loop(False)
    assert g.level_loop_start() == -1
    g.set_level_loop(True)
    assert g.level_loop_start() == 6
    for leaves, depth in ((255, 10), (8, 64)):      # C4's shape: only level 9 would be left; < 8 pairs
        g2 = Grower(1000, 8, leaves, depth, False, "cuda")
        g2.set_level_wait(False)
        assert g2.level_loop_start() == -1


def test_loop_regraphs_when_parameters_change():
    """The graph bakes in the grower's parameters: a second fit on the same
    grower-sized problem with another lambda must give that lambda's trees."""
    from yabt_b200.boosting import BoostParams, MSELoss
    X, y = _data(n=12000, seed=5)
    for lam in (1.0, 7.5):
        params = BoostParams(n_estimators=3, max_leaves=31, max_depth=64, learning_rate=0.3, reg_lambda=lam,
                             neural_leaves=False, levelwise=True)
        on, _, dev_on = _fit(params, X, y, MSELoss(), True)
        off, _, _ = _fit(params, X, y, MSELoss(), False)
        _same(on, off, X[:2000])
        assert dev_on > 0


def test_multiclass_streams_with_loop():
    from yabt_b200.boosting import BoostParams
    from yabt_b200.multiclass import MulticlassBooster
    X, y = _data(n=8000, seed=9)
    cls = np.digitize(y, np.quantile(y, [0.25, 0.5, 0.75])).astype(np.float32)
    params = BoostParams(n_estimators=4, max_leaves=31, max_depth=64, learning_rate=0.3, neural_leaves=True,
                         leaf_net_min_samples=40, min_samples_leaf=5)
    a = MulticlassBooster(params).fit(X, cls)
    b = MulticlassBooster(params)
    orig = b.fit
    # loop off in every class booster: set before the boosters grow their first tree
    import yabt_b200.boosting as boosting
    saved = getattr(boosting.Booster, "_level_loop", None)
    boosting.Booster._level_loop = False
    try:
        orig(X, cls)
    finally:
        if saved is None:
            del boosting.Booster._level_loop
        else:
            boosting.Booster._level_loop = saved
    for ba, bb in zip(a.boosters_, b.boosters_):
        _same(ba, bb, X[:1000])
