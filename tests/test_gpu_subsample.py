"""Row subsampling (yabt/boosting.py:374-376, 392-393, 486): each tree grows on
rows[:m] of a permutation drawn from the CPU generator, and the leaf models and
the margin update route every row. The GPU booster must draw the same rows as
the oracle restatement and grow the same trees: every tree's structure is
identical, predictions agree within 1e-4 relative."""
import os
import sys

import numpy as np
import pytest

from oracle.boost import Booster as OBooster, BoostParams as OBP, LogLoss as OLog, MSELoss as OMSE

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_golden import _data  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("loss,neural", [("mse", False), ("mse", True), ("logloss", True)])
def test_subsample_matches_oracle(loss, neural):
    from yabt_b200 import Booster, BoostParams, LogLoss, MSELoss
    X, y = _data(51, 6000, 9, 0.02)
    if loss == "logloss":
        y = (y > np.median(y)).astype(np.float32)
    kw = dict(n_estimators=4, max_leaves=15, learning_rate=0.2, subsample=0.6, seed=3, neural_leaves=neural)
    ob = OBooster(OBP(**kw), OMSE() if loss == "mse" else OLog()).fit(X, y)
    gb = Booster(BoostParams(**kw), MSELoss() if loss == "mse" else LogLoss()).fit(X, y)
    for t in range(4):
        np.testing.assert_array_equal(gb.trees[t].feature.cpu().numpy(), ob.trees[t].feature, err_msg=f"tree {t}")
        np.testing.assert_array_equal(gb.trees[t].threshold.cpu().numpy(), ob.trees[t].threshold, err_msg=f"tree {t}")
    np.testing.assert_allclose(gb.predict_margin(X), ob.predict_margin(X), rtol=1e-4, atol=1e-4)


def test_group_rows_is_a_stable_grouping():
    """yabt_group_rows: rows of each leaf in increasing order, ranges tile [0, n)."""
    import torch
    from yabt_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(5)
    for n, L in ((100_000, 63), (8193, 7), (1, 1), (300_000, 511)):
        leaf = rng.integers(0, L, size=n).astype(np.int32)
        leaf[rng.random(n) < 0.3] = L - 1                     # a crowded leaf
        d = torch.from_numpy(leaf).cuda()
        ws = torch.empty(int(lib.yabt_group_rows_workspace_bytes(n, L)), dtype=torch.uint8, device="cuda")
        b = torch.empty(L, dtype=torch.int32, device="cuda")
        c = torch.empty(L, dtype=torch.int32, device="cuda")
        r = torch.empty(n, dtype=torch.int32, device="cuda")
        _lib.check(lib.yabt_group_rows(d.data_ptr(), n, L, ws.data_ptr(), ws.numel(), b.data_ptr(), c.data_ptr(),
                                       r.data_ptr(), _lib.stream_ptr()), "yabt_group_rows")
        np.testing.assert_array_equal(r.cpu().numpy(), np.argsort(leaf, kind="stable"))
        np.testing.assert_array_equal(c.cpu().numpy(), np.bincount(leaf, minlength=L))
        np.testing.assert_array_equal(b.cpu().numpy(), np.concatenate([[0], np.cumsum(np.bincount(leaf, minlength=L))[:-1]]))
