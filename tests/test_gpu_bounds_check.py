"""The bounds-checked build (GPU test).

``python -m yabt_b200.build --bounds-check`` compiles the library with
``-DYABT_BOUNDS_CHECK`` into ``libyabt_b200_checked.so``: every row id the
histogram kernel and the row partition read from a row list, every row the
leaf assignment writes and every node the routing of all rows follows is
checked before the access; a failing check sets a device error bit (which
``Booster.fit`` raises on) and skips the access. This test fits small models
with that build in a child process (``YABT_LIB_VARIANT=checked``) -- the
level-wise grower with leaf models, the best-first grower, row subsampling
and a log-loss fit -- and requires no error bit and the same trees as the
ordinary build fits in this process."""

import json
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECKED = os.path.join(ROOT, "yabt_b200", "libyabt_b200_checked.so")

SCRIPT = r"""
import json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from yabt_b200 import Booster, BoostParams, LogLoss, MSELoss, _lib
assert _lib.LIB_PATH.endswith(sys.argv[2])
rng = np.random.default_rng(5)
X = rng.normal(size=(6000, 23)).astype(np.float32)
X[rng.random(size=X.shape) < 0.02] = np.nan
z = np.nan_to_num(X)
y = (np.sin(z[:, 0]) + z[:, 1] * z[:, 2] + 0.1 * rng.normal(size=6000)).astype(np.float32)
cases = {
    "levelwise": (dict(n_estimators=4, max_leaves=63), MSELoss(), y),
    "bestfirst": (dict(n_estimators=3, max_leaves=12), MSELoss(), y),
    "subsample": (dict(n_estimators=3, max_leaves=31, subsample=0.7), MSELoss(), y),
    "logloss": (dict(n_estimators=3, max_leaves=31), LogLoss(), (y > np.median(y)).astype(np.float32)),
}
out = {}
for name, (kw, loss, target) in cases.items():
    b = Booster(BoostParams(**kw), loss).fit(X, target)
    out[name] = {"trees": [[t.feature.cpu().tolist(), t.threshold.cpu().tolist(), t.left.cpu().tolist()]
                           for t in b.trees],
                 "pred": b.predict_margin(X[:500]).tolist()}
print(json.dumps(out))
"""


def _run(variant: str, libname: str) -> dict:
    env = dict(os.environ)
    env.pop("YABT_LIB_VARIANT", None)
    if variant:
        env["YABT_LIB_VARIANT"] = variant
    r = subprocess.run([sys.executable, "-c", SCRIPT, ROOT, libname], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_bounds_checked_build_matches_and_reports_nothing():
    if not os.path.exists(CHECKED):
        pytest.fail("libyabt_b200_checked.so missing: python -m yabt_b200.build --bounds-check")
    checked = _run("checked", "libyabt_b200_checked.so")
    plain = _run("", "libyabt_b200.so")
    for name in plain:
        assert checked[name]["trees"] == plain[name]["trees"], name
        np.testing.assert_array_equal(np.array(checked[name]["pred"]), np.array(plain[name]["pred"]))
