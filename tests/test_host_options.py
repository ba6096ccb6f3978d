"""Host-side option handling on the CPU: options outside the GPU tree-growth
path raise NotImplementedError naming the option (nothing falls back to a CPU
implementation), the device must be CUDA, and the grower is chosen as the
reference chooses it on a CUDA device (yabt/boosting.py:415-426). No GPU is used."""

import numpy as np
import pytest

from yabt_b200.boosting import BoostParams, _check_supported, use_bestfirst, use_c_grower_math

UNSUPPORTED = [("kernel_splits", True), ("refine_steps", 2), ("refit_every", 5), ("adaptive_features", True),
               ("product_features", True), ("auto_tune", True), ("stochastic_routing", True),
               ("leaf_net_hidden", 16), ("subsample", 0.0), ("levelwise", "sometimes")]


@pytest.mark.parametrize("name,value", UNSUPPORTED)
def test_unsupported_option_raises_with_its_name(name, value):
    with pytest.raises(NotImplementedError, match=name):
        _check_supported(BoostParams(**{name: value}))


def test_supported_defaults_pass_and_cpu_device_raises():
    _check_supported(BoostParams())                              # "auto" resolves to CUDA
    _check_supported(BoostParams(subsample=0.5, colsample=0.5, goss_enabled=True, levelwise=False))
    with pytest.raises(NotImplementedError, match="CUDA"):
        _check_supported(BoostParams(device="cpu"))


def test_estimator_fit_rejects_before_any_device_work():
    from yabt_b200 import YABTClassifier, YABTRegressor
    X = np.random.default_rng(0).normal(size=(50, 3)).astype(np.float32)
    y = X[:, 0]
    with pytest.raises(NotImplementedError, match="CUDA"):
        YABTRegressor(n_estimators=2, device="cpu").fit(X, y)
    with pytest.raises(NotImplementedError, match="kernel_splits"):
        YABTRegressor(n_estimators=2, kernel_splits=True).fit(X, y)
    with pytest.raises(NotImplementedError, match="categorical"):
        YABTClassifier(n_estimators=2).fit(X, (y > 0).astype(int), categorical_features=[1])


@pytest.mark.parametrize("levelwise,max_leaves,numba,bestfirst,cmath", [
    (True, 8, "auto", False, False),       # level-wise on request
    ("auto", 16, "auto", False, False),    # "auto": level-wise from 16 leaves
    ("auto", 15, "auto", True, False),     # "auto": best-first below 16 leaves
    (False, 255, "auto", True, False),     # best-first on request
    (False, 255, True, True, True),        # the C / Numba grower's arithmetic
    (True, 255, True, False, False),       # level-wise wins over numba_grower
])
def test_grower_choice(levelwise, max_leaves, numba, bestfirst, cmath):
    p = BoostParams(levelwise=levelwise, max_leaves=max_leaves, numba_grower=numba)
    assert use_bestfirst(p) is bestfirst
    assert use_c_grower_math(p) is cmath
