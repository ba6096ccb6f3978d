"""yabt_b200: B200-native tree-growth path of the YABT gradient-boosting library.

The public surface mirrors the reference package (``yabt``): the estimators
``YABTRegressor`` / ``YABTClassifier``, ``Booster`` / ``BoostParams`` /
``LogLoss`` / ``MSELoss``, ``Tree``, ``Binner``, ``grow_tree_levelwise`` and
``cuda_hist.build_hist``. Compute runs in hand-written sm_100a CUDA kernels of
``libyabt_b200.so`` behind a C ABI (include/yabt_b200.h); there is no CPU
fallback.
"""

from .binning import Binner  # noqa: F401
from .boosting import Booster, BoostParams, LogLoss, MSELoss  # noqa: F401
from .grower import grow_tree, grow_tree_c, grow_tree_levelwise  # noqa: F401
from .multiclass import MulticlassBooster  # noqa: F401
from .multitask import MultiTaskBooster  # noqa: F401
from .sklearn_api import YABTClassifier, YABTMultiTaskRegressor, YABTRegressor  # noqa: F401
from .tree import LEAF, Tree, TreeParams  # noqa: F401

__all__ = [
    "Binner", "Booster", "BoostParams", "LogLoss", "MSELoss", "MulticlassBooster",
    "YABTClassifier", "YABTRegressor", "YABTMultiTaskRegressor", "MultiTaskBooster", "Tree", "TreeParams", "LEAF", "grow_tree", "grow_tree_c", "grow_tree_levelwise",
]
