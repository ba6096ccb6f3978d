"""yabt_b200: B200-native tree-growth path of the YABT gradient-boosting library.

The public surface mirrors the reference package (``yabt``): estimators,
``Booster`` / ``BoostParams``, ``Tree``, ``grow_tree_levelwise`` and
``cuda_hist.build_hist``. Compute runs in hand-written sm_100a CUDA kernels
of ``libyabt_b200.so`` behind a C ABI (include/yabt_b200.h).
"""

from .tree import LEAF, Tree, TreeParams  # noqa: F401

__all__ = ["LEAF", "Tree", "TreeParams"]
