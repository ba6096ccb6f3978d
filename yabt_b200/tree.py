"""Tree layout (unchanged from the reference) and tree-level entry points.

``Tree`` keeps the field layout of yabt/tree.py:39-76 so that pickled models
and callers that read the arrays see the same structure. Its inference
methods run on the CUDA kernels of ``libyabt_b200.so``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

LEAF = -1
KERNEL_SPLIT = -2


@dataclass
class TreeParams:
    """yabt/tree.py:22-36 (axis-split fields; kernel splits are not supported
    by the level-wise path, yabt/tree.py:396-397)."""
    max_leaves: int = 31
    max_depth: int = 64
    reg_lambda: float = 1.0
    gamma: float = 0.0
    min_child_weight: float = 1e-3
    min_samples_leaf: int = 20
    learning_rate: float = 0.1
    kernel_splits: bool = False
    kernel_candidates: int = 8
    kernel_gamma: float = 0.0
    kernel_min_samples: int = 64
    kernel_importance_weighting: bool = False


@dataclass
class Tree:
    """Flat tensor tree, yabt/tree.py:39-76. Internal nodes split as
    ``x[f] <= threshold`` (left). ``feature`` is -1 at leaves."""

    feature: torch.Tensor
    threshold: torch.Tensor
    left: torch.Tensor
    right: torch.Tensor
    value: torch.Tensor
    depth: int
    kernel_id: torch.Tensor | None = None
    kernel_centers: torch.Tensor | None = None
    kernel_prec: torch.Tensor | None = None
    leaf_net_feats: torch.Tensor | None = None
    leaf_net_linear: torch.Tensor | None = None
    leaf_net_W1: torch.Tensor | None = None
    leaf_net_b1: torch.Tensor | None = None
    leaf_net_W2: torch.Tensor | None = None
    leaf_net_lo: torch.Tensor | None = None
    leaf_net_hi: torch.Tensor | None = None
    gate_scale: torch.Tensor | None = None

    @property
    def is_leaf(self) -> torch.Tensor:
        return self.feature == LEAF

    def num_leaves(self) -> int:
        return int((self.feature == LEAF).sum())

    def apply(self, X: torch.Tensor) -> torch.Tensor:
        """Leaf (node) index per row of raw X (n, F), yabt/tree.py:82-116."""
        from .predict import apply_tree
        return apply_tree(self, X)

    def net_contribution(self, X: torch.Tensor, node: torch.Tensor) -> torch.Tensor:
        """yabt/tree.py:118-128 (linear leaves)."""
        from .predict import net_contribution
        return net_contribution(self, X, node)

    def predict(self, X: torch.Tensor) -> torch.Tensor:
        """yabt/tree.py:130-135."""
        from .predict import predict_forest
        return predict_forest([self], X, base=0.0)

    def path_feature_pairs(self) -> list[tuple[int, int]]:
        """(ancestor feature, descendant feature) pairs along root-to-leaf
        paths, yabt/tree.py:186-203 (same DFS order)."""
        feature = self.feature.tolist()
        left, right = self.left.tolist(), self.right.tolist()
        pairs: list[tuple[int, int]] = []
        stack: list[tuple[int, tuple[int, ...]]] = [(0, ())]
        while stack:
            nid, anc = stack.pop()
            f = feature[nid]
            if f == LEAF:
                continue
            if f >= 0:
                pairs.extend((a, f) for a in anc)
                anc = anc + (f,)
            stack.append((left[nid], anc))
            stack.append((right[nid], anc))
        return pairs
