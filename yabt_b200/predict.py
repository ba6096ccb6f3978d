"""Inference on the device: packed-forest prediction and single-tree routing
(yabt/tree.py:82-135, yabt/boosting.py:542-550) through the C ABI."""

from __future__ import annotations

import torch

from . import _lib


class Packed:
    """All trees' node arrays concatenated (child indices local to each tree)."""

    def __init__(self, trees, device):
        self.ntrees = len(trees)
        self.device = device
        if not trees:
            self.K = 0
            return
        sizes = [int(t.feature.numel()) for t in trees]
        off = [0]
        for s in sizes[:-1]:
            off.append(off[-1] + s)
        self.tree_off = torch.tensor(off, dtype=torch.int64, device=device)
        self.feature = torch.cat([t.feature for t in trees]).to(torch.int32)
        self.threshold = torch.cat([t.threshold for t in trees]).float().contiguous()
        self.left = torch.cat([t.left for t in trees]).to(torch.int32)
        self.right = torch.cat([t.right for t in trees]).to(torch.int32)
        self.value = torch.cat([t.value for t in trees]).float().contiguous()
        Ks = {int(t.leaf_net_feats.numel()) for t in trees if t.leaf_net_feats is not None}
        if len(Ks) > 1:
            raise ValueError("trees with different leaf-model widths")
        self.K = Ks.pop() if Ks else 0
        if self.K:
            K = self.K
            self.has_nets = torch.tensor([int(t.leaf_net_feats is not None) for t in trees],
                                         dtype=torch.int32, device=device)
            z = lambda s: torch.zeros(s, K, dtype=torch.float32, device=device)
            self.feats = torch.stack([t.leaf_net_feats if t.leaf_net_feats is not None
                                      else torch.zeros(K, dtype=torch.int64, device=device) for t in trees])
            self.linear = torch.cat([t.leaf_net_linear if t.leaf_net_linear is not None else z(s)
                                     for t, s in zip(trees, sizes)]).contiguous()
            self.lo = torch.cat([t.leaf_net_lo if t.leaf_net_lo is not None else z(s)
                                 for t, s in zip(trees, sizes)]).contiguous()
            self.hi = torch.cat([t.leaf_net_hi if t.leaf_net_hi is not None else z(s)
                                 for t, s in zip(trees, sizes)]).contiguous()


def pack_trees(trees) -> Packed:
    dev = trees[0].feature.device if trees else torch.device("cuda")
    return Packed(trees, dev)


def predict_packed(pk: Packed, X: torch.Tensor, base: float) -> torch.Tensor:
    """base + sum of all packed trees' contributions for imputed row-major X."""
    X = X.contiguous()
    n, F = X.shape
    out = torch.empty(n, dtype=torch.float32, device=X.device)
    if pk.ntrees == 0:
        out.fill_(base)
        return out
    nets = pk.K > 0
    _lib.check(_lib.load().yabt_predict_forest(
        X.data_ptr(), n, F, pk.ntrees, pk.tree_off.data_ptr(), pk.feature.data_ptr(),
        pk.threshold.data_ptr(), pk.left.data_ptr(), pk.right.data_ptr(), pk.value.data_ptr(),
        pk.has_nets.data_ptr() if nets else None, pk.feats.data_ptr() if nets else None, pk.K,
        pk.linear.data_ptr() if nets else None, pk.lo.data_ptr() if nets else None,
        pk.hi.data_ptr() if nets else None, float(base), out.data_ptr(), _lib.stream_ptr()),
        "yabt_predict_forest")
    return out


def predict_forest(trees, X: torch.Tensor, base: float = 0.0) -> torch.Tensor:
    return predict_packed(pack_trees(list(trees)), X, base)


def predict_forest_arrays(forest, t0: int, t1: int, X: torch.Tensor, base: float) -> torch.Tensor:
    """Contribution of trees [t0, t1) stored in a boosting Forest (sizes read
    from the device meta: one small synchronisation)."""
    from .tree import Tree
    meta = forest.meta[t0:t1].cpu()
    trees = []
    for t in range(t0, t1):
        k = int(meta[t - t0, 0])
        tr = Tree(feature=forest.feature[t, :k], threshold=forest.threshold[t, :k], left=forest.left[t, :k],
                  right=forest.right[t, :k], value=forest.value[t, :k], depth=int(meta[t - t0, 1]))
        if forest.K and bool(forest.has_nets[t]):
            K = forest.K
            tr.leaf_net_feats = forest.feats[t, :K]
            tr.leaf_net_linear = forest.linear[t, :k, :K]
            tr.leaf_net_lo = forest.lo[t, :k, :K]
            tr.leaf_net_hi = forest.hi[t, :k, :K]
        trees.append(tr)
    return predict_forest(trees, X, base)


def apply_tree(tree, X: torch.Tensor) -> torch.Tensor:
    """Leaf index per row (yabt/tree.py:82-116)."""
    if tree.kernel_id is not None:
        raise NotImplementedError("kernel splits are not supported")
    X = X.to(torch.float32).contiguous()
    n, F = X.shape
    out = torch.empty(n, dtype=torch.int64, device=X.device)
    _lib.check(_lib.load().yabt_apply_tree(X.data_ptr(), n, F, tree.feature.contiguous().data_ptr(),
                                           tree.threshold.contiguous().data_ptr(),
                                           tree.left.contiguous().data_ptr(),
                                           tree.right.contiguous().data_ptr(), out.data_ptr(),
                                           _lib.stream_ptr()), "yabt_apply_tree")
    return out


def net_contribution(tree, X: torch.Tensor, node: torch.Tensor) -> torch.Tensor:
    """Per-row leaf-model output (yabt/tree.py:118-128): the forest kernel with
    the leaf values zeroed."""
    if tree.leaf_net_feats is None:
        return torch.zeros(X.shape[0], device=X.device)
    from .tree import Tree
    t0 = Tree(feature=tree.feature, threshold=tree.threshold, left=tree.left, right=tree.right,
              value=torch.zeros_like(tree.value), depth=tree.depth, leaf_net_feats=tree.leaf_net_feats,
              leaf_net_linear=tree.leaf_net_linear, leaf_net_lo=tree.leaf_net_lo,
              leaf_net_hi=tree.leaf_net_hi)
    return predict_forest([t0], X, 0.0)
