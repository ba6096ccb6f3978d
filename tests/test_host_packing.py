"""Forest packing for batched prediction on the CPU (yabt_b200.predict.Packed):
node arrays concatenated per tree with tree offsets, child indices kept local
to each tree, leaf-model tables zero-filled for trees without leaf models, and
mixed leaf-model widths rejected. Pure host logic: no GPU is used."""

import pytest
import torch

from yabt_b200.predict import Packed
from yabt_b200.tree import Tree


def _tree(nodes, K=None, seed=0):
    g = torch.Generator().manual_seed(seed)
    feature = torch.full((nodes,), -1, dtype=torch.int64)
    left = torch.full((nodes,), -1, dtype=torch.int64)
    right = torch.full((nodes,), -1, dtype=torch.int64)
    if nodes >= 3:
        feature[0], left[0], right[0] = 2, 1, 2
    t = Tree(feature=feature, threshold=torch.rand(nodes, generator=g), left=left, right=right,
             value=torch.rand(nodes, generator=g), depth=1 if nodes >= 3 else 0)
    if K:
        t.leaf_net_feats = torch.arange(K, dtype=torch.int64)
        t.leaf_net_linear = torch.rand(nodes, K, generator=g)
        t.leaf_net_lo = -torch.rand(nodes, K, generator=g)
        t.leaf_net_hi = torch.rand(nodes, K, generator=g)
    return t


def test_layout_and_zero_filled_tables():
    trees = [_tree(3, K=4, seed=1), _tree(1, seed=2), _tree(3, K=4, seed=3)]
    pk = Packed(trees, torch.device("cpu"))
    assert pk.ntrees == 3 and pk.K == 4
    assert pk.tree_off.tolist() == [0, 3, 4]
    assert pk.feature.dtype == torch.int32 and pk.left.dtype == torch.int32
    assert pk.feature.tolist() == [2, -1, -1, -1, 2, -1, -1]
    assert pk.left.tolist() == [1, -1, -1, -1, 1, -1, -1]          # child ids stay local to each tree
    assert torch.equal(pk.value, torch.cat([t.value for t in trees]))
    assert pk.has_nets.tolist() == [1, 0, 1]
    assert pk.linear.shape == (7, 4) and pk.lo.shape == (7, 4) and pk.hi.shape == (7, 4)
    assert torch.equal(pk.linear[3], torch.zeros(4))                 # the tree without leaf models
    assert torch.equal(pk.linear[4:], trees[2].leaf_net_linear)
    assert pk.feats.shape == (3, 4) and pk.feats[1].tolist() == [0, 0, 0, 0]


def test_constant_leaves_only_and_empty_forest():
    pk = Packed([_tree(3), _tree(1)], torch.device("cpu"))
    assert pk.K == 0 and not hasattr(pk, "linear")
    empty = Packed([], torch.device("cpu"))
    assert empty.ntrees == 0 and empty.K == 0


def test_mixed_leaf_model_widths_rejected():
    with pytest.raises(ValueError, match="widths"):
        Packed([_tree(3, K=4), _tree(3, K=8)], torch.device("cpu"))
