"""Multi-task boosting on the device: one shared tree structure for T targets
with a leaf value per target (yabt/multitask.py:31-251).

Each tree is grown by ``yabt_grow_tree_multitask`` (best-first on the summed
per-task gain, yabt/multitask.py:60-150 with yabt/histogram.py:120-188) and the
margins and squared-loss gradients of all tasks are updated by
``yabt_mt_update``; the binning, the bin matrix and row subsampling / feature
masks are those of the single-task booster.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .binning import to_device_f32
from .boosting import BoostParams, DeviceData, MSELoss
from .grower import Grower
from .tree import TreeParams

MAX_TASKS = 8


@dataclass
class MultiTaskTree:
    """Shared split structure with vector leaf values (yabt/multitask.py:31-57)."""
    feature: torch.Tensor     # (nodes,) int64; -1 at leaves
    threshold: torch.Tensor   # (nodes,) float32
    left: torch.Tensor        # (nodes,) int64
    right: torch.Tensor       # (nodes,) int64
    value: torch.Tensor       # (nodes, T) float32
    depth: int

    def apply(self, X: torch.Tensor) -> torch.Tensor:
        """Leaf of every row of the imputed raw matrix X (n, F)."""
        X = X.to(torch.float32).contiguous()
        n, F = X.shape
        out = torch.empty(n, dtype=torch.int64, device=X.device)
        _lib.check(_lib.load().yabt_apply_tree(X.data_ptr(), n, F, self.feature.data_ptr(), self.threshold.data_ptr(),
                                               self.left.data_ptr(), self.right.data_ptr(), out.data_ptr(),
                                               _lib.stream_ptr()), "yabt_apply_tree")
        return out

    def predict(self, X: torch.Tensor) -> torch.Tensor:
        """(n, T) per-task contributions."""
        margin = torch.zeros(self.value.shape[1], X.shape[0], dtype=torch.float32, device=X.device)
        _add_tree(self, X, margin)
        return margin.t()


def _add_tree(tree: MultiTaskTree, X: torch.Tensor, margin_tm: torch.Tensor) -> None:
    leaf = tree.apply(X).to(torch.int32)
    T, n = margin_tm.shape
    _lib.check(_lib.load().yabt_mt_update(leaf.data_ptr(), tree.value.contiguous().data_ptr(), T, n,
                                          margin_tm.data_ptr(), None, None, _lib.stream_ptr()), "yabt_mt_update")


def grow_multitask_tree(binned: torch.Tensor, grad: torch.Tensor, hess: torch.Tensor, binner, params: BoostParams,
                        feature_mask: torch.Tensor | None = None, *, return_leaf: bool = False):
    """Drop-in for yabt/multitask.py:60-150 on a CUDA device: binned (n, F)
    uint8, grad and hess (n, T) with unit hessians (the squared loss the
    reference's multi-task estimator uses). Returns the MultiTaskTree (and the
    leaf of every row when ``return_leaf``)."""
    from .grower import EdgePack, pack_bins
    if binned.device.type != "cuda":
        raise ValueError("grow_multitask_tree (yabt_b200) needs CUDA tensors")
    if not bool(torch.all(hess == 1.0)):
        raise NotImplementedError("multi-task growth supports unit hessians (squared loss)")
    n, F = binned.shape
    T = grad.shape[1]
    if not 1 <= T <= MAX_TASKS:
        raise NotImplementedError(f"multi-task growth supports 1..{MAX_TASKS} targets, got {T}")
    dev = binned.device
    lib = _lib.load()
    grower = Grower(n, F, params.max_leaves, params.max_depth, True, dev)
    ws = torch.empty(int(lib.yabt_mt_workspace_bytes(grower.h, T)), dtype=torch.uint8, device=dev)
    out = grower.new_outputs()
    values = torch.empty(grower.max_nodes, T, dtype=torch.float32, device=dev)
    g_tm = grad.to(torch.float32).t().contiguous()
    tp = TreeParams(max_leaves=params.max_leaves, max_depth=params.max_depth, reg_lambda=params.reg_lambda,
                    gamma=params.gamma, min_child_weight=params.min_child_weight,
                    min_samples_leaf=params.min_samples_leaf, learning_rate=params.learning_rate)
    fm = feature_mask.to(device=dev, dtype=torch.uint8).contiguous() if feature_mask is not None else None
    a = grower.args(pack_bins(binned), g_tm[0], g_tm[0], EdgePack(list(binner.edges_), binner.scales_, dev), tp, out,
                    fm, None, 0.5)
    _lib.check(lib.yabt_grow_tree_multitask(grower.h, ctypes.byref(a), T, g_tm.data_ptr(), ws.data_ptr(), ws.numel(),
                                            values.data_ptr(), _lib.stream_ptr()), "yabt_grow_tree_multitask")
    meta = out["meta"].tolist()
    if meta[2] != 0:
        raise _lib.YabtError(f"device error bits 0x{meta[2]:x} while growing a tree")
    k = meta[0]
    tree = MultiTaskTree(feature=out["feature"][:k], threshold=out["threshold"][:k], left=out["left"][:k],
                         right=out["right"][:k], value=values[:k], depth=meta[1])
    if return_leaf:
        return tree, out["leaf_of_row"].to(torch.int64)
    return tree


class MultiTaskBooster:
    """Newton boosting with shared-structure trees over T targets at once
    (yabt/multitask.py:153-251), squared loss."""

    def __init__(self, params: BoostParams, loss=None):
        self.p = params
        self.loss = loss if loss is not None else MSELoss()
        self.trees: list[MultiTaskTree] = []
        self.binner = None
        self.base_score: torch.Tensor | None = None
        self.best_iter: int | None = None

    def fit(self, X, Y, eval_set=None) -> "MultiTaskBooster":
        p = self.p
        if getattr(self.loss, "kind", None) != 0:
            raise NotImplementedError("multi-task growth supports the squared loss (YABTMultiTaskRegressor)")
        dev = torch.device(p.resolve_device())
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device_ = str(dev)
        gen = torch.Generator(device="cpu").manual_seed(p.seed)
        data = DeviceData(X, p.max_bins, dev)
        self.binner = data.binner
        n, F = data.n, data.F
        Y = np.asarray(Y, dtype=np.float32)
        if Y.ndim == 1:
            Y = Y[:, None]
        T = Y.shape[1]
        if not 1 <= T <= MAX_TASKS:
            raise NotImplementedError(f"multi-task growth supports 1..{MAX_TASKS} targets, got {T}")
        self.n_tasks_ = T
        Yd = torch.as_tensor(Y).to(dev)
        # yabt/multitask.py:163-167,197-198: per-task base scores (the column means)
        self.base_score = torch.tensor([self.loss.base_score(Yd[:, t]) for t in range(T)], device=dev)
        y_tm = Yd.t().contiguous()
        margin = self.base_score[:, None].expand(T, n).contiguous()
        grad = torch.empty(T, n, dtype=torch.float32, device=dev)
        lib = _lib.load()
        s = _lib.stream_ptr()
        _lib.check(lib.yabt_mt_update(None, None, T, n, margin.data_ptr(), y_tm.data_ptr(), grad.data_ptr(), s),
                   "yabt_mt_update")
        tp = TreeParams(max_leaves=p.max_leaves, max_depth=p.max_depth, reg_lambda=p.reg_lambda,
                        gamma=p.gamma, min_child_weight=p.min_child_weight,
                        min_samples_leaf=p.min_samples_leaf, learning_rate=p.learning_rate)
        grower = Grower(n, F, p.max_leaves, p.max_depth, True, dev)
        mt_ws = torch.empty(int(lib.yabt_mt_workspace_bytes(grower.h, T)), dtype=torch.uint8, device=dev)
        out = grower.new_outputs()
        values = torch.empty(grower.max_nodes, T, dtype=torch.float32, device=dev)

        class _Edges:   # EdgePack-compatible view of the fitted device edges
            values, off, cnt, scales = data.edges, data.edge_off, data.edge_cnt, data.scales

        Xv = yv = margin_v = None
        if eval_set is not None:
            Xv = to_device_f32(eval_set[0], dev).clone()
            self.binner.impute_device(Xv)
            Yv = np.asarray(eval_set[1], dtype=np.float32)
            yv = torch.as_tensor(Yv[:, None] if Yv.ndim == 1 else Yv).to(dev)
            margin_v = self.base_score[:, None].expand(T, Xv.shape[0]).contiguous()
            best_val, rounds_since_best = float("inf"), 0

        self.trees = []
        for t in range(p.n_estimators):
            root = None
            if p.subsample < 1.0:
                m = int(n * p.subsample)
                root = torch.sort(torch.randperm(n, generator=gen)[:m]).values.to(torch.int32).to(dev)
            fmask = None
            if p.colsample < 1.0:
                k = max(1, int(F * p.colsample))
                fm = torch.zeros(F, dtype=torch.uint8)
                fm[torch.randperm(F, generator=gen)[:k]] = 1
                fmask = fm.to(dev)
            a = grower.args(data.bins, grad[0], grad[0], _Edges, tp, out, fmask, None, 0.5,
                            bins_fm=data.bins_fm, root_rows=root)
            _lib.check(lib.yabt_grow_tree_multitask(grower.h, ctypes.byref(a), T, grad.data_ptr(), mt_ws.data_ptr(),
                                                    mt_ws.numel(), values.data_ptr(), s), "yabt_grow_tree_multitask")
            if root is not None:
                # yabt/multitask.py:226: the margin update routes every row
                _lib.check(lib.yabt_grow_apply_all(grower.h, ctypes.byref(a), s), "yabt_grow_apply_all")
            _lib.check(lib.yabt_mt_update(out["leaf_of_row"].data_ptr(), values.data_ptr(), T, n, margin.data_ptr(),
                                          y_tm.data_ptr(), grad.data_ptr(), s), "yabt_mt_update")
            meta = out["meta"].tolist()
            if meta[2] != 0:
                raise _lib.YabtError(f"device error bits 0x{meta[2]:x} while growing a tree")
            k = meta[0]
            tree = MultiTaskTree(feature=out["feature"][:k].clone(), threshold=out["threshold"][:k].clone(),
                                 left=out["left"][:k].clone(), right=out["right"][:k].clone(),
                                 value=values[:k].clone(), depth=meta[1])
            self.trees.append(tree)
            if eval_set is not None:
                _add_tree(tree, Xv, margin_v)
                vl = float(self.loss.loss(margin_v.t(), yv))
                if vl < best_val - 1e-7:
                    best_val, self.best_iter, rounds_since_best = vl, t, 0
                else:
                    rounds_since_best += 1
                if p.early_stopping_rounds and rounds_since_best >= p.early_stopping_rounds:
                    break
        return self

    def _margin(self, Xt: torch.Tensor, n_trees: int | None = None) -> torch.Tensor:
        margin = self.base_score[:, None].expand(self.n_tasks_, Xt.shape[0]).contiguous()
        for tree in self.trees[:n_trees]:
            _add_tree(tree, Xt, margin)
        return margin.t()

    def predict_margin(self, X, use_best_iter: bool = True) -> np.ndarray:
        """(n, T) margins (yabt/multitask.py:236-251)."""
        dev = torch.device(getattr(self, "device_", None) or "cuda")
        Xt = to_device_f32(X, dev).clone()
        self.binner.impute_device(Xt)
        n_trees = self.best_iter + 1 if (use_best_iter and self.best_iter is not None) else None
        return self._margin(Xt, n_trees).cpu().numpy()

