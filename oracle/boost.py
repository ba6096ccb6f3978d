"""Oracle restatement of the boosting loop (test infrastructure only).

Restates the GPU-path pieces of ``Booster.fit`` (yabt/boosting.py:271-534)
that the CUDA build replaces: the losses (:27-58), the interaction detector
(yabt/adaptive_features.py:113-177), the level-wise grower call (:428-431),
neural leaves (:495-497) and the margin update (:511-514); plus
``predict_margin`` (:542-561) and the one-vs-rest multiclass wrapper
(yabt/multiclass.py:9-48).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .binning import Binner
from .grow import OTree, TreeParams, grow_bestfirst, grow_levelwise
from .leafnet import column_stats, fit_leaf_networks

f32 = np.float32
INTERACTION_MIN_ROWS = 2000  # yabt/boosting.py:24


class MSELoss:
    """yabt/boosting.py:45-58."""
    is_classification = False

    @staticmethod
    def base_score(y):
        return float(np.float32(y.astype(np.float64).mean()))

    @staticmethod
    def grad_hess(m, y):
        return (m - y).astype(np.float32), np.ones_like(y, dtype=np.float32)


class LogLoss:
    """yabt/boosting.py:27-42."""
    is_classification = True

    @staticmethod
    def base_score(y):
        p = float(np.clip(np.float32(y.astype(np.float64).mean()), f32(1e-6), f32(1 - 1e-6)))
        return float(np.log(p / (1 - p)))

    @staticmethod
    def grad_hess(m, y):
        p = (f32(1) / (f32(1) + np.exp(-m.astype(np.float32)))).astype(np.float32)
        return (p - y).astype(np.float32), np.maximum(p * (f32(1) - p), f32(1e-6)).astype(np.float32)


class InteractionDetector:
    """yabt/adaptive_features.py:113-160."""

    def __init__(self, F: int):
        self.scores = np.zeros((F, F), np.float32)

    def update(self, pairs):
        for a, b in pairs:
            if a != b:
                self.scores[a, b] += 1
                self.scores[b, a] += 1

    def normalized(self) -> np.ndarray:
        m = self.scores
        mx = m.max()
        if mx <= 0:
            return m.copy()
        nz = m[m > 0]
        bg = f32(nz.astype(np.float64).sum()) / f32(nz.size)
        return np.maximum((m - bg) / (mx - bg + f32(1e-8)), f32(0)).astype(np.float32)


@dataclass
class BoostParams:
    """Subset of yabt/boosting.py:61-198 used on the GPU tree-growth path."""
    n_estimators: int = 500
    learning_rate: float = 0.1
    max_leaves: int = 31
    max_depth: int = 64
    reg_lambda: float = 1.0
    gamma: float = 0.0
    min_child_weight: float = 1e-3
    min_samples_leaf: int = 20
    max_bins: int = 256
    interaction_aware: bool = True
    interaction_boost: float = 0.5
    neural_leaves: bool = True
    leaf_net_features: int = 8
    leaf_net_l2: float = 1.0
    leaf_net_min_samples: int = 50
    subsample: float = 1.0
    seed: int = 0
    levelwise: bool | str = "auto"
    goss_enabled: bool = False
    goss_ratio: float = 0.9
    goss_device: str = "cpu"      # the device of the sampler's generator (the reference's is the fit device)


def _goss_rows(g: np.ndarray, ratio: float, gen, device: str):
    """The GOSS draw, yabt/adaptive_features.py:75-110: the ceil-free budget
    keep = max(1, round(n ratio)), top = max(1, min(keep, round(n (1 - ratio)))),
    the top rows by |g| from a descending argsort, then randperm(rest)[:keep - top]
    from the sampler's own generator, weighted (n - top) / drawn. The sort and the
    generator are torch's on ``device`` (the reference draws on the fit device).
    Returns (rows, weights or None) as numpy arrays."""
    import torch
    n = g.shape[0]
    ratio = min(max(ratio, 0.0), 1.0)
    keep_n = max(1, round(n * ratio))
    top_n = max(1, min(keep_n, round(n * (1.0 - ratio))))
    order = torch.argsort(torch.from_numpy(g).to(device).abs(), descending=True)
    if keep_n - top_n <= 0 or order.numel() == top_n:
        return order[:top_n].cpu().numpy(), None
    rest = order[top_n:]
    drawn = rest[torch.randperm(rest.numel(), generator=gen, device=device)[:keep_n - top_n]]
    w = np.ones(top_n + drawn.numel(), np.float32)
    w[top_n:] = np.float32((n - top_n) / drawn.numel())
    return torch.cat([order[:top_n], drawn]).cpu().numpy(), w


class Booster:
    """Newton boosting on CPU (yabt/boosting.py:271-561) with the grower the
    reference picks on a CUDA device (yabt/boosting.py:415-421): level-wise
    for ``levelwise=True`` or ``"auto"`` with max_leaves >= 16, else the
    best-first heap grower."""

    def __init__(self, params: BoostParams, loss):
        self.p = params
        self.loss = loss
        self.trees: list[OTree] = []
        self.binner: Binner | None = None
        self.base_score = 0.0

    def fit(self, X, y, n_trees: int | None = None, record: bool = False):
        p = self.p
        self.binner = Binner(p.max_bins).fit(X)
        binned = self.binner.transform(X)
        Xraw = self.binner.impute(X)
        y = np.asarray(y, np.float32)
        n, F = Xraw.shape
        use_ia = p.interaction_aware and n >= INTERACTION_MIN_ROWS
        det = InteractionDetector(F) if use_ia else None
        self.base_score = self.loss.base_score(y)
        margin = np.full(n, self.base_score, np.float32)
        tp = TreeParams(p.max_leaves, p.max_depth, p.reg_lambda, p.gamma,
                        p.min_child_weight, p.min_samples_leaf, p.learning_rate)
        col_mean, col_std = column_stats(Xraw)
        # the reference's CPU generator (yabt/boosting.py:286) drives row subsampling
        import torch
        gen = torch.Generator(device="cpu").manual_seed(p.seed)
        goss_gen = torch.Generator(device=p.goss_device).manual_seed(p.seed) if p.goss_enabled else None
        self.records = []
        for t in range(p.n_estimators if n_trees is None else n_trees):
            g, h = self.loss.grad_hess(margin, y)
            imat = det.normalized() if det is not None else None
            lw = p.levelwise is True or (p.levelwise == "auto" and p.max_leaves >= 16)

            def grow(b_, g_, h_):
                if lw:
                    tree_, leaf_, _ = grow_levelwise(b_, g_, h_, self.binner.edges_, self.binner.scales_,
                                                     tp, None, imat, p.interaction_boost)
                else:
                    tree_, leaf_ = grow_bestfirst(b_, g_, h_, self.binner.edges_, self.binner.scales_,
                                                  tp, None, imat, p.interaction_boost)
                return tree_, leaf_
            if p.goss_enabled:
                # yabt/boosting.py:371-374,393-396; sampler yabt/adaptive_features.py:75-110
                rows, w = _goss_rows(g, p.goss_ratio, goss_gen, p.goss_device)
                gs, hs = g[rows], h[rows]
                if w is not None:
                    gs, hs = (gs * w).astype(np.float32), (hs * w).astype(np.float32)
                tree, _ = grow(binned[rows], gs, hs)
                leaf = tree.apply(Xraw)
            elif p.subsample < 1.0:
                # yabt/boosting.py:374-376, 392-393: grow on rows[:m] of a permutation,
                # then route every row through the tree (:486)
                m = int(n * p.subsample)
                rows = torch.randperm(n, generator=gen)[:m].numpy()
                tree, _ = grow(binned[rows], g[rows], h[rows])
                leaf = tree.apply(Xraw)
            else:
                tree, leaf = grow(binned, g, h)
            if p.neural_leaves:
                tree = fit_leaf_networks(tree, Xraw, y, margin, self.loss, p, leaf,
                                         col_mean, col_std)
            if det is not None:
                det.update(tree.path_feature_pairs())
            contrib = tree.value[leaf]
            if tree.leaf_net_feats is not None:
                contrib = contrib + tree.net_contribution(Xraw, leaf)
            if record:
                self.records.append(dict(margin=margin.copy(), g=g, h=h, imat=imat, leaf=leaf))
            margin = (margin + contrib).astype(np.float32)
            self.trees.append(tree)
        self.margin_ = margin
        return self

    def predict_margin(self, X) -> np.ndarray:
        Xt = self.binner.impute(X)
        out = np.full(Xt.shape[0], self.base_score, np.float32)
        for tree in self.trees:
            out = (out + tree.predict(Xt)).astype(np.float32)
        return out
