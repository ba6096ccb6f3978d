"""Newton boosting loop on the device (yabt/boosting.py:27-561).

Per tree the loop is a fixed sequence of CUDA launches with no host
synchronisation: interaction-matrix normalisation, level-wise growth,
ridge-linear leaves, interaction-score update and the fused margin update that
also produces the next tree's gradients. Trees are written straight into
device-resident forest arrays; ``Tree`` objects are views of those arrays,
materialised once at the end of ``fit``.

Supported ``BoostParams`` (the reference's defaults are the supported path):
level-wise growth, the best-first grower (the heap order of yabt/tree.py, or
the C / Numba grower's arithmetic with ``numba_grower=True``), interaction
steering, ridge-linear neural leaves, row subsampling (``subsample``), GOSS
(``goss_enabled``), feature subsampling (``colsample``),
``min_split_gain_rel``, eval-set early stopping. Options outside the GPU
tree-growth path (kernel splits, refinement / refit, adaptive features,
product features, auto-tune, MLP leaves, stochastic routing) raise
NotImplementedError.
"""

from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass, fields

import numpy as np
import torch

from . import _lib
from .binning import Binner, to_device_f32, to_feature_major
from .grower import Grower
from .tree import Tree, TreeParams

_INTERACTION_MIN_ROWS = 2000   # yabt/boosting.py:24


class LogLoss:
    """yabt/boosting.py:27-42 (loss id 1 on the device)."""
    is_classification = True
    kind = 1

    @staticmethod
    def base_score(y: torch.Tensor) -> float:
        p = float(y.mean().clamp(1e-6, 1 - 1e-6))
        return float(np.log(p / (1 - p)))

    @staticmethod
    def base_from_mean(m: float) -> float:
        p = float(np.clip(np.float32(m), np.float32(1e-6), np.float32(1 - 1e-6)))
        return float(np.log(p / (1 - p)))

    @staticmethod
    def grad_hess(margin: torch.Tensor, y: torch.Tensor):
        p = torch.sigmoid(margin)
        return p - y, (p * (1 - p)).clamp_min(1e-6)

    @staticmethod
    def loss(margin: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        return torch.nn.functional.binary_cross_entropy_with_logits(margin, y)


class MSELoss:
    """yabt/boosting.py:45-58 (loss id 0; unit hessian)."""
    is_classification = False
    kind = 0

    @staticmethod
    def base_score(y: torch.Tensor) -> float:
        return float(y.mean())

    @staticmethod
    def base_from_mean(m: float) -> float:
        return float(np.float32(m))

    @staticmethod
    def grad_hess(margin: torch.Tensor, y: torch.Tensor):
        return margin - y, torch.ones_like(y)

    @staticmethod
    def loss(margin: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        return 0.5 * (margin - y).square().mean()


@dataclass
class BoostParams:
    """Same fields and defaults as yabt/boosting.py:61-198."""
    n_estimators: int = 500
    learning_rate: float = 0.1
    max_leaves: int = 31
    max_depth: int = 64
    reg_lambda: float = 1.0
    gamma: float = 0.0
    min_split_gain_rel: float = 0.0
    min_child_weight: float = 1e-3
    min_samples_leaf: int = 20
    subsample: float = 1.0
    colsample: float = 1.0
    max_bins: int = 256
    refine_steps: int = 0
    refine_lr: float = 0.02
    refine_min_gain: float = 1e-4
    refit_every: int = 0
    refit_steps: int = 30
    refit_lr: float = 0.05
    adaptive_features: bool = False
    feature_importance_alpha: float = 0.1
    goss_enabled: bool = False
    goss_ratio: float = 0.9
    detect_interactions: bool = False
    interaction_aware: bool = True
    interaction_boost: float = 0.5
    product_features: bool = False
    product_max_features: int = 5
    product_max_order: int = 3
    product_min_corr: float = 0.03
    product_corr_gain: float = 1.3
    kernel_splits: bool = False
    kernel_candidates: int = 8
    kernel_gamma: float = 0.0
    kernel_min_samples: int = 64
    kernel_importance_weighting: bool | str = False
    neural_leaves: bool = True
    leaf_net_hidden: int = 0
    leaf_net_features: int = 8
    leaf_net_l2: float = 1.0
    leaf_net_steps: int = 40
    leaf_net_lr: float = 0.05
    leaf_net_min_samples: int = 50
    auto_tune: bool = False
    stochastic_routing: bool = False
    routing_tau: float = 0.05
    levelwise: bool | str = "auto"
    numba_grower: bool | str = "auto"
    c_grower: bool | str = "auto"
    c_grower_threads: int = 0
    sparse_hist: bool | str = "auto"
    sparse_hist_max_density: float = 0.5
    early_stopping_rounds: int = 0
    seed: int = 0
    device: str = "auto"
    verbose: bool = False

    def resolve_device(self) -> str:
        if self.device == "auto":
            return "cuda"
        return self.device


def use_bestfirst(p: BoostParams) -> bool:
    """The grower the reference picks on a CUDA device, yabt/boosting.py:415-421:
    level-wise for ``levelwise=True``, or ``"auto"`` with max_leaves >= 16;
    otherwise the best-first heap grower (kernel splits, which also force the
    heap there, are not part of this path)."""
    return not (p.levelwise is True or (p.levelwise == "auto" and p.max_leaves >= 16))


def use_c_grower_math(p: BoostParams) -> bool:
    """Best-first trees in the C / Numba grower's arithmetic: the reference runs
    that grower on a CUDA device when ``numba_grower=True`` and the level-wise
    grower is off (yabt/boosting.py:424-426; ``c_grower`` only picks between
    the C and Numba builds, which grow identical trees)."""
    return use_bestfirst(p) and p.numba_grower is True


def _check_supported(p: BoostParams) -> None:
    bad = []
    for name, ok in (("kernel_splits", not p.kernel_splits), ("refine_steps", p.refine_steps == 0),
                     ("refit_every", p.refit_every == 0), ("adaptive_features", not p.adaptive_features),
                     ("product_features", not p.product_features),
                     ("auto_tune", not p.auto_tune), ("stochastic_routing", not p.stochastic_routing),
                     ("leaf_net_hidden", p.leaf_net_hidden == 0), ("subsample", 0.0 < p.subsample <= 1.0),
                     ("levelwise", p.levelwise in (True, False, "auto"))):
        if not ok:
            bad.append(name)
    if bad:
        raise NotImplementedError(f"yabt_b200 implements the GPU tree-growth path; unsupported "
                                  f"options: {', '.join(bad)}")
    dev = p.resolve_device()
    if not str(dev).startswith("cuda"):
        raise NotImplementedError("yabt_b200 runs on CUDA devices only (device=%r)" % (dev,))


class DeviceData:
    """Training matrix prepared once on the device: binner, tiled bin matrix,
    imputed feature-major features and their column moments. Shared by the
    one-vs-rest boosters of a multiclass fit."""

    def __init__(self, X, max_bins: int, device: torch.device, comm=None):
        """``comm`` (a ``distributed.ShardComm``): X holds this rank's rows of a
        row-sharded training set; binning and column moments cover every rank."""
        lib = _lib.load()
        # host wall time of each preparation stage (the stream is drained at
        # each boundary; these stages run once per fit)
        stamps = [time.perf_counter()]

        def stage_done():
            torch.cuda.synchronize(device)
            stamps.append(time.perf_counter())
        self.Xfm = to_feature_major(X, device)
        stage_done()
        self.F, self.n = int(self.Xfm.shape[0]), int(self.Xfm.shape[1])
        n, F = self.n, self.F
        self.comm = comm
        if comm is None:
            self.binner = Binner(max_bins).fit_device(self.Xfm, n)
        else:
            self.binner = Binner(max_bins).fit_device_sharded(self.Xfm, n, comm)
        stage_done()
        # imputes Xfm in place; the feature-major copy feeds the row partition
        self.bins, _, self.bins_fm = self.binner.transform_device(self.Xfm, n, feature_major=True)
        stage_done()
        if comm is None:
            self.col_mean = torch.empty(F, dtype=torch.float32, device=device)
            self.col_std = torch.empty(F, dtype=torch.float32, device=device)
            _lib.check(lib.yabt_column_stats(self.Xfm.data_ptr(), n, F, self.col_mean.data_ptr(),
                                             self.col_std.data_ptr(), _lib.stream_ptr()), "yabt_column_stats")
        else:
            from .distributed import column_stats
            self.col_mean, self.col_std = column_stats(self.Xfm, n, comm)
        stage_done()
        self.timings = {k: stamps[i + 1] - stamps[i] for i, k in
                        enumerate(("to_device_s", "bin_fit_s", "bin_transform_s", "column_stats_s"))}
        med, edges, ecnt, scales = self.binner._dev
        self.edges = edges                      # [F][255]
        self.edge_off = (torch.arange(F, dtype=torch.int32, device=device) * 255).contiguous()
        self.edge_cnt = ecnt
        self.scales = scales
        self.device = device


class Forest:
    """Device-resident arrays of up to T trees (one row per tree)."""

    def __init__(self, T: int, max_nodes: int, K: int, device):
        z = dict(device=device)
        self.T, self.max_nodes, self.K = T, max_nodes, K
        self.feature = torch.full((T, max_nodes), -1, dtype=torch.int64, **z)
        self.threshold = torch.zeros(T, max_nodes, dtype=torch.float32, **z)
        self.left = torch.full((T, max_nodes), -1, dtype=torch.int64, **z)
        self.right = torch.full((T, max_nodes), -1, dtype=torch.int64, **z)
        self.value = torch.zeros(T, max_nodes, dtype=torch.float32, **z)
        self.gate = torch.ones(T, max_nodes, dtype=torch.float32, **z)
        self.meta = torch.zeros(T, 4, dtype=torch.int32, **z)
        self.feats = torch.zeros(T, max(K, 1), dtype=torch.int64, **z)
        self.linear = torch.zeros(T, max_nodes, max(K, 1), dtype=torch.float32, **z)
        self.lo = torch.zeros(T, max_nodes, max(K, 1), dtype=torch.float32, **z)
        self.hi = torch.zeros(T, max_nodes, max(K, 1), dtype=torch.float32, **z)
        self.has_nets = torch.zeros(T, dtype=torch.int32, **z)


class Booster:
    """yabt/boosting.py:201-561 on the device."""

    def __init__(self, params: BoostParams, loss):
        self.p = params
        self.loss = loss
        self.trees: list[Tree] = []
        self.binner: Binner | None = None
        self.base_score: float = 0.0
        self.best_iter: int | None = None
        self.interaction_detector = None
        self.tuning_report_ = None
        self.product_spec_: list = []
        self._packed = None

    # ------------------------------------------------------------------ fit
    def fit(self, X, y, eval_set=None, data: DeviceData | None = None, tree_callback=None,
            comm=None) -> "Booster":
        """yabt/boosting.py:271-534. ``tree_callback(t, grower)``, if given, is
        called after the launches of tree t are queued (no synchronisation).

        ``comm`` (a ``distributed.ShardComm``): X and y hold this rank's rows of
        a row-sharded training set; every rank must call ``fit`` with the same
        parameters and ends with the same model."""
        for _ in self.fit_steps(X, y, eval_set, data, tree_callback, comm):
            pass
        return self

    def fit_steps(self, X, y, eval_set=None, data: DeviceData | None = None, tree_callback=None, comm=None):
        """``fit`` as a generator: yields the tree index after queuing each
        tree's launches on the current CUDA stream (callers can interleave
        several boosters on several streams); the model is complete when the
        generator is exhausted."""
        p = self.p
        _check_supported(p)
        if comm is not None and (eval_set is not None or p.min_split_gain_rel > 0.0 or p.goss_enabled):
            raise NotImplementedError("row-sharded fits support neither eval_set, min_split_gain_rel nor GOSS")
        dev = torch.device(p.resolve_device())
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device_ = str(dev)
        t_fit = time.perf_counter()
        own_data = data is None
        if data is None:
            data = DeviceData(X, p.max_bins, dev, comm=comm)
        elif comm is not None and data.comm is None:
            raise ValueError("a row-sharded fit needs DeviceData built with the same comm")
        self.binner = data.binner
        n, F = data.n, data.F
        n_total = n if comm is None else sum(comm.int_values(n))
        lib = _lib.load()
        s = _lib.stream_ptr()
        yt = torch.as_tensor(np.asarray(y, dtype=np.float32)).to(dev)
        general = self.loss.kind != 0
        gen = torch.Generator(device="cpu").manual_seed(p.seed)

        use_ia = p.interaction_aware and n_total >= _INTERACTION_MIN_ROWS
        scores = torch.zeros(F, F, dtype=torch.float32, device=dev) if (use_ia or p.detect_interactions) else None
        imat = torch.empty(F, F, dtype=torch.float32, device=dev) if use_ia else None

        if comm is None:
            self.base_score = self.loss.base_score(yt)
        else:
            self.base_score = self.loss.base_from_mean(comm.sum_float(float(yt.double().sum())) / n_total)
        margin = torch.full((n,), self.base_score, dtype=torch.float32, device=dev)
        grad = torch.empty(n, dtype=torch.float32, device=dev)
        hess = torch.empty(n, dtype=torch.float32, device=dev) if general else None
        _lib.check(lib.yabt_grad_init(margin.data_ptr(), yt.data_ptr(), n, self.loss.kind, grad.data_ptr(),
                                      hess.data_ptr() if hess is not None else None, s), "yabt_grad_init")

        bestfirst = use_bestfirst(p)
        tp = TreeParams(max_leaves=p.max_leaves, max_depth=p.max_depth, reg_lambda=p.reg_lambda,
                        gamma=p.gamma, min_child_weight=p.min_child_weight,
                        min_samples_leaf=p.min_samples_leaf, learning_rate=p.learning_rate)
        goss = p.goss_enabled
        # GOSS reweights the sampled rows' hessians, so the tree needs the hessian channel
        grower = Grower(n, F, p.max_leaves, p.max_depth, general or goss, dev)
        _lib.check(lib.yabt_grower_set_bestfirst_f64(grower.h, 1 if use_c_grower_math(p) else 0),
                   "yabt_grower_set_bestfirst_f64")
        # the bin matrix is fixed for the fit: root histograms over all rows reuse
        # the first tree's per-bin row counts (trees grown on a row sample do not)
        _lib.check(lib.yabt_grower_set_root_count_cache(grower.h, 1), "yabt_grower_set_root_count_cache")
        # level-wise trees queue their levels without host waits (a finished
        # tree's remaining levels are device-side no-ops, or are skipped by the
        # device-side level loop below, both cheaper than the host waiting to
        # stop and leaving the GPU idle while it queues the next tree); best-first
        # trees, with up to max_leaves - 1 steps, stop queuing once complete
        lw = getattr(self, "_level_wait", None)
        grower.set_level_wait(bestfirst if lw is None else lw)
        # levels past level_loop_start() run in the device-side level loop
        # (one CUDA graph per tree, repeated on the device while the tree grows)
        grower.set_level_loop(getattr(self, "_level_loop", True))
        self.grower_ = grower
        K = min(p.leaf_net_features, F) if p.neural_leaves else 0
        if p.neural_leaves and not 1 <= K <= 8:
            raise NotImplementedError("leaf_net_features must be in [1, 8]")
        T = p.n_estimators
        forest = Forest(T, grower.max_nodes, K, dev)
        leaf_of_row = torch.empty(n, dtype=torch.int32, device=dev)
        parent = torch.empty(grower.max_nodes, dtype=torch.int32, device=dev)
        ln_ws = None
        if p.neural_leaves:
            ln_ws = torch.empty(int(lib.yabt_leafnet_workspace_bytes(n, F, grower.max_nodes)),
                                dtype=torch.uint8, device=dev)
        rows = grower.leaf_rows()
        sub = p.subsample < 1.0 or goss
        if goss:
            # yabt/boosting.py:337-338: the sampler's device generator, seeded once per fit
            goss_gen = torch.Generator(device=dev).manual_seed(p.seed)
            g_goss = torch.zeros(n, dtype=torch.float32, device=dev)
            h_goss = torch.zeros(n, dtype=torch.float32, device=dev)
        if sub:
            # row subsampling: trees grow on a sample, leaf models and the margin
            # update route every row (ranges from a stable grouping by leaf)
            offset = 0
            if comm is not None:
                from .distributed import shard_layout
                offset, _ = shard_layout(comm, n)
            mn = grower.max_nodes
            grp_ws = torch.empty(int(lib.yabt_group_rows_workspace_bytes(n, mn)), dtype=torch.uint8, device=dev)
            grp_begin = torch.empty(mn, dtype=torch.int32, device=dev)
            grp_count = torch.empty(mn, dtype=torch.int32, device=dev)
            grp_rows = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
            grp_src = torch.zeros(mn, dtype=torch.int32, device=dev)     # every leaf range is in grp_rows

        margin_v = yv = Xv = None
        if eval_set is not None:
            Xv = to_device_f32(eval_set[0], dev).clone()
            self.binner.impute_device(Xv)
            yv = torch.as_tensor(np.asarray(eval_set[1], dtype=np.float32)).to(dev)
            margin_v = torch.full((Xv.shape[0],), self.base_score, dtype=torch.float32, device=dev)
            best_val, rounds_since_best = float("inf"), 0

        class _Edges:   # EdgePack-compatible view of the fitted device edges
            values, off, cnt, scales = data.edges, data.edge_off, data.edge_cnt, data.scales

        n_built = 0
        for t in range(T):
            root = None
            g_tree, h_tree = grad, hess
            if goss:
                # yabt/boosting.py:371-374,393-396 (GOSS takes precedence over subsample):
                # the tree grows on the sampled rows with grad, hess times the row weights
                from .sampling import goss_sample
                sel, w = goss_sample(grad, p.goss_ratio, goss_gen)
                g_goss.index_copy_(0, sel, grad[sel] * w if w is not None else grad[sel])
                hs = hess[sel] if hess is not None else torch.ones(sel.numel(), device=dev)
                h_goss.index_copy_(0, sel, hs * w if w is not None else hs)
                g_tree, h_tree = g_goss, h_goss
                root = torch.sort(sel).values.to(torch.int32)   # row order only affects locality
            elif sub:
                # yabt/boosting.py:374-376: rows[:m] of a permutation drawn from the
                # CPU generator before the feature mask (the same draw order)
                m = int(n_total * p.subsample)
                perm = torch.randperm(n_total, generator=gen)[:m]
                if comm is not None:
                    perm = perm[(perm >= offset) & (perm < offset + n)] - offset
                root = torch.sort(perm).values.to(torch.int32).to(dev)   # row order only affects locality
            if use_ia:
                _lib.check(lib.yabt_interaction_normalize(scores.data_ptr(), F, imat.data_ptr(), s),
                           "yabt_interaction_normalize")
            fmask = None
            if p.colsample < 1.0:
                k = max(1, int(F * p.colsample))
                fm = torch.zeros(F, dtype=torch.uint8)
                fm[torch.randperm(F, generator=gen)[:k]] = 1
                fmask = fm.to(dev)
            tp_t = tp
            if p.min_split_gain_rel > 0.0:
                g_var = float(grad.var())
                tp_t = TreeParams(**{f.name: getattr(tp, f.name) for f in fields(tp)})
                tp_t.gamma = p.gamma + p.min_split_gain_rel * g_var
            out = dict(feature=forest.feature[t], threshold=forest.threshold[t], left=forest.left[t],
                       right=forest.right[t], value=forest.value[t], gate_scale=forest.gate[t],
                       leaf_of_row=leaf_of_row, meta=forest.meta[t])
            a = grower.args(data.bins, g_tree, h_tree, _Edges, tp_t, out, fmask, imat, p.interaction_boost,
                            bins_fm=data.bins_fm, root_rows=root)
            if comm is None:
                grower.grow(a, bestfirst=bestfirst, f64=use_c_grower_math(p))
            elif bestfirst:
                from .distributed import grow_tree_bestfirst
                grow_tree_bestfirst(grower, a, comm)
            else:
                from .distributed import grow_tree
                grow_tree(grower, a, comm)
            if sub:
                # every row's leaf (the tree saw only the sample), grouped by leaf
                _lib.check(lib.yabt_grow_apply_all(grower.h, ctypes.byref(a), s), "yabt_grow_apply_all")
                _lib.check(lib.yabt_group_rows(leaf_of_row.data_ptr(), n, grower.max_nodes, grp_ws.data_ptr(),
                                               grp_ws.numel(), grp_begin.data_ptr(), grp_count.data_ptr(),
                                               grp_rows.data_ptr(), s), "yabt_group_rows")
            if p.neural_leaves:
                la = _lib.LeafNetArgs()
                la.feature = forest.feature[t].data_ptr(); la.value = forest.value[t].data_ptr()
                la.max_nodes = grower.max_nodes; la.meta = forest.meta[t].data_ptr()
                la.leaf_src, la.leaf_begin, la.leaf_count = rows["src"], rows["begin"], rows["count"]
                la.fin, la.list0, la.list1 = rows["fin"], rows["list0"], rows["list1"]
                if sub:
                    la.leaf_src, la.leaf_begin, la.leaf_count = (grp_src.data_ptr(), grp_begin.data_ptr(),
                                                                 grp_count.data_ptr())
                    la.fin = grp_rows.data_ptr()
                la.leaf_of_row = leaf_of_row.data_ptr(); la.Xfm = data.Xfm.data_ptr()
                la.col_mean = data.col_mean.data_ptr(); la.col_std = data.col_std.data_ptr()
                la.margin = margin.data_ptr(); la.y = yt.data_ptr(); la.n = n; la.F = F; la.K = K
                la.loss = self.loss.kind; la.min_samples = p.leaf_net_min_samples; la.l2 = p.leaf_net_l2
                la.learning_rate = p.learning_rate
                la.feats = forest.feats[t].data_ptr(); la.linear = forest.linear[t].data_ptr()
                la.lo = forest.lo[t].data_ptr(); la.hi = forest.hi[t].data_ptr()
                la.has_nets = forest.has_nets[t:t + 1].data_ptr()
                if comm is None:
                    _lib.check(lib.yabt_leafnet_fit(ctypes.byref(la), ln_ws.data_ptr(), ln_ws.numel(), s),
                               "yabt_leafnet_fit")
                else:
                    from .distributed import fit_leaf_models
                    fit_leaf_models(la, ln_ws, comm, grower)
            if scores is not None:
                _lib.check(lib.yabt_interaction_update(forest.feature[t].data_ptr(), forest.left[t].data_ptr(),
                                                       forest.right[t].data_ptr(), forest.meta[t].data_ptr(),
                                                       F, grower.max_nodes, scores.data_ptr(), parent.data_ptr(),
                                                       s), "yabt_interaction_update")
            u = _lib.UpdateArgs()
            u.leaf_of_row = leaf_of_row.data_ptr(); u.value = forest.value[t].data_ptr()
            u.max_nodes = grower.max_nodes
            if p.neural_leaves:
                u.linear = forest.linear[t].data_ptr(); u.lo = forest.lo[t].data_ptr()
                u.hi = forest.hi[t].data_ptr(); u.feats = forest.feats[t].data_ptr()
                u.has_nets = forest.has_nets[t:t + 1].data_ptr()
            u.K = K; u.Xfm = data.Xfm.data_ptr(); u.n = n; u.margin = margin.data_ptr(); u.y = yt.data_ptr()
            u.grad = grad.data_ptr(); u.hess = hess.data_ptr() if hess is not None else None
            u.loss = self.loss.kind
            _lib.check(lib.yabt_update_margin(ctypes.byref(u), s), "yabt_update_margin")
            n_built = t + 1
            if tree_callback is not None:
                tree_callback(t, grower)
            if eval_set is not None:
                margin_v = margin_v + self._predict_trees(forest, t, t + 1, Xv, base=0.0, n_nodes=None)
                vl = float(self.loss.loss(margin_v, yv))
                if vl < best_val - 1e-7:
                    best_val, self.best_iter, rounds_since_best = vl, t, 0
                else:
                    rounds_since_best += 1
                if p.verbose and t % 50 == 0:
                    print(f"[{t}] train={float(self.loss.loss(margin, yt)):.5f} val={vl:.5f}")
                if p.early_stopping_rounds and rounds_since_best >= p.early_stopping_rounds:
                    break
            yield t
        if comm is not None and getattr(grower, "_exchange", None) is not None:
            try:
                grower._exchange.check()
            finally:
                grower._exchange.close()
                grower._exchange = None
        self._forest = forest
        self._margin_train = margin
        self.interaction_scores_ = scores
        meta = forest.meta[:n_built].cpu()
        # host wall time of the fit's stages: preparing the matrix (when fit built
        # it) and everything after it (trees, leaf models, margins)
        t_end = time.perf_counter()
        prep = sum(data.timings.values()) if own_data else 0.0
        self.fit_timings_ = dict(data.timings if own_data else {}, trees_s=t_end - t_fit - prep,
                                 total_s=t_end - t_fit)
        err = int(meta[:, 2].abs().sum()) if n_built else 0
        if err:
            raise _lib.YabtError(f"device error bits set while growing trees (0x{err:x})")
        has = forest.has_nets[:n_built].cpu().tolist()
        self.trees = []
        for t in range(n_built):
            k = int(meta[t, 0])
            tr = Tree(feature=forest.feature[t, :k], threshold=forest.threshold[t, :k],
                      left=forest.left[t, :k], right=forest.right[t, :k], value=forest.value[t, :k],
                      depth=int(meta[t, 1]), gate_scale=forest.gate[t, :k])
            if p.neural_leaves and has[t]:
                tr.leaf_net_feats = forest.feats[t, :K]
                tr.leaf_net_linear = forest.linear[t, :k, :K]
                tr.leaf_net_lo = forest.lo[t, :k, :K]
                tr.leaf_net_hi = forest.hi[t, :k, :K]
            self.trees.append(tr)
        self._packed = None

    # ------------------------------------------------------------------ predict
    def _predict_trees(self, forest: Forest, t0: int, t1: int, X: torch.Tensor, base: float, n_nodes):
        """Contribution of trees [t0, t1) of a Forest (device, row-major X)."""
        from .predict import predict_forest_arrays
        return predict_forest_arrays(forest, t0, t1, X, base)

    def packed(self):
        if self._packed is None:
            from .predict import pack_trees
            self._packed = pack_trees(self.trees)
        return self._packed

    def top_interactions(self, k: int = 5):
        """Top-k (i, j, score) pairs by accumulated path-pair counts
        (yabt/adaptive_features.py:162-177)."""
        if getattr(self, "interaction_scores_", None) is None:
            return []
        sc = (self.interaction_scores_ / (len(self.trees) + 1e-8)).cpu()
        F = sc.shape[0]
        out = [(i, j, float(sc[i, j])) for i in range(F) for j in range(i + 1, F)]
        out.sort(key=lambda x: x[2], reverse=True)
        return out[:k]

    def _margin(self, Xt: torch.Tensor, n_trees: int | None = None, soft=None) -> torch.Tensor:
        from .predict import predict_packed
        trees = self.trees[:n_trees] if n_trees is not None else self.trees
        if n_trees is not None and n_trees != len(self.trees):
            from .predict import pack_trees
            pk = pack_trees(trees)
        else:
            pk = self.packed()
        return predict_packed(pk, Xt, self.base_score)

    def predict_margin(self, X, use_best_iter: bool = True) -> np.ndarray:
        """yabt/boosting.py:552-561."""
        dev = torch.device(getattr(self, "device_", None) or "cuda")
        Xt = to_device_f32(X, dev).clone()
        self.binner.impute_device(Xt)
        n_trees = None
        if use_best_iter and self.best_iter is not None and self.p.refit_every == 0:
            n_trees = self.best_iter + 1
        return self._margin(Xt, n_trees).cpu().numpy()
