"""Generate the golden parity fixtures by running the reference itself.

Run in a container where the reference source tree is importable:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/yabt-reference

It imports the reference's ``yabt`` package (CPU torch; no CUDA needed) and
records, for small seeded inputs, what the reference computes on the GPU
tree-growth path:

* ``binning.npz``  Binner.fit/transform (yabt/binning.py:29-129): edges,
                   medians, scales and the uint8 bin matrix;
* ``grow.npz``     grow_tree_levelwise (yabt/tree.py:362-625) on its torch
                   scatter branch, for several parameter sets, with feature
                   masks and interaction steering; the tree arrays plus the
                   leaf of every row (Tree.apply, yabt/tree.py:82-116);
* ``leafnet.npz``  fit_leaf_networks (yabt/neural_leaves.py:131-184);
* ``boost.npz``    Booster(levelwise=True, device="cpu") fits
                   (yabt/boosting.py:271-561) and their predict_margin, for
                   MSE and LogLoss, plus YABTClassifier multiclass
                   predict_proba (yabt/multiclass.py:40-44);
* ``bestfirst.npz`` the best-first (heap) grower grow_tree (yabt/tree.py:206-360,
                   axis splits), written by ``make_golden.py --bestfirst``;
* ``hist.npz``     the torch scatter histogram the reference CUDA kernel is
                   tested against (tests/test_cuda_hist.py:13-22 of the reference).

The inputs are stored next to the outputs so the fixtures are self-contained.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _data(seed: int, n: int, F: int, nan_frac: float = 0.0):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, F)).astype(np.float32)
    if F > 3:
        X[:, 1] = np.exp(X[:, 1])                         # heavy tail
        X[:, 2] = rng.integers(0, 8, size=n)              # low cardinality
        X[:, 3] = np.where(rng.random(n) < 0.3, 0.0, X[:, 3])  # exact zeros
    if nan_frac:
        X[rng.random(size=X.shape) < nan_frac] = np.nan
    Xc = np.nan_to_num(X)
    y = (np.sin(Xc[:, 0]) + Xc[:, 1 % F] * Xc[:, 2 % F] * 0.3 + 0.5 * Xc[:, 3 % F] ** 2
         + 0.1 * rng.normal(size=n)).astype(np.float32)
    return X, y


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import torch
    from yabt.binning import Binner
    from yabt.boosting import Booster, BoostParams, LogLoss, MSELoss
    from yabt.neural_leaves import fit_leaf_networks
    from yabt.sklearn_api import YABTClassifier
    from yabt.tree import TreeParams, grow_tree_levelwise
    from yabt.adaptive_features import FeatureInteractionDetector

    assert not torch.cuda.is_available(), "run on a CPU-only host (numpy binner path)"
    torch.manual_seed(0)

    # ---------------- binning ----------------
    out = {}
    cases = [(0, 3000, 7, 0.0), (1, 1001, 5, 0.05), (2, 210_000, 3, 0.02), (3, 599, 4, 0.0)]
    for i, (seed, n, F, nanf) in enumerate(cases):
        X, _ = _data(seed, n, F, nanf)
        if i == 0:
            X[:, 4] = 1.5          # constant column
            X[:, 5] = np.nan       # all-NaN column
        b = Binner(256).fit(X)
        if n <= 50_000:  # large inputs are regenerated from the seed by the tests
            out[f"c{i}_X"] = X
        out[f"c{i}_bins"] = b.transform(X).numpy()
        out[f"c{i}_medians"] = b.medians_.astype(np.float32)
        out[f"c{i}_scales"] = b.scales_.numpy()
        out[f"c{i}_nedges"] = np.array([len(e) for e in b.edges_], np.int64)
        out[f"c{i}_edges"] = np.concatenate([e.numpy() for e in b.edges_])
    out["ncases"] = np.array(len(cases))
    out["cases"] = np.array(cases, np.float64)
    np.savez_compressed(os.path.join(HERE, "binning.npz"), **out)

    # ---------------- grower ----------------
    out = {}
    gcases = [
        dict(seed=10, n=3000, F=8, leaves=31, depth=64, msl=20, imat=False, fmask=False),
        dict(seed=11, n=4000, F=12, leaves=63, depth=5, msl=5, imat=True, fmask=False),
        dict(seed=12, n=2500, F=6, leaves=15, depth=64, msl=20, imat=True, fmask=True),
        dict(seed=13, n=1500, F=10, leaves=255, depth=10, msl=1, imat=False, fmask=False),
    ]
    for i, c in enumerate(gcases):
        X, y = _data(c["seed"], c["n"], c["F"], 0.02)
        binner = Binner(256).fit(X)
        binned = binner.transform(X)
        Xraw = torch.from_numpy(binner.impute(X))
        rng = np.random.default_rng(c["seed"] + 100)
        g = torch.from_numpy(rng.normal(size=c["n"]).astype(np.float32))
        h = torch.from_numpy(rng.uniform(0.05, 0.25, size=c["n"]).astype(np.float32))
        imat = None
        if c["imat"]:
            det = FeatureInteractionDetector(c["F"], device="cpu")
            pairs = [(int(a), int(b)) for a, b in rng.integers(0, c["F"], size=(40, 2))]
            pairs += [(0, 1)] * 6
            det.update_from_path_pairs(pairs)
            imat = det.normalized_matrix()
        fm = None
        if c["fmask"]:
            fm = torch.from_numpy(rng.random(c["F"]) < 0.7)
        tp = TreeParams(max_leaves=c["leaves"], max_depth=c["depth"], min_samples_leaf=c["msl"],
                        learning_rate=0.1)
        tree = grow_tree_levelwise(binned, g, h, binner, tp, fm, interaction_matrix=imat,
                                   interaction_boost=0.5)
        out[f"g{i}_X"] = X
        out[f"g{i}_g"] = g.numpy(); out[f"g{i}_h"] = h.numpy()
        out[f"g{i}_params"] = np.array([c["leaves"], c["depth"], c["msl"]], np.int64)
        out[f"g{i}_imat"] = imat.numpy() if imat is not None else np.zeros((0, 0), np.float32)
        out[f"g{i}_fmask"] = fm.numpy() if fm is not None else np.zeros(0, bool)
        for k in ("feature", "threshold", "left", "right", "value", "gate_scale"):
            out[f"g{i}_{k}"] = getattr(tree, k).numpy()
        out[f"g{i}_depth"] = np.array(tree.depth)
        out[f"g{i}_leaf"] = tree.apply(Xraw).numpy()
    out["ncases"] = np.array(len(gcases))
    np.savez_compressed(os.path.join(HERE, "grow.npz"), **out)

    # ---------------- neural leaves ----------------
    out = {}
    for i, (seed, n, F, leaves) in enumerate([(20, 4000, 10, 31), (21, 3000, 5, 8)]):
        X, y = _data(seed, n, F, 0.0)
        binner = Binner(256).fit(X)
        binned = binner.transform(X)
        Xraw = torch.from_numpy(binner.impute(X))
        yt = torch.from_numpy(y)
        margin = torch.full((n,), float(yt.mean()))
        g, h = MSELoss.grad_hess(margin, yt)
        tree = grow_tree_levelwise(binned, g, h, binner, TreeParams(max_leaves=leaves), None)
        leaf = tree.apply(Xraw)
        p = BoostParams(learning_rate=0.1)
        gen = torch.Generator().manual_seed(0)
        t2 = fit_leaf_networks(tree, Xraw, yt, margin, MSELoss(), p, gen, leaf_idx=leaf)
        out[f"l{i}_X"] = X; out[f"l{i}_y"] = y
        for k in ("feature", "threshold", "left", "right", "value"):
            out[f"l{i}_tree_{k}"] = getattr(tree, k).numpy()
        out[f"l{i}_tree_depth"] = np.array(tree.depth)
        out[f"l{i}_leaf"] = leaf.numpy()
        out[f"l{i}_margin"] = margin.numpy()
        out[f"l{i}_feats"] = t2.leaf_net_feats.numpy()
        out[f"l{i}_linear"] = t2.leaf_net_linear.numpy()
        out[f"l{i}_lo"] = t2.leaf_net_lo.numpy(); out[f"l{i}_hi"] = t2.leaf_net_hi.numpy()
        out[f"l{i}_value"] = t2.value.numpy()
    np.savez_compressed(os.path.join(HERE, "leafnet.npz"), **out)

    # ---------------- boosting ----------------
    out = {}
    X, y = _data(30, 2500, 6, 0.01)
    p = BoostParams(n_estimators=12, max_leaves=15, learning_rate=0.1, levelwise=True,
                    device="cpu", seed=0)
    bm = Booster(p, MSELoss()).fit(X, y)
    out["mse_X"] = X; out["mse_y"] = y
    out["mse_pred"] = bm.predict_margin(X)
    out["mse_base"] = np.array(bm.base_score)
    for t_i, t in enumerate(bm.trees[:3]):
        out[f"mse_t{t_i}_feature"] = t.feature.numpy()
        out[f"mse_t{t_i}_value"] = t.value.numpy()
    Xc, yc = _data(31, 2200, 5, 0.0)
    ycls = (yc > np.median(yc)).astype(np.float32)
    bl = Booster(BoostParams(n_estimators=10, max_leaves=15, learning_rate=0.2, levelwise=True,
                             device="cpu", seed=0), LogLoss()).fit(Xc, ycls)
    out["log_X"] = Xc; out["log_y"] = ycls
    out["log_pred"] = bl.predict_margin(Xc)
    out["log_base"] = np.array(bl.base_score)
    Xm, ym = _data(32, 2100, 5, 0.0)
    ymc = np.digitize(ym, np.quantile(ym, [0.33, 0.66])).astype(np.float32)
    clf = YABTClassifier(n_estimators=6, max_leaves=15, levelwise=True, device="cpu",
                         seed=0).fit(Xm, ymc)
    out["mc_X"] = Xm; out["mc_y"] = ymc
    out["mc_proba"] = clf.predict_proba(Xm)
    np.savez_compressed(os.path.join(HERE, "boost.npz"), **out)

    # ---------------- scatter histogram (CUDA-kernel reference) ----------------
    out = {}
    torch.manual_seed(0)
    n, F, K = 3000, 9, 5
    binned = torch.randint(0, 256, (n, F), dtype=torch.uint8)
    g = torch.randn(n); h = torch.rand(n) + 0.1
    w = (torch.rand(n) > 0.5).float()
    slot = torch.randint(0, K, (n,))
    flat = (slot[:, None] * (F * 256) + torch.arange(F)[None, :] * 256 + binned.long()).reshape(-1)
    ref = torch.zeros(3, K * F * 256)
    ref[0].scatter_add_(0, flat, (g * w)[:, None].expand(n, F).reshape(-1))
    ref[1].scatter_add_(0, flat, (h * w)[:, None].expand(n, F).reshape(-1))
    ref[2].scatter_add_(0, flat, w[:, None].expand(n, F).reshape(-1))
    out.update(binned=binned.numpy(), g=g.numpy(), h=h.numpy(), w=w.numpy(),
               slot=slot.numpy(), hist=ref.view(3, K, F, 256).numpy())
    np.savez_compressed(os.path.join(HERE, "hist.npz"), **out)
    print("golden fixtures written to", HERE)


def bestfirst(ref_root: str) -> None:
    """``bestfirst.npz``: the reference's best-first (heap) grower
    (yabt/tree.py:206-360, axis splits) on seeded cases, run on a CPU-only host."""
    sys.path.insert(0, ref_root)
    import torch
    from yabt.adaptive_features import FeatureInteractionDetector
    from yabt.binning import Binner
    from yabt.tree import TreeParams, grow_tree

    assert not torch.cuda.is_available(), "run on a CPU-only host (numpy binner path)"
    out = {}
    bcases = [
        dict(seed=30, n=3000, F=8, leaves=15, depth=64, msl=20, imat=False, fmask=False),
        dict(seed=31, n=4000, F=12, leaves=31, depth=4, msl=5, imat=True, fmask=False),
        dict(seed=32, n=2500, F=6, leaves=7, depth=64, msl=20, imat=True, fmask=True),
        dict(seed=33, n=1500, F=10, leaves=63, depth=10, msl=1, imat=False, fmask=False),
    ]
    for i, c in enumerate(bcases):
        X, _ = _data(c["seed"], c["n"], c["F"], 0.02)
        binner = Binner(256).fit(X)
        binned = binner.transform(X)
        Xraw = torch.from_numpy(binner.impute(X))
        rng = np.random.default_rng(c["seed"] + 100)
        g = torch.from_numpy(rng.normal(size=c["n"]).astype(np.float32))
        h = torch.from_numpy(rng.uniform(0.05, 0.25, size=c["n"]).astype(np.float32))
        imat = None
        if c["imat"]:
            det = FeatureInteractionDetector(c["F"], device="cpu")
            pairs = [(int(a), int(b)) for a, b in rng.integers(0, c["F"], size=(40, 2))]
            pairs += [(0, 1)] * 6
            det.update_from_path_pairs(pairs)
            imat = det.normalized_matrix()
        fm = None
        if c["fmask"]:
            fm = torch.from_numpy(rng.random(c["F"]) < 0.7)
        tp = TreeParams(max_leaves=c["leaves"], max_depth=c["depth"], min_samples_leaf=c["msl"],
                        learning_rate=0.1)
        tree = grow_tree(binned, g, h, binner, tp, fm, interaction_matrix=imat, interaction_boost=0.5)
        out[f"b{i}_X"] = X
        out[f"b{i}_g"] = g.numpy(); out[f"b{i}_h"] = h.numpy()
        out[f"b{i}_params"] = np.array([c["leaves"], c["depth"], c["msl"]], np.int64)
        out[f"b{i}_imat"] = imat.numpy() if imat is not None else np.zeros((0, 0), np.float32)
        out[f"b{i}_fmask"] = fm.numpy() if fm is not None else np.zeros(0, bool)
        for k in ("feature", "threshold", "left", "right", "value", "gate_scale"):
            out[f"b{i}_{k}"] = getattr(tree, k).numpy()
        out[f"b{i}_leaf"] = tree.apply(Xraw).numpy()
    out["ncases"] = np.array(len(bcases))
    np.savez_compressed(os.path.join(HERE, "bestfirst.npz"), **out)
    print("bestfirst fixtures written to", HERE)


def multitask(ref_root: str) -> None:
    """``multitask.npz``: the reference's multi-task grower
    (yabt/multitask.py:60-150) on seeded cases with squared-loss gradients, and
    a YABTMultiTaskRegressor fit (yabt/sklearn_api.py:366-402), on a CPU-only
    host."""
    sys.path.insert(0, ref_root)
    import torch
    from yabt.binning import Binner
    from yabt.boosting import BoostParams
    from yabt.multitask import grow_multitask_tree
    from yabt.sklearn_api import YABTMultiTaskRegressor

    assert not torch.cuda.is_available(), "run on a CPU-only host (numpy binner path)"
    out = {}
    mcases = [
        dict(seed=40, n=3000, F=8, T=2, leaves=15, depth=64, msl=20, fmask=False),
        dict(seed=41, n=4000, F=12, T=3, leaves=31, depth=5, msl=5, fmask=False),
        dict(seed=42, n=2500, F=6, T=1, leaves=9, depth=64, msl=20, fmask=True),
        dict(seed=43, n=2000, F=10, T=5, leaves=24, depth=8, msl=10, fmask=False),
    ]
    for i, c in enumerate(mcases):
        X, _ = _data(c["seed"], c["n"], c["F"], 0.02)
        binner = Binner(256).fit(X)
        binned = binner.transform(X)
        Xraw = torch.from_numpy(binner.impute(X))
        rng = np.random.default_rng(c["seed"] + 100)
        g = torch.from_numpy(rng.normal(size=(c["n"], c["T"])).astype(np.float32))
        h = torch.ones_like(g)
        fm = torch.from_numpy(rng.random(c["F"]) < 0.7) if c["fmask"] else None
        p = BoostParams(max_leaves=c["leaves"], max_depth=c["depth"], min_samples_leaf=c["msl"],
                        learning_rate=0.1, device="cpu")
        tree = grow_multitask_tree(binned, g, h, binner, p, fm)
        out[f"m{i}_X"] = X
        out[f"m{i}_g"] = g.numpy()
        out[f"m{i}_params"] = np.array([c["leaves"], c["depth"], c["msl"]], np.int64)
        out[f"m{i}_fmask"] = fm.numpy() if fm is not None else np.zeros(0, bool)
        for k in ("feature", "threshold", "left", "right", "value"):
            out[f"m{i}_{k}"] = getattr(tree, k).numpy()
        out[f"m{i}_leaf"] = tree.apply(Xraw).numpy()
    out["ncases"] = np.array(len(mcases))
    # an estimator fit: three correlated targets
    X, _ = _data(44, 3000, 8, 0.02)
    z = np.nan_to_num(X)
    rng = np.random.default_rng(45)
    Y = np.stack([np.sin(z[:, 0]) + z[:, 1], z[:, 1] * z[:, 2], 0.5 * z[:, 0] - z[:, 3]], axis=1)
    Y = (Y + 0.1 * rng.normal(size=Y.shape)).astype(np.float32)
    est = YABTMultiTaskRegressor(n_estimators=8, max_leaves=15, learning_rate=0.2, device="cpu").fit(X, Y)
    out["est_X"], out["est_Y"] = X, Y
    out["est_pred"] = est.predict(X).astype(np.float32)
    out["est_feature0"] = est.booster_.trees[0].feature.numpy()
    np.savez_compressed(os.path.join(HERE, "multitask.npz"), **out)
    print("multitask fixtures written to", HERE)


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 and not sys.argv[1].startswith("--") else "/root/reference"
    if "--bestfirst" in sys.argv:
        bestfirst(ref)
    elif "--multitask" in sys.argv:
        multitask(ref)
    else:
        main(ref)
