"""CUDA level-wise grower vs the CPU oracle (GPU tests)."""
import numpy as np
import pytest
import torch

from oracle.binning import Binner as OBinner
from oracle.grow import TreeParams as OTP, grow_levelwise

pytestmark = pytest.mark.gpu


def _run(X, g, h, leaves, depth, msl, imat=None, fmask=None, dyadic=False):
    from yabt_b200.grower import grow_tree_levelwise
    from yabt_b200.tree import TreeParams
    b = OBinner().fit(X)
    binned = b.transform(X)
    ot, oleaf, _ = grow_levelwise(binned, g, h, b.edges_, b.scales_,
                                  OTP(max_leaves=leaves, max_depth=depth, min_samples_leaf=msl),
                                  fmask, imat, 0.5)
    dev = "cuda"
    tb = torch.from_numpy(binned).to(dev)
    gt, ht = torch.from_numpy(g).to(dev), torch.from_numpy(h).to(dev)
    im = torch.from_numpy(imat).to(dev) if imat is not None else None
    fm = torch.from_numpy(fmask).to(dev) if fmask is not None else None
    gtree, gleaf = grow_tree_levelwise(tb, gt, ht, b, TreeParams(max_leaves=leaves, max_depth=depth,
                                                                 min_samples_leaf=msl),
                                       fm, im, 0.5, return_leaf=True)
    return ot, oleaf, gtree, gleaf.cpu().numpy()


def _check(ot, oleaf, gtree, gleaf, exact_values=False):
    np.testing.assert_array_equal(gtree.feature.cpu().numpy(), ot.feature)
    np.testing.assert_array_equal(gtree.left.cpu().numpy(), ot.left)
    np.testing.assert_array_equal(gtree.right.cpu().numpy(), ot.right)
    np.testing.assert_array_equal(gtree.threshold.cpu().numpy(), ot.threshold)
    np.testing.assert_array_equal(gtree.gate_scale.cpu().numpy(), ot.gate_scale)
    assert gtree.depth == ot.depth
    v = gtree.value.cpu().numpy()
    if exact_values:
        np.testing.assert_array_equal(v, ot.value)
    else:
        np.testing.assert_allclose(v, ot.value, rtol=1e-5, atol=1e-7)
    np.testing.assert_array_equal(gleaf, oleaf)


@pytest.mark.parametrize("seed,n,F,leaves,depth", [(0, 3000, 8, 31, 64), (1, 20000, 20, 31, 64),
                                                   (2, 5000, 70, 63, 6), (3, 1500, 10, 255, 10),
                                                   (4, 257, 3, 15, 64), (5, 31, 1, 7, 64)])
def test_grow_dyadic_exact(seed, n, F, leaves, depth):
    """Gradients/hessians on a dyadic grid: every sum is exact in float32, so the
    GPU tree must equal the oracle tree bit for bit (structure and values)."""
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, F)).astype(np.float32)
    g = (rng.integers(-512, 512, size=n) / 256.0).astype(np.float32)
    h = (rng.integers(1, 64, size=n) / 256.0).astype(np.float32)
    ot, oleaf, gt, gl = _run(X, g, h, leaves, depth, 5 if n < 2000 else 20)
    _check(ot, oleaf, gt, gl)


def test_grow_unit_hessian_path():
    rng = np.random.default_rng(7)
    n, F = 40000, 33
    X = rng.normal(size=(n, F)).astype(np.float32)
    g = (rng.integers(-1000, 1000, size=n) / 128.0).astype(np.float32)
    h = np.ones(n, np.float32)
    ot, oleaf, gt, gl = _run(X, g, h, 63, 64, 20)
    _check(ot, oleaf, gt, gl)


@pytest.mark.parametrize("case", range(4))
def test_grow_matches_golden_inputs(golden, case):
    """Reference golden inputs (continuous gradients): structure must match."""
    z = golden("grow")
    leaves, depth, msl = (int(v) for v in z[f"g{case}_params"])
    imat = z[f"g{case}_imat"]
    fm = z[f"g{case}_fmask"]
    ot, oleaf, gt, gl = _run(z[f"g{case}_X"], z[f"g{case}_g"], z[f"g{case}_h"], leaves, depth, msl,
                             imat if imat.size else None, fm if fm.size else None)
    _check(ot, oleaf, gt, gl)
    np.testing.assert_array_equal(gt.feature.cpu().numpy(), z[f"g{case}_feature"])


@pytest.mark.parametrize("general", [False, True])
def test_root_count_cache_reproduces_uncached_trees(general):
    """yabt_grower_set_root_count_cache: after the first tree records the root's
    per-bin row counts, later root histograms skip the count channel and copy
    them in; the trees must equal those of a grower without the cache."""
    from yabt_b200 import _lib
    from yabt_b200.grower import EdgePack, Grower, pack_bins
    from yabt_b200.tree import TreeParams
    rng = np.random.default_rng(21)
    n, F = 30000, 70
    X = rng.normal(size=(n, F)).astype(np.float32)
    b = OBinner().fit(X)
    bins = pack_bins(torch.from_numpy(b.transform(X)).cuda())
    ep = EdgePack(list(b.edges_), b.scales_, "cuda")
    tp = TreeParams(max_leaves=63, max_depth=8, min_samples_leaf=20)
    outs = []
    for cached in (True, False):
        gr = Grower(n, F, 63, 8, general, "cuda")
        _lib.check(gr.lib.yabt_grower_set_root_count_cache(gr.h, 1 if cached else 0), "cache")
        trees = []
        for t in range(3):
            r = np.random.default_rng(100 + t)
            g = torch.from_numpy((r.integers(-512, 512, size=n) / 256.0).astype(np.float32)).cuda()
            h = (torch.from_numpy((r.integers(1, 64, size=n) / 256.0).astype(np.float32)).cuda() if general
                 else torch.ones(n, device="cuda"))
            out = gr.new_outputs()
            gr.grow(gr.args(bins, g, h, ep, tp, out))
            torch.cuda.synchronize()
            k = int(out["meta"][0].item())
            trees.append({key: out[key][:k].cpu().numpy() for key in ("feature", "threshold", "left", "value")}
                         | {"leaf": out["leaf_of_row"].cpu().numpy()})
        outs.append(trees)
    for t in range(3):
        for key in ("feature", "threshold", "left", "value", "leaf"):
            np.testing.assert_array_equal(outs[0][t][key], outs[1][t][key], err_msg=f"tree {t} {key}")


@pytest.mark.parametrize("case", ["constant_columns", "fewer_rows_than_two_leaves", "max_leaves_2",
                                  "max_depth_1", "one_constant_column"])
def test_grow_degenerate_trees(case):
    """Trees that stop early: a root-only tree (constant columns, or fewer rows
    than two leaves of min_samples_leaf), a single split (max_leaves = 2,
    max_depth = 1) and a constant column among others (never chosen). Dyadic
    gradients: the structure and leaf of every row equal the oracle's; values
    within 1e-5."""
    rng = np.random.default_rng(7)
    n, F, leaves, depth, msl = 500, 5, 31, 64, 20
    X = rng.normal(size=(n, F)).astype(np.float32)
    g = (rng.integers(-512, 512, size=n) / 256.0).astype(np.float32)
    h = (rng.integers(1, 64, size=n) / 256.0).astype(np.float32)
    if case == "constant_columns":
        X = np.full((n, 4), 3.0, np.float32)
    elif case == "fewer_rows_than_two_leaves":
        X, g, h = X[:30], g[:30], h[:30]
    elif case == "max_leaves_2":
        leaves = 2
    elif case == "max_depth_1":
        leaves, depth = 255, 1
    else:
        X[:, 2] = 1.0
        msl = 5
    ot, oleaf, gt, gl = _run(X, g, h, leaves, depth, msl)
    _check(ot, oleaf, gt, gl)
    if case in ("constant_columns", "fewer_rows_than_two_leaves"):
        assert gt.feature.numel() == 1 and int(gt.feature[0]) == -1
    if case == "one_constant_column":
        assert not bool((gt.feature == 2).any())
