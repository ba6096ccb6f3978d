"""The reference's own CUDA histogram kernels against this library's, on the
same B200 (GPU tests).

``oracle/_ref/yabt_hist_cuda.so`` is the reference's ``yabt/_cuda/hist.cu``
compiled from its source by ``oracle/build_ref_hist.py`` (the build its loader,
yabt/cuda_hist.py:42-67, performs on first use). Both sides build the same
fused ``(3, K, F, 256)`` histogram from the same inputs: the reference with
``hist_priv_kernel`` (K = 1, shared-memory tiles of 8 features, float atomics)
or ``hist_kernel`` (K > 1, float atomics in global memory); this library with
``yabt_hist_build`` (the drop-in of ``build_hist``) and, at the root of a
tree, the grower's ``k_hist`` on the tiled bin matrix. The results agree
within the reference's own bound (1e-5 of the largest bin,
tests/test_cuda_hist.py of the reference); the times are CUDA-event medians
after warm-up, written as JSON lines to stdout and, if ``YABT_HIST_TIMING``
names a file, appended there.
"""

import importlib.machinery
import importlib.util
import json
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REF_SO = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                      "yabt_hist_cuda.so")


def _ref_module():
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref/yabt_hist_cuda.so not built (oracle/build_ref_hist.py)")
    loader = importlib.machinery.ExtensionFileLoader("yabt_hist_cuda", REF_SO)
    spec = importlib.util.spec_from_file_location("yabt_hist_cuda", REF_SO, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def _time(fn, reps=10, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return float(np.median(ts))


def _report(rec):
    line = json.dumps(rec)
    print(line)
    path = os.environ.get("YABT_HIST_TIMING")
    if path:
        with open(path, "a") as f:
            f.write(line + "\n")


def _inputs(n, F, K, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    binned = torch.randint(0, 256, (n, F), generator=g, device="cuda", dtype=torch.uint8)
    slot = (torch.zeros(n, dtype=torch.int64, device="cuda") if K == 1
            else torch.randint(0, K, (n,), generator=g, device="cuda"))
    gr = torch.randn(n, generator=g, device="cuda")
    hs = torch.rand(n, generator=g, device="cuda") + 0.1
    w = torch.ones(n, device="cuda")
    return binned, slot, gr, hs, w


@pytest.mark.parametrize("n,F,K", [(20000, 24, 1), (20000, 24, 4), (20000, 24, 31),
                                   (2_000_000, 200, 1), (2_000_000, 200, 64)])
def test_build_hist_vs_reference_kernel(n, F, K):
    from yabt_b200.cuda_hist import build_hist
    ref = _ref_module()
    binned, slot, gr, hs, w = _inputs(n, F, K)
    want = ref.hist_build(binned, slot, gr, hs, w, K, F, 256)
    got = build_hist(binned, slot, gr, hs, w, K, F, 256)
    torch.cuda.synchronize()
    scale = float(want.abs().max())
    err = float((got.double() - want.double()).abs().max()) / max(scale, 1e-9)
    assert err <= 1e-5, err
    t_ref = _time(lambda: ref.hist_build(binned, slot, gr, hs, w, K, F, 256))
    t_ours = _time(lambda: build_hist(binned, slot, gr, hs, w, K, F, 256))
    _report({"case": "build_hist", "n": n, "F": F, "K": K, "reference_ms": t_ref, "yabt_hist_build_ms": t_ours,
             "speedup": t_ref / t_ours, "max_rel_diff": err})


def test_tree_root_histogram_vs_reference_kernel():
    """The C4 root (2,000,000 x 200, one node) as the grower builds it: k_hist on
    the tiled bin matrix, exact sums, against the reference's hist_priv_kernel
    on the row-major matrix with the same gradients."""
    from yabt_b200.grower import EdgePack, Grower, pack_bins
    from yabt_b200.tree import TreeParams
    ref = _ref_module()
    n, F = 2_000_000, 200
    binned, slot, gr, hs, w = _inputs(n, F, 1, seed=3)
    ones = torch.ones(n, device="cuda")
    tiled = pack_bins(binned)
    edges = [torch.arange(1, 256, dtype=torch.float32) for _ in range(F)]
    ep = EdgePack(edges, torch.ones(F), "cuda")
    gw = Grower(n, F, 2, 1, False, "cuda")
    tp = TreeParams(max_leaves=2, max_depth=1, min_samples_leaf=20)

    def grow_root():
        out = gw.new_outputs()
        gw.grow(gw.args(tiled, gr, ones, ep, tp, out))
    for _ in range(3):
        grow_root()
    torch.cuda.synchronize()
    gw.set_timing(16)
    for _ in range(10):
        grow_root()
    torch.cuda.synchronize()
    times = gw.hist_times()
    assert times, "no k_hist launch recorded"
    t_khist = float(np.median(times))
    t_ref = _time(lambda: ref.hist_build(binned, slot, gr, ones, w, 1, F, 256))
    _report({"case": "tree_root", "n": n, "F": F, "K": 1, "reference_ms": t_ref, "k_hist_ms": t_khist,
             "speedup": t_ref / t_khist})
