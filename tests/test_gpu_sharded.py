"""GPU parity of the row-sharded fit: ranks that each hold a block of the
rows (contiguous blocks in rank order) must end with the model a single-GPU
fit builds on the concatenated rows.

Two ranks run as two processes on GPU 0 over gloo (the collectives are staged
through host memory and no kernel waits on another process), so the test needs
one GPU; with two or more GPUs the same check also runs over NCCL, one rank
per GPU. Binning (medians, edges, scales) and, without leaf models, every tree
are bit-identical; with leaf models the float64 normal equations are summed in
a different order, so leaf values and predictions are compared within 1e-5 /
1e-4 relative, the first tree's structure exactly."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

N, F = 8192, 10          # a power of two: the mean of dyadic targets is exact either way
SPLIT = (5000, 3192)


def _data():
    rng = np.random.default_rng(7)
    X = rng.normal(size=(N, F)).astype(np.float32)
    X[:, 3] = np.exp(X[:, 3])
    X[rng.random(size=X.shape) < 0.02] = np.nan
    z = np.nan_to_num(X)
    y = np.sin(z[:, 0]) + z[:, 1] * z[:, 2] + 0.5 * z[:, 4] + 0.1 * rng.normal(size=N)
    y = (np.round(np.clip(y, -7, 7) * 4) / 4).astype(np.float32)   # dyadic: the mean is exact in float32
    return X, y


def _params(neural: bool, subsample: float = 1.0, levelwise="auto"):
    """max_leaves=15: "auto" grows best-first (yabt/boosting.py:420), True level-wise."""
    from yabt_b200.boosting import BoostParams
    return BoostParams(n_estimators=4, max_leaves=15, max_depth=5, learning_rate=0.3, neural_leaves=neural,
                       leaf_net_min_samples=50, min_samples_leaf=20, subsample=subsample, levelwise=levelwise)


def _summary(b, Xt):
    med, edges, ecnt, scales = b.binner._dev
    trees = [dict(feature=t.feature.cpu().numpy(), threshold=t.threshold.cpu().numpy(),
                  left=t.left.cpu().numpy(), right=t.right.cpu().numpy(), value=t.value.cpu().numpy())
             for t in b.trees]
    return dict(med=med.cpu().numpy(), edges=edges.cpu().numpy(), ecnt=ecnt.cpu().numpy(),
                scales=scales.cpu().numpy(), trees=trees, pred=b.predict_margin(Xt))


def _worker(rank, world, port, backend, neural, q, subsample=1.0, levelwise="auto", fits=1):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = rank if backend == "nccl" else 0
    torch.cuda.set_device(dev)
    kw = dict(device_id=torch.device("cuda", dev)) if backend == "nccl" else {}
    dist.init_process_group(backend, rank=rank, world_size=world, **kw)
    try:
        from yabt_b200.boosting import Booster, MSELoss
        from yabt_b200.distributed import ShardComm
        X, y = _data()
        off = sum(SPLIT[:rank])
        sl = slice(off, off + SPLIT[rank])
        comm = ShardComm()
        sums = []
        for _ in range(fits):          # later fits reuse the group's mapped exchange buffers
            b = Booster(_params(neural, subsample, levelwise), MSELoss())
            b.fit(X[sl], y[sl], comm=comm)
            torch.cuda.synchronize()
            sums.append(_summary(b, X[:1500]))
        for other in sums[1:]:
            np.testing.assert_array_equal(other["pred"], sums[0]["pred"])
        q.put((rank, sums[0]))
        comm.release_exchange()
    except Exception as e:          # report instead of hanging the parent
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _run_sharded(backend, neural, subsample=1.0, levelwise="auto", fits=1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_worker, args=(r, 2, port, backend, neural, q, subsample, levelwise, fits))
             for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert isinstance(res[r], dict), res[r]
    return res


def _single(neural, subsample=1.0, levelwise="auto"):
    from yabt_b200.boosting import Booster, MSELoss
    X, y = _data()
    b = Booster(_params(neural, subsample, levelwise), MSELoss())
    b.fit(X, y)
    return _summary(b, X[:1500])


def _compare(res, ref, neural):
    for r in (0, 1):
        got = res[r]
        np.testing.assert_array_equal(got["med"], ref["med"])
        np.testing.assert_array_equal(got["ecnt"], ref["ecnt"])
        for f in range(F):
            c = ref["ecnt"][f]
            np.testing.assert_array_equal(got["edges"][f, :c], ref["edges"][f, :c])
        np.testing.assert_array_equal(got["scales"], ref["scales"])
        assert len(got["trees"]) == len(ref["trees"])
        for t, (a, b) in enumerate(zip(got["trees"], ref["trees"])):
            if neural and t > 0:
                continue
            for k in ("feature", "threshold", "left", "right"):
                np.testing.assert_array_equal(a[k], b[k], err_msg=f"tree {t} {k}")
            if neural:
                np.testing.assert_allclose(a["value"], b["value"], rtol=1e-5, atol=1e-6)
            else:
                np.testing.assert_array_equal(a["value"], b["value"], err_msg=f"tree {t} value")
        if neural:
            np.testing.assert_allclose(got["pred"], ref["pred"], rtol=1e-4, atol=1e-4)
        else:
            np.testing.assert_array_equal(got["pred"], ref["pred"])
    # both ranks hold the same model
    np.testing.assert_array_equal(res[0]["pred"], res[1]["pred"])


@pytest.mark.parametrize("levelwise", [True, "auto"])
@pytest.mark.parametrize("neural", [False, True])
def test_two_ranks_one_gpu_gloo(neural, levelwise):
    _compare(_run_sharded("gloo", neural, levelwise=levelwise), _single(neural, levelwise=levelwise), neural)


def test_two_ranks_subsample_gloo():
    """Row subsampling draws over the global rows: each rank grows on its share."""
    _compare(_run_sharded("gloo", False, 0.6), _single(False, 0.6), False)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("levelwise", [True, "auto"])
def test_two_ranks_nccl(levelwise):
    """One rank per GPU: the level (or best-first step) histograms are summed by
    the NVLink exchange kernel."""
    _compare(_run_sharded("nccl", True, levelwise=levelwise), _single(True, levelwise=levelwise), True)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_nccl_two_fits():
    """Two fits in a row on one process group: the second reuses the mapped
    exchange buffers (the exchange sequence numbers carry on) and grows the
    same model as the first."""
    _compare(_run_sharded("nccl", True, levelwise=True, fits=2), _single(True, levelwise=True), True)


def _worker_classifier(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from yabt_b200 import YABTClassifier
        from yabt_b200.distributed import ShardComm
        X, y = _data()
        yb = np.where(y > 0, 3.0, -1.0).astype(np.float32)       # labels other than 0 / 1
        off = sum(SPLIT[:rank])
        sl = slice(off, off + SPLIT[rank])
        comm = ShardComm()
        est = YABTClassifier(n_estimators=4, max_leaves=31, learning_rate=0.3, neural_leaves=False)
        est.fit(X[sl], yb[sl], comm=comm)
        torch.cuda.synchronize()
        q.put((rank, dict(classes=est.classes_.tolist(), proba=est.predict_proba(X[:1500]))))
        comm.release_exchange()
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_nccl_classifier():
    """The estimator's own sharded fit (YABTClassifier.fit(..., comm=)): the
    class labels are gathered over NCCL from host arrays, and the sharded model
    equals the single-GPU one (no leaf models: bit for bit)."""
    from yabt_b200 import YABTClassifier
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_worker_classifier, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    X, y = _data()
    yb = np.where(y > 0, 3.0, -1.0).astype(np.float32)
    ref = YABTClassifier(n_estimators=4, max_leaves=31, learning_rate=0.3, neural_leaves=False).fit(X, yb)
    for r in range(2):
        assert isinstance(res[r], dict), res[r]
        assert res[r]["classes"] == [-1.0, 3.0]
        np.testing.assert_array_equal(res[r]["proba"], ref.predict_proba(X[:1500]))


def _chain(n=8192, F=12, seed=3, chain=10):
    """Nested target (the level-loop tests' data): trees grow about `chain`
    levels deep, past the device-side loop's first level."""
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, F)).astype(np.float32)
    on = np.ones(n, dtype=bool)
    y = np.zeros(n, dtype=np.float32)
    for k in range(chain):
        on &= X[:, k] > -0.3
        y += 2.0 * on
    return X, y


def _loop_params():
    from yabt_b200.boosting import BoostParams
    return BoostParams(n_estimators=4, max_leaves=31, max_depth=64, learning_rate=0.3, neural_leaves=False,
                       min_samples_leaf=5, levelwise=True)


def _worker_loop(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from yabt_b200 import _lib
        from yabt_b200.boosting import Booster, MSELoss
        from yabt_b200.distributed import ShardComm
        lib = _lib.load()
        X, y = _chain()
        off = sum(SPLIT[:rank])
        sl = slice(off, off + SPLIT[rank])
        comm = ShardComm()
        out = {}
        for loop in (True, False):
            torch.cuda.synchronize()
            _lib.check(lib.yabt_launch_count_device_reset(_lib.stream_ptr()), "reset")
            b = Booster(_loop_params(), MSELoss())
            b._level_loop = loop
            b.fit(X[sl], y[sl], comm=comm)
            torch.cuda.synchronize()
            out[loop] = dict(trees=[{k: getattr(t, k).cpu().numpy() for k in ("feature", "threshold", "left",
                                                                              "right", "value")} for t in b.trees],
                             pred=b.predict_margin(X[:2000]), dev=int(lib.yabt_launch_count_device()),
                             start=b.grower_.level_loop_start())
        q.put((rank, out))
        comm.release_exchange()
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_nccl_level_loop():
    """Sharded feature-sliced trees with their deeper levels in the device-side
    level loop (reduce-scatter and best-split gather inside the loop's body):
    the same bits as the same fit with every level driven by the host, and as
    a single-GPU fit; the loop ran on every rank."""
    from yabt_b200.boosting import Booster, MSELoss
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_worker_loop, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    X, y = _chain()
    ref = Booster(_loop_params(), MSELoss()).fit(X, y)
    for r in range(2):
        assert isinstance(res[r], dict), res[r]
        on, off = res[r][True], res[r][False]
        assert on["start"] > 0
        assert on["dev"] >= 9 and off["dev"] == 0, (on["dev"], off["dev"])
        for t, (a, b, c) in enumerate(zip(on["trees"], off["trees"], ref.trees)):
            for k in ("feature", "threshold", "left", "right", "value"):
                np.testing.assert_array_equal(a[k], b[k], err_msg=f"rank {r} tree {t} {k}")
                np.testing.assert_array_equal(a[k], getattr(c, k).cpu().numpy(), err_msg=f"rank {r} tree {t} {k}")
        np.testing.assert_array_equal(on["pred"], ref.predict_margin(X[:2000]))
