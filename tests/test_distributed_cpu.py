"""Host logic of the row-sharded fit on CPU: two gloo ranks exercise the
collectives wrapper (sums, maxima, minima, gathers of
ragged column blocks), the shard layout and the split of the reference's
quantile sample across ranks. No GPU is used."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from yabt_b200.distributed import QUANTILE_SAMPLE, local_sample, sample_rows


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from yabt_b200.distributed import ShardComm, shard_layout
        c = ShardComm()
        out = {}
        t = torch.arange(6, dtype=torch.int64) * (rank + 1)
        out["sum"] = c.sum_(t).tolist()
        f = torch.tensor([1.5, -2.0, float("inf")]) * (1 if rank == 0 else -1)
        out["max"] = c.max_(f.clone()).tolist()
        out["min"] = c.min_(f.clone()).tolist()
        # bit patterns of non-negative floats (the quantisation words) order as int32
        w = torch.tensor([np.float32(1.5 * (rank + 1)).view(np.int32), 0 if rank == 0 else 0x3F000000],
                         dtype=torch.int32)
        out["fmax"] = c.max_(w).tolist()
        n_local = [7, 3][rank]
        out["layout"] = shard_layout(c, n_local)
        blk = torch.full((2, n_local), float(rank)) + torch.arange(n_local).float()
        out["gather"] = c.gather_columns(blk).tolist()
        out["fsum"] = c.sum_float(0.25 * (rank + 1))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def test_collectives_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        o = res[r]
        assert o["sum"] == [3 * i for i in range(6)]
        assert o["max"] == [1.5, 2.0, float("inf")]
        assert o["min"] == [-1.5, -2.0, float("-inf")]
        assert o["fmax"] == [int(np.float32(3.0).view(np.int32)), 0x3F000000]
        assert o["layout"] == ((0, 10) if r == 0 else (7, 10))
        assert o["gather"] == [[0, 1, 2, 3, 4, 5, 6, 1, 2, 3], [0, 1, 2, 3, 4, 5, 6, 1, 2, 3]]
        assert o["fsum"] == 0.75


@pytest.mark.parametrize("n_total,sizes", [(1000, [600, 400]), (450_000, [100_000, 250_000, 100_000])])
def test_quantile_sample_split(n_total, sizes):
    """The ranks' local sample rows, shifted by their offsets, are exactly the
    reference's sample (yabt/binning.py:36-40) drawn over the global rows."""
    rows = sample_rows(n_total)
    assert len(rows) == min(n_total, QUANTILE_SAMPLE)
    got, off = [], 0
    for n in sizes:
        loc = local_sample(rows, off, n)
        assert loc.min() >= 0 and loc.max() < n
        got.append(loc + off)
        off += n
    np.testing.assert_array_equal(np.sort(np.concatenate(got)), np.sort(rows))
    if n_total > QUANTILE_SAMPLE:
        ref = np.random.default_rng(0).choice(n_total, QUANTILE_SAMPLE, replace=False)
        np.testing.assert_array_equal(rows, ref)


def test_reserve_epochs_blocks_never_wrap():
    """The exchange epochs a device-side level loop numbers from: consecutive,
    after every epoch already handed out, never containing 0 and never
    wrapping inside a block (every rank computes the same numbers)."""
    from types import SimpleNamespace

    from yabt_b200.distributed import ExchangeBuffers
    x = SimpleNamespace(epoch=0)
    assert ExchangeBuffers.next_epoch(x) == 1
    first = ExchangeBuffers.reserve_epochs(x, 20)
    assert first == 2 and x.epoch == 21
    assert ExchangeBuffers.next_epoch(x) == 22
    x.epoch = 0xFFFFFFFF - 5
    first = ExchangeBuffers.reserve_epochs(x, 10)       # would cross 2^32: restarts at 1
    assert first == 1 and x.epoch == 10
    x.epoch = 0xFFFFFFFF - 12
    first = ExchangeBuffers.reserve_epochs(x, 10)
    assert first == 0xFFFFFFFF - 11 and first + 9 <= 0xFFFFFFFF
