"""Row-sharded fitting over several GPUs, one process per GPU.

Each rank holds a contiguous block of the training rows (its shard) and runs
the same sequence of kernels as a single-GPU fit on its own rows. Wherever the
reference's fit reads statistics of ALL rows, the ranks reduce their partial
statistics with ``torch.distributed`` collectives (NCCL over NVLink on GPUs;
gloo, staged through host memory, in the CPU tests), so that every rank takes
identical decisions and holds an identical model:

* binning (yabt/binning.py:29-69): the three radix-selection passes of the
  medians sum their digit histograms and NaN counts; the quantile sample is the
  reference's own draw over the global row count, gathered from the ranks
  that own the rows;
* column moments for the leaf models: sums, then centred sums of squares;
* per tree: the max |g| / max |h| quantisation words (max), every level's
  smaller-child histograms (exact int64 sums, so split decisions are
  bit-identical to a single-GPU fit on the concatenated rows), and the leaf
  models' statistics (gradient correlations, leaf counts, normal equations,
  input envelopes);
* the base score (sum of y).

With the NVLink exchange (one rank per GPU), the per-tree reductions (the
quantisation words and the leaf-model statistics) run through the same mapped
buffers as the level histograms (yabt_grow_xallreduce: one small kernel, summed
in rank order, no host round trip); otherwise through the process group.

Margins, gradients, row partitions and leaf assignments stay rank-local.
Float64 sums of the leaf-model statistics change order with the rank count,
so leaf values agree with a single-GPU fit to rounding, not bit for bit.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib

QUANTILE_SAMPLE = 200_000
LOOKAHEAD = 3         # levels the GPU keeps queued while the host checks for a complete tree


class ShardComm:
    """Collectives of one process group. With the NCCL backend tensors are
    reduced in place on the device; with any other backend (gloo) they are
    staged through host memory."""

    def __init__(self, group=None, peer_exchange: bool = True, feature_sliced: bool = True):
        """``peer_exchange``: sum the level histograms with the library's own
        NVLink kernel (yabt_grow_xreduce) when every rank has its own GPU on
        this node and the backend is NCCL; otherwise with all-reduces.
        ``feature_sliced`` (with the exchange, level-wise trees): each rank
        reduces and scans only its slice of the features and the ranks
        exchange each node's best split."""
        import torch.distributed as dist
        if not dist.is_initialized():
            raise RuntimeError("ShardComm needs an initialised torch.distributed process group")
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.on_device = dist.get_backend(group) == "nccl"
        self.peer_exchange = bool(peer_exchange) and self.on_device and 1 < self.world <= 8
        self.feature_sliced = bool(feature_sliced)
        if self.peer_exchange:
            import hashlib
            uuid = str(torch.cuda.get_device_properties(torch.cuda.current_device()).uuid)
            key = int.from_bytes(hashlib.sha1(uuid.encode()).digest()[:7], "little")
            self.peer_exchange = len(set(self.int_values(key))) == self.world

    # in-place reductions -------------------------------------------------
    def _reduce(self, t: torch.Tensor, op) -> torch.Tensor:
        if self.world == 1:
            return t
        if self.on_device:
            from .phases import host_phase
            with host_phase():
                self.dist.all_reduce(t, op=op, group=self.group)
            return t
        if t.device.type == "cpu":
            self.dist.all_reduce(t, op=op, group=self.group)
            return t
        h = t.cpu()
        self.dist.all_reduce(h, op=op, group=self.group)
        t.copy_(h)
        return t

    def sum_(self, t: torch.Tensor) -> torch.Tensor:
        return self._reduce(t, self.dist.ReduceOp.SUM)

    def max_(self, t: torch.Tensor) -> torch.Tensor:
        return self._reduce(t, self.dist.ReduceOp.MAX)

    def min_(self, t: torch.Tensor) -> torch.Tensor:
        return self._reduce(t, self.dist.ReduceOp.MIN)

    # NVLink exchange buffers (held across fits) ---------------------------
    def exchange_buffers(self, nbytes: int) -> "ExchangeBuffers":
        """This group's exchange buffers of at least ``nbytes`` data bytes
        (collective when they have to be created or grown: every rank asks for
        the same size at the same point of the fit)."""
        x = getattr(self, "_xbufs", None)
        if x is not None and x.nbytes >= nbytes:
            return x
        if x is not None:
            x.release()
        self._xbufs = ExchangeBuffers(self, nbytes)
        return self._xbufs

    def release_exchange(self) -> None:
        """Collective: free the exchange buffers (they are otherwise kept until exit)."""
        x = getattr(self, "_xbufs", None)
        if x is not None:
            x.release()
            self._xbufs = None

    # scalars and gathers -------------------------------------------------
    def int_values(self, v: int) -> list[int]:
        """Every rank's value of an integer, in rank order."""
        dev = "cuda" if self.on_device else "cpu"
        mine = torch.tensor([int(v)], dtype=torch.int64, device=dev)
        out = [torch.empty_like(mine) for _ in range(self.world)]
        self.dist.all_gather(out, mine, group=self.group)
        return [int(x.item()) for x in out]

    def sum_float(self, v: float) -> float:
        dev = "cuda" if self.on_device else "cpu"
        t = torch.tensor([float(v)], dtype=torch.float64, device=dev)
        self.sum_(t)
        return float(t.item())

    def gather_columns(self, x: torch.Tensor) -> torch.Tensor:
        """Concatenate every rank's (F, m_r) float32 block along columns, in
        rank order; the result is on x's device."""
        F, m = x.shape
        sizes = self.int_values(m)
        mx = max(max(sizes), 1)
        # the collective runs where the backend works (NCCL: this rank's GPU,
        # even for a host tensor such as an estimator's class labels)
        dev = torch.device("cuda", torch.cuda.current_device()) if self.on_device else torch.device("cpu")
        pad = torch.zeros(F, mx, dtype=x.dtype, device=dev)
        pad[:, :m] = x.to(dev)
        parts = [torch.empty_like(pad) for _ in range(self.world)]
        self.dist.all_gather(parts, pad, group=self.group)
        return torch.cat([p[:, :s] for p, s in zip(parts, sizes)], dim=1).to(x.device).contiguous()


def _view(base: torch.Tensor, ptr: int, count: int, dtype: torch.dtype) -> torch.Tensor:
    """``count`` elements of ``dtype`` at device address ``ptr`` inside the
    uint8 workspace tensor ``base``."""
    size = torch.empty(0, dtype=dtype).element_size()
    off = int(ptr) - base.data_ptr()
    if off < 0 or off + count * size > base.numel() or off % size:
        raise _lib.YabtError("buffer outside its workspace")
    return base[off:off + count * size].view(dtype)


def shard_layout(comm: ShardComm, n_local: int) -> tuple[int, int]:
    """(first global row of this rank, total rows): ranks hold contiguous
    blocks in rank order."""
    sizes = comm.int_values(n_local)
    return sum(sizes[:comm.rank]), sum(sizes)


def sample_rows(n_total: int) -> np.ndarray:
    """Global quantile-sample rows: the reference's draw (yabt/binning.py:36-40)."""
    if n_total > QUANTILE_SAMPLE:
        return np.random.default_rng(0).choice(n_total, QUANTILE_SAMPLE, replace=False)
    return np.arange(n_total)


def local_sample(rows: np.ndarray, offset: int, n_local: int) -> np.ndarray:
    """The sample rows this rank owns, as local row indices (draw order)."""
    mine = rows[(rows >= offset) & (rows < offset + n_local)]
    return (mine - offset).astype(np.int64)


def fit_binner(Xfm: torch.Tensor, n_local: int, max_bins: int, comm: ShardComm):
    """Device binner state (medians, edges [F][255], edge counts, scales)
    fitted over the rows of every rank."""
    lib = _lib.load()
    F = Xfm.shape[0]
    dev = Xfm.device
    s = _lib.stream_ptr()
    offset, n_total = shard_layout(comm, n_local)
    ws = torch.empty(int(lib.yabt_bin_fit_workspace_bytes(max(n_local, 1), F, 1)), dtype=torch.uint8, device=dev)
    hp, words, nanp = ctypes.c_void_p(), ctypes.c_longlong(), ctypes.c_void_p()
    _lib.check(lib.yabt_bin_median_bufs(F, ws.data_ptr(), ctypes.byref(hp), ctypes.byref(words),
                                        ctypes.byref(nanp)), "yabt_bin_median_bufs")
    hist = _view(ws, hp.value, words.value, torch.int32)
    nanc = _view(ws, nanp.value, F, torch.int64)
    for p in range(3):
        _lib.check(lib.yabt_bin_median_hist(Xfm.data_ptr(), n_local, F, p, ws.data_ptr(), ws.numel(), s),
                   "yabt_bin_median_hist")
        comm.sum_(hist)                      # uint32 counts: int32 sums wrap identically
        if p == 0:
            comm.sum_(nanc)
        _lib.check(lib.yabt_bin_median_pick(n_total, F, p, ws.data_ptr(), ws.numel(), s), "yabt_bin_median_pick")
    med = torch.empty(F, dtype=torch.float32, device=dev)
    _lib.check(lib.yabt_bin_median_final(F, ws.data_ptr(), ws.numel(), med.data_ptr(), s), "yabt_bin_median_final")
    del ws
    idx = torch.from_numpy(local_sample(sample_rows(n_total), offset, n_local)).to(dev)
    Xs = comm.gather_columns(Xfm.index_select(1, idx))
    nq = Xs.shape[1]
    ws = torch.empty(int(lib.yabt_bin_fit_workspace_bytes(nq, F, nq)), dtype=torch.uint8, device=dev)
    edges = torch.empty(F, 255, dtype=torch.float32, device=dev)
    ecnt = torch.empty(F, dtype=torch.int32, device=dev)
    scales = torch.empty(F, dtype=torch.float32, device=dev)
    _lib.check(lib.yabt_bin_fit_edges(Xs.data_ptr(), nq, F, max_bins, ws.data_ptr(), ws.numel(), edges.data_ptr(),
                                      ecnt.data_ptr(), scales.data_ptr(), s), "yabt_bin_fit_edges")
    return med, edges, ecnt, scales


def column_stats(Xfm: torch.Tensor, n_local: int, comm: ShardComm) -> tuple[torch.Tensor, torch.Tensor]:
    """Column means and unbiased stds over the rows of every rank."""
    lib = _lib.load()
    F = Xfm.shape[0]
    dev = Xfm.device
    s = _lib.stream_ptr()
    _, n_total = shard_layout(comm, n_local)
    acc = torch.zeros(2 * F, dtype=torch.float64, device=dev)
    for p in range(2):
        _lib.check(lib.yabt_column_sums(Xfm.data_ptr(), n_local, n_total, F, p, acc.data_ptr(), s), "yabt_column_sums")
        comm.sum_(acc[p * F:(p + 1) * F])
    mean = torch.empty(F, dtype=torch.float32, device=dev)
    std = torch.empty(F, dtype=torch.float32, device=dev)
    _lib.check(lib.yabt_column_finish(acc.data_ptr(), n_total, F, mean.data_ptr(), std.data_ptr(), s),
               "yabt_column_finish")
    return mean, std


class ExchangeBuffers:
    """Every rank's exchange buffer, mapped into this process (CUDA IPC over
    NVLink, plain peer loads and stores). Held by the ShardComm across fits:
    setting up and tearing down the IPC mappings costs a synchronisation of the
    ranks and can take longer than a whole fit, so a fit binds its grower to
    the buffers instead and leaves them mapped (``ShardComm.release_exchange``
    frees them). ``epoch`` numbers the exchange calls; every rank makes the
    same calls in the same order, so the sequences agree."""

    def __init__(self, comm: "ShardComm", nbytes: int):
        self.lib = lib = _lib.load()
        self.comm = comm
        handle = (ctypes.c_char * 64)()
        own = ctypes.c_void_p()
        _lib.check(lib.yabt_xchg_alloc(nbytes, ctypes.byref(own), handle), "yabt_xchg_alloc")
        self.own = own.value
        self.header = int(lib.yabt_xchg_header_bytes())
        dev = torch.device("cuda", torch.cuda.current_device())
        mine = torch.frombuffer(bytearray(handle.raw), dtype=torch.uint8).to(dev)
        parts = [torch.empty_like(mine) for _ in range(comm.world)]
        comm.dist.all_gather(parts, mine, group=comm.group)
        self.opened = []
        ptrs = []
        for q, t in enumerate(parts):
            if q == comm.rank:
                ptrs.append(self.own)
                continue
            hq = (ctypes.c_char * 64).from_buffer_copy(bytes(t.cpu().numpy()))
            pq = ctypes.c_void_p()
            _lib.check(lib.yabt_xchg_open(hq, ctypes.byref(pq)), "yabt_xchg_open")
            self.opened.append(pq.value)
            ptrs.append(pq.value)
        self.bufs = (ctypes.c_void_p * comm.world)(*ptrs)
        self.nbytes = nbytes
        self.epoch = 0
        comm.dist.barrier(group=comm.group)

    def next_epoch(self) -> int:
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF or 1
        return self.epoch

    def reserve_epochs(self, count: int) -> int:
        """The first of ``count`` consecutive epochs (a device-side level loop
        numbers its exchange calls from it); no wrap-around inside the block."""
        if self.epoch + count + 1 > 0xFFFFFFFF:
            self.epoch = 0
        first = self.epoch + 1
        self.epoch += count
        return first

    def release(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's."""
        torch.cuda.synchronize()
        self.comm.dist.barrier(group=self.comm.group)     # no rank still reads or writes a peer buffer
        for p in self.opened:
            self.lib.yabt_xchg_close(p)
        self.opened = []
        self.comm.dist.barrier(group=self.comm.group)
        if self.own:
            self.lib.yabt_xchg_free(self.own)
            self.own = None


def feature_slice(F: int, rank: int, world: int) -> tuple[int, int]:
    """Features [lo, hi) that rank scans in feature-sliced growth (the rule of
    yabt_grow_xreduce_sliced)."""
    return F * rank // world, F * (rank + 1) // world


class PeerExchange:
    """A grower bound to the ShardComm's exchange buffers (its smaller-child
    histogram buffer is this rank's exchange buffer). ``reduce(level)``
    launches yabt_grow_xreduce: no host synchronisation and exactly the level's
    bytes; ``allreduce_`` the small per-tree reductions. With ``sliced`` (the
    level-wise grower, at least one feature per rank) each level is instead
    reduce-scattered by feature slices (``reduce_sliced``), scanned on the
    rank's slice and the ranks' best splits gathered (``gather``). ``close()``
    must be called on every rank at the end of the fit; the buffers stay mapped
    for the next fit."""

    def __init__(self, grower, comm: ShardComm):
        self.lib = lib = grower.lib
        self.grower, self.comm = grower, comm
        hist = int(lib.yabt_grow_small_count(grower.h, 62)) * 8          # the largest level
        self.rec_offset = (hist + 255) // 256 * 256                       # per-node best-split records after it
        need = self.rec_offset + int(lib.yabt_grow_xgather_bytes(grower.h))
        self.x = comm.exchange_buffers(need)
        _lib.check(lib.yabt_grower_set_small(grower.h, self.x.own + self.x.header, self.x.nbytes),
                   "yabt_grower_set_small")
        self.bufs, self.nbytes = self.x.bufs, self.x.nbytes
        self.sliced = False

    def set_sliced(self, on: bool) -> None:
        """Feature-sliced levels (needs at least one feature per rank)."""
        F = self.grower.F
        on = bool(on) and F >= self.comm.world
        lo, hi = feature_slice(F, self.comm.rank, self.comm.world) if on else (0, F)
        _lib.check(self.lib.yabt_grower_set_feature_slice(self.grower.h, lo, hi), "yabt_grower_set_feature_slice")
        self.sliced = on

    def reduce_sliced(self, level: int) -> None:
        _lib.check(self.lib.yabt_grow_xreduce_sliced(self.grower.h, self.bufs, self.comm.rank, self.comm.world,
                                                     level, self.x.next_epoch(), _lib.stream_ptr()),
                   "yabt_grow_xreduce_sliced")

    def gather(self, level: int) -> None:
        _lib.check(self.lib.yabt_grow_xgather(self.grower.h, self.bufs, self.comm.rank, self.comm.world, level,
                                              self.x.next_epoch(), self.rec_offset, _lib.stream_ptr()),
                   "yabt_grow_xgather")

    def level_loop(self, a: _lib.TreeArgs) -> bool:
        """The tree's remaining levels (from the grower's level_loop_start())
        as one device-side loop with the sliced exchange inside it; False when
        the loop cannot run now (the caller then drives those levels)."""
        g = self.grower
        first = g.level_loop_start()
        e0 = self.x.reserve_epochs(2 * max(g.levels - first, 0))
        used = ctypes.c_int()
        _lib.check(self.lib.yabt_grow_level_loop_sharded(g.h, ctypes.byref(a), self.bufs, self.comm.rank,
                                                         self.comm.world, self.rec_offset, e0, ctypes.byref(used),
                                                         _lib.stream_ptr()), "yabt_grow_level_loop_sharded")
        return bool(used.value)

    def reduce(self, level: int) -> None:
        _lib.check(self.lib.yabt_grow_xreduce(self.grower.h, self.bufs, self.comm.rank, self.comm.world, level,
                                              self.x.next_epoch(), _lib.stream_ptr()), "yabt_grow_xreduce")

    _KINDS = {(torch.int64, "sum"): 0, (torch.float64, "sum"): 1, (torch.int32, "max"): 2,
              (torch.float32, "max"): 3}

    def allreduce_(self, t: torch.Tensor, op: str) -> bool:
        """In-place all-reduce of a small contiguous device tensor through the
        exchange buffers (yabt_grow_xallreduce: one kernel, rank-ordered, no
        host round trip). False when the dtype / op or the size does not fit
        (the caller then uses the process group)."""
        kind = self._KINDS.get((t.dtype, op))
        if kind is None or not t.is_contiguous() or t.numel() * t.element_size() > self.nbytes:
            return False
        _lib.check(self.lib.yabt_grow_xallreduce(self.grower.h, self.bufs, self.nbytes, self.comm.rank,
                                                 self.comm.world, t.data_ptr(), t.data_ptr(), t.numel(), kind,
                                                 self.x.next_epoch(), _lib.stream_ptr()), "yabt_grow_xallreduce")
        return True

    def check(self) -> None:
        """Raises if a per-tree all-reduce timed out (reads one device word)."""
        bits = ctypes.c_uint()
        _lib.check(self.lib.yabt_grow_xerr(self.grower.h, ctypes.byref(bits)), "yabt_grow_xerr")
        if bits.value:
            raise _lib.YabtError(f"peer all-reduce timed out (device error bits 0x{bits.value:x})")

    def close(self) -> None:
        """End of the fit: the grower lets go of the buffers (which stay mapped)."""
        if self.sliced:
            self.set_sliced(False)
        self.grower = None


def _reduce_sum(comm: ShardComm, xchg, t: torch.Tensor) -> None:
    """Sum over the ranks in place: the exchange kernel when it can, else the process group."""
    if xchg is None or not xchg.allreduce_(t, "sum"):
        comm.sum_(t)


def _reduce_max(comm: ShardComm, xchg, t: torch.Tensor) -> None:
    if xchg is None or not xchg.allreduce_(t, "max"):
        comm.max_(t)


def grow_tree(grower, a: _lib.TreeArgs, comm: ShardComm) -> None:
    """One tree over the rows of every rank: the grower's step API with the
    quantisation words and each level's smaller-child histograms summed
    between the steps. With the peer exchange the sums are one kernel per
    level that reads the level's size from the device. Otherwise they are
    all-reduces: the level state (pairs, active) of the previous split is
    copied to host memory while the next level's histogram kernels run, so
    each all-reduce covers exactly that level's histograms and the loop stops
    with the tree; the state is identical on every rank, so every rank makes
    the same collective calls."""
    lib = grower.lib
    h = grower.h
    s = _lib.stream_ptr()
    ref = ctypes.byref(a)
    if not hasattr(grower, "_level_host"):
        grower._level_host = torch.zeros(4, dtype=torch.int32).pin_memory()
        grower._level_event = torch.cuda.Event()
    info, ev = grower._level_host, grower._level_event
    state = _view(grower.ws, lib.yabt_grow_level_ptr(h), 4, torch.int32)
    xchg = getattr(grower, "_exchange", None)
    if xchg is None and comm.peer_exchange:
        xchg = grower._exchange = PeerExchange(grower, comm)
    _lib.check(lib.yabt_grow_begin(h, ref, s), "yabt_grow_begin")
    _reduce_max(comm, xchg, _view(grower.ws, lib.yabt_grow_amax_ptr(h), 2, torch.int32))   # non-negative float bits
    _lib.check(lib.yabt_grow_init(h, ref, s), "yabt_grow_init")
    if xchg is not None:
        # the NVLink exchange sizes itself from the device state; the host reads
        # each level's state LOOKAHEAD levels later (the GPU keeps that many
        # levels queued) and stops launching once the tree is complete. With
        # feature slices each rank sums and scans only its slice of the
        # features, and the ranks' best splits per node are gathered before
        # the splits are chosen.
        if not xchg.sliced and comm.feature_sliced:
            xchg.set_sliced(True)
        if not hasattr(grower, "_level_ring"):
            grower._level_ring = [(torch.cuda.Event(), torch.zeros(4, dtype=torch.int32).pin_memory())
                                  for _ in range(8)]
        ring = grower._level_ring
        # feature-sliced trees run their levels from level_loop_start() on in
        # the device-side level loop (every rank takes the same branch)
        loop_from = grower.level_loop_start() if xchg.sliced else -1
        for d in range(grower.levels):
            if d == loop_from and xchg.level_loop(a):
                break
            _lib.check(lib.yabt_grow_hist(h, ref, d, s), "yabt_grow_hist")
            if xchg.sliced:
                xchg.reduce_sliced(d)
                _lib.check(lib.yabt_grow_scan(h, ref, d, s), "yabt_grow_scan")
                xchg.gather(d)
                _lib.check(lib.yabt_grow_choose(h, ref, d, s), "yabt_grow_choose")
            else:
                xchg.reduce(d)
                _lib.check(lib.yabt_grow_split(h, ref, d, s), "yabt_grow_split")
            if not getattr(grower, "level_wait", True):
                continue                         # every level queued (finished levels are no-ops on every rank)
            ev_d, host_d = ring[d % 8]
            host_d.copy_(state, non_blocking=True)
            ev_d.record()
            if d >= LOOKAHEAD:
                ev_o, host_o = ring[(d - LOOKAHEAD) % 8]
                ev_o.synchronize()
                if not int(host_o[1]):           # identical on every rank
                    break
        _lib.check(lib.yabt_grow_end(h, ref, s), "yabt_grow_end")
        return
    per_job = int(lib.yabt_grow_small_count(h, 0))
    small = _view(grower.ws, lib.yabt_grow_small_ptr(h), int(lib.yabt_grow_small_count(h, grower.levels - 1)),
                  torch.int64)
    jobs = 1
    for d in range(grower.levels):
        _lib.check(lib.yabt_grow_hist(h, ref, d, s), "yabt_grow_hist")
        if d > 0:
            ev.synchronize()                 # the previous split's state; level d's histogram runs meanwhile
            _, active, _, jobs = info.tolist()
            if not active:
                break
        comm.sum_(small[:jobs * per_job])
        _lib.check(lib.yabt_grow_split(h, ref, d, s), "yabt_grow_split")
        info.copy_(state, non_blocking=True)
        ev.record()
    _lib.check(lib.yabt_grow_end(h, ref, s), "yabt_grow_end")


def grow_tree_bestfirst(grower, a: _lib.TreeArgs, comm: ShardComm) -> None:
    """Best-first growth (yabt/tree.py:206-360) over the rows of every rank:
    the step-wise best-first API with the quantisation words, the root
    histogram and each step's smaller-child histogram (one job) summed between
    the halves of a step. The candidate choice reads only summed histograms,
    so every rank splits the same nodes and makes the same collective calls;
    the host stops LOOKAHEAD steps after the device reports the tree complete."""
    lib = grower.lib
    h = grower.h
    s = _lib.stream_ptr()
    ref = ctypes.byref(a)
    if not hasattr(grower, "_level_ring"):
        grower._level_ring = [(torch.cuda.Event(), torch.zeros(4, dtype=torch.int32).pin_memory())
                              for _ in range(8)]
    ring = grower._level_ring
    state = _view(grower.ws, lib.yabt_grow_level_ptr(h), 4, torch.int32)
    xchg = getattr(grower, "_exchange", None)
    if xchg is None and comm.peer_exchange:
        xchg = grower._exchange = PeerExchange(grower, comm)
    _lib.check(lib.yabt_grow_begin(h, ref, s), "yabt_grow_begin")
    _reduce_max(comm, xchg, _view(grower.ws, lib.yabt_grow_amax_ptr(h), 2, torch.int32))   # non-negative float bits
    _lib.check(lib.yabt_grow_init(h, ref, s), "yabt_grow_init")
    small = None
    if xchg is None:   # with the exchange the histograms live in its buffer, outside the workspace
        small = _view(grower.ws, lib.yabt_grow_small_ptr(h), int(lib.yabt_grow_small_count(h, 0)), torch.int64)

    def reduce(level):
        if xchg is not None:
            xchg.reduce(level)           # sizes itself from the device state (a no-op step skips)
        else:
            comm.sum_(small)

    _lib.check(lib.yabt_grow_bf_root_hist(h, ref, s), "yabt_grow_bf_root_hist")
    reduce(0)
    _lib.check(lib.yabt_grow_bf_scan(h, ref, 0, s), "yabt_grow_bf_scan")
    for k in range(1, max(1, grower.max_leaves - 1) + 1):
        _lib.check(lib.yabt_grow_bf_split(h, ref, k, s), "yabt_grow_bf_split")
        reduce(1)                            # the best-first histogram runs at level 1
        _lib.check(lib.yabt_grow_bf_scan(h, ref, k, s), "yabt_grow_bf_scan")
        ev_k, host_k = ring[k % 8]
        host_k.copy_(state, non_blocking=True)
        ev_k.record()
        if k > LOOKAHEAD:
            ev_o, host_o = ring[(k - LOOKAHEAD) % 8]
            ev_o.synchronize()
            if not int(host_o[1]):           # identical on every rank
                break
    _lib.check(lib.yabt_grow_end(h, ref, s), "yabt_grow_end")


def fit_leaf_models(la: _lib.LeafNetArgs, ws: torch.Tensor, comm: ShardComm, grower=None) -> None:
    """Leaf models of one tree over the rows of every rank: the three stages
    of yabt_leafnet_stage with the statistics reduced in between."""
    lib = _lib.load()
    s = _lib.stream_ptr()
    ref = ctypes.byref(la)
    ptr = [ctypes.c_void_p() for _ in range(3)]
    cnt = [ctypes.c_longlong() for _ in range(3)]
    _lib.check(lib.yabt_leafnet_bufs(ref, ws.data_ptr(), ws.numel(), ctypes.byref(ptr[0]), ctypes.byref(cnt[0]),
                                     ctypes.byref(ptr[1]), ctypes.byref(cnt[1]), ctypes.byref(ptr[2]),
                                     ctypes.byref(cnt[2])), "yabt_leafnet_bufs")
    stats = _view(ws, ptr[0].value, cnt[0].value, torch.float64)
    totals = _view(ws, ptr[1].value, cnt[1].value, torch.float64)
    env = _view(ws, ptr[2].value, cnt[2].value, torch.float32)

    def stage(k):
        _lib.check(lib.yabt_leafnet_stage(ref, k, ws.data_ptr(), ws.numel(), s), "yabt_leafnet_stage")
    xchg = getattr(grower, "_exchange", None) if grower is not None else None
    stage(0)
    _reduce_sum(comm, xchg, stats)
    stage(1)
    _reduce_sum(comm, xchg, totals)
    _reduce_max(comm, xchg, env)
    stage(2)
