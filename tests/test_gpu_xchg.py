"""The NVLink level exchange (yabt_grow_xreduce) on one GPU, without faulting
or hanging it.

1. A two-rank exchange whose second rank never arrives: the first rank's
   kernel polls the peer's "histograms written" flag, gives up after its
   bounded wait (about a second), sets the exchange-timeout bit in the tree's
   error word and returns; the host reads the bit and the context stays
   usable.
2. A one-rank exchange (the kernel's own flags only) leaves the level's
   histograms unchanged, so a tree grown with it equals a tree grown without.
3. The small-vector all-reduce (yabt_grow_xallreduce): identity on one rank
   for every element kind, a refused oversized vector, and the same bounded
   wait and persistent error bit when a peer never arrives.
4. Feature-sliced levels (reduce-scatter, slice scan, best-split gather,
   choice) on one rank grow the same tree as the whole-tree call.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

XCHG_TIMEOUT_BIT = 1 << 7


def _setup(n=5000, F=12, seed=0):
    from yabt_b200.grower import EdgePack, Grower, pack_bins
    from yabt_b200.tree import TreeParams
    rng = np.random.default_rng(seed)
    binned = torch.from_numpy(rng.integers(0, 40, size=(n, F)).astype(np.uint8)).cuda()
    grad = torch.from_numpy(rng.normal(size=n).astype(np.float32)).cuda()
    hess = torch.ones(n, device="cuda")

    class _B:   # edges: bin b <-> threshold b
        edges_ = [torch.arange(39, dtype=torch.float32) for _ in range(F)]
        scales_ = torch.ones(F)
    gr = Grower(n, F, 15, 5, False, "cuda")
    ep = EdgePack(list(_B.edges_), _B.scales_, "cuda")
    out = gr.new_outputs()
    a = gr.args(pack_bins(binned), grad, hess, ep, TreeParams(max_leaves=15, max_depth=5), out)
    return gr, a, out


def _xchg_buffers(gr, count):
    from yabt_b200 import _lib
    lib = gr.lib
    nbytes = int(lib.yabt_grow_small_count(gr.h, 62)) * 8
    bufs = []
    for _ in range(count):
        p, hnd = ctypes.c_void_p(), (ctypes.c_char * 64)()
        _lib.check(lib.yabt_xchg_alloc(nbytes, ctypes.byref(p), hnd), "yabt_xchg_alloc")
        bufs.append(p.value)
    return bufs, nbytes


def test_exchange_wait_times_out_and_reports():
    from yabt_b200 import _lib
    gr, a, out = _setup()
    lib = gr.lib
    s = _lib.stream_ptr()
    (b0, b1), nbytes = _xchg_buffers(gr, 2)
    hdr = int(lib.yabt_xchg_header_bytes())
    try:
        _lib.check(lib.yabt_grower_set_small(gr.h, b0 + hdr, nbytes), "set_small")
        ref = ctypes.byref(a)
        _lib.check(lib.yabt_grow_begin(gr.h, ref, s), "begin")
        _lib.check(lib.yabt_grow_init(gr.h, ref, s), "init")
        _lib.check(lib.yabt_grow_hist(gr.h, ref, 0, s), "hist")
        bufs = (ctypes.c_void_p * 2)(b0, b1)
        # rank 0 of 2; rank 1 (buffer b1) never runs, so its flag is never set
        _lib.check(lib.yabt_grow_xreduce(gr.h, bufs, 0, 2, 0, 1, s), "xreduce")
        _lib.check(lib.yabt_grow_end(gr.h, ref, s), "end")
        torch.cuda.synchronize()
        assert int(out["meta"][2].item()) & XCHG_TIMEOUT_BIT
        # the context is still usable: an ordinary tree grows cleanly afterwards
        gr2, a2, out2 = _setup(seed=1)
        gr2.grow(a2)
        torch.cuda.synchronize()
        assert int(out2["meta"][2].item()) == 0
    finally:
        torch.cuda.synchronize()
        lib.yabt_xchg_free(b0)
        lib.yabt_xchg_free(b1)


def test_single_rank_exchange_is_identity():
    from yabt_b200 import _lib
    gr_ref, a_ref, out_ref = _setup(seed=2)
    gr_ref.grow(a_ref)
    gr, a, out = _setup(seed=2)
    lib = gr.lib
    s = _lib.stream_ptr()
    (b0,), nbytes = _xchg_buffers(gr, 1)
    hdr = int(lib.yabt_xchg_header_bytes())
    try:
        _lib.check(lib.yabt_grower_set_small(gr.h, b0 + hdr, nbytes), "set_small")
        ref = ctypes.byref(a)
        bufs = (ctypes.c_void_p * 1)(b0)
        _lib.check(lib.yabt_grow_begin(gr.h, ref, s), "begin")
        _lib.check(lib.yabt_grow_init(gr.h, ref, s), "init")
        for d in range(gr.levels):
            _lib.check(lib.yabt_grow_hist(gr.h, ref, d, s), "hist")
            _lib.check(lib.yabt_grow_xreduce(gr.h, bufs, 0, 1, d, d + 1, s), "xreduce")
            _lib.check(lib.yabt_grow_split(gr.h, ref, d, s), "split")
        _lib.check(lib.yabt_grow_end(gr.h, ref, s), "end")
        torch.cuda.synchronize()
        assert int(out["meta"][2].item()) == 0
        nn = int(out_ref["meta"][0].item())
        assert int(out["meta"][0].item()) == nn > 1
        for k in ("feature", "threshold", "left", "right", "value"):      # the tree's nodes
            np.testing.assert_array_equal(out[k][:nn].cpu().numpy(), out_ref[k][:nn].cpu().numpy(), err_msg=k)
        np.testing.assert_array_equal(out["leaf_of_row"].cpu().numpy(), out_ref["leaf_of_row"].cpu().numpy())
    finally:
        torch.cuda.synchronize()
        lib.yabt_xchg_free(b0)


@pytest.mark.parametrize("kind,dtype", [(0, torch.int64), (1, torch.float64), (2, torch.int32), (3, torch.float32)])
def test_single_rank_allreduce_is_identity(kind, dtype):
    """yabt_grow_xallreduce with one rank copies src to dst (separate and aliased)."""
    from yabt_b200 import _lib
    gr, a, out = _setup(seed=3)
    lib = gr.lib
    s = _lib.stream_ptr()
    (b0,), nbytes = _xchg_buffers(gr, 1)
    try:
        bufs = (ctypes.c_void_p * 1)(b0)
        src = (torch.arange(1000, device="cuda") * 7 - 3000).to(dtype)
        dst = torch.zeros_like(src)
        _lib.check(lib.yabt_grow_xallreduce(gr.h, bufs, nbytes, 0, 1, src.data_ptr(), dst.data_ptr(), src.numel(),
                                            kind, 1, s), "xallreduce")
        x = src.clone()
        _lib.check(lib.yabt_grow_xallreduce(gr.h, bufs, nbytes, 0, 1, x.data_ptr(), x.data_ptr(), x.numel(),
                                            kind, 2, s), "xallreduce in place")
        torch.cuda.synchronize()
        assert torch.equal(dst, src) and torch.equal(x, src)
        bits = ctypes.c_uint()
        _lib.check(lib.yabt_grow_xerr(gr.h, ctypes.byref(bits)), "xerr")
        assert bits.value == 0
        # a vector larger than the buffers is refused before any launch
        big = int(nbytes // src.element_size()) + 1
        assert lib.yabt_grow_xallreduce(gr.h, bufs, nbytes, 0, 1, src.data_ptr(), dst.data_ptr(), big, kind, 3,
                                        s) != 0
    finally:
        torch.cuda.synchronize()
        lib.yabt_xchg_free(b0)


def test_allreduce_wait_times_out_and_reports():
    """A two-rank all-reduce whose second rank never arrives gives up after its
    bounded wait and sets the persistent exchange-timeout bit, which the next
    tree's meta reports too; the context stays usable."""
    from yabt_b200 import _lib
    gr, a, out = _setup(seed=4)
    lib = gr.lib
    s = _lib.stream_ptr()
    (b0, b1), nbytes = _xchg_buffers(gr, 2)
    try:
        bufs = (ctypes.c_void_p * 2)(b0, b1)
        t = torch.ones(64, dtype=torch.float64, device="cuda")
        _lib.check(lib.yabt_grow_xallreduce(gr.h, bufs, nbytes, 0, 2, t.data_ptr(), t.data_ptr(), t.numel(), 1, 1,
                                            s), "xallreduce")
        torch.cuda.synchronize()
        bits = ctypes.c_uint()
        _lib.check(lib.yabt_grow_xerr(gr.h, ctypes.byref(bits)), "xerr")
        assert bits.value & XCHG_TIMEOUT_BIT
        gr.grow(a)
        torch.cuda.synchronize()
        assert int(out["meta"][2].item()) & XCHG_TIMEOUT_BIT
    finally:
        torch.cuda.synchronize()
        lib.yabt_xchg_free(b0)
        lib.yabt_xchg_free(b1)


def test_single_rank_sliced_levels_are_identity():
    """Feature-sliced levels on one rank (the slice is every feature): the
    reduce-scatter, the split scan, the gather of the best split per node and
    the choice grow the same tree as yabt_grow_tree."""
    from yabt_b200 import _lib
    gr_ref, a_ref, out_ref = _setup(seed=6)
    gr_ref.grow(a_ref)
    gr, a, out = _setup(seed=6)
    lib = gr.lib
    s = _lib.stream_ptr()
    hist = int(lib.yabt_grow_small_count(gr.h, 62)) * 8
    rec_off = (hist + 255) // 256 * 256
    nbytes = rec_off + int(lib.yabt_grow_xgather_bytes(gr.h))
    p, hnd = ctypes.c_void_p(), (ctypes.c_char * 64)()
    _lib.check(lib.yabt_xchg_alloc(nbytes, ctypes.byref(p), hnd), "yabt_xchg_alloc")
    b0 = p.value
    hdr = int(lib.yabt_xchg_header_bytes())
    try:
        _lib.check(lib.yabt_grower_set_small(gr.h, b0 + hdr, nbytes), "set_small")
        _lib.check(lib.yabt_grower_set_feature_slice(gr.h, 0, gr.F), "slice")
        assert lib.yabt_grower_set_feature_slice(gr.h, 3, 3) != 0          # an empty slice is refused
        ref = ctypes.byref(a)
        bufs = (ctypes.c_void_p * 1)(b0)
        _lib.check(lib.yabt_grow_begin(gr.h, ref, s), "begin")
        _lib.check(lib.yabt_grow_init(gr.h, ref, s), "init")
        e = 0
        for d in range(gr.levels):
            _lib.check(lib.yabt_grow_hist(gr.h, ref, d, s), "hist")
            e += 1
            _lib.check(lib.yabt_grow_xreduce_sliced(gr.h, bufs, 0, 1, d, e, s), "xreduce_sliced")
            _lib.check(lib.yabt_grow_scan(gr.h, ref, d, s), "scan")
            e += 1
            _lib.check(lib.yabt_grow_xgather(gr.h, bufs, 0, 1, d, e, rec_off, s), "xgather")
            _lib.check(lib.yabt_grow_choose(gr.h, ref, d, s), "choose")
        _lib.check(lib.yabt_grow_end(gr.h, ref, s), "end")
        torch.cuda.synchronize()
        assert int(out["meta"][2].item()) == 0
        nn = int(out_ref["meta"][0].item())
        assert int(out["meta"][0].item()) == nn > 1
        for k in ("feature", "threshold", "left", "right", "value"):
            np.testing.assert_array_equal(out[k][:nn].cpu().numpy(), out_ref[k][:nn].cpu().numpy(), err_msg=k)
        np.testing.assert_array_equal(out["leaf_of_row"].cpu().numpy(), out_ref["leaf_of_row"].cpu().numpy())
    finally:
        torch.cuda.synchronize()
        lib.yabt_xchg_free(b0)
