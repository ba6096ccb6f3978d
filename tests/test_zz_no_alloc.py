"""The allocation-free bin fit (GPU test).

``yabt_bin_fit_static`` serves callers that cannot allocate device memory when
they fit -- for example a process whose GPU memory is reserved up front by
another framework's caching allocator, or a latency-critical loop where a
cudaMalloc (which may synchronise the device and can fail under memory
pressure) is not allowed. It keeps its scratch in a fixed array inside the
library instead of a caller workspace. This test calls it through the C ABI
twice in a row, on different data, and checks every output bit for bit
against ``yabt_bin_fit`` with a caller-allocated workspace, checks that the
call leaves torch's allocated bytes and the device's free memory unchanged,
and that a fit too large for the fixed array is refused with a clear error.

The file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _xfm(X: np.ndarray) -> torch.Tensor:
    from yabt_b200 import _lib
    Xd = torch.from_numpy(np.ascontiguousarray(X, dtype=np.float32)).cuda()
    n, F = Xd.shape
    Xfm = torch.empty(F, n, dtype=torch.float32, device="cuda")
    _lib.check(_lib.load().yabt_transpose(Xd.data_ptr(), n, F, Xfm.data_ptr(), _lib.stream_ptr()), "transpose")
    return Xfm


def _outs(F: int):
    return (torch.empty(F, dtype=torch.float32, device="cuda"),
            torch.empty(F, 255, dtype=torch.float32, device="cuda"),
            torch.empty(F, dtype=torch.int32, device="cuda"),
            torch.empty(F, dtype=torch.float32, device="cuda"))


def _fit_workspace(Xfm, n, F, nq):
    from yabt_b200 import _lib
    lib = _lib.load()
    ws = torch.empty(int(lib.yabt_bin_fit_workspace_bytes(n, F, nq)), dtype=torch.uint8, device="cuda")
    med, edges, cnt, sc = _outs(F)
    _lib.check(lib.yabt_bin_fit(Xfm.data_ptr(), n, F, None, nq, 256, ws.data_ptr(), ws.numel(), med.data_ptr(),
                                edges.data_ptr(), cnt.data_ptr(), sc.data_ptr(), _lib.stream_ptr()), "yabt_bin_fit")
    return med, edges, cnt, sc


def _fit_static(Xfm, n, F, nq):
    from yabt_b200 import _lib
    lib = _lib.load()
    med, edges, cnt, sc = _outs(F)
    rc = lib.yabt_bin_fit_static(Xfm.data_ptr(), n, F, None, nq, 256, med.data_ptr(), edges.data_ptr(),
                                 cnt.data_ptr(), sc.data_ptr(), _lib.stream_ptr())
    return rc, (med, edges, cnt, sc)


def _data(seed, n, F):
    rng = np.random.default_rng(seed)
    X = rng.normal(size=(n, F)).astype(np.float32)
    X[:, 1] = np.exp(X[:, 1])
    X[:, 2] = rng.integers(0, 5, size=n)
    X[rng.random(size=X.shape) < 0.03] = np.nan
    return X


def _free_device_bytes() -> int:
    free, _ = torch.cuda.mem_get_info()
    return int(free)


def test_static_bin_fit_matches_workspace_fit_twice():
    from yabt_b200 import _lib
    for seed, n, F in ((0, 6000, 12), (1, 3001, 7)):      # two calls in a row, different shapes
        X = _data(seed, n, F)
        Xfm = _xfm(X)
        ref = _fit_workspace(Xfm, n, F, n)
        outs = _outs(F)                                   # outputs allocated before the measured call
        torch.cuda.synchronize()
        torch_before, free_before = torch.cuda.memory_allocated(), _free_device_bytes()
        rc = _lib.load().yabt_bin_fit_static(Xfm.data_ptr(), n, F, None, n, 256, *[t.data_ptr() for t in outs],
                                             _lib.stream_ptr())
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        # the call allocates nothing: neither torch's allocator nor the device's free memory moves
        assert torch.cuda.memory_allocated() == torch_before
        assert _free_device_bytes() == free_before
        got = outs
        for a, b, name in zip(got, ref, ("medians", "edges", "edge_cnt", "scales")):
            if name == "edges":
                c = ref[2].cpu().numpy()
                for f in range(F):
                    np.testing.assert_array_equal(a[f, :c[f]].cpu().numpy(), b[f, :c[f]].cpu().numpy())
            else:
                np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy(), err_msg=name)


def test_static_bin_fit_rejects_oversized_fit():
    from yabt_b200 import _lib
    lib = _lib.load()
    cap = int(lib.yabt_bin_fit_static_capacity())
    n, F = 200_000, 200
    assert int(lib.yabt_bin_fit_workspace_bytes(n, F, n)) > cap
    Xfm = torch.zeros(F, 16, dtype=torch.float32, device="cuda")   # never read: refused before any launch
    rc, _ = _fit_static(Xfm, n, F, n)
    assert rc == 5
    assert "static buffer" in _lib.last_error()
