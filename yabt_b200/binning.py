"""Quantile binner on the device (yabt/binning.py:12-129).

``Binner.fit`` computes per-feature medians (over all rows), quantile edges
and robust scales with the CUDA kernels of ``libyabt_b200.so``; the edges are
bit-identical to the reference's numpy path. The row sample for quantile
estimation is drawn on the host with the reference's own RNG call
(``np.random.default_rng(0).choice``, yabt/binning.py:36-38) -- an index
draw, not compute.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib

MAX_BINS = 256
QUANTILE_SAMPLE = 200_000


def _device(device) -> torch.device:
    d = torch.device(device if device is not None else "cuda")
    if d.type != "cuda":
        raise ValueError("yabt_b200 runs on CUDA devices only")
    return d


def to_device_f32(X, device) -> torch.Tensor:
    """(n, F) float32 contiguous tensor on ``device`` (host arrays are copied
    through pinned memory)."""
    if isinstance(X, torch.Tensor):
        return X.to(device=device, dtype=torch.float32).contiguous()
    a = np.ascontiguousarray(np.asarray(X, dtype=np.float32))
    t = torch.from_numpy(a)
    if t.numel() > (1 << 20):
        t = t.pin_memory()
    return t.to(device, non_blocking=True)


def to_feature_major(X, device, chunk_bytes: int = 64 << 20) -> torch.Tensor:
    """(F, n) float32 device matrix of a row-major (n, F) input. Host input is
    copied in chunks through two device staging buffers on a copy stream, each
    chunk transposed while the next one is in flight, so no (n, F) device
    copy of the whole matrix is made."""
    lib = _lib.load()
    dev = _device(device)
    if isinstance(X, torch.Tensor) and X.device.type == "cuda":
        Xd = X.to(device=dev, dtype=torch.float32).contiguous()
        n, F = Xd.shape
        Xfm = torch.empty(F, n, dtype=torch.float32, device=dev)
        _lib.check(lib.yabt_transpose(Xd.data_ptr(), n, F, Xfm.data_ptr(), _lib.stream_ptr()), "yabt_transpose")
        return Xfm
    Xh = X if isinstance(X, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(np.asarray(X, dtype=np.float32)))
    Xh = Xh.to(torch.float32).contiguous()
    n, F = Xh.shape
    Xfm = torch.empty(F, n, dtype=torch.float32, device=dev)
    if n == 0:
        return Xfm
    rows = max(1, min(n, chunk_bytes // (4 * F)))
    main = torch.cuda.current_stream(dev)
    copy = torch.cuda.Stream(dev)
    stage = [torch.empty(rows, F, dtype=torch.float32, device=dev) for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    for i, r0 in enumerate(range(0, n, rows)):
        m = min(rows, n - r0)
        k = i & 1
        with torch.cuda.stream(copy):
            if i >= 2:
                copy.wait_event(freed[k])        # the transpose of chunk i-2 is done with this buffer
            stage[k][:m].copy_(Xh[r0:r0 + m], non_blocking=True)
            copied[k].record(copy)
        main.wait_event(copied[k])
        _lib.check(lib.yabt_transpose_block(stage[k].data_ptr(), m, F, Xfm.data_ptr() + 4 * r0, n,
                                            _lib.stream_ptr()), "yabt_transpose_block")
        freed[k].record(main)
    for t in stage:
        t.record_stream(copy)
    return Xfm


class Binner:
    """Quantile-bins float features into uint8 codes; same semantics as the
    reference: bin(x) = #{e_j < x}, so bin(x) <= b  <=>  x <= edges[b]."""

    def __init__(self, max_bins: int = MAX_BINS):
        if not 2 <= max_bins <= 256:
            raise ValueError("max_bins must be in [2, 256]")
        self.max_bins = max_bins
        self.edges_: list[torch.Tensor] | None = None
        self.medians_: np.ndarray | None = None
        self.scales_: torch.Tensor | None = None
        self._dev = None       # device copies: medians, edges [F][255], edge counts, scales

    # ------------------------------------------------------------------ fit
    def fit_device(self, Xfm: torch.Tensor, n: int) -> "Binner":
        """Fit from a feature-major (F, n) float32 device tensor (NaN allowed)."""
        lib = _lib.load()
        F = Xfm.shape[0]
        dev = Xfm.device
        s = _lib.stream_ptr()
        if n > QUANTILE_SAMPLE:
            idx_np = np.random.default_rng(0).choice(n, QUANTILE_SAMPLE, replace=False)
            idx = torch.from_numpy(idx_np.astype(np.int32)).to(dev)
            nq = QUANTILE_SAMPLE
        else:
            idx, nq = None, n
        ws = torch.empty(int(lib.yabt_bin_fit_workspace_bytes(n, F, nq)), dtype=torch.uint8, device=dev)
        med = torch.empty(F, dtype=torch.float32, device=dev)
        edges = torch.empty(F, 255, dtype=torch.float32, device=dev)
        ecnt = torch.empty(F, dtype=torch.int32, device=dev)
        scales = torch.empty(F, dtype=torch.float32, device=dev)
        _lib.check(lib.yabt_bin_fit(Xfm.data_ptr(), n, F, idx.data_ptr() if idx is not None else None, nq,
                                    self.max_bins, ws.data_ptr(), ws.numel(), med.data_ptr(),
                                    edges.data_ptr(), ecnt.data_ptr(), scales.data_ptr(), s), "yabt_bin_fit")
        return self._set_state(med, edges, ecnt, scales)

    def fit_device_sharded(self, Xfm: torch.Tensor, n: int, comm) -> "Binner":
        """Fit over the rows of every rank of ``comm`` (a ``ShardComm``): this
        rank holds the feature-major (F, n) block of its rows. The result equals
        a fit on the concatenation of every rank's rows."""
        from .distributed import fit_binner
        return self._set_state(*fit_binner(Xfm, n, self.max_bins, comm))

    def _set_state(self, med, edges, ecnt, scales) -> "Binner":
        F = med.shape[0]
        self._dev = (med, edges, ecnt, scales)
        # host views of the fitted state (the reference's attribute layout)
        med_h = med.cpu().numpy()
        cnt_h = ecnt.cpu().numpy()
        e_h = edges.cpu()
        self.medians_ = med_h
        self.edges_ = [e_h[f, : int(cnt_h[f])].clone() for f in range(F)]
        self.scales_ = scales.cpu()
        return self

    def fit(self, X) -> "Binner":
        """yabt/binning.py:29-69 (numpy semantics, computed on the device)."""
        dev = _device(X.device if isinstance(X, torch.Tensor) else None)
        Xd = to_device_f32(X, dev)
        n, F = Xd.shape
        Xfm = torch.empty(F, n, dtype=torch.float32, device=dev)
        _lib.check(_lib.load().yabt_transpose(Xd.data_ptr(), n, F, Xfm.data_ptr(), _lib.stream_ptr()),
                   "yabt_transpose")
        return self.fit_device(Xfm, n)

    # ------------------------------------------------------------------ transform
    def transform_device(self, Xfm: torch.Tensor, n: int, plain: bool = False, feature_major: bool = False):
        """Bins of a feature-major (F, n) device matrix. Imputes NaN in place.
        Returns (tiled bin matrix, plain (n, F) uint8 or None), plus the
        feature-major (F, n) uint8 bins when ``feature_major``."""
        assert self._dev is not None, "Binner not fitted"
        lib = _lib.load()
        F = Xfm.shape[0]
        med, edges, ecnt, _ = self._dev
        tiled = torch.empty(int(lib.yabt_bin_matrix_bytes(n, F)), dtype=torch.uint8, device=Xfm.device)
        pl = torch.empty(n, F, dtype=torch.uint8, device=Xfm.device) if plain else None
        fm = torch.empty(F, n, dtype=torch.uint8, device=Xfm.device) if feature_major else None
        _lib.check(lib.yabt_bin_transform(Xfm.data_ptr(), n, F, med.data_ptr(), edges.data_ptr(),
                                          ecnt.data_ptr(), tiled.data_ptr(),
                                          pl.data_ptr() if pl is not None else None,
                                          fm.data_ptr() if fm is not None else None, _lib.stream_ptr()),
                   "yabt_bin_transform")
        if feature_major:
            return tiled, pl, fm
        return tiled, pl

    def transform(self, X, device: str = "cuda") -> torch.Tensor:
        """(n, F) uint8 bin codes on ``device`` (yabt/binning.py:97-112)."""
        dev = _device(device)
        Xd = to_device_f32(X, dev)
        n, F = Xd.shape
        Xfm = torch.empty(F, n, dtype=torch.float32, device=dev)
        _lib.check(_lib.load().yabt_transpose(Xd.data_ptr(), n, F, Xfm.data_ptr(), _lib.stream_ptr()),
                   "yabt_transpose")
        _, pl = self.transform_device(Xfm, n, plain=True)
        return pl

    def impute_device(self, X: torch.Tensor) -> torch.Tensor:
        """NaN -> median on a row-major (n, F) device tensor (in place)."""
        n, F = X.shape
        _lib.check(_lib.load().yabt_impute_rows(X.data_ptr(), n, F, self._dev[0].data_ptr(),
                                                _lib.stream_ptr()), "yabt_impute_rows")
        return X

    def impute(self, X) -> np.ndarray:
        """Median-imputed raw matrix (yabt/binning.py:121-124), imputed on the device."""
        Xd = to_device_f32(X, self._dev[0].device).clone()
        return self.impute_device(Xd).cpu().numpy()

    def edge_value(self, feature: int, bin_idx: int) -> float:
        """Raw threshold equivalent to ``bin <= bin_idx`` (yabt/binning.py:126-129)."""
        e = self.edges_[feature]
        return float(e[min(bin_idx, len(e) - 1)])

    def __getstate__(self):
        d = dict(self.__dict__)
        d["_dev"] = None if self._dev is None else tuple(t.cpu() for t in self._dev)
        return d

    def __setstate__(self, d):
        self.__dict__.update(d)
        if self._dev is not None and torch.cuda.is_available():
            self._dev = tuple(t.cuda() for t in self._dev)
