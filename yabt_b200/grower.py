"""Host side of the level-wise grower: workspace management and the drop-in
``grow_tree_levelwise`` (yabt/tree.py:362-625).

A ``Grower`` owns one device workspace (a torch uint8 tensor) sized by the C
ABI for a problem shape, and grows trees with no host synchronisation: the
tree arrays are written into caller-provided device tensors. The drop-in
function ``grow_tree_levelwise`` returns a ``Tree`` sized to its node count
(one small device-to-host read, as the reference's per-level ``.tolist()``).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .tree import Tree, TreeParams


def _i32(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.int32).contiguous()


class EdgePack:
    """Per-feature interior edges packed for the device (concatenated values,
    offsets, counts) plus scales."""

    def __init__(self, edges: list[torch.Tensor], scales: torch.Tensor, device):
        cnt = torch.tensor([int(len(e)) for e in edges], dtype=torch.int32)
        off = torch.zeros_like(cnt)
        if cnt.numel() > 1:
            off[1:] = torch.cumsum(cnt, 0)[:-1].to(torch.int32)
        self.values = torch.cat([torch.as_tensor(e, dtype=torch.float32).reshape(-1).cpu()
                                 for e in edges]).to(device)
        self.off = off.to(device)
        self.cnt = cnt.to(device)
        self.scales = torch.as_tensor(scales, dtype=torch.float32).to(device).contiguous()
        self.F = len(edges)


class Grower:
    """One grower context (C ABI ``yabt_grower``) bound to a workspace tensor."""

    def __init__(self, n: int, F: int, max_leaves: int, max_depth: int, general: bool,
                 device: torch.device | str = "cuda"):
        self.lib = _lib.load()
        self.device = torch.device(device)
        self.n, self.F, self.general = int(n), int(F), bool(general)
        self.max_leaves, self.max_depth = int(max_leaves), int(max_depth)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(self.lib.yabt_grower_create(self.n, self.F, self.max_leaves, self.max_depth,
                                                   1 if general else 0, ctypes.byref(h)),
                       "yabt_grower_create")
            self.h = h
            nbytes = int(self.lib.yabt_grower_workspace_bytes(h))
            self.ws = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
            _lib.check(self.lib.yabt_grower_bind(h, self.ws.data_ptr(), nbytes, _lib.stream_ptr()),
                       "yabt_grower_bind")
        self.max_nodes = int(self.lib.yabt_grower_max_nodes(h))
        self.levels = int(self.lib.yabt_grower_levels(h))

    def __del__(self):
        try:
            if getattr(self, "h", None) is not None:
                self.lib.yabt_grower_destroy(self.h)
        except Exception:
            pass

    def new_outputs(self) -> dict:
        dev, m = self.device, self.max_nodes
        return dict(
            feature=torch.empty(m, dtype=torch.int64, device=dev),
            threshold=torch.empty(m, dtype=torch.float32, device=dev),
            left=torch.empty(m, dtype=torch.int64, device=dev),
            right=torch.empty(m, dtype=torch.int64, device=dev),
            value=torch.empty(m, dtype=torch.float32, device=dev),
            gate_scale=torch.empty(m, dtype=torch.float32, device=dev),
            leaf_of_row=torch.empty(self.n, dtype=torch.int32, device=dev),
            meta=torch.zeros(4, dtype=torch.int32, device=dev),
        )

    def args(self, bins: torch.Tensor, grad: torch.Tensor, hess: torch.Tensor | None,
             edges: EdgePack, params: TreeParams, out: dict,
             feature_mask: torch.Tensor | None = None,
             interaction: torch.Tensor | None = None, interaction_boost: float = 0.5,
             bins_fm: torch.Tensor | None = None, root_rows: torch.Tensor | None = None) -> _lib.TreeArgs:
        """``bins_fm``: optional feature-major (F, n) copy of the bins, read by
        the row partition. ``root_rows``: optional int32 device tensor of the
        rows to grow the tree on (row subsampling)."""
        a = _lib.TreeArgs()
        a.bins = bins.data_ptr()
        a.bins_fm = bins_fm.data_ptr() if bins_fm is not None else None
        a.root_rows = root_rows.data_ptr() if (root_rows is not None and root_rows.numel()) else None
        a.n_root = int(root_rows.numel()) if root_rows is not None else 0
        if root_rows is not None and root_rows.numel() == 0:
            a.root_rows = self._empty_root().data_ptr()
        a.grad = grad.data_ptr()
        a.hess = hess.data_ptr() if (hess is not None and self.general) else None
        a.edges, a.edge_off, a.edge_cnt = edges.values.data_ptr(), edges.off.data_ptr(), edges.cnt.data_ptr()
        a.scales = edges.scales.data_ptr()
        a.feature_mask = feature_mask.data_ptr() if feature_mask is not None else None
        a.interaction = interaction.data_ptr() if interaction is not None else None
        a.reg_lambda = float(params.reg_lambda)
        a.gamma = float(params.gamma)
        a.min_child_weight = float(params.min_child_weight)
        a.learning_rate = float(params.learning_rate)
        a.interaction_boost = float(interaction_boost)
        a.min_samples_leaf = int(params.min_samples_leaf)
        for k in ("feature", "threshold", "left", "right", "value", "gate_scale", "leaf_of_row", "meta"):
            setattr(a, k, out[k].data_ptr())
        # the struct holds raw device addresses: keep every tensor behind them
        # alive for as long as the struct is (a caller may pass temporaries)
        a._keep = (bins, grad, hess, edges, out, feature_mask, interaction, bins_fm, root_rows)
        return a

    def grow(self, a: _lib.TreeArgs, stream=None, bestfirst: bool = False, f64: bool = False) -> None:
        """One tree: level-wise (yabt/tree.py:362-625), or best-first: the heap
        grower of yabt/tree.py:206-360, or with ``f64`` the C / Numba grower's
        arithmetic (yabt/_cgrow/grow.c:243-427)."""
        if bestfirst:
            _lib.check(self.lib.yabt_grower_set_bestfirst_f64(self.h, 1 if f64 else 0),
                       "yabt_grower_set_bestfirst_f64")
            _lib.check(self.lib.yabt_grow_tree_bestfirst(self.h, ctypes.byref(a), _lib.stream_ptr(stream)),
                       "yabt_grow_tree_bestfirst")
        else:
            _lib.check(self.lib.yabt_grow_tree(self.h, ctypes.byref(a), _lib.stream_ptr(stream)),
                       "yabt_grow_tree")

    def _empty_root(self) -> torch.Tensor:
        if getattr(self, "_empty", None) is None:
            self._empty = torch.zeros(1, dtype=torch.int32, device=self.device)
        return self._empty

    def set_level_wait(self, wait: bool) -> None:
        """Whether growing a tree may wait on the device to stop queuing levels
        once the tree is complete (off: every level is queued, no host waits)."""
        _lib.check(self.lib.yabt_grower_set_level_wait(self.h, 1 if wait else 0), "yabt_grower_set_level_wait")
        self.level_wait = bool(wait)

    def set_level_loop(self, on: bool) -> None:
        """Device-side level loop (a CUDA graph with a WHILE node) for the
        levels past level_loop_start(); on by default."""
        _lib.check(self.lib.yabt_grower_set_level_loop(self.h, 1 if on else 0), "yabt_grower_set_level_loop")

    def level_loop_start(self) -> int:
        """First level grown inside the device-side level loop, or -1 when the
        loop is off or would not pay for this grower."""
        return int(self.lib.yabt_grower_level_loop_start(self.h))

    def set_timing(self, max_launches: int) -> None:
        """Record CUDA events around up to max_launches histogram launches."""
        _lib.check(self.lib.yabt_grower_set_timing(self.h, int(max_launches)), "yabt_grower_set_timing")

    def hist_times(self, cap: int = 4096) -> list[float]:
        buf = (ctypes.c_float * cap)()
        cnt = ctypes.c_int()
        _lib.check(self.lib.yabt_grower_hist_times(self.h, buf, cap, ctypes.byref(cnt)), "yabt_grower_hist_times")
        return [buf[i] for i in range(min(cnt.value, cap))]

    def acc_reset(self) -> None:
        _lib.check(self.lib.yabt_grower_acc_reset(self.h, _lib.stream_ptr()), "yabt_grower_acc_reset")

    def acc_read(self) -> tuple[int, int, int]:
        buf = (ctypes.c_longlong * 3)()
        _lib.check(self.lib.yabt_grower_acc_read(self.h, buf), "yabt_grower_acc_read")
        return int(buf[0]), int(buf[1]), int(buf[2])

    def root_counts(self) -> torch.Tensor:
        """(F, 256) int64 per-bin row counts of this grower's rows, recorded by
        the last root histogram over all rows (the root-count cache must be on)."""
        out = torch.empty(self.F, 256, dtype=torch.int64, device=self.device)
        _lib.check(self.lib.yabt_grower_root_counts(self.h, out.data_ptr(), _lib.stream_ptr()),
                   "yabt_grower_root_counts")
        return out

    def hist_rows(self) -> list[int]:
        buf = (ctypes.c_longlong * 64)()
        _lib.check(self.lib.yabt_grower_hist_rows(self.h, buf, 64), "yabt_grower_hist_rows")
        return [int(buf[i]) for i in range(64)]

    def leaf_rows(self) -> dict:
        ptrs = [ctypes.c_void_p() for _ in range(6)]
        _lib.check(self.lib.yabt_grow_leaf_rows(self.h, *[ctypes.byref(p) for p in ptrs]),
                   "yabt_grow_leaf_rows")
        return dict(zip(("src", "begin", "count", "fin", "list0", "list1"), [p.value for p in ptrs]))


def bin_matrix_bytes(n: int, F: int) -> int:
    return int(_lib.load().yabt_bin_matrix_bytes(int(n), int(F)))


def pack_bins(binned: torch.Tensor) -> torch.Tensor:
    """Plain row-major (n, F) uint8 -> tiled layout (device)."""
    binned = binned.contiguous()
    n, F = binned.shape
    out = torch.empty(bin_matrix_bytes(n, F), dtype=torch.uint8, device=binned.device)
    _lib.check(_lib.load().yabt_pack_bins(binned.data_ptr(), n, F, out.data_ptr(), _lib.stream_ptr()),
               "yabt_pack_bins")
    return out


def trim_tree(out: dict, n_nodes: int, depth: int) -> Tree:
    k = n_nodes
    return Tree(feature=out["feature"][:k], threshold=out["threshold"][:k], left=out["left"][:k],
                right=out["right"][:k], value=out["value"][:k], depth=depth,
                gate_scale=out["gate_scale"][:k])


_GROWERS: dict = {}


def _grow_one(binned, grad, hess, binner, params, feature_mask, interaction_matrix, interaction_boost,
              return_leaf, bestfirst, name, f64=False):
    if binned.device.type != "cuda":
        raise ValueError(f"{name} (yabt_b200) needs CUDA tensors")
    n, F = binned.shape
    dev = binned.device
    general = not bool(torch.all(hess == 1.0))
    key = (n, F, params.max_leaves, params.max_depth, general, dev.index)
    gr = _GROWERS.get(key)
    if gr is None:
        gr = _GROWERS[key] = Grower(n, F, params.max_leaves, params.max_depth, general, dev)
    tiled = pack_bins(binned)
    ep = EdgePack(list(binner.edges_), binner.scales_, dev)
    out = gr.new_outputs()
    fm = feature_mask.to(device=dev, dtype=torch.uint8).contiguous() if feature_mask is not None else None
    im = interaction_matrix.to(device=dev, dtype=torch.float32).contiguous() if interaction_matrix is not None else None
    g = grad.to(torch.float32).contiguous()
    h = hess.to(torch.float32).contiguous()
    a = gr.args(tiled, g, h, ep, params, out, fm, im, interaction_boost)
    gr.grow(a, bestfirst=bestfirst, f64=f64)
    meta = out["meta"].tolist()
    if meta[2] != 0:
        raise _lib.YabtError(f"device error bits 0x{meta[2]:x} while growing a tree")
    tree = trim_tree(out, meta[0], meta[1])
    if return_leaf:
        return tree, out["leaf_of_row"].to(torch.int64)
    return tree


def grow_tree_levelwise(binned: torch.Tensor, grad: torch.Tensor, hess: torch.Tensor, binner,
                        params: TreeParams, feature_mask: torch.Tensor | None = None,
                        interaction_matrix: torch.Tensor | None = None,
                        interaction_boost: float = 0.5, *, return_leaf: bool = False):
    """Drop-in for yabt/tree.py:362-625 on a CUDA device.

    ``binned`` is the plain (n, F) uint8 bin matrix (it is packed into the
    tiled layout on the device). The hessian channel is dropped when every
    hessian equals 1 (squared loss), which the reference's float32 sums of
    ones reproduce exactly. Returns the ``Tree`` (and the leaf of every row
    when ``return_leaf``)."""
    return _grow_one(binned, grad, hess, binner, params, feature_mask, interaction_matrix, interaction_boost,
                     return_leaf, False, "grow_tree_levelwise")


def grow_tree(binned: torch.Tensor, grad: torch.Tensor, hess: torch.Tensor, binner,
              params: TreeParams, feature_mask: torch.Tensor | None = None,
              interaction_matrix: torch.Tensor | None = None,
              interaction_boost: float = 0.5, *, return_leaf: bool = False):
    """Drop-in for the best-first (heap) grower yabt/tree.py:206-360 on a CUDA
    device, axis splits (kernel splits are not part of this path): the leaf
    with the largest split gain is split first (ties: the earlier-pushed,
    i.e. lower node id), up to ``max_leaves`` leaves and ``max_depth``.
    Arguments and results as :func:`grow_tree_levelwise`."""
    return _grow_one(binned, grad, hess, binner, params, feature_mask, interaction_matrix, interaction_boost,
                     return_leaf, True, "grow_tree")


def grow_tree_c(binned: torch.Tensor, grad: torch.Tensor, hess: torch.Tensor, binner,
                params: TreeParams, feature_mask: torch.Tensor | None = None,
                interaction_matrix: torch.Tensor | None = None,
                interaction_boost: float = 0.5, *, return_leaf: bool = False):
    """Drop-in for the reference's OpenMP C grower ``grow_tree_c``
    (yabt/grow_c.py:336-456, kernel yabt/_cgrow/grow.c:243-427; the Numba
    grower computes the same trees) on a CUDA device: best-first growth with
    the C grower's float64 split scan and leaf values and its tie order.
    Histograms are exact sums, so trees equal the C grower's wherever its
    float32 histogram bins are exact (and agree to rounding elsewhere)."""
    return _grow_one(binned, grad, hess, binner, params, feature_mask, interaction_matrix, interaction_boost,
                     return_leaf, True, "grow_tree_c", f64=True)
