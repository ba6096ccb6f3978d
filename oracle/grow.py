"""Oracle restatement of the level-wise tree grower (test infrastructure only).

Restates ``grow_tree_levelwise`` (yabt/tree.py:362-625) on its torch-scatter
branch (yabt/tree.py:442-452), which is the CPU execution of the exact math
that the reference's CUDA histogram kernel (yabt/_cuda/hist.cu:27-133)
replaces. Float arithmetic follows what torch does on the CPU for the same
expressions, which the golden vectors pin:

* histogram bins: float32 additions in row order (torch CPU ``scatter_add_``
  is sequential; ``np.add.at`` performs the same sequence of float32 adds);
* ``cumsum`` over bins: accumulated in float64, each prefix rounded to float32
  (torch CPU accumulates float cumsum in double);
* split gain, validity, boost and leaf values: float32 element-wise operations
  in the reference's operand order, Python scalars rounded to float32;
* argmax: first maximum in flat (feature * 256 + bin) order.

Two places where the reference's order is implementation-defined are fixed
here and documented as "parity unpinned" where they matter:
* the ``topk`` leaf-budget cut (yabt/tree.py:527-530): kept splits are the
  highest gains, ties broken by the lower active position;
* ``Gtot/Htot/Ctot`` (yabt/tree.py:533-534) are float32 sums whose torch
  reduction order is ISA specific; they are summed in float64 here and rounded.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

B = 256
LEAF = -1
f32 = np.float32


@dataclass
class TreeParams:
    """yabt/tree.py:22-36 (axis-split fields)."""
    max_leaves: int = 31
    max_depth: int = 64
    reg_lambda: float = 1.0
    gamma: float = 0.0
    min_child_weight: float = 1e-3
    min_samples_leaf: int = 20
    learning_rate: float = 0.1


@dataclass
class OTree:
    """Flat tree arrays, the layout of ``Tree`` (yabt/tree.py:39-76)."""
    feature: np.ndarray
    threshold: np.ndarray
    left: np.ndarray
    right: np.ndarray
    value: np.ndarray
    depth: int
    gate_scale: np.ndarray
    leaf_net_feats: np.ndarray | None = None
    leaf_net_linear: np.ndarray | None = None
    leaf_net_lo: np.ndarray | None = None
    leaf_net_hi: np.ndarray | None = None
    # split bins (not part of Tree, kept for parity checks)
    split_bin: np.ndarray | None = None
    extras: dict = field(default_factory=dict)

    def apply(self, X: np.ndarray) -> np.ndarray:
        """Leaf index per row of raw X (yabt/tree.py:82-116)."""
        n = X.shape[0]
        node = np.zeros(n, dtype=np.int64)
        is_leaf = self.feature == LEAF
        for _ in range(self.depth):
            f = np.maximum(self.feature[node], 0)
            x = X[np.arange(n), f]
            go_left = x <= self.threshold[node]
            nxt = np.where(go_left, self.left[node], self.right[node])
            node = np.where(is_leaf[node], node, nxt)
        return node

    def apply_bins(self, binned: np.ndarray) -> np.ndarray:
        """Leaf index per row of the bin matrix: bin <= split bin goes left."""
        n = binned.shape[0]
        node = np.zeros(n, dtype=np.int64)
        is_leaf = self.feature == LEAF
        for _ in range(self.depth):
            f = np.maximum(self.feature[node], 0)
            go_left = binned[np.arange(n), f].astype(np.int64) <= self.split_bin[node]
            nxt = np.where(go_left, self.left[node], self.right[node])
            node = np.where(is_leaf[node], node, nxt)
        return node

    def net_contribution(self, X: np.ndarray, node: np.ndarray) -> np.ndarray:
        """yabt/tree.py:118-128 (linear leaves)."""
        if self.leaf_net_feats is None:
            return np.zeros(X.shape[0], dtype=np.float32)
        Xs = X[:, self.leaf_net_feats]
        Xs = np.minimum(np.maximum(Xs, self.leaf_net_lo[node]), self.leaf_net_hi[node])
        return (self.leaf_net_linear[node] * Xs).sum(axis=1, dtype=np.float32)

    def predict(self, X: np.ndarray) -> np.ndarray:
        """yabt/tree.py:130-135."""
        node = self.apply(X)
        out = self.value[node]
        if self.leaf_net_feats is not None:
            out = out + self.net_contribution(X, node)
        return out

    def path_feature_pairs(self) -> list[tuple[int, int]]:
        """(ancestor feature, descendant feature) pairs, yabt/tree.py:186-203."""
        pairs: list[tuple[int, int]] = []
        stack: list[tuple[int, tuple[int, ...]]] = [(0, ())]
        while stack:
            nid, anc = stack.pop()
            f = int(self.feature[nid])
            if f == LEAF:
                continue
            pairs.extend((a, f) for a in anc)
            anc = anc + (f,)
            stack.append((int(self.left[nid]), anc))
            stack.append((int(self.right[nid]), anc))
        return pairs


def feature_major(a: np.ndarray) -> np.ndarray:
    """(F, n) contiguous copy of an (n, F) matrix, transposed in row blocks
    (a whole-matrix transpose copy is cache-unfriendly at millions of rows)."""
    n, F = a.shape
    out = np.empty((F, n), dtype=a.dtype)
    for r0 in range(0, n, 1 << 15):
        out[:, r0:r0 + (1 << 15)] = a[r0:r0 + (1 << 15)].T
    return out


def scatter_hist(binned: np.ndarray, slot: np.ndarray, g: np.ndarray, h: np.ndarray,
                 w: np.ndarray | None, K: int) -> np.ndarray:
    """(3, K, F, 256) float32 histogram, sequential float32 adds in row order
    (yabt/tree.py:442-452; yabt/_cuda/hist.cu:27-49 computes the same sums with
    atomics)."""
    return scatter_hist_fm(feature_major(binned), slot, g, h, w, K)


def scatter_hist_fm(binned_fm: np.ndarray, slot: np.ndarray, g: np.ndarray, h: np.ndarray,
                    w: np.ndarray | None, K: int) -> np.ndarray:
    """``scatter_hist`` of a feature-major (F, n) bin matrix.

    Every bin belongs to one feature, so adding feature by feature performs the
    same sequence of float32 additions into each bin as one pass in row-major
    element order (``np.add.at`` is sequential). Channels whose values are all
    one (the row count, a unit hessian) are integer counts below 2^24, which a
    sequential float32 sum represents exactly, so they are counted directly."""
    F, n = binned_fm.shape
    out = np.zeros((3, K, F, B), dtype=np.float32)
    if n == 0:
        return out
    base = slot.astype(np.int64) * B
    g32 = g.astype(np.float32)
    h32 = h.astype(np.float32)
    w32 = None if w is None else w.astype(np.float32)
    unit_h = bool(np.all(h32 == 1.0))
    unit_w = w32 is None or bool(np.all(w32 == 1.0))
    for f in range(F):
        idx = base + binned_fm[f]
        cnt = np.bincount(idx, minlength=K * B).astype(np.float32).reshape(K, B)
        acc = np.zeros(K * B, np.float32)
        np.add.at(acc, idx, g32)
        out[0, :, f] = acc.reshape(K, B)
        if unit_h:
            out[1, :, f] = cnt
        else:
            acc = np.zeros(K * B, np.float32)
            np.add.at(acc, idx, h32)
            out[1, :, f] = acc.reshape(K, B)
        if unit_w:
            out[2, :, f] = cnt
        else:
            acc = np.zeros(K * B, np.float32)
            np.add.at(acc, idx, w32)
            out[2, :, f] = acc.reshape(K, B)
    return out


def split_scan(hist: np.ndarray, lam: float, gamma: float, mcw: float, msl: int,
               feature_mask: np.ndarray | None = None,
               boost: np.ndarray | None = None):
    """Per-node best split over (feature, bin), yabt/tree.py:504-525.

    hist: (3, M, F, 256) float32. boost: (M, F) float32 selection multiplier
    or None. Returns (best_idx (M,), best_gain (M,) float32, cum (3,M,F,256))."""
    cum = np.cumsum(hist.astype(np.float64), axis=-1).astype(np.float32)
    GL, HL, CL = cum[0], cum[1], cum[2]
    G, H, C = GL[..., -1:], HL[..., -1:], CL[..., -1:]
    GR, HR, CR = G - GL, H - HL, C - CL
    lam32 = f32(lam)
    t = GL * GL / (HL + lam32) + GR * GR / (HR + lam32) - G * G / (H + lam32)
    gain = f32(0.5) * t - f32(gamma)
    mcw32 = f32(mcw)
    valid = (CL >= msl) & (CR >= msl) & (HL >= mcw32) & (HR >= mcw32)
    valid[..., -1] = False
    if feature_mask is not None:
        valid &= feature_mask.reshape(1, -1, 1)
    gain = np.where(valid, gain, f32(-np.inf)).astype(np.float32)
    M = gain.shape[0]
    flat = gain.reshape(M, -1)
    if boost is None:
        idx = flat.argmax(axis=1)
    else:
        sel = (gain * boost[:, :, None]).reshape(M, -1)
        idx = sel.argmax(axis=1)
    best_gain = flat[np.arange(M), idx]
    return idx, best_gain, cum


def budget_keep(best_gain: np.ndarray, remaining: int) -> np.ndarray:
    """Leaf budget, yabt/tree.py:526-530: keep the ``remaining`` highest gains
    among positive ones; ties go to the lower active position (the reference's
    ``topk`` tie order is implementation defined)."""
    do = best_gain > 0
    if int(do.sum()) <= remaining:
        return do
    pos = np.arange(best_gain.shape[0])
    cand = np.where(do, best_gain, -np.inf)
    order = np.lexsort((pos, -cand.astype(np.float64)))
    keep = np.zeros_like(do)
    keep[order[:remaining]] = True
    return keep


def grow_levelwise(binned: np.ndarray, grad: np.ndarray, hess: np.ndarray,
                   edges: list[np.ndarray], scales: np.ndarray, params: TreeParams,
                   feature_mask: np.ndarray | None = None,
                   interaction_matrix: np.ndarray | None = None,
                   interaction_boost: float = 0.5):
    """Restates yabt/tree.py:362-625. Returns (OTree, node_of_row, trace) where
    trace records per level the histograms and chosen splits for parity tests."""
    n, F = binned.shape
    lam, gamma = params.reg_lambda, params.gamma
    mcw, msl, lr = params.min_child_weight, params.min_samples_leaf, params.learning_rate
    scales_c = np.maximum(scales.astype(np.float32), f32(1e-12))
    imat = None if interaction_matrix is None else interaction_matrix.astype(np.float32)

    feature, threshold, left, right, value, node_depth, gate, sbin = [], [], [], [], [], [], [], []

    def add_leaf(v: float, d: int) -> int:
        feature.append(LEAF); threshold.append(0.0); left.append(-1); right.append(-1)
        value.append(v); node_depth.append(d); gate.append(1.0); sbin.append(-1)
        return len(feature) - 1

    # yabt/tree.py:473 (Python float arithmetic on the float32 sums)
    gsum = float(np.sum(grad.astype(np.float64)).astype(np.float32))
    hsum = float(np.sum(hess.astype(np.float64)).astype(np.float32))
    add_leaf(-lr * gsum / (hsum + lam), 0)
    node_of_row = np.zeros(n, dtype=np.int64)
    active = [0]
    binned_fm = feature_major(binned)
    hist = scatter_hist_fm(binned_fm, np.zeros(n, np.int64), grad, hess, None, 1)
    pathmax = np.zeros((1, F), np.float32) if imat is not None else None
    remaining = params.max_leaves - 1
    depth = 0
    trace = []
    while active and depth < params.max_depth and remaining > 0:
        M = len(active)
        if depth == 0:
            pr = np.zeros(n, np.int64)
            row_active = np.ones(n, bool)
        else:
            node_to_pos = np.full(len(feature), -1, np.int64)
            node_to_pos[np.array(active)] = np.arange(M)
            pos = node_to_pos[node_of_row]
            row_active = pos >= 0
            pr = np.maximum(pos, 0)
        boost = None
        if imat is not None:
            boost = (f32(1.0) + f32(interaction_boost) * pathmax).astype(np.float32)
        idx, best_gain, cum = split_scan(hist, lam, gamma, mcw, msl, feature_mask, boost)
        f, b = idx // B, idx % B
        do = budget_keep(best_gain, remaining)
        Gtot = hist[0, :, 0, :].astype(np.float64).sum(-1).astype(np.float32)
        Htot = hist[1, :, 0, :].astype(np.float64).sum(-1).astype(np.float32)
        Ctot = hist[2, :, 0, :].astype(np.float64).sum(-1).astype(np.float32)
        mi = np.arange(M)
        gL, hL, cL = cum[0][mi, f, b], cum[1][mi, f, b], cum[2][mi, f, b]
        vL = (f32(-lr) * gL) / (hL + f32(lam))
        vR = (f32(-lr) * (Gtot - gL)) / ((Htot - hL) + f32(lam))
        small_left = cL <= (Ctot - cL)
        trace.append(dict(hist=hist.copy(), f=f.copy(), b=b.copy(), gain=best_gain.copy(),
                          do=do.copy(), active=list(active)))

        child_l = [-1] * M
        child_r = [-1] * M
        nxt: list[int] = []
        split_pos: list[int] = []
        d1 = depth + 1
        for m in range(M):
            if not do[m]:
                continue
            split_pos.append(m)
            gid, fm, bm = active[m], int(f[m]), int(b[m])
            feature[gid] = fm
            e = edges[fm]
            threshold[gid] = float(e[min(bm, len(e) - 1)])
            gate[gid] = float(scales_c[fm])
            sbin[gid] = bm
            value[gid] = 0.0
            nl, nr = add_leaf(float(vL[m]), d1), add_leaf(float(vR[m]), d1)
            left[gid], right[gid] = nl, nr
            child_l[m], child_r[m] = nl, nr
            nxt += (nl, nr)
        remaining -= len(nxt) // 2

        # yabt/tree.py:562-570 repartition
        cl = np.array(child_l, np.int64)
        cr = np.array(child_r, np.int64)
        xb = binned[np.arange(n), f[pr]].astype(np.int64)
        go_left = xb <= b[pr]
        newn = np.where(go_left, cl[pr], cr[pr])
        moved = row_active & do[pr]
        node_of_row = np.where(moved, newn, node_of_row)

        # yabt/tree.py:576-612 smaller-child histogram + sibling subtraction.
        # Skipped once the loop cannot run again (the result is never read).
        more = bool(nxt) and d1 < params.max_depth and remaining > 0
        if more:
            sp = np.array(split_pos, np.int64)
            P = sp.shape[0]
            pos_to_pair = np.full(M, -1, np.int64)
            pos_to_pair[sp] = np.arange(P)
            sil = small_left[sp]
            pair_row = pos_to_pair[pr]
            part = row_active & (pair_row >= 0)
            sil_row = sil[np.maximum(pair_row, 0)]
            small = part & (go_left == sil_row)
            rows = np.nonzero(small)[0]
            hs = scatter_hist_fm(binned_fm[:, rows], pair_row[rows], grad[rows], hess[rows], None, P)
            hp = hist[:, sp]
            ho = hp - hs
            s4 = sil.reshape(1, P, 1, 1)
            lh = np.where(s4, hs, ho)
            rh = np.where(s4, ho, hs)
            hist = np.empty((3, 2 * P, F, B), np.float32)
            hist[:, 0::2] = lh
            hist[:, 1::2] = rh
            if imat is not None:
                cpm = np.maximum(pathmax[sp], imat[f[sp]])
                pathmax = np.repeat(cpm, 2, axis=0)
        active = nxt if more else []
        depth = d1

    tree = OTree(
        feature=np.array(feature, np.int64), threshold=np.array(threshold, np.float32),
        left=np.array(left, np.int64), right=np.array(right, np.int64),
        value=np.array(value, np.float32), depth=max(node_depth) + 1,
        gate_scale=np.array(gate, np.float32), split_bin=np.array(sbin, np.int64))
    return tree, node_of_row, trace


def grow_bestfirst(binned: np.ndarray, grad: np.ndarray, hess: np.ndarray,
                   edges: list[np.ndarray], scales: np.ndarray, params: TreeParams,
                   feature_mask: np.ndarray | None = None,
                   interaction_matrix: np.ndarray | None = None,
                   interaction_boost: float = 0.5):
    """Restates the best-first (heap) grower, yabt/tree.py:206-360, for axis
    splits: a heap of candidate leaves keyed by (-gain, push order); pop the
    best, partition its rows (stable), histogram the smaller child, subtract
    for the sibling, push both children. Returns (OTree, node_of_row)."""
    import heapq
    import itertools
    n, F = binned.shape
    lam, gamma = params.reg_lambda, params.gamma
    mcw, msl, lr = params.min_child_weight, params.min_samples_leaf, params.learning_rate
    scales_c = np.maximum(scales.astype(np.float32), f32(1e-12))
    imat = None if interaction_matrix is None else interaction_matrix.astype(np.float32)
    feature, threshold, left, right, value, node_depth, gate, sbin = [], [], [], [], [], [], [], []

    def tot(x):   # float32 sum of a float32 vector (summed in float64 and rounded)
        return float(np.sum(x.astype(np.float64)).astype(np.float32))

    def new_node(g_sum: float, h_sum: float, depth: int) -> int:   # yabt/tree.py:233-243
        feature.append(LEAF); threshold.append(0.0); left.append(-1); right.append(-1)
        value.append(-lr * g_sum / (h_sum + lam)); node_depth.append(depth); gate.append(1.0)
        sbin.append(-1)
        return len(feature) - 1

    def hist_of(rows):
        return scatter_hist(binned[rows], np.zeros(rows.size, np.int64), grad[rows], hess[rows], None, 1)[:, 0]

    all_rows = np.arange(n)
    root_hist = hist_of(all_rows)
    root = new_node(tot(grad), tot(hess), 0)
    tiebreak = itertools.count()
    heap: list = []

    def push_candidate(nid, rows, hist, path=()):                   # yabt/tree.py:252-290
        if node_depth[nid] >= params.max_depth:
            return
        boost = None
        if imat is not None and path:
            pf = np.array(sorted(set(path)), np.int64)
            boost = (f32(1.0) + f32(interaction_boost) * imat[pf].max(axis=0)).astype(np.float32)[None, :]
        idx, gain, _ = split_scan(hist[:, None], lam, gamma, mcw, msl, feature_mask, boost)
        g = float(gain[0])
        if g > 0:
            heapq.heappush(heap, (-g, next(tiebreak), nid, rows, hist, int(idx[0]) // B, int(idx[0]) % B, path))

    push_candidate(root, all_rows, root_hist)
    n_leaves = 1
    while heap and n_leaves < params.max_leaves:                     # yabt/tree.py:295-348
        _, _, nid, rows, hist, f, b, path = heapq.heappop(heap)
        go_left = binned[rows, f] <= b
        rows_l, rows_r = rows[go_left], rows[~go_left]
        if rows_l.size <= rows_r.size:
            hist_l = hist_of(rows_l)
            hist_r = hist - hist_l
        else:
            hist_r = hist_of(rows_r)
            hist_l = hist - hist_r
        d = node_depth[nid] + 1
        nl = new_node(tot(hist_l[0, 0]), tot(hist_l[1, 0]), d)
        nr = new_node(tot(hist_r[0, 0]), tot(hist_r[1, 0]), d)
        feature[nid] = f
        e = edges[f]
        threshold[nid] = float(e[min(b, len(e) - 1)])
        gate[nid] = float(scales_c[f])
        sbin[nid] = b
        left[nid], right[nid] = nl, nr
        value[nid] = 0.0
        n_leaves += 1
        push_candidate(nl, rows_l, hist_l, path + (f,))
        push_candidate(nr, rows_r, hist_r, path + (f,))

    tree = OTree(
        feature=np.array(feature, np.int64), threshold=np.array(threshold, np.float32),
        left=np.array(left, np.int64), right=np.array(right, np.int64),
        value=np.array(value, np.float32), depth=max(node_depth) + 1,
        gate_scale=np.array(gate, np.float32), split_bin=np.array(sbin, np.int64))
    return tree, tree.apply_bins(binned)
