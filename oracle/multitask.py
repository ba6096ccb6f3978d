"""CPU restatement of the multi-task grower (test infrastructure only).

grow_multitask restates yabt/multitask.py:60-150 with build_histogram_multi and
find_best_split_multi (yabt/histogram.py:120-188) in numpy float32: a
(2T+1, F, 256) histogram (T gradient channels, T hessian channels, counts;
sequential float32 adds in row-major order like the reference's CPU
scatter_add_), float32 prefix sums, the summed per-task Newton gain, shared
counts and summed hessians for validity, best-first (heap) growth with the
smaller child histogrammed and the sibling obtained by subtraction.
Pinned against the reference's own runs in tests/golden/multitask.npz.
"""

from __future__ import annotations

import heapq
import itertools

import numpy as np

from .grow import B, LEAF, TreeParams

f32 = np.float32


def hist_multi(binned: np.ndarray, grad: np.ndarray, hess: np.ndarray) -> np.ndarray:
    """(2T+1, F, 256) float32, yabt/histogram.py:120-140."""
    n, F = binned.shape
    T = grad.shape[1]
    flat = (np.arange(F, dtype=np.int64)[None, :] * B + binned.astype(np.int64)).reshape(-1)
    out = np.zeros((2 * T + 1, F * B), np.float32)
    for t in range(T):
        np.add.at(out[t], flat, np.repeat(grad[:, t].astype(np.float32), F))
        np.add.at(out[T + t], flat, np.repeat(hess[:, t].astype(np.float32), F))
    np.add.at(out[2 * T], flat, np.ones(n * F, np.float32))
    return out.reshape(2 * T + 1, F, B)


def best_split_multi(hist: np.ndarray, T: int, lam: float, gamma: float, mcw: float, msl: int,
                     fmask: np.ndarray | None):
    """(gain, f, b), yabt/histogram.py:143-188 (float32, first maximum)."""
    lam32 = f32(lam)
    CL = np.cumsum(hist[2 * T], axis=1, dtype=np.float32)
    C = CL[:, -1:]
    CR = C - CL
    total = np.zeros_like(CL)
    sum_HL = np.zeros_like(CL)
    for t in range(T):
        GL = np.cumsum(hist[t], axis=1, dtype=np.float32)
        HL = np.cumsum(hist[T + t], axis=1, dtype=np.float32)
        G, H = GL[:, -1:], HL[:, -1:]
        GR, HR = G - GL, H - HL
        total = total + f32(0.5) * (GL * GL / (HL + lam32) + GR * GR / (HR + lam32) - G * G / (H + lam32))
        sum_HL = sum_HL + HL
    sum_HR = sum_HL[:, -1:] - sum_HL
    total = total - f32(gamma)
    mcw32 = f32(mcw)
    valid = (CL >= msl) & (CR >= msl) & (sum_HL >= mcw32) & (sum_HR >= mcw32)
    valid[:, -1] = False
    if fmask is not None:
        valid &= fmask.reshape(-1, 1)
    total = np.where(valid, total, f32(-np.inf)).astype(np.float32)
    idx = int(total.reshape(-1).argmax())
    f, b = divmod(idx, B)
    return float(total[f, b]), f, b


def grow_multitask(binned: np.ndarray, grad: np.ndarray, hess: np.ndarray, edges: list[np.ndarray],
                   params: TreeParams, fmask: np.ndarray | None = None):
    """yabt/multitask.py:60-150. Returns (feature, threshold, left, right,
    value (nodes, T), depth, leaf of every row)."""
    n, F = binned.shape
    T = grad.shape[1]
    lam, lr = params.reg_lambda, params.learning_rate
    feature, threshold, left, right, depth_of, values, sbin = [], [], [], [], [], [], []

    def new_node(g_sum: np.ndarray, h_sum: np.ndarray, depth: int) -> int:
        feature.append(LEAF); threshold.append(0.0); left.append(-1); right.append(-1); sbin.append(-1)
        # -lr * g / (h + lam) as float32 tensor arithmetic
        values.append((g_sum * f32(-lr) / (h_sum + f32(lam))).astype(np.float32))
        depth_of.append(depth)
        return len(feature) - 1

    def totals(hist):
        return hist[:T, 0, :].sum(axis=1, dtype=np.float32), hist[T:2 * T, 0, :].sum(axis=1, dtype=np.float32)

    rows_all = np.arange(n)
    root_hist = hist_multi(binned, grad, hess)
    root = new_node(*totals(root_hist), 0)
    order = itertools.count()
    heap: list = []

    def push(nid, rows, hist):
        if depth_of[nid] >= params.max_depth:
            return
        gain, f, b = best_split_multi(hist, T, lam, params.gamma, params.min_child_weight,
                                      params.min_samples_leaf, fmask)
        if gain > 0:
            heapq.heappush(heap, (-gain, next(order), nid, rows, hist, f, b))

    push(root, rows_all, root_hist)
    n_leaves = 1
    while heap and n_leaves < params.max_leaves:
        _, _, nid, rows, hist, f, b = heapq.heappop(heap)
        go_left = binned[rows, f] <= b
        rows_l, rows_r = rows[go_left], rows[~go_left]
        if rows_l.size <= rows_r.size:
            hist_l = hist_multi(binned[rows_l], grad[rows_l], hess[rows_l])
            hist_r = hist - hist_l
        else:
            hist_r = hist_multi(binned[rows_r], grad[rows_r], hess[rows_r])
            hist_l = hist - hist_r
        d = depth_of[nid] + 1
        nl = new_node(*totals(hist_l), d)
        nr = new_node(*totals(hist_r), d)
        feature[nid] = f
        e = edges[f]
        threshold[nid] = float(e[min(b, len(e) - 1)])
        sbin[nid] = b
        left[nid], right[nid] = nl, nr
        values[nid] = np.zeros(T, np.float32)
        n_leaves += 1
        push(nl, rows_l, hist_l)
        push(nr, rows_r, hist_r)

    feature = np.array(feature, np.int64)
    left_a, right_a = np.array(left, np.int64), np.array(right, np.int64)
    thr = np.array(threshold, np.float32)
    # leaf of every row, routed on the bins (bin <= split bin <=> x <= threshold)
    sbin = np.array(sbin, np.int64)
    node = np.zeros(n, np.int64)
    for _ in range(max(depth_of) + 1):
        fr = feature[node]
        inner = fr >= 0
        go = binned[np.arange(n), np.where(inner, fr, 0)] <= sbin[node]
        node = np.where(inner, np.where(go, left_a[node], right_a[node]), node)
    return feature, thr, left_a, right_a, np.stack(values), max(depth_of) + 1, node
