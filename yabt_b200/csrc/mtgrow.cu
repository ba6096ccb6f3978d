// Multi-task trees: one split structure for T targets, a leaf value per task.
//
// Restates grow_multitask_tree (yabt/multitask.py:60-150) with
// find_best_split_multi (yabt/histogram.py:143-188): best-first (heap) growth
// on the sum over tasks of the per-task Newton gains; validity from the shared
// counts and the summed child hessians; each node's value per task is
// -lr * G_t / (H_t + lambda). The reference's tasks all use squared loss
// (YABTMultiTaskRegressor, yabt/sklearn_api.py:366-402), so every per-task
// hessian channel equals the count channel and H_t = row count.
//
// The best-first grower does the work: k_bf_pick (heap pop, tree arrays,
// partition plan), k_partition, k_plan and the histogram kernels. Per step
// the smaller child's histogram is built in ceil(T/2) passes of the general
// (two-channel) histogram kernel, one task in each channel under one shared
// quantisation scale, into a [2P][F][256] value + count buffer. The kernels
// here add what differs: the multi-channel scan (both children's histograms
// by subtraction, the summed gain, the per-task sums of the chosen bin) and
// the per-task leaf values.
#include "grow.cuh"

namespace yabt {

// -lr * G / (H + lambda) in float32 on the float32 sums (torch float32 ops,
// yabt/multitask.py:84-90)
__device__ __forceinline__ float mt_value(const GrowParams& p, float ginv, long long g, long long c) {
  const float G = __fmul_rn(__ll2float_rn(g), ginv);
  return __fdiv_rn(__fmul_rn(G, -p.lr), __fadd_rn(__ll2float_rn(c), p.lam));
}

__device__ __forceinline__ void warp_prefix8(long long (&v)[8], long long* total) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 1; i < 8; ++i) v[i] += v[i - 1];
  long long x = v[7];
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  *total = __shfl_sync(0xffffffffu, x, 31);
  const long long excl = x - v[7];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] += excl;
}

__device__ __forceinline__ void load8(const long long* src, long long (&v)[8]) {
  const longlong2* q = reinterpret_cast<const longlong2*>(src);
#pragma unroll
  for (int i = 0; i < 4; ++i) { const longlong2 t = q[i]; v[2 * i] = t.x; v[2 * i + 1] = t.y; }
}

__device__ __forceinline__ void store8(long long* dst, const long long (&v)[8]) {
  longlong2* q = reinterpret_cast<longlong2*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) q[i] = make_longlong2(v[2 * i], v[2 * i + 1]);
}

// Root (root != 0: its histogram in mb.small) or the two children of the node
// the last k_bf_pick split. Blocks [0, fblocks): one warp per feature for both
// children (the left child's slot is the parent's: each channel of the parent
// is read before that channel of either child is written). Blocks beyond: the
// children's row ranges, as in k_bf_scan.
__global__ void __launch_bounds__(SCAN_WARPS * 32)
k_mt_scan(GrowParams p, GrowBufs b, MtBufs mb, TreeIO io, int root) {
  GrowState* st = b.st;
  const int fblocks = (p.F + SCAN_WARPS - 1) / SCAN_WARPS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t FB = (size_t)p.F * YABT_NB;
  const size_t HN = (size_t)(mb.T + 1) * FB;
  if (root) {
    if (!st->active) return;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      b.leaf_src[0] = SRC_IDENTITY; b.leaf_begin[0] = 0; b.leaf_count[0] = (int)io.n_root;
      b.node_slot[0] = 0;
      st->bf_next_slot = 1; st->bf_split = -2; st->bf_scan = 1;
    }
  } else {
    if (st->bf_split < 0) return;
    if (blockIdx.x >= fblocks) {
      const int nl = st->n_nodes - 2, nr = nl + 1;
      const int B = b.seg_begin[0][0], cnt = b.seg_count[0][0];
      const int keep = st->bf_scan;
      if (blockIdx.x == fblocks && threadIdx.x == 0) {
        const int src = keep ? SRC_LIST0 : SRC_LIST1;
        b.leaf_src[nl] = src; b.leaf_begin[nl] = b.seg_begin[1][0]; b.leaf_count[nl] = b.seg_count[1][0];
        b.leaf_src[nr] = src; b.leaf_begin[nr] = b.seg_begin[1][1]; b.leaf_count[nr] = b.seg_count[1][1];
      }
      if (keep) {
        const int nb = gridDim.x - fblocks;
        for (int i = (blockIdx.x - fblocks) * blockDim.x + threadIdx.x; i < cnt; i += nb * blockDim.x)
          b.rows[0][B + i] = b.rows[1][B + i];
      }
      return;
    }
    if (!st->bf_scan) return;
  }
  const int f = blockIdx.x * SCAN_WARPS + warp;
  if (blockIdx.x >= fblocks || f >= p.F) return;
  const int T = mb.T, nch = root ? 1 : 2;
  const float ginv = st->ginv, lam = p.lam, fmsl = (float)p.msl, mcw = p.mcw;
  const bool fok = !(p.use_fmask && io.fmask && !io.fmask[f]);
  int slot[2] = {0, 0};
  bool sil = true;
  if (!root) {
    const int nl = st->n_nodes - 2;
    slot[0] = b.node_slot[nl]; slot[1] = b.node_slot[nl + 1];
    sil = b.pair_sil[0] != 0;
  }
  const size_t off = (size_t)f * YABT_NB + lane * 8;
  // counts: the small child's (packed two bins per word) and the parent's
  long long cnt[2][8];
  {
    const longlong2* q = reinterpret_cast<const longlong2*>(mb.small + (size_t)2 * mb.P * FB +
                                                            (size_t)f * (YABT_NB / 2) + lane * 4);
    long long cs[8];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const longlong2 t = q[i];
      cs[4 * i + 0] = (long long)((unsigned long long)t.x & 0xffffffffULL);
      cs[4 * i + 1] = (long long)((unsigned long long)t.x >> 32);
      cs[4 * i + 2] = (long long)((unsigned long long)t.y & 0xffffffffULL);
      cs[4 * i + 3] = (long long)((unsigned long long)t.y >> 32);
    }
    if (root) {
#pragma unroll
      for (int i = 0; i < 8; ++i) cnt[0][i] = cs[i];
    } else {
      long long cp[8];
      load8(mb.hist + (size_t)slot[0] * HN + (size_t)T * FB + off, cp);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        cnt[0][i] = sil ? cs[i] : cp[i] - cs[i];
        cnt[1][i] = sil ? cp[i] - cs[i] : cs[i];
      }
    }
  }
  __syncwarp();
  long long ctot[2] = {0, 0};
#pragma unroll
  for (int ch = 0; ch < 2; ++ch) {
    if (ch >= nch) break;
    store8(mb.hist + (size_t)slot[ch] * HN + (size_t)T * FB + off, cnt[ch]);
    warp_prefix8(cnt[ch], &ctot[ch]);
  }
  // summed gain over tasks, in task order
  float tot[2][8];
#pragma unroll
  for (int i = 0; i < 8; ++i) tot[0][i] = tot[1][i] = 0.f;
  for (int t = 0; t < T; ++t) {
    long long v[2][8];
    long long vs[8];
    load8(mb.small + (size_t)t * FB + off, vs);
    if (root) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[0][i] = vs[i];
    } else {
      long long vp[8];
      load8(mb.hist + (size_t)slot[0] * HN + (size_t)t * FB + off, vp);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[0][i] = sil ? vs[i] : vp[i] - vs[i];
        v[1][i] = sil ? vp[i] - vs[i] : vs[i];
      }
    }
    __syncwarp();
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      if (ch >= nch) break;
      store8(mb.hist + (size_t)slot[ch] * HN + (size_t)t * FB + off, v[ch]);
      long long gt;
      warp_prefix8(v[ch], &gt);
      const float G = __fmul_rn(__ll2float_rn(gt), ginv);
      const float H = __ll2float_rn(ctot[ch]);
      const float t3 = __fdiv_rn(__fmul_rn(G, G), __fadd_rn(H, lam));
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float GL = __fmul_rn(__ll2float_rn(v[ch][i]), ginv);
        const float HL = __ll2float_rn(cnt[ch][i]);
        const float GR = __fsub_rn(G, GL), HR = __fsub_rn(H, HL);
        const float t1 = __fdiv_rn(__fmul_rn(GL, GL), __fadd_rn(HL, lam));
        const float t2 = __fdiv_rn(__fmul_rn(GR, GR), __fadd_rn(HR, lam));
        tot[ch][i] = __fadd_rn(tot[ch][i], __fmul_rn(0.5f, __fsub_rn(__fadd_rn(t1, t2), t3)));
      }
    }
  }
  // validity and the first maximum per child
  int bbin[2] = {0, 0};
  float bgain[2] = {-INFINITY, -INFINITY};
  long long bcl[2] = {0, 0};
#pragma unroll
  for (int ch = 0; ch < 2; ++ch) {
    if (ch >= nch) break;
    const float H = __ll2float_rn(ctot[ch]);
    float sumH = 0.f;                          // sum over tasks of the hessian totals
    for (int t = 0; t < T; ++t) sumH = __fadd_rn(sumH, H);
    float bg = -INFINITY;
    int bb = 0;
    long long bc = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int bin = lane * 8 + i;
      const float CL = __ll2float_rn(cnt[ch][i]);
      const float CR = __fsub_rn(H, CL);
      float sumHL = 0.f;
      for (int t = 0; t < T; ++t) sumHL = __fadd_rn(sumHL, CL);
      const float sumHR = __fsub_rn(sumH, sumHL);
      const bool valid = fok && bin != YABT_NB - 1 && CL >= fmsl && CR >= fmsl && sumHL >= mcw && sumHR >= mcw;
      const float gain = valid ? __fsub_rn(tot[ch][i], p.gamma) : -INFINITY;
      if (i == 0 || gain > bg) { bg = gain; bb = bin; bc = cnt[ch][i]; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float og = __shfl_xor_sync(0xffffffffu, bg, o);
      const int ob = __shfl_xor_sync(0xffffffffu, bb, o);
      const long long oc = __shfl_xor_sync(0xffffffffu, bc, o);
      if (og > bg || (og == bg && ob < bb)) { bg = og; bb = ob; bc = oc; }
    }
    bgain[ch] = bg; bbin[ch] = bb; bcl[ch] = bc;
  }
  // per-task left sums at the chosen bins (the children's channels were just written)
#pragma unroll
  for (int ch = 0; ch < 2; ++ch) {
    if (ch >= nch) break;
    MtRec* rec = mb.feat + (size_t)ch * p.F + f;
    for (int t = 0; t < MT_MAX; ++t) {
      long long gl = 0, gt = 0;
      if (t < T) {
        long long v[8];
        load8(mb.hist + (size_t)slot[ch] * HN + (size_t)t * FB + off, v);
        warp_prefix8(v, &gt);
        long long mine = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (lane * 8 + i == bbin[ch]) mine = v[i];
        gl = __shfl_sync(0xffffffffu, mine, bbin[ch] >> 3);
      }
      if (lane == 0) { rec->gl[t] = gl; rec->g[t] = gt; }
    }
    if (lane == 0) {
      BfCand r;
      r.sel = bgain[ch]; r.gain = bgain[ch]; r.f = f; r.bin = bbin[ch]; r.flag = 0;
      r.cl = bcl[ch]; r.c = ctot[ch]; r.gl = 0; r.hl = bcl[ch]; r.g = 0; r.h = ctot[ch];
      b.bf_feat[(size_t)ch * p.F + f] = r;
      atomicMax(&b.node_key[ch], ((unsigned long long)f2ord(bgain[ch]) << 32) | (0xffffffffu - (unsigned)f));
    }
  }
}

// Before k_bf_pick: the per-task sums of the nodes the last scan produced
// follow their chosen feature (k_bf_pick commits the structure record), and
// the root's values.
__global__ void k_mt_commit(GrowParams p, GrowBufs b, MtBufs mb) {
  GrowState* st = b.st;
  if (!st->active || !st->bf_scan) return;
  const int split = st->bf_split;
  const int nc = split == -2 ? 1 : split >= 0 ? 2 : 0;
  for (int c = 0; c < nc; ++c) {
    const int gid = split == -2 ? 0 : st->n_nodes - 2 + c;
    const int f = (int)(0xffffffffu - (unsigned)(b.node_key[c] & 0xffffffffULL));
    const MtRec r = mb.feat[(size_t)c * p.F + ((unsigned)f < (unsigned)p.F ? f : 0)];
    if (threadIdx.x == 0) mb.cand[gid] = r;
    if (split == -2) {
      const long long cnt = b.bf_feat[(unsigned)f < (unsigned)p.F ? f : 0].c;
      for (int t = threadIdx.x; t < mb.T; t += blockDim.x) mb.values[t] = mt_value(p, st->ginv, r.g[t], cnt);
    }
  }
}

// After k_bf_pick: the per-task values of the two children of the node it
// split (the split node's own values become zero), yabt/multitask.py:122-132.
__global__ void k_mt_values(GrowParams p, GrowBufs b, MtBufs mb) {
  GrowState* st = b.st;
  const int m = st->bf_split;
  if (m < 0) return;
  const int nl = st->n_nodes - 2, nr = nl + 1;
  const MtRec r = mb.cand[m];
  const BfCand c = b.bf_cand[m];
  for (int t = threadIdx.x; t < mb.T; t += blockDim.x) {
    mb.values[(size_t)nl * mb.T + t] = mt_value(p, st->ginv, r.gl[t], c.cl);
    mb.values[(size_t)nr * mb.T + t] = mt_value(p, st->ginv, r.g[t] - r.gl[t], c.c - c.cl);
    mb.values[(size_t)m * mb.T + t] = 0.f;
  }
}

// margin[t][i] += values[leaf[i]][t] (when values is given), then the squared
// loss gradient grad[t][i] = margin[t][i] - y[t][i] (when grad is given).
__global__ void k_mt_update(const int* __restrict__ leaf, const float* __restrict__ values, int T, long long n,
                            float* __restrict__ margin, const float* __restrict__ y, float* __restrict__ grad) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long l = values ? (long long)leaf[i] : 0;
    for (int t = 0; t < T; ++t) {
      float m = margin[t * n + i];
      if (values) { m = __fadd_rn(m, values[l * T + t]); margin[t * n + i] = m; }
      if (grad) grad[t * n + i] = __fsub_rn(m, y[t * n + i]);
    }
  }
}

cudaError_t launch_mt_scan(const GrowParams& p, const GrowBufs& b, const MtBufs& mb, const TreeIO& io, int root,
                           int nsm, cudaStream_t s) {
  const int fblocks = (p.F + SCAN_WARPS - 1) / SCAN_WARPS;
  const int grid = root ? fblocks : fblocks + std::max(1, std::min<int>(nsm, (int)((p.n + 2047) / 2048)));
  k_mt_scan<<<grid, SCAN_WARPS * 32, 0, s>>>(p, b, mb, io, root);
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_mt_commit(const GrowParams& p, const GrowBufs& b, const MtBufs& mb, cudaStream_t s) {
  k_mt_commit<<<1, 32, 0, s>>>(p, b, mb);
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_mt_values(const GrowParams& p, const GrowBufs& b, const MtBufs& mb, cudaStream_t s) {
  k_mt_values<<<1, 32, 0, s>>>(p, b, mb);
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_mt_update(const int* leaf, const float* values, int T, long long n, float* margin, const float* y,
                             float* grad, int nsm, cudaStream_t s) {
  const int grid = (int)std::min<long long>((n + 255) / 256, 8LL * nsm);
  k_mt_update<<<std::max(grid, 1), 256, 0, s>>>(leaf, values, T, n, margin, y, grad);
  count_launches(1);
  return cudaGetLastError();
}

}  // namespace yabt
