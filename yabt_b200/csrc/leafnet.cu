// Ridge-linear neural leaves, the fused margin update + loss gradients, and
// the interaction detector, all on the device.
//
// Restates fit_leaf_networks with leaf_net_hidden == 0
// (yabt/neural_leaves.py:131-184, _select_features :21-39, _fit_linear :42-90),
// the loss gradients (yabt/boosting.py:36-38,53-54), the margin update
// (yabt/boosting.py:511-514, Tree.net_contribution yabt/tree.py:118-128) and
// FeatureInteractionDetector (yabt/adaptive_features.py:129-160).
//
// Per tree, with no host synchronisation:
//   k_ln_select   split-feature use counts -> top-K (count desc, feature asc);
//                 flags whether gradient-correlation padding is needed
//   k_ln_corr     (only if padding is needed) |X^T g - mean * sum g| / std
//   k_ln_pad      completes the feature list
//   k_ln_rows     natural row order: per-row record (x_norm[K], g, h), per-leaf
//                 min/max envelope of the raw inputs
//   k_ln_gram     per leaf segment chunk: fp64 normal-equation partial sums
//                 M = sum h x1 x1^T (upper triangle), b = -sum g x1, every
//                 accumulator in registers of the lane that owns the row,
//                 fixed order (deterministic)
//   k_ln_solve    per leaf: reduce chunk partials in order, add the ridge,
//                 Cholesky solve, fold normalisation + learning rate
//   k_update      margin += value[leaf] + sum_k linear * clamp(x, lo, hi);
//                 next tree's gradient / hessian
#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "../../include/yabt_b200.h"

namespace yabt {

constexpr int KMAX = 8;                 // leaf-model inputs (leaf_net_features <= 8)
constexpr int NE = (KMAX + 1) * (KMAX + 2) / 2 + (KMAX + 1);   // 45 + 9 = 54 accumulators
constexpr int GRAM_CHUNK = 2048;        // smallest rows per Gram partial (enough blocks at small n)
constexpr long long GRAM_SPLIT = 296;   // large fits: about 2 x 148 partials of full size (see gram_rows)

// Rows per Gram partial: 2,048 x m, m = n / (2,048 x 296) clamped to [1, 8].
// Each partial pays fixed costs (its start-up loads, the warp sums of 54
// accumulators); large fits give each lane more rows to spread them over.
// A function of n alone, so a fit's partials, and hence its sums, do not
// depend on the device.
inline int gram_rows(long long n) {
  const long long m = n / (GRAM_CHUNK * GRAM_SPLIT);
  return GRAM_CHUNK * (int)(m < 1 ? 1 : (m > 8 ? 8 : m));
}

struct LeafNetArgs {
  // tree (device)
  const long long* feature;   // [maxn]
  float* value;               // [maxn] updated in place (fold)
  int n_nodes_cap;            // maxn
  const int* meta;            // [4] from the grower: n_nodes, ...
  // leaf ranges (grower workspace)
  const int* leaf_src;
  const int* leaf_begin;
  const int* leaf_count;
  const int* fin;
  const int* list0;
  const int* list1;
  const int* leaf_of_row;
  // data
  const float* Xfm;           // [F][n] imputed
  const float* col_mean;      // [F]
  const float* col_std;       // [F] unbiased, unclamped
  const float* margin;        // [n] ensemble margin excluding this tree
  const float* y;             // [n]
  long long n;
  int F;
  int K;                      // min(leaf_net_features, F)
  int loss;                   // 0 squared error, 1 logistic
  int min_samples;
  float l2;
  float lr;
  // outputs (device)
  long long* feats;           // [K]
  float* linear;              // [maxn][K]
  float* lo;                  // [maxn][K]
  float* hi;                  // [maxn][K]
  int* has_nets;              // [1]
  // scratch (device)
  int* fcount;                // [F]
  int* flags;                 // [4]: n_used, need_pad, n_chunks, n_eligible
  double* stats;              // [F + 1 + maxn]: sum_i x_fi g_i [F], sum g, leaf row counts [maxn]
  double* corr;               // stats
  double* gsum;               // stats + F
  float* env;                 // [maxn][2 * KMAX]: -min x, max x (the leaf input envelopes)
  float* rec;                 // [n][REC] records
  float* pmin;                // [max_chunks][KMAX] chunk envelope
  float* pmax;                // [max_chunks][KMAX]
  int* counts;                // [maxn]
  int* leaf_first;            // [maxn] first chunk of a leaf
  int* leaf_nch;              // [maxn] chunks of a leaf
  int* chunk_leaf;            // [max_chunks]
  int* chunk_begin;           // [max_chunks]
  int* chunk_end;             // [max_chunks]
  double* partial;            // [max_chunks][NE]
  double* totals;             // [maxn][NE] per-node sums of the chunk partials
  int max_chunks;
  int chunk_rows;             // rows per Gram partial (gram_rows(n))
};

constexpr int REC = 12;   // floats per row record: raw x[8], g, h, pad[2] (48 bytes)

__device__ __forceinline__ void loss_gh(int loss, float m, float y, float* g, float* h) {
  if (loss == 0) { *g = __fsub_rn(m, y); *h = 1.f; return; }
  // p = sigmoid(m) = 1 / (1 + exp(-m)), g = p - y, h = max(p (1 - p), 1e-6)
  const float p = __fdiv_rn(1.f, __fadd_rn(1.f, expf(-m)));
  *g = __fsub_rn(p, y);
  *h = fmaxf(__fmul_rn(p, __fsub_rn(1.f, p)), 1e-6f);
}

// ------------------------------------------------------------------ feature choice
__global__ void __launch_bounds__(1024) k_ln_select(LeafNetArgs a) {
  __shared__ int s_used;
  const int nn = a.meta[0];
  for (int f = threadIdx.x; f < a.F; f += blockDim.x) a.fcount[f] = 0;
  __syncthreads();
  for (int g = threadIdx.x; g < nn; g += blockDim.x) {
    const long long f = a.feature[g];
    if (f >= 0) atomicAdd(&a.fcount[f], 1);
  }
  if (threadIdx.x == 0) s_used = 0;
  __syncthreads();
  // rank used features by (count desc, feature asc)
  for (int f = threadIdx.x; f < a.F; f += blockDim.x) {
    const int c = a.fcount[f];
    if (c <= 0) continue;
    atomicAdd(&s_used, 1);
    int rank = 0;
    for (int q = 0; q < a.F; ++q) {
      const int cq = a.fcount[q];
      if (cq > c || (cq == c && cq > 0 && q < f)) ++rank;
    }
    if (rank < a.K) a.feats[rank] = f;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int used = min(s_used, a.K);
    a.flags[0] = used;
    a.flags[1] = used < a.K;
    a.gsum[0] = 0.0;
  }
  for (int f = threadIdx.x; f < a.F; f += blockDim.x) a.corr[f] = 0.0;
  // this rank's leaf row counts, summed over the ranks with the correlations
  double* cnt = a.stats + a.F + 1;
  for (int g = threadIdx.x; g < a.n_nodes_cap; g += blockDim.x)
    cnt[g] = (g < nn && a.feature[g] < 0) ? (double)a.leaf_count[g] : 0.0;
}

// grid (chunks, ceil(F/8)): sum_i x_fi g_i and sum g (only when padding is needed)
__global__ void k_ln_corr(LeafNetArgs a) {
  if (!a.flags[1]) return;
  const int f0 = blockIdx.y * 8;
  double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  double gs = 0.0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < a.n;
       i += (long long)gridDim.x * blockDim.x) {
    const int l = a.leaf_of_row[i];
    float g, h;
    loss_gh(a.loss, __fadd_rn(a.margin[i], a.value[l]), a.y[i], &g, &h);
    gs += (double)g;
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (f0 + q < a.F) acc[q] += (double)a.Xfm[(long long)(f0 + q) * a.n + i] * (double)g;
  }
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    double v = acc[q];
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) atomicAdd(&a.corr[min(f0 + q, a.F - 1)], f0 + q < a.F ? v : 0.0);
  }
  for (int o = 16; o; o >>= 1) gs += __shfl_xor_sync(0xffffffffu, gs, o);
  if (lane == 0 && blockIdx.y == 0) atomicAdd(a.gsum, gs);
}

__global__ void __launch_bounds__(1024) k_ln_pad(LeafNetArgs a) {
  if (!a.flags[1]) return;
  // score = |X^T g - mean * sum g| / max(std, 1e-6); used features excluded
  __shared__ int s_base;
  if (threadIdx.x == 0) s_base = a.flags[0];
  __syncthreads();
  const int need = a.K - s_base;
  for (int f = threadIdx.x; f < a.F; f += blockDim.x) {
    if (a.fcount[f] > 0) continue;
    const float sf = (float)(fabs(a.corr[f] - (double)a.col_mean[f] * a.gsum[0]) /
                             fmax((double)a.col_std[f], 1e-6));
    int rank = 0;
    for (int q = 0; q < a.F; ++q) {
      if (a.fcount[q] > 0) continue;
      const float sq = (float)(fabs(a.corr[q] - (double)a.col_mean[q] * a.gsum[0]) /
                               fmax((double)a.col_std[q], 1e-6));
      if (sq > sf || (sq == sf && q < f)) ++rank;
    }
    if (rank < need) a.feats[s_base + rank] = f;
  }
}

// ------------------------------------------------------------------ per-row records
// Natural row order, streaming: record = (raw x[K], g, h) at margin + value[leaf].
// A thread takes two rows per step (i and i + grid stride) and issues every
// load of both before it stores either record.
__global__ void __launch_bounds__(256) k_ln_rows(LeafNetArgs a) {
  const int K = a.K;
  int fk[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) fk[k] = k < K ? (int)a.feats[k] : 0;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i0 = blockIdx.x * (long long)blockDim.x + threadIdx.x; i0 < a.n; i0 += 2 * stride) {
    int l[2];
    float m[2], y[2], v[2], x[2][KMAX];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const long long i = i0 + r * stride;
      const bool ok = i < a.n;
      l[r] = ok ? a.leaf_of_row[i] : 0;
      m[r] = ok ? a.margin[i] : 0.f;
      y[r] = ok ? a.y[i] : 0.f;
#pragma unroll
      for (int k = 0; k < KMAX; ++k) x[r][k] = (ok && k < K) ? a.Xfm[(long long)fk[k] * a.n + i] : 0.f;
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) v[r] = i0 + r * stride < a.n ? a.value[l[r]] : 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const long long i = i0 + r * stride;
      if (i >= a.n) break;
      float g, h;
      loss_gh(a.loss, __fadd_rn(m[r], v[r]), y[r], &g, &h);
      float4* dst = reinterpret_cast<float4*>(a.rec + i * REC);
      dst[0] = make_float4(x[r][0], x[r][1], x[r][2], x[r][3]);
      dst[1] = make_float4(x[r][4], x[r][5], x[r][6], x[r][7]);
      dst[2] = make_float4(g, h, 0.f, 0.f);
    }
  }
}

// one block: counts, eligibility and the chunk plan (every non-empty leaf;
// chunks of a leaf are contiguous: leaf_first[g], leaf_nch[g])
__global__ void __launch_bounds__(1024) k_ln_plan(LeafNetArgs a) {
  const int nn = a.meta[0];
  __shared__ int s_ne;
  if (threadIdx.x == 0) s_ne = 0;
  __syncthreads();
  for (int g = threadIdx.x; g < nn; g += blockDim.x) {
    const bool leaf = a.feature[g] < 0;
    const int c = leaf ? a.leaf_count[g] : 0;
    a.counts[g] = c;
    a.leaf_nch[g] = (c + a.chunk_rows - 1) / a.chunk_rows;
    if (leaf && c >= a.min_samples) atomicAdd(&s_ne, 1);
  }
  __syncthreads();
  if ((threadIdx.x >> 5) == 0) {
    const int lane = threadIdx.x & 31;
    int carry = 0;
    for (int base = 0; base < nn; base += 32) {
      const int g = base + lane;
      const int v = g < nn ? a.leaf_nch[g] : 0;
      int x = v;
      for (int o = 1; o < 32; o <<= 1) { const int y = __shfl_up_sync(0xffffffffu, x, o); if (lane >= o) x += y; }
      if (g < nn) a.leaf_first[g] = carry + x - v;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) {
      a.flags[2] = min(carry, a.max_chunks);
      a.flags[3] = s_ne;
      a.has_nets[0] = s_ne > 0;
    }
  }
  __syncthreads();
  for (int g = threadIdx.x; g < nn; g += blockDim.x) {
    const int c = a.counts[g], f0 = a.leaf_first[g];
    for (int q = 0; q < a.leaf_nch[g]; ++q) {
      const int idx = f0 + q;
      if (idx >= a.max_chunks) break;
      a.chunk_leaf[idx] = g;
      a.chunk_begin[idx] = a.leaf_begin[g] + q * a.chunk_rows;
      a.chunk_end[idx] = a.leaf_begin[g] + min(c, (q + 1) * a.chunk_rows);
    }
  }
}

// One block (8 warps) per chunk of a leaf's rows; each lane owns rows (the
// lane's share of its warp's rows) and keeps every normal-equation
// accumulator in registers: with x1 = (x_norm[K], 1) padded with zeros to
// KMAX + 1 entries, M_ij += (h x1_i) x1_j for i <= j (45 fused products) and
// b_i += (-g) x1_i (9). The records of the next two rows and the list index
// of the one after are in flight while the current row is used (the index
// load never stalls a record load), and the raw-x envelope is tracked on the
// way. At the end of the chunk each warp adds its lanes' sums (butterfly), the
// warps are added in order, and the chunk partial is written in the packed
// layout of the D = K + 1 system: the chunk partial is deterministic.
__global__ void __launch_bounds__(256, 1) k_ln_gram(LeafNetArgs a) {
  __shared__ double sp[8][NE];
  __shared__ float smin[8][KMAX], smax[8][KMAX];
  const int c = blockIdx.x;
  if (c >= a.flags[2]) return;
  const int g = a.chunk_leaf[c];
  const bool elig = a.counts[g] >= a.min_samples;
  const int src = a.leaf_src[g];
  const int* lst = src == 0 ? a.fin : (src == 1 ? a.list0 : (src == 2 ? a.list1 : nullptr));
  const int b0 = a.chunk_begin[c], b1 = a.chunk_end[c];
  const int K = a.K, D = K + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int DM = KMAX + 1;                 // padded system size
  constexpr int NT = DM * (DM + 1) / 2;        // upper-triangle entries of the padded system
  float mu[KMAX], sd[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    const int f = k < K ? (int)a.feats[k] : 0;
    mu[k] = k < K ? a.col_mean[f] : 0.f;
    sd[k] = k < K ? fmaxf(a.col_std[f], 1e-6f) : 1.f;
  }
  double acc[NT], accb[DM];
#pragma unroll
  for (int e = 0; e < NT; ++e) acc[e] = 0.0;
#pragma unroll
  for (int i = 0; i < DM; ++i) accb[i] = 0.0;
  float mn[KMAX], mx[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) { mn[k] = INFINITY; mx[k] = -INFINITY; }
  const int per = (b1 - b0 + 7) / 8;
  const int w0 = b0 + warp * per, w1 = min(b1, w0 + per);
  auto row_of = [&](int q) { return lst ? __ldg(lst + q) : q; };
  auto fetch = [&](int row, float4& r0, float4& r1, float2& r2) {   // raw x[8]; g, h
    const float* r = a.rec + (long long)row * REC;
    r0 = __ldg(reinterpret_cast<const float4*>(r));
    r1 = __ldg(reinterpret_cast<const float4*>(r) + 1);
    r2 = __ldg(reinterpret_cast<const float2*>(r + KMAX));
  };
  float4 c0 = make_float4(0.f, 0.f, 0.f, 0.f), c1 = c0, n0 = c0, n1 = c0;
  float2 c2 = make_float2(0.f, 0.f), n2 = c2;
  int p = w0 + lane, i2 = 0;
  if (p < w1) fetch(row_of(p), c0, c1, c2);
  if (p + 32 < w1) fetch(row_of(p + 32), n0, n1, n2);
  if (p + 64 < w1) i2 = row_of(p + 64);
  for (; p < w1; p += 32) {
    float4 m0 = n0, m1 = n1;
    float2 m2 = n2;
    if (p + 64 < w1) fetch(i2, m0, m1, m2);       // record two rows ahead
    if (p + 96 < w1) i2 = row_of(p + 96);          // list index three rows ahead
    const float xr[KMAX] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    double x[DM];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      if (k < K) { mn[k] = fminf(mn[k], xr[k]); mx[k] = fmaxf(mx[k], xr[k]); }
      x[k] = k < K ? (double)__fdiv_rn(__fsub_rn(xr[k], mu[k]), sd[k]) : (k == K ? 1.0 : 0.0);
    }
    x[KMAX] = K == KMAX ? 1.0 : 0.0;            // the bias input sits at index K
    if (elig) {
      const double hh = (double)c2.y, ng = -(double)c2.x;
      int e = 0;
#pragma unroll
      for (int i = 0; i < DM; ++i) {
        const double hx = __dmul_rn(hh, x[i]);
#pragma unroll
        for (int j = i; j < DM; ++j, ++e) acc[e] = __fma_rn(hx, x[j], acc[e]);
        accb[i] = __fma_rn(ng, x[i], accb[i]);
      }
    }
    c0 = n0; c1 = n1; c2 = n2;
    n0 = m0; n1 = m1; n2 = m2;
  }
  // warp sums (every lane ends with them), then lane 0 writes the packed entries
#pragma unroll
  for (int e = 0; e < NT; ++e)
#pragma unroll
    for (int o = 16; o; o >>= 1) acc[e] = __dadd_rn(acc[e], __shfl_xor_sync(0xffffffffu, acc[e], o));
#pragma unroll
  for (int i = 0; i < DM; ++i)
#pragma unroll
    for (int o = 16; o; o >>= 1) accb[i] = __dadd_rn(accb[i], __shfl_xor_sync(0xffffffffu, accb[i], o));
  const int ntri = D * (D + 1) / 2;
  for (int e = lane; e < NE; e += 32) sp[warp][e] = 0.0;
  __syncwarp();
  if (lane == 0) {
    int e = 0;
#pragma unroll
    for (int i = 0; i < DM; ++i) {
#pragma unroll
      for (int j = i; j < DM; ++j, ++e)
        if (j < D) sp[warp][i * D - i * (i - 1) / 2 + (j - i)] = acc[e];
      if (i < D) sp[warp][ntri + i] = accb[i];
    }
  }
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    float a0 = mn[k], a1 = mx[k];
    for (int o = 16; o; o >>= 1) {
      a0 = fminf(a0, __shfl_xor_sync(0xffffffffu, a0, o));
      a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, o));
    }
    if (lane == 0) { smin[warp][k] = a0; smax[warp][k] = a1; }
  }
  __syncthreads();
  if (threadIdx.x < NE) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t = __dadd_rn(t, sp[w][threadIdx.x]);
    a.partial[(long long)c * NE + threadIdx.x] = t;
  } else if (threadIdx.x >= 64 && threadIdx.x < 64 + KMAX) {
    const int k = threadIdx.x - 64;
    float a0 = INFINITY, a1 = -INFINITY;
    for (int w = 0; w < 8; ++w) { a0 = fminf(a0, smin[w][k]); a1 = fmaxf(a1, smax[w][k]); }
    a.pmin[(long long)c * KMAX + k] = a0;
    a.pmax[(long long)c * KMAX + k] = a1;
  }
}

// One warp per node: lanes reduce the node's chunk partials (contiguous, in
// chunk order) into its totals and its envelope into lo / hi.
__global__ void __launch_bounds__(128) k_ln_total(LeafNetArgs a) {
  const int nn = a.meta[0];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x * 4 + warp;
  if (g >= nn) return;
  const int K = a.K;
  const bool leaf = a.feature[g] < 0;
  const int c0 = leaf ? a.leaf_first[g] : 0, nc = leaf ? a.leaf_nch[g] : 0;
  if (lane < K) {
    float lo = INFINITY, hi = -INFINITY;
    for (int c = c0; c < c0 + nc; ++c) {
      lo = fminf(lo, a.pmin[(long long)c * KMAX + lane]);
      hi = fmaxf(hi, a.pmax[(long long)c * KMAX + lane]);
    }
    a.env[(long long)g * 2 * KMAX + lane] = -lo;
    a.env[(long long)g * 2 * KMAX + KMAX + lane] = hi;
  }
  for (int e = lane; e < NE; e += 32) {
    double t = 0.0;
    for (int c = c0; c < c0 + nc; ++c) t = __dadd_rn(t, a.partial[(long long)c * NE + e]);
    a.totals[(long long)g * NE + e] = t;
  }
}

// eligibility from the (all-ranks) leaf counts: counts, eligible-leaf count and has_nets
__global__ void __launch_bounds__(1024) k_ln_elig(LeafNetArgs a) {
  __shared__ int s_ne;
  const int nn = a.meta[0];
  const double* cnt = a.stats + a.F + 1;
  if (threadIdx.x == 0) s_ne = 0;
  __syncthreads();
  for (int g = threadIdx.x; g < nn; g += blockDim.x) {
    const bool leaf = a.feature[g] < 0;
    const int c = leaf ? (int)cnt[g] : 0;
    a.counts[g] = c;
    if (leaf && c >= a.min_samples) atomicAdd(&s_ne, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) { a.flags[3] = s_ne; a.has_nets[0] = s_ne > 0; }
}

// One warp per node: lane 0 adds the ridge to the node's totals, solves by
// Cholesky and folds (yabt/neural_leaves.py:85-89,180-184).
__global__ void __launch_bounds__(128) k_ln_solve(LeafNetArgs a) {
  __shared__ double se[4][NE];
  const int nn = a.meta[0];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x * 4 + warp;
  if (g >= nn) return;
  const int K = a.K, D = K + 1;
  const bool leaf = a.feature[g] < 0;
  const bool elig = leaf && a.counts[g] >= a.min_samples;
  if (lane < K) {
    a.lo[(long long)g * K + lane] = -a.env[(long long)g * 2 * KMAX + lane];
    a.hi[(long long)g * K + lane] = a.env[(long long)g * 2 * KMAX + KMAX + lane];
  }
  for (int e = lane; e < NE; e += 32) se[warp][e] = elig ? a.totals[(long long)g * NE + e] : 0.0;
  __syncwarp();
  if (lane != 0) return;
  float W[KMAX], db = 0.f;
#pragma unroll
  for (int k = 0; k < KMAX; ++k) W[k] = 0.f;
  if (elig) {
    const double* e = se[warp];
    double M[KMAX + 1][KMAX + 1], bv[KMAX + 1];
    int idx = 0;
    for (int i = 0; i < D; ++i)
      for (int j = i; j < D; ++j) { M[i][j] = e[idx]; M[j][i] = e[idx]; ++idx; }
    for (int i = 0; i < D; ++i) bv[i] = e[idx + i];
    for (int i = 0; i < K; ++i) M[i][i] = __dadd_rn(M[i][i], (double)a.l2);
    M[K][K] = __dadd_rn(M[K][K], 1e-8);
    bool ok = true;
    for (int j = 0; j < D && ok; ++j) {
      double s = M[j][j];
      for (int k = 0; k < j; ++k) s -= M[j][k] * M[j][k];
      if (!(s > 0.0)) { ok = false; break; }
      const double d = sqrt(s);
      M[j][j] = d;
      for (int i = j + 1; i < D; ++i) {
        double t = M[i][j];
        for (int k = 0; k < j; ++k) t -= M[i][k] * M[j][k];
        M[i][j] = t / d;
      }
    }
    if (ok) {
      double z[KMAX + 1], th[KMAX + 1];
      for (int i = 0; i < D; ++i) {
        double t = bv[i];
        for (int k = 0; k < i; ++k) t -= M[i][k] * z[k];
        z[i] = t / M[i][i];
      }
      for (int i = D - 1; i >= 0; --i) {
        double t = z[i];
        for (int k = i + 1; k < D; ++k) t -= M[k][i] * th[k];
        th[i] = t / M[i][i];
      }
      for (int k = 0; k < K; ++k) W[k] = (float)th[k];
      db = (float)th[K];
    }
  }
  // fold: value += lr * (db - sum_k W_k * (mu_k / sd_k)); linear = lr * W / sd
  float s = 0.f;
  for (int k = 0; k < K; ++k) {
    const int f = (int)a.feats[k];
    const float sd = fmaxf(a.col_std[f], 1e-6f);
    const float mu = a.col_mean[f];
    s = __fadd_rn(s, __fmul_rn(W[k], __fdiv_rn(mu, sd)));
    a.linear[(long long)g * K + k] = __fdiv_rn(__fmul_rn(a.lr, W[k]), sd);
  }
  if (a.flags[3] > 0) a.value[g] = __fadd_rn(a.value[g], __fmul_rn(a.lr, __fsub_rn(db, s)));
}

// ------------------------------------------------------------------ margin update + gradients
struct UpdateArgs {
  const int* leaf_of_row;
  const float* value;         // [maxn] (leaf values incl. folded bias)
  const float* linear;        // [maxn][K] or nullptr
  const float* lo;
  const float* hi;
  const long long* feats;     // [K]
  const int* has_nets;        // [1] or nullptr
  int K;
  const float* Xfm;
  long long n;
  float* margin;
  const float* y;
  float* grad;                // next tree's gradient (or nullptr)
  float* hess;                // next tree's hessian (or nullptr: unit hessian)
  int loss;
};

// Per-leaf tables (value, linear, lo, hi) are staged in shared memory; rows
// stream in natural order, two a thread per step (i and i + grid stride) with
// every load of both issued before either row's margin and gradient are stored.
__global__ void __launch_bounds__(256) k_update(UpdateArgs u, int nn) {
  // per-leaf tables in shared memory: linear / lo / hi as [nn][KMAX] (padded,
  // so a row reads each table with two 16-byte loads), then value[nn]
  extern __shared__ __align__(16) float tb[];
  const bool nets = u.linear && u.has_nets && u.has_nets[0];
  const int K = nets ? u.K : 0;
  float* slin = tb;
  float* slo = slin + (size_t)nn * KMAX;
  float* shi = slo + (size_t)nn * KMAX;
  float* sval = nets ? shi + (size_t)nn * KMAX : tb;   // without leaf models only the values
  for (int i = threadIdx.x; i < nn; i += blockDim.x) sval[i] = u.value[i];
  if (nets) {
    for (int i = threadIdx.x; i < nn * KMAX; i += blockDim.x) {
      const int l = i / KMAX, k = i % KMAX;
      const bool in = k < K;
      slin[i] = in ? u.linear[l * K + k] : 0.f;
      slo[i] = in ? u.lo[l * K + k] : 0.f;
      shi[i] = in ? u.hi[l * K + k] : 0.f;
    }
  }
  __syncthreads();
  int fk[KMAX];
#pragma unroll
  for (int k = 0; k < KMAX; ++k) fk[k] = (k < K) ? (int)u.feats[k] : 0;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i0 = blockIdx.x * (long long)blockDim.x + threadIdx.x; i0 < u.n; i0 += 2 * stride) {
    int lr[2];
    float mr[2], yr[2], xr[2][KMAX];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const long long i = i0 + r * stride;
      const bool ok = i < u.n;
      lr[r] = ok ? u.leaf_of_row[i] : 0;
      mr[r] = ok ? u.margin[i] : 0.f;
      yr[r] = (ok && u.grad) ? u.y[i] : 0.f;
#pragma unroll
      for (int k = 0; k < KMAX; ++k) xr[r][k] = (ok && k < K) ? u.Xfm[(long long)fk[k] * u.n + i] : 0.f;
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const long long i = i0 + r * stride;
      if (i >= u.n) break;
      const int l = lr[r];
      float c = sval[l];
      if (nets) {
        float lin[KMAX], lo[KMAX], hi[KMAX];
        const float4* p4 = reinterpret_cast<const float4*>(slin + (size_t)l * KMAX);
        const float4* q4 = reinterpret_cast<const float4*>(slo + (size_t)l * KMAX);
        const float4* r4 = reinterpret_cast<const float4*>(shi + (size_t)l * KMAX);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float4 a = p4[h], b = q4[h], d = r4[h];
          lin[4 * h] = a.x; lin[4 * h + 1] = a.y; lin[4 * h + 2] = a.z; lin[4 * h + 3] = a.w;
          lo[4 * h] = b.x; lo[4 * h + 1] = b.y; lo[4 * h + 2] = b.z; lo[4 * h + 3] = b.w;
          hi[4 * h] = d.x; hi[4 * h + 1] = d.y; hi[4 * h + 2] = d.z; hi[4 * h + 3] = d.w;
        }
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < KMAX; ++k) {
          if (k < K) {
            const float xc = fminf(fmaxf(xr[r][k], lo[k]), hi[k]);
            s = __fadd_rn(s, __fmul_rn(lin[k], xc));
          }
        }
        c = __fadd_rn(c, s);
      }
      const float m = __fadd_rn(mr[r], c);
      u.margin[i] = m;
      if (u.grad) {
        float g, h;
        loss_gh(u.loss, m, yr[r], &g, &h);
        u.grad[i] = g;
        if (u.hess) u.hess[i] = h;
      }
    }
  }
}

__global__ void k_grad_init(const float* margin, const float* y, long long n, int loss, float* grad, float* hess) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float g, h;
    loss_gh(loss, margin[i], y[i], &g, &h);
    grad[i] = g;
    if (hess) hess[i] = h;
  }
}

// ------------------------------------------------------------------ column moments
// mean and unbiased std of every feature column (fp64 two-pass), float32 results
__global__ void __launch_bounds__(512) k_colstats(const float* __restrict__ Xfm, long long n, float* mean, float* std) {
  __shared__ double s[512];
  const int f = blockIdx.x;
  const float* col = Xfm + (long long)f * n;
  double acc = 0.0;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) acc += (double)col[i];
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int o = 256; o; o >>= 1) { if (threadIdx.x < o) s[threadIdx.x] += s[threadIdx.x + o]; __syncthreads(); }
  const double mu = s[0] / (double)n;
  __syncthreads();
  acc = 0.0;
  for (long long i = threadIdx.x; i < n; i += blockDim.x) { const double d = (double)col[i] - mu; acc += d * d; }
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int o = 256; o; o >>= 1) { if (threadIdx.x < o) s[threadIdx.x] += s[threadIdx.x + o]; __syncthreads(); }
  if (threadIdx.x == 0) {
    mean[f] = (float)mu;
    std[f] = (float)sqrt(s[0] / (double)(n > 1 ? n - 1 : 1));
  }
}

// Row-sharded column moments: pass 0 writes acc[f] = sum x over this rank's
// rows; after acc[0..F) holds the all-ranks sum, pass 1 writes
// acc[F + f] = sum (x - mu)^2 with mu = acc[f] / n_total. Same block reduction
// as k_colstats, so one rank reproduces it exactly.
__global__ void __launch_bounds__(512) k_colsum(const float* __restrict__ Xfm, long long n, long long n_total,
                                                int F, int pass, double* acc) {
  __shared__ double s[512];
  const int f = blockIdx.x;
  const float* col = Xfm + (long long)f * n;
  const double mu = pass == 0 ? 0.0 : acc[f] / (double)n_total;
  double v = 0.0;
  if (pass == 0) for (long long i = threadIdx.x; i < n; i += blockDim.x) v += (double)col[i];
  else for (long long i = threadIdx.x; i < n; i += blockDim.x) { const double d = (double)col[i] - mu; v += d * d; }
  s[threadIdx.x] = v;
  __syncthreads();
  for (int o = 256; o; o >>= 1) { if (threadIdx.x < o) s[threadIdx.x] += s[threadIdx.x + o]; __syncthreads(); }
  if (threadIdx.x == 0) acc[pass * F + f] = s[0];
}

__global__ void k_colfinish(const double* acc, long long n_total, int F, float* mean, float* std) {
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= F) return;
  mean[f] = (float)(acc[f] / (double)n_total);
  std[f] = (float)sqrt(acc[F + f] / (double)(n_total > 1 ? n_total - 1 : 1));
}

// ------------------------------------------------------------------ interaction detector
// scores (F x F, float counts) += 1 for every (ancestor feature, node feature)
// pair with a != f along root-to-node paths, both directions
// (yabt/tree.py:186-203, yabt/adaptive_features.py:129-145)
__global__ void __launch_bounds__(512) k_ia_update(const long long* feature, const long long* left,
                                                   const long long* right, const int* meta, int F,
                                                   float* scores, int* parent) {
  const int nn = meta[0];
  for (int g = threadIdx.x; g < nn; g += blockDim.x) parent[g] = -1;
  __syncthreads();
  for (int g = threadIdx.x; g < nn; g += blockDim.x) {
    if (feature[g] >= 0) { parent[left[g]] = g; parent[right[g]] = g; }
  }
  __syncthreads();
  for (int g = threadIdx.x; g < nn; g += blockDim.x) {
    const long long f = feature[g];
    if (f < 0) continue;
    for (int p = parent[g]; p >= 0; p = parent[p]) {
      const long long a = feature[p];
      if (a == f) continue;
      atomicAdd(&scores[a * F + f], 1.f);
      atomicAdd(&scores[f * F + a], 1.f);
    }
  }
}

// normalized_matrix (yabt/adaptive_features.py:147-160): one block
__global__ void __launch_bounds__(1024) k_ia_normalize(const float* scores, int F, float* imat) {
  __shared__ float s_mx[32];
  __shared__ double s_sum[32];
  __shared__ long long s_cnt[32];
  const long long FF = (long long)F * F;
  float mx = 0.f;
  double sum = 0.0;
  long long cnt = 0;
  for (long long i = threadIdx.x; i < FF; i += blockDim.x) {
    const float v = scores[i];
    mx = fmaxf(mx, v);
    if (v > 0.f) { sum += (double)v; ++cnt; }
  }
  for (int o = 16; o; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    sum += __shfl_xor_sync(0xffffffffu, sum, o);
    cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  }
  if ((threadIdx.x & 31) == 0) { s_mx[threadIdx.x >> 5] = mx; s_sum[threadIdx.x >> 5] = sum; s_cnt[threadIdx.x >> 5] = cnt; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) { s_mx[0] = fmaxf(s_mx[0], s_mx[w]); s_sum[0] += s_sum[w]; s_cnt[0] += s_cnt[w]; }
  }
  __syncthreads();
  mx = s_mx[0];
  if (!(mx > 0.f)) {
    for (long long i = threadIdx.x; i < FF; i += blockDim.x) imat[i] = scores[i];
    return;
  }
  // bg = mean of the positive entries: float32 sum (exact for integer counts) / count
  const float bg = __fdiv_rn((float)s_sum[0], (float)s_cnt[0]);
  const float den = __fadd_rn(__fsub_rn(mx, bg), 1e-8f);
  for (long long i = threadIdx.x; i < FF; i += blockDim.x)
    imat[i] = fmaxf(__fdiv_rn(__fsub_rn(scores[i], bg), den), 0.f);
}

}  // namespace yabt

// ------------------------------------------------------------------ C ABI
using namespace yabt;

#define LCUDA(x)                                                                         \
  do {                                                                                   \
    cudaError_t e__ = (x);                                                               \
    if (e__ != cudaSuccess) {                                                            \
      set_error("%s: %s (%s:%d)", #x, cudaGetErrorString(e__), __FILE__, __LINE__);      \
      return YABT_ERR_CUDA;                                                              \
    }                                                                                    \
  } while (0)

extern "C" {

long long yabt_leafnet_workspace_bytes(long long n, int F, int max_nodes) {
  auto al = [](long long x) { return (x + 255) & ~255LL; };
  const long long max_chunks = n / GRAM_CHUNK + max_nodes + 1;
  long long b = 0;
  b += al((long long)F * 4);                 // fcount
  b += al(16);                               // flags
  b += al((long long)(F + 1 + max_nodes) * 8);   // stats: corr, gsum, leaf counts
  b += al(n * REC * 4);                      // rec
  b += 2 * al(max_chunks * KMAX * 4);        // pmin, pmax
  b += 3 * al((long long)max_nodes * 4);     // counts, leaf_first, leaf_nch
  b += 3 * al(max_chunks * 4);               // chunk arrays
  b += al(max_chunks * NE * 8);              // partials
  b += al((long long)max_nodes * NE * 8);    // totals
  b += al((long long)max_nodes * 2 * KMAX * 4);   // envelopes
  return b;
}

}  // extern "C"

namespace yabt {

static int leafnet_carve(const yabt_leafnet_args* p, void* workspace, long long ws_bytes, LeafNetArgs* out,
                         const char* who) {
  if (!p || !workspace || p->K < 1 || p->K > KMAX || p->n < 0 || p->F <= 0) {
    set_error("%s: bad arguments (K must be in [1, %d])", who, KMAX);
    return YABT_ERR_ARG;
  }
  if (ws_bytes < yabt_leafnet_workspace_bytes(p->n, p->F, p->max_nodes)) {
    set_error("%s: workspace too small", who);
    return YABT_ERR_WORKSPACE;
  }
  auto al = [](long long x) { return (x + 255) & ~255LL; };
  LeafNetArgs a;
  a.feature = (const long long*)p->feature; a.value = p->value; a.n_nodes_cap = p->max_nodes; a.meta = p->meta;
  a.leaf_src = p->leaf_src; a.leaf_begin = p->leaf_begin; a.leaf_count = p->leaf_count;
  a.fin = p->fin; a.list0 = p->list0; a.list1 = p->list1; a.leaf_of_row = p->leaf_of_row;
  a.Xfm = p->Xfm; a.col_mean = p->col_mean; a.col_std = p->col_std; a.margin = p->margin; a.y = p->y;
  a.n = p->n; a.F = p->F; a.K = p->K; a.loss = p->loss; a.min_samples = p->min_samples;
  a.l2 = p->l2; a.lr = p->learning_rate;
  a.feats = (long long*)p->feats; a.linear = p->linear; a.lo = p->lo; a.hi = p->hi; a.has_nets = p->has_nets;
  const long long max_chunks = p->n / GRAM_CHUNK + p->max_nodes + 1;
  char* w = (char*)workspace;
  a.fcount = (int*)w; w += al((long long)p->F * 4);
  a.flags = (int*)w; w += al(16);
  a.stats = (double*)w; w += al((long long)(p->F + 1 + p->max_nodes) * 8);
  a.corr = a.stats;
  a.gsum = a.stats + p->F;
  a.rec = (float*)w; w += al(p->n * REC * 4);
  a.pmin = (float*)w; w += al(max_chunks * KMAX * 4);
  a.pmax = (float*)w; w += al(max_chunks * KMAX * 4);
  a.counts = (int*)w; w += al((long long)p->max_nodes * 4);
  a.leaf_first = (int*)w; w += al((long long)p->max_nodes * 4);
  a.leaf_nch = (int*)w; w += al((long long)p->max_nodes * 4);
  a.chunk_leaf = (int*)w; w += al(max_chunks * 4);
  a.chunk_begin = (int*)w; w += al(max_chunks * 4);
  a.chunk_end = (int*)w; w += al(max_chunks * 4);
  a.partial = (double*)w; w += al(max_chunks * NE * 8);
  a.totals = (double*)w; w += al((long long)p->max_nodes * NE * 8);
  a.env = (float*)w;
  a.max_chunks = (int)max_chunks;
  a.chunk_rows = gram_rows(p->n);
  *out = a;
  return YABT_OK;
}

// Stage s of the leaf-model fit (see yabt_leafnet_stage in the header).
static cudaError_t leafnet_launch(const LeafNetArgs& a, int stage, cudaStream_t s) {
  const int nsm = YABT_SMS_HINT;
  const int nblk = (a.n_nodes_cap + 3) / 4;
  PhaseScope ph(PH_LEAFNET, s);
  switch (stage) {
    case 0: {
      k_ln_select<<<1, 1024, 0, s>>>(a);
      if (a.n > 0) {
        dim3 grid((unsigned)std::min<long long>((a.n + 255) / 256, 4LL * nsm), (unsigned)((a.F + 7) / 8));
        k_ln_corr<<<grid, 256, 0, s>>>(a);
        count_launches(1);
      }
      count_launches(1);
      break;
    }
    case 1: {
      k_ln_pad<<<1, 1024, 0, s>>>(a);
      if (a.n > 0) {
        const int grid = (int)std::min<long long>((a.n + 255) / 256, 16LL * nsm);
        k_ln_rows<<<grid, 256, 0, s>>>(a);
        count_launches(1);
      }
      k_ln_plan<<<1, 1024, 0, s>>>(a);
      k_ln_elig<<<1, 1024, 0, s>>>(a);
      k_ln_gram<<<(unsigned)std::min<long long>(a.max_chunks, a.n / a.chunk_rows + a.n_nodes_cap + 1), 256, 0,
                  s>>>(a);
      k_ln_total<<<nblk, 128, 0, s>>>(a);
      count_launches(5);
      break;
    }
    default: {
      k_ln_solve<<<nblk, 128, 0, s>>>(a);
      count_launches(1);
      break;
    }
  }
  return cudaGetLastError();
}

}  // namespace yabt

extern "C" {

// Fit ridge-linear leaf models for one grown tree and fold them into
// value / linear / lo / hi (yabt/neural_leaves.py:131-184).
int yabt_leafnet_fit(const yabt_leafnet_args* p, void* workspace, long long ws_bytes, void* stream) {
  LeafNetArgs a;
  int rc = leafnet_carve(p, workspace, ws_bytes, &a, "yabt_leafnet_fit");
  if (rc) return rc;
  if (p->n <= 0) { set_error("yabt_leafnet_fit: n must be > 0"); return YABT_ERR_ARG; }
  for (int st = 0; st < 3; ++st) LCUDA(leafnet_launch(a, st, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_leafnet_stage(const yabt_leafnet_args* p, int stage, void* workspace, long long ws_bytes, void* stream) {
  LeafNetArgs a;
  int rc = leafnet_carve(p, workspace, ws_bytes, &a, "yabt_leafnet_stage");
  if (rc) return rc;
  if (stage < 0 || stage > 2) { set_error("yabt_leafnet_stage: stage must be 0..2"); return YABT_ERR_ARG; }
  LCUDA(leafnet_launch(a, stage, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_leafnet_bufs(const yabt_leafnet_args* p, void* workspace, long long ws_bytes, void** stats,
                      long long* stats_count, void** totals, long long* totals_count, void** envelope,
                      long long* envelope_count) {
  LeafNetArgs a;
  int rc = leafnet_carve(p, workspace, ws_bytes, &a, "yabt_leafnet_bufs");
  if (rc) return rc;
  if (stats) *stats = a.stats;
  if (stats_count) *stats_count = (long long)p->F + 1 + p->max_nodes;
  if (totals) *totals = a.totals;
  if (totals_count) *totals_count = (long long)p->max_nodes * NE;
  if (envelope) *envelope = a.env;
  if (envelope_count) *envelope_count = (long long)p->max_nodes * 2 * KMAX;
  return YABT_OK;
}

int yabt_update_margin(const yabt_update_args* p, void* stream) {
  if (!p || !p->leaf_of_row || !p->value || !p->margin || p->n < 0) { set_error("yabt_update_margin: bad arguments"); return YABT_ERR_ARG; }
  UpdateArgs u;
  u.leaf_of_row = p->leaf_of_row; u.value = p->value; u.linear = p->linear; u.lo = p->lo; u.hi = p->hi;
  u.feats = (const long long*)p->feats; u.has_nets = p->has_nets; u.K = p->K; u.Xfm = p->Xfm; u.n = p->n;
  u.margin = p->margin; u.y = p->y; u.grad = p->grad; u.hess = p->hess; u.loss = p->loss;
  if (p->n == 0) return YABT_OK;
  if (p->max_nodes <= 0) { set_error("yabt_update_margin: max_nodes must be > 0"); return YABT_ERR_ARG; }
  const size_t smem = (size_t)p->max_nodes * (p->linear ? 1 + 3 * KMAX : 1) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k_update, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) { set_error("k_update smem: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  }
  // one wave of resident blocks (the tables are staged once per block)
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_update, 256, smem) != cudaSuccess || occ < 1) occ = 1;
  const int grid = (int)std::min<long long>((p->n + 511) / 512, (long long)YABT_SMS_HINT * occ);
  PhaseScope ph(PH_UPDATE, (cudaStream_t)stream);
  k_update<<<grid, 256, smem, (cudaStream_t)stream>>>(u, p->max_nodes);
  count_launches(1);
  LCUDA(cudaGetLastError());
  return YABT_OK;
}

int yabt_grad_init(const float* margin, const float* y, long long n, int loss, float* grad, float* hess, void* stream) {
  if (!margin || !y || !grad || n < 0) { set_error("yabt_grad_init: bad arguments"); return YABT_ERR_ARG; }
  if (n == 0) return YABT_OK;
  const int grid = (int)std::min<long long>((n + 255) / 256, (long long)YABT_SMS_HINT * 8);
  PhaseScope ph(PH_UPDATE, (cudaStream_t)stream);
  k_grad_init<<<grid, 256, 0, (cudaStream_t)stream>>>(margin, y, n, loss, grad, hess);
  count_launches(1);
  LCUDA(cudaGetLastError());
  return YABT_OK;
}

int yabt_column_stats(const float* Xfm, long long n, int F, float* mean, float* std, void* stream) {
  if (!Xfm || n <= 0 || F <= 0 || !mean || !std) { set_error("yabt_column_stats: bad arguments"); return YABT_ERR_ARG; }
  k_colstats<<<F, 512, 0, (cudaStream_t)stream>>>(Xfm, n, mean, std);
  count_launches(1);
  LCUDA(cudaGetLastError());
  return YABT_OK;
}

int yabt_column_sums(const float* Xfm, long long n, long long n_total, int F, int pass, double* acc, void* stream) {
  if ((n > 0 && !Xfm) || n < 0 || n_total <= 0 || F <= 0 || pass < 0 || pass > 1 || !acc) {
    set_error("yabt_column_sums: bad arguments");
    return YABT_ERR_ARG;
  }
  k_colsum<<<F, 512, 0, (cudaStream_t)stream>>>(Xfm, n, n_total, F, pass, acc);
  count_launches(1);
  LCUDA(cudaGetLastError());
  return YABT_OK;
}

int yabt_column_finish(const double* acc, long long n_total, int F, float* mean, float* std, void* stream) {
  if (!acc || n_total <= 0 || F <= 0 || !mean || !std) { set_error("yabt_column_finish: bad arguments"); return YABT_ERR_ARG; }
  k_colfinish<<<(F + 255) / 256, 256, 0, (cudaStream_t)stream>>>(acc, n_total, F, mean, std);
  count_launches(1);
  LCUDA(cudaGetLastError());
  return YABT_OK;
}

int yabt_interaction_update(const int64_t* feature, const int64_t* left, const int64_t* right, const int32_t* meta,
                            int F, int max_nodes, float* scores, int32_t* parent_scratch, void* stream) {
  if (!feature || !left || !right || !meta || !scores || !parent_scratch || F <= 0) {
    set_error("yabt_interaction_update: bad arguments");
    return YABT_ERR_ARG;
  }
  (void)max_nodes;
  PhaseScope ph(PH_INTERACT, (cudaStream_t)stream);
  k_ia_update<<<1, 512, 0, (cudaStream_t)stream>>>((const long long*)feature, (const long long*)left,
                                                   (const long long*)right, meta, F, scores, parent_scratch);
  count_launches(1);
  LCUDA(cudaGetLastError());
  return YABT_OK;
}

int yabt_interaction_normalize(const float* scores, int F, float* imat, void* stream) {
  if (!scores || !imat || F <= 0) { set_error("yabt_interaction_normalize: bad arguments"); return YABT_ERR_ARG; }
  PhaseScope ph(PH_INTERACT, (cudaStream_t)stream);
  k_ia_normalize<<<1, 1024, 0, (cudaStream_t)stream>>>(scores, F, imat);
  count_launches(1);
  LCUDA(cudaGetLastError());
  return YABT_OK;
}

}  // extern "C"
