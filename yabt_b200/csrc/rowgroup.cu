// Stable grouping of row ids by leaf: for leaf l, rows[begin[l] ..
// begin[l] + count[l]) are the rows i with leaf_of_row[i] == l in increasing
// order. The leaf models read their rows through such ranges; after a tree is
// grown on a row sample, every row's leaf comes from yabt_grow_apply_all and
// this grouping gives the leaf models all rows (yabt/boosting.py:486-497 fits
// them on the full training set).
//
//   k_grp_count   block per chunk of GRP_CHUNK rows: rows per leaf -> cnt[leaf][chunk]
//   k_grp_scan    block per leaf: exclusive scan over the chunks -> off[leaf][chunk], total
//   k_grp_begin   one block: begin = exclusive scan of the totals over leaves
//   k_grp_place   block per chunk, 8 warps on 8 consecutive sub-ranges: per-warp
//                 counts, their prefix over warps, then each warp places its rows
//                 in order (rank among equal leaves in a 32-row batch by
//                 __match_any_sync). Deterministic, no global atomics.
#include <algorithm>

#include "../../include/yabt_b200.h"
#include "common.cuh"

namespace yabt {
namespace {

constexpr int GRP_CHUNK = 8192;
constexpr int GRP_WARPS = 8;

__global__ void __launch_bounds__(256) k_grp_count(const int* __restrict__ leaf, long long n, int L,
                                                   int nch, int* __restrict__ cnt, int* __restrict__ err) {
  extern __shared__ int sc[];      // [L]
  for (int i = threadIdx.x; i < L; i += blockDim.x) sc[i] = 0;
  __syncthreads();
  const long long r0 = (long long)blockIdx.x * GRP_CHUNK;
  const long long r1 = min(n, r0 + GRP_CHUNK);
  bool bad = false;
  for (long long i = r0 + threadIdx.x; i < r1; i += blockDim.x) {
    const int l = leaf[i];
    if (l < 0 || l >= L) { bad = true; continue; }
    atomicAdd(&sc[l], 1);
  }
  if (bad) atomicOr(err, 1);
  __syncthreads();
  for (int l = threadIdx.x; l < L; l += blockDim.x) cnt[(long long)l * nch + blockIdx.x] = sc[l];
}

__global__ void __launch_bounds__(256) k_grp_scan(int* __restrict__ cnt, int nch, int* __restrict__ total) {
  __shared__ int sw[8];
  __shared__ int s_carry;
  const int l = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int* row = cnt + (long long)l * nch;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  for (int c0 = 0; c0 < nch; c0 += blockDim.x) {
    const int c = c0 + threadIdx.x;
    const int v = c < nch ? row[c] : 0;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) { const int y = __shfl_up_sync(0xffffffffu, x, o); if (lane >= o) x += y; }
    if (lane == 31) sw[warp] = x;
    __syncthreads();
    int wpre = 0;
    for (int w = 0; w < warp; ++w) wpre += sw[w];
    const int carry = s_carry;
    if (c < nch) row[c] = carry + wpre + x - v;      // exclusive offset within the leaf
    __syncthreads();
    if (threadIdx.x == 0) { int t = 0; for (int w = 0; w < 8; ++w) t += sw[w]; s_carry = carry + t; }
    __syncthreads();
  }
  if (threadIdx.x == 0) total[l] = s_carry;
}

__global__ void __launch_bounds__(1024) k_grp_begin(const int* __restrict__ total, int L, int* __restrict__ begin,
                                                    int* __restrict__ count) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  int carry = 0;
  for (int l0 = 0; l0 < L; l0 += 32) {
    const int l = l0 + lane;
    const int v = l < L ? total[l] : 0;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) { const int y = __shfl_up_sync(0xffffffffu, x, o); if (lane >= o) x += y; }
    if (l < L) { begin[l] = carry + x - v; count[l] = v; }
    carry += __shfl_sync(0xffffffffu, x, 31);
  }
}

__global__ void __launch_bounds__(GRP_WARPS * 32) k_grp_place(const int* __restrict__ leaf, long long n, int L, int nch,
                                                              const int* __restrict__ off, const int* __restrict__ begin,
                                                              int* __restrict__ rows) {
  extern __shared__ int sm[];      // wc[GRP_WARPS][L] counts, then running positions
  int* wc = sm;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long r0 = (long long)blockIdx.x * GRP_CHUNK;
  const long long r1 = min(n, r0 + GRP_CHUNK);
  const long long per = (GRP_CHUNK + GRP_WARPS - 1) / GRP_WARPS;
  const long long w0 = min(r1, r0 + warp * per), w1 = min(r1, w0 + per);
  for (int i = threadIdx.x; i < GRP_WARPS * L; i += blockDim.x) wc[i] = 0;
  __syncthreads();
  int* my = wc + warp * L;
  // per-warp counts (one leader per group of equal leaves: no conflicts)
  for (long long b = w0; b < w1; b += 32) {
    const long long i = b + lane;
    const int l = i < w1 ? leaf[i] : -1;
    const bool ok = l >= 0 && l < L;
    const unsigned peers = __match_any_sync(0xffffffffu, ok ? l : -1);
    if (ok && lane == __ffs(peers) - 1) my[l] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  // start of each warp's rows of leaf l: begin + chunk offset + earlier warps
  for (int l = threadIdx.x; l < L; l += blockDim.x) {
    int run = begin[l] + off[(long long)l * nch + blockIdx.x];
    for (int w = 0; w < GRP_WARPS; ++w) {
      const int c = wc[w * L + l];
      wc[w * L + l] = run;
      run += c;
    }
  }
  __syncthreads();
  for (long long b = w0; b < w1; b += 32) {
    const long long i = b + lane;
    const int l = i < w1 ? leaf[i] : -1;
    const bool ok = l >= 0 && l < L;
    const unsigned peers = __match_any_sync(0xffffffffu, ok ? l : -1);
    if (ok) rows[my[l] + __popc(peers & ((1u << lane) - 1u))] = (int)i;
    __syncwarp();
    if (ok && lane == __ffs(peers) - 1) my[l] += __popc(peers);
    __syncwarp();
  }
}

long long grp_carve(long long n, int L, char* base, int** cnt, int** total, int** err) {
  const int nch = (int)((n + GRP_CHUNK - 1) / GRP_CHUNK);
  auto al = [](long long x) { return (x + 255) & ~255LL; };
  long long o = 0;
  if (cnt) *cnt = reinterpret_cast<int*>(base + o);
  o += al(4LL * L * std::max(nch, 1));
  if (total) *total = reinterpret_cast<int*>(base + o);
  o += al(4LL * L);
  if (err) *err = reinterpret_cast<int*>(base + o);
  o += al(4);
  return o;
}

}  // namespace
}  // namespace yabt

using namespace yabt;

extern "C" {

long long yabt_group_rows_workspace_bytes(long long n, int num_leaves) {
  if (n < 0 || num_leaves <= 0) return -1;
  return grp_carve(n, num_leaves, nullptr, nullptr, nullptr, nullptr);
}

int yabt_group_rows(const int32_t* leaf_of_row, long long n, int num_leaves, void* workspace, long long ws_bytes,
                    int32_t* begin, int32_t* count, int32_t* rows, void* stream) {
  if (n < 0 || n > INT32_MAX || num_leaves <= 0 || num_leaves > 4096 || !begin || !count ||
      (n > 0 && (!leaf_of_row || !rows)) || !workspace) {
    set_error("yabt_group_rows: bad arguments (num_leaves <= 4096)");
    return YABT_ERR_ARG;
  }
  if (ws_bytes < yabt_group_rows_workspace_bytes(n, num_leaves)) {
    set_error("yabt_group_rows: workspace too small");
    return YABT_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PhaseScope ph(PH_PARTITION, s);
  int *cnt, *total, *err;
  grp_carve(n, num_leaves, static_cast<char*>(workspace), &cnt, &total, &err);
  const int nch = (int)((n + GRP_CHUNK - 1) / GRP_CHUNK);
  const int L = num_leaves;
  cudaError_t e = cudaMemsetAsync(err, 0, 4, s);
  if (e == cudaSuccess && nch == 0) e = cudaMemsetAsync(total, 0, 4LL * L, s);
  if (e == cudaSuccess && nch > 0) {
    const size_t place_smem = (size_t)GRP_WARPS * L * 4;
    if (place_smem > 48 * 1024)
      e = cudaFuncSetAttribute(k_grp_place, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)place_smem);
    if (e == cudaSuccess) {
      k_grp_count<<<nch, 256, (size_t)L * 4, s>>>(leaf_of_row, n, L, nch, cnt, err);
      k_grp_scan<<<L, 256, 0, s>>>(cnt, nch, total);
      count_launches(2);
    }
  }
  if (e == cudaSuccess) {
    k_grp_begin<<<1, 1024, 0, s>>>(total, L, begin, count);
    count_launches(1);
    if (nch > 0) {
      k_grp_place<<<nch, GRP_WARPS * 32, (size_t)GRP_WARPS * L * 4, s>>>(leaf_of_row, n, L, nch, cnt, begin, rows);
      count_launches(1);
    }
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) { set_error("yabt_group_rows: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

}  // extern "C"
