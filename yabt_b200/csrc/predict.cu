// Inference: batched multi-tree prediction and single-tree routing.
//
// Restates Tree.apply / Tree.predict / Tree.net_contribution
// (yabt/tree.py:82-135) and Booster._margin (yabt/boosting.py:542-550):
// out[i] = base + sum_t ( value_t[leaf_t(x_i)] + sum_k linear_t[leaf, k] *
// clamp(x_i[feat_tk], lo_t[leaf, k], hi_t[leaf, k]) ), trees in order, float32
// additions in the reference's order (per tree: value + net, then margin +
// contribution). One warp per 32 rows; every lane walks its row through all
// trees of the packed forest (nodes of all trees concatenated, child indices
// local to their tree).
#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "../../include/yabt_b200.h"

namespace yabt {

__global__ void __launch_bounds__(256)
k_predict_forest(const float* __restrict__ X, long long n, int F, int ntrees,
                 const long long* __restrict__ tree_off, const int* __restrict__ feature,
                 const float* __restrict__ threshold, const int* __restrict__ left,
                 const int* __restrict__ right, const float* __restrict__ value,
                 const int* __restrict__ has_nets, const long long* __restrict__ feats, int K,
                 const float* __restrict__ linear, const float* __restrict__ lo,
                 const float* __restrict__ hi, float base, float* __restrict__ out) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float* x = X + i * F;
  float m = base;
  for (int t = 0; t < ntrees; ++t) {
    const long long o = tree_off[t];
    int node = 0;
    for (int d = 0; d < 4096; ++d) {           // bounded walk (trees are finite)
      const int f = __ldg(feature + o + node);
      if (f < 0) break;
      node = (__ldg(x + f) <= __ldg(threshold + o + node)) ? __ldg(left + o + node) : __ldg(right + o + node);
    }
    float c = __ldg(value + o + node);
    if (has_nets && has_nets[t]) {
      float s = 0.f;
      const long long b = (o + node) * K;
      for (int k = 0; k < K; ++k) {
        const float xv = __ldg(x + feats[(long long)t * K + k]);
        const float xc = fminf(fmaxf(xv, __ldg(lo + b + k)), __ldg(hi + b + k));
        s = __fadd_rn(s, __fmul_rn(__ldg(linear + b + k), xc));
      }
      c = __fadd_rn(c, s);
    }
    m = __fadd_rn(m, c);
  }
  out[i] = m;
}

__global__ void k_apply_tree(const float* __restrict__ X, long long n, int F, const long long* __restrict__ feature,
                             const float* __restrict__ threshold, const long long* __restrict__ left,
                             const long long* __restrict__ right, long long* __restrict__ out) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float* x = X + i * F;
  long long node = 0;
  for (int d = 0; d < 4096; ++d) {
    const long long f = feature[node];
    if (f < 0) break;
    node = (x[f] <= threshold[node]) ? left[node] : right[node];
  }
  out[i] = node;
}

__global__ void k_impute_rows(float* __restrict__ X, long long n, int F, const float* __restrict__ medians) {
  const long long total = n * F;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const float v = X[e];
    if (isnan(v)) X[e] = medians[e % F];
  }
}

}  // namespace yabt

using namespace yabt;

extern "C" {

int yabt_predict_forest(const float* X, long long n, int F, int ntrees, const int64_t* tree_off,
                        const int32_t* feature, const float* threshold, const int32_t* left,
                        const int32_t* right, const float* value, const int32_t* has_nets,
                        const int64_t* feats, int K, const float* linear, const float* lo, const float* hi,
                        float base, float* out, void* stream) {
  if (n == 0 && F > 0 && ntrees >= 0) return YABT_OK;   // no rows: nothing is read (buffers may be NULL)
  if (!X || n < 0 || F <= 0 || ntrees < 0 || !out || (ntrees > 0 && (!tree_off || !feature || !threshold ||
      !left || !right || !value))) {
    set_error("yabt_predict_forest: bad arguments");
    return YABT_ERR_ARG;
  }
  if (n == 0) return YABT_OK;
  k_predict_forest<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      X, n, F, ntrees, (const long long*)tree_off, feature, threshold, left, right, value, has_nets,
      (const long long*)feats, K, linear, lo, hi, base, out);
  count_launches(1);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { set_error("yabt_predict_forest: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

int yabt_apply_tree(const float* X, long long n, int F, const int64_t* feature, const float* threshold,
                    const int64_t* left, const int64_t* right, int64_t* out, void* stream) {
  if (n == 0 && F > 0) return YABT_OK;   // no rows: nothing is read (buffers may be NULL)
  if (!X || n < 0 || F <= 0 || !feature || !threshold || !left || !right || !out) {
    set_error("yabt_apply_tree: bad arguments");
    return YABT_ERR_ARG;
  }
  if (n == 0) return YABT_OK;
  k_apply_tree<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      X, n, F, (const long long*)feature, threshold, (const long long*)left, (const long long*)right,
      (long long*)out);
  count_launches(1);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { set_error("yabt_apply_tree: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

int yabt_impute_rows(float* X, long long n, int F, const float* medians, void* stream) {
  if (n == 0 && F > 0) return YABT_OK;   // no rows: nothing is read (buffers may be NULL)
  if (!X || n < 0 || F <= 0 || !medians) { set_error("yabt_impute_rows: bad arguments"); return YABT_ERR_ARG; }
  if (n == 0) return YABT_OK;
  const int grid = (int)std::min<long long>((n * F + 255) / 256, (long long)YABT_SMS_HINT * 16);
  k_impute_rows<<<grid, 256, 0, (cudaStream_t)stream>>>(X, n, F, medians);
  count_launches(1);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { set_error("yabt_impute_rows: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

}  // extern "C"
