// Quantile binning on the device, bit-exact with the reference's numpy path.
//
// Restates Binner.fit / transform / impute (yabt/binning.py:29-124):
//   medians   np.nanmedian over ALL rows of each feature (binning.py:32-33):
//             3-pass MSB radix select (11/11/10-bit digits) of the two middle
//             order statistics of the non-NaN values; median = f32(a+b)/2.
//   edges     quantiles k/max_bins (k = 1..max_bins-1) of the non-NaN values of
//             a row sample (all rows if n <= 200000, else the host-drawn
//             default_rng(0).choice indices, binning.py:36-40), computed with
//             numpy's 'linear' method in float64 without FMA contraction, cast
//             to float32 and de-duplicated (binning.py:56-61). The sample
//             columns are sorted by a bitonic network (keys = order-preserving
//             u32 of the floats, NaN and padding sort last).
//   scales    q75 - q25 of the same sample, else the column std, else 1 (:62-66).
//   transform NaN -> median, bin = #{edges < x} (searchsorted left) written as
//             uint8 into the tiled bin layout; the imputed feature-major float
//             matrix is kept for the leaf models and the margin update.
#include <algorithm>
#include <cstdint>
#include <vector>

#include "common.cuh"

namespace yabt {

constexpr unsigned KEY_NAN = 0xFFFFFFFFu;

__device__ __forceinline__ unsigned fkey(float x) { return isnan(x) ? KEY_NAN : f2ord(x); }

// ---------------------------------------------------------------- transpose
// X (n, F) row-major -> Xfm (F, n)
// rows [0, n) of X (n, F) row-major -> Xfm[f * ld + r]
__global__ void k_transpose(const float* __restrict__ X, long long n, int F, float* __restrict__ Xfm, long long ld) {
  __shared__ float t[32][33];
  const long long r0 = (long long)blockIdx.x * 32;
  const int f0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const long long r = r0 + i;
    const int f = f0 + tx;
    t[i][tx] = (r < n && f < F) ? X[r * F + f] : 0.f;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int f = f0 + i;
    const long long r = r0 + tx;
    if (f < F && r < n) Xfm[(long long)f * ld + r] = t[tx][i];
  }
}

// ---------------------------------------------------------------- radix select (medians)
// sel[F]: struct of per-feature selection state
struct SelState {
  unsigned prefix[2];   // key bits selected so far for targets 0/1
  long long k[2];       // remaining rank inside the current prefix
  long long m;          // non-NaN count
  int done;             // 1 if m == 0
  int pad;
};

__device__ __forceinline__ int sel_shift(int pass) { return pass == 0 ? 21 : (pass == 1 ? 10 : 0); }
__device__ __forceinline__ int sel_bits(int pass) { return pass == 2 ? 10 : 11; }

// grid: (chunks, F); histogram of the pass digit for elements matching each target prefix
__global__ void k_sel_hist(const float* __restrict__ Xfm, long long n, int pass,
                           const SelState* __restrict__ sel, unsigned* __restrict__ hist,
                           unsigned long long* __restrict__ nan_count) {
  __shared__ unsigned sh[2][2048];
  const int f = blockIdx.y;
  const int shift = sel_shift(pass), bits = sel_bits(pass);
  const unsigned dmask = (1u << bits) - 1u;
  unsigned pre0 = 0, pre1 = 0;
  bool two = false;
  if (pass > 0) {
    const SelState s = sel[f];
    if (s.done) return;
    pre0 = s.prefix[0]; pre1 = s.prefix[1];
    two = pre0 != pre1;
  }
  for (int i = threadIdx.x; i < 2 * 2048; i += blockDim.x) (&sh[0][0])[i] = 0;
  __syncthreads();
  const float* col = Xfm + (long long)f * n;
  const int hshift = shift + bits;       // bits above the digit
  unsigned nn = 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const unsigned key = fkey(col[i]);
    if (key == KEY_NAN) { ++nn; continue; }
    const unsigned d = (key >> shift) & dmask;
    const unsigned hi = hshift >= 32 ? 0u : (key >> hshift);
    if (pass == 0 || hi == pre0) atomicAdd(&sh[0][d], 1u);
    if (two && hi == pre1) atomicAdd(&sh[1][d], 1u);
  }
  if (pass == 0) {
    for (int o = 16; o; o >>= 1) nn += __shfl_xor_sync(0xffffffffu, nn, o);
    if ((threadIdx.x & 31) == 0 && nn) atomicAdd(&nan_count[f], (unsigned long long)nn);
  }
  __syncthreads();
  unsigned* gh = hist + (size_t)f * 2 * 2048;
  for (int i = threadIdx.x; i < 2048; i += blockDim.x) {
    if (sh[0][i]) atomicAdd(&gh[i], sh[0][i]);
    if (two && sh[1][i]) atomicAdd(&gh[2048 + i], sh[1][i]);
  }
}

// one warp per feature: for both targets, pick the digit bucket holding the
// remaining rank (state is read before it is updated, in warp order)
__global__ void k_sel_pick(long long n, int F, int pass, SelState* __restrict__ sel,
                           const unsigned* __restrict__ hist, const unsigned long long* __restrict__ nan_count) {
  const int f = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (f >= F) return;
  SelState st = sel[f];
  if (pass == 0) {
    st.m = n - (long long)nan_count[f];
    st.done = st.m == 0;
    st.prefix[0] = st.prefix[1] = 0;
    st.k[0] = (st.m - 1) / 2;
    st.k[1] = st.m / 2;
  }
  if (st.done) { if (lane == 0) sel[f] = st; return; }
  const bool two = pass > 0 && st.prefix[0] != st.prefix[1];
  const int bits = sel_bits(pass);
  const int nb = 1 << bits;
  for (int t = 0; t < 2; ++t) {
    const unsigned* h = hist + (size_t)f * 2 * 2048 + ((two && t == 1) ? 2048 : 0);
    const long long k = st.k[t];
    long long run = 0, before = 0;
    int found = -1;
    for (int base = 0; base < nb && found < 0; base += 32) {
      const long long c = h[base + lane];
      long long x = c;
      for (int o = 1; o < 32; o <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      const bool hit = (run + x > k) && (run + x - c <= k);
      const unsigned bal = __ballot_sync(0xffffffffu, hit);
      if (bal) {
        const int l = __ffs(bal) - 1;
        found = base + l;
        before = __shfl_sync(0xffffffffu, run + x - c, l);
      }
      run += __shfl_sync(0xffffffffu, x, 31);
    }
    if (found >= 0) {
      st.prefix[t] = (pass == 0 ? 0u : (st.prefix[t] << bits)) | (unsigned)found;
      st.k[t] = k - before;
    }
  }
  if (lane == 0) sel[f] = st;
}

__global__ void k_sel_zero(unsigned* hist, long long count) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count;
       i += (long long)gridDim.x * blockDim.x) hist[i] = 0;
}

__global__ void k_sel_final(int F, const SelState* __restrict__ sel, float* __restrict__ medians) {
  const int f = blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= F) return;
  const SelState s = sel[f];
  if (s.done) { medians[f] = 0.f; return; }   // all-NaN column -> 0 (binning.py:33)
  const float a = ord2f(s.prefix[0]), b = ord2f(s.prefix[1]);
  medians[f] = (s.m & 1) ? a : __fdiv_rn(__fadd_rn(a, b), 2.f);
}

// ---------------------------------------------------------------- sample + bitonic sort
// keys[F][P]: sample column keys (row idx[i] or i), NaN / padding -> KEY_NAN
__global__ void k_sample_keys(const float* __restrict__ Xfm, long long n, int F, const int* __restrict__ idx,
                              long long nq, long long P, unsigned* __restrict__ keys) {
  const long long total = (long long)F * P;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int f = (int)(e / P);
    const long long i = e % P;
    unsigned k = KEY_NAN;
    if (i < nq) {
      const long long r = idx ? (long long)idx[i] : i;
      k = fkey(Xfm[(long long)f * n + r]);
    }
    keys[e] = k;
  }
}

constexpr int BL = 2048;   // elements per shared-memory bitonic block (1024 threads x 2)

// all stages k <= min(P, BL) inside each block-sized chunk
__global__ void __launch_bounds__(1024) k_bitonic_local(unsigned* __restrict__ keys, long long P, int kmax) {
  __shared__ unsigned s[BL];
  const int L = (int)min((long long)BL, P);            // chunk = L elements of one column
  const long long base = (long long)blockIdx.x * L;
  for (int i = threadIdx.x; i < L; i += blockDim.x) s[i] = keys[base + i];
  __syncthreads();
  const long long colbase = (base / P) * P;            // chunk lies inside one column
  for (int k = 2; k <= kmax; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < L; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const long long gi = base + i - colbase;
          const bool asc = (gi & k) == 0;
          const unsigned a = s[i], b = s[ixj];
          if ((a > b) == asc) { s[i] = b; s[ixj] = a; }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < L; i += blockDim.x) keys[base + i] = s[i];
}

// merge stage k: strides j < BL inside shared memory
__global__ void __launch_bounds__(1024) k_bitonic_merge_local(unsigned* __restrict__ keys, long long P, long long k) {
  __shared__ unsigned s[BL];
  const long long base = (long long)blockIdx.x * BL;
  for (int i = threadIdx.x; i < BL; i += blockDim.x) s[i] = keys[base + i];
  __syncthreads();
  const long long colbase = (base / P) * P;
  for (int j = BL >> 1; j > 0; j >>= 1) {
    for (int i = threadIdx.x; i < BL; i += blockDim.x) {
      const int ixj = i ^ j;
      if (ixj > i) {
        const long long gi = base + i - colbase;
        const bool asc = (gi & k) == 0;
        const unsigned a = s[i], b = s[ixj];
        if ((a > b) == asc) { s[i] = b; s[ixj] = a; }
      }
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < BL; i += blockDim.x) keys[base + i] = s[i];
}

// one global compare-exchange stage (stride j >= BL)
__global__ void k_bitonic_global(unsigned* __restrict__ keys, long long P, int F, long long k, long long j) {
  const long long half = (long long)F * P / 2;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < half;
       t += (long long)gridDim.x * blockDim.x) {
    // t-th pair: low index i has bit j clear
    const int lj = __ffsll(j) - 1;                    // log2(j)
    const long long lo = t & (j - 1), hi = t >> lj;
    const long long i = (hi << (lj + 1)) | lo;        // insert a 0 bit at position lj
    const long long ixj = i | j;
    const long long gi = i % P;
    const bool asc = (gi & k) == 0;
    const unsigned a = keys[i], b = keys[ixj];
    if ((a > b) == asc) { keys[i] = b; keys[ixj] = a; }
  }
}

// ---------------------------------------------------------------- quantiles
// numpy 'linear' quantile of sorted float keys (m valid) at q, float64 result
__device__ double quantile_sorted(const unsigned* s, long long m, double q) {
  const double v = __dmul_rn((double)(m - 1), q);
  double lo = floor(v);
  const bool top = v >= (double)(m - 1);
  if (top) lo = -1.0;
  const double t = __dsub_rn(v, lo);
  const long long li = top ? m - 1 : (long long)lo;
  const long long hi = top ? m - 1 : li + 1;
  const float a = ord2f(s[li]), b = ord2f(s[hi]);
  const double d = (double)__fsub_rn(b, a);
  if (t >= 0.5) return __dsub_rn((double)b, __dmul_rn(d, __dsub_rn(1.0, t)));
  return __dadd_rn((double)a, __dmul_rn(d, t));
}

// one block (256 threads) per feature: edges (sorted unique float32 quantiles) and scale
__global__ void __launch_bounds__(256)
k_quantiles(const unsigned* __restrict__ keys, long long P, int max_bins, float* __restrict__ edges,
            int* __restrict__ ecnt, float* __restrict__ scales) {
  __shared__ float q[256];
  __shared__ long long s_m;
  __shared__ double s_sum[256];
  const int f = blockIdx.x;
  const unsigned* col = keys + (long long)f * P;
  if (threadIdx.x == 0) {
    long long lo = 0, hi = P;                 // first KEY_NAN
    while (lo < hi) { const long long mid = (lo + hi) >> 1; if (col[mid] < KEY_NAN) lo = mid + 1; else hi = mid; }
    s_m = lo;
  }
  __syncthreads();
  const long long m = s_m;
  // an all-NaN sample column is quantised as the single value 0 (binning.py:57-58)
  const unsigned zero_key = f2ord(0.f);
  const unsigned* src = m > 0 ? col : &zero_key;
  const long long mm = m > 0 ? m : 1;
  const int nq = max_bins - 1;
  const double step = 1.0 / (double)max_bins;
  const int t = threadIdx.x;
  q[t] = INFINITY;
  if (t < nq) q[t] = (float)quantile_sorted(src, mm, __dmul_rn((double)(t + 1), step));
  __syncthreads();
  // bitonic sort of 256 floats (np.unique sorts); +inf padding
  for (int k = 2; k <= 256; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      const int ixj = t ^ j;
      if (ixj > t) {
        const bool asc = (t & k) == 0;
        const float a = q[t], b = q[ixj];
        if ((a > b) == asc) { q[t] = b; q[ixj] = a; }
      }
      __syncthreads();
    }
  // unique: keep first of each run of equal values among the nq real entries
  const bool keep = t < nq && (t == 0 || !(q[t] == q[t - 1]));
  const unsigned bal = __ballot_sync(0xffffffffu, keep);
  __shared__ int wc[8];
  if ((t & 31) == 0) wc[t >> 5] = __popc(bal);
  __syncthreads();
  int off = 0;
  for (int w = 0; w < (t >> 5); ++w) off += wc[w];
  off += __popc(bal & ((1u << (t & 31)) - 1u));
  if (keep) edges[(long long)f * 255 + off] = q[t];
  if (t == 0) { int tot = 0; for (int w = 0; w < 8; ++w) tot += wc[w]; ecnt[f] = tot; }
  // scale: IQR, else std of the sample column, else 1
  __syncthreads();
  if (t == 0) {
    const double q25 = quantile_sorted(src, mm, 0.25), q75 = quantile_sorted(src, mm, 0.75);
    s_sum[0] = q75 - q25;
  }
  __syncthreads();
  double iqr = s_sum[0];
  if (iqr == 0.0) {
    __syncthreads();
    double acc = 0.0;
    for (long long i = t; i < mm; i += 256) acc += (double)ord2f(src[i]);
    s_sum[t] = acc;
    __syncthreads();
    for (int o = 128; o; o >>= 1) { if (t < o) s_sum[t] += s_sum[t + o]; __syncthreads(); }
    const double mean = s_sum[0] / (double)mm;
    __syncthreads();
    acc = 0.0;
    for (long long i = t; i < mm; i += 256) { const double d = (double)ord2f(src[i]) - mean; acc += d * d; }
    s_sum[t] = acc;
    __syncthreads();
    for (int o = 128; o; o >>= 1) { if (t < o) s_sum[t] += s_sum[t + o]; __syncthreads(); }
    const float sd = (float)sqrt(s_sum[0] / (double)mm);
    iqr = sd != 0.f ? (double)sd : 1.0;
  }
  if (t == 0) scales[f] = (float)iqr;
}

// ---------------------------------------------------------------- transform
// grid: (row blocks of 64, feature groups of 32). Imputes NaN in Xfm (in place),
// writes bins in the tiled layout (plain_out != nullptr: also row-major (n, F)).
__global__ void __launch_bounds__(256)
k_transform(float* __restrict__ Xfm, long long n, int F, const float* __restrict__ medians,
            const float* __restrict__ edges, const int* __restrict__ ecnt, uint8_t* __restrict__ tiled,
            uint8_t* __restrict__ plain_out, uint8_t* __restrict__ fm_out) {
  __shared__ float se[32][256];
  __shared__ int sc[32];
  __shared__ uint8_t sb[64][36];
  const int f0 = blockIdx.y * 32;
  const int nf = min(32, F - f0);
  const long long r0 = (long long)blockIdx.x * 64;
  for (int i = threadIdx.x; i < nf * 255; i += blockDim.x) {
    const int ff = i / 255, e = i % 255;
    se[ff][e] = edges[(long long)(f0 + ff) * 255 + e];
  }
  for (int i = threadIdx.x; i < nf; i += blockDim.x) sc[i] = ecnt[f0 + i];
  __syncthreads();
  const int lane = threadIdx.x & 63, grp = threadIdx.x >> 6;   // 64 rows x 4 groups
  for (int ff = grp; ff < nf; ff += 4) {
    const long long r = r0 + lane;
    if (r >= n) continue;
    float* p = Xfm + (long long)(f0 + ff) * n + r;
    float x = *p;
    if (isnan(x)) { x = medians[f0 + ff]; *p = x; }
    int lo = 0, hi = sc[ff];
    while (lo < hi) { const int mid = (lo + hi) >> 1; if (se[ff][mid] < x) lo = mid + 1; else hi = mid; }
    sb[lane][ff] = (uint8_t)lo;
    if (fm_out) fm_out[(long long)(f0 + ff) * n + r] = (uint8_t)lo;   // feature-major copy
  }
  __syncthreads();
  // write: thread -> (row, feature) pairs, byte addresses from the tiled layout
  for (int i = threadIdx.x; i < 64 * nf; i += blockDim.x) {
    const int rr = i / nf, ff = i % nf;
    const long long r = r0 + rr;
    if (r >= n) continue;
    const FeatAddr a = feat_addr(F, n, f0 + ff);
    tiled[a.off + r * a.width + a.pos] = sb[rr][ff];
    if (plain_out) plain_out[r * F + f0 + ff] = sb[rr][ff];
  }
}

}  // namespace yabt

// ---------------------------------------------------------------- C ABI
#include "../../include/yabt_b200.h"

using namespace yabt;

#define BCUDA(x)                                                                         \
  do {                                                                                   \
    cudaError_t e__ = (x);                                                               \
    if (e__ != cudaSuccess) {                                                            \
      set_error("%s: %s (%s:%d)", #x, cudaGetErrorString(e__), __FILE__, __LINE__);      \
      return YABT_ERR_CUDA;                                                              \
    }                                                                                    \
  } while (0)

static long long pow2_at_least(long long x) {
  long long p = 1;
  while (p < x) p <<= 1;
  return p;
}

extern "C" {

long long yabt_bin_fit_workspace_bytes(long long n, int F, long long nq) {
  const long long P = pow2_at_least(std::max(nq, 2LL));
  long long b = 0;
  b += ((long long)F * sizeof(SelState) + 255) & ~255LL;
  b += ((long long)F * 2 * 2048 * 4 + 255) & ~255LL;
  b += ((long long)F * 8 + 255) & ~255LL;
  b += ((long long)F * P * 4 + 255) & ~255LL;
  return b;
}

int yabt_transpose(const float* X, long long n, int F, float* Xfm, void* stream) {
  if (n == 0 && F > 0) return YABT_OK;   // no rows: nothing is read (buffers may be NULL)
  if (!X || !Xfm || n < 0 || F <= 0) { set_error("yabt_transpose: bad arguments"); return YABT_ERR_ARG; }
  if (n == 0) return YABT_OK;
  dim3 grid((unsigned)((n + 31) / 32), (unsigned)((F + 31) / 32));
  k_transpose<<<grid, 256, 0, (cudaStream_t)stream>>>(X, n, F, Xfm, n);
  count_launches(1);
  BCUDA(cudaGetLastError());
  return YABT_OK;
}

int yabt_transpose_block(const float* X, long long m, int F, float* Xfm, long long ld, void* stream) {
  if (!X || !Xfm || m < 0 || F <= 0 || ld < m) { set_error("yabt_transpose_block: bad arguments"); return YABT_ERR_ARG; }
  if (m == 0) return YABT_OK;
  dim3 grid((unsigned)((m + 31) / 32), (unsigned)((F + 31) / 32));
  k_transpose<<<grid, 256, 0, (cudaStream_t)stream>>>(X, m, F, Xfm, ld);
  count_launches(1);
  BCUDA(cudaGetLastError());
  return YABT_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- fit steps
// The bin fit in steps: the median selection passes (a digit histogram over
// the caller's rows, then a pick on the -- possibly all-reduced -- histogram),
// and the edge fit on a row sample. yabt_bin_fit runs them back to back; a
// row-sharded fit all-reduces the histograms and NaN counts between the steps
// and fits the edges on the gathered sample.
namespace yabt {

struct FitWs {
  SelState* sel;
  unsigned* hist;               // [F][2][2048]
  unsigned long long* nanc;     // [F]
  unsigned* keys;               // [F][P]
};

static FitWs carve_fit(void* workspace, int F) {
  char* w = (char*)workspace;
  FitWs r;
  r.sel = (SelState*)w; w += ((long long)F * sizeof(SelState) + 255) & ~255LL;
  r.hist = (unsigned*)w; w += ((long long)F * 2 * 2048 * 4 + 255) & ~255LL;
  r.nanc = (unsigned long long*)w; w += ((long long)F * 8 + 255) & ~255LL;
  r.keys = (unsigned*)w;
  return r;
}

static cudaError_t median_hist(const float* Xfm, long long n, int F, int pass, const FitWs& w, cudaStream_t s) {
  cudaError_t e = cudaSuccess;
  if (pass == 0) e = cudaMemsetAsync(w.nanc, 0, (size_t)F * 8, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(w.hist, 0, (size_t)F * 2 * 2048 * 4, s);
  if (e != cudaSuccess) return e;
  if (n > 0) {
    const int chunks = (int)std::max(1LL, std::min(64LL, (n + 65535) / 65536));
    k_sel_hist<<<dim3(chunks, F), 512, 0, s>>>(Xfm, n, pass, w.sel, w.hist, w.nanc);
    count_launches(1);
  }
  return cudaGetLastError();
}

static cudaError_t median_pick(long long n_total, int F, int pass, const FitWs& w, cudaStream_t s) {
  k_sel_pick<<<(F * 32 + 255) / 256, 256, 0, s>>>(n_total, F, pass, w.sel, w.hist, w.nanc);
  count_launches(1);
  return cudaGetLastError();
}

static cudaError_t median_final(int F, const FitWs& w, float* medians, cudaStream_t s) {
  k_sel_final<<<(F + 255) / 256, 256, 0, s>>>(F, w.sel, medians);
  count_launches(1);
  return cudaGetLastError();
}

// edges and scales from the sample rows idx[0..nq) of Xfm (all of its first nq
// columns when idx is NULL)
static cudaError_t fit_edges(const float* Xfm, long long n, int F, const int32_t* idx, long long nq, int max_bins,
                             const FitWs& w, float* edges, int32_t* edge_cnt, float* scales, cudaStream_t s) {
  const long long P = pow2_at_least(std::max(nq, 2LL));
  unsigned* keys = w.keys;
  {
    const long long total = (long long)F * P;
    const int grid = (int)std::min<long long>((total + 255) / 256, (long long)YABT_SMS_HINT * 16);
    k_sample_keys<<<grid, 256, 0, s>>>(Xfm, n, F, idx, nq, P, keys);
    count_launches(2);   // sample keys + first bitonic pass
  }
  if (P <= BL) {
    k_bitonic_local<<<(unsigned)F, 1024, 0, s>>>(keys, P, (int)P);
  } else {
    k_bitonic_local<<<(unsigned)(F * P / BL), 1024, 0, s>>>(keys, P, BL);
    for (long long k = 2 * BL; k <= P; k <<= 1) {
      for (long long j = k >> 1; j >= BL; j >>= 1) {
        const long long half = (long long)F * P / 2;
        const int grid = (int)std::min<long long>((half + 255) / 256, (long long)YABT_SMS_HINT * 16);
        k_bitonic_global<<<grid, 256, 0, s>>>(keys, P, F, k, j);
        count_launches(1);
      }
      k_bitonic_merge_local<<<(unsigned)(F * P / BL), 1024, 0, s>>>(keys, P, k);
      count_launches(1);
    }
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_quantiles<<<F, 256, 0, s>>>(keys, P, max_bins, edges, edge_cnt, scales);
  count_launches(1);
  return cudaGetLastError();
}

}  // namespace yabt

extern "C" {

int yabt_bin_fit(const float* Xfm, long long n, int F, const int32_t* sample_idx, long long nq,
                 int max_bins, void* workspace, long long ws_bytes, float* medians, float* edges,
                 int32_t* edge_cnt, float* scales, void* stream) {
  if (!Xfm || n <= 0 || F <= 0 || nq <= 0 || max_bins < 2 || max_bins > 256 || !workspace || !medians ||
      !edges || !edge_cnt || !scales) {
    set_error("yabt_bin_fit: bad arguments");
    return YABT_ERR_ARG;
  }
  if (ws_bytes < yabt_bin_fit_workspace_bytes(n, F, nq)) { set_error("yabt_bin_fit: workspace too small"); return YABT_ERR_WORKSPACE; }
  cudaStream_t s = (cudaStream_t)stream;
  PhaseScope ph(PH_BINNING, s);
  const FitWs w = carve_fit(workspace, F);
  // medians: radix select over all rows
  for (int pass = 0; pass < 3; ++pass) {
    BCUDA(median_hist(Xfm, n, F, pass, w, s));
    BCUDA(median_pick(n, F, pass, w, s));
  }
  BCUDA(median_final(F, w, medians, s));
  // edges: sample keys, bitonic sort per column, quantiles
  BCUDA(fit_edges(Xfm, n, F, sample_idx, nq, max_bins, w, edges, edge_cnt, scales, s));
  return YABT_OK;
}

int yabt_bin_median_hist(const float* Xfm, long long n, int F, int pass, void* workspace, long long ws_bytes,
                         void* stream) {
  if ((n > 0 && !Xfm) || n < 0 || F <= 0 || pass < 0 || pass > 2 || !workspace) {
    set_error("yabt_bin_median_hist: bad arguments");
    return YABT_ERR_ARG;
  }
  if (ws_bytes < yabt_bin_fit_workspace_bytes(std::max(n, 1LL), F, 1)) {
    set_error("yabt_bin_median_hist: workspace too small");
    return YABT_ERR_WORKSPACE;
  }
  BCUDA(median_hist(Xfm, n, F, pass, carve_fit(workspace, F), (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_bin_median_pick(long long n_total, int F, int pass, void* workspace, long long ws_bytes, void* stream) {
  if (n_total <= 0 || F <= 0 || pass < 0 || pass > 2 || !workspace) {
    set_error("yabt_bin_median_pick: bad arguments");
    return YABT_ERR_ARG;
  }
  if (ws_bytes < yabt_bin_fit_workspace_bytes(1, F, 1)) {
    set_error("yabt_bin_median_pick: workspace too small");
    return YABT_ERR_WORKSPACE;
  }
  BCUDA(median_pick(n_total, F, pass, carve_fit(workspace, F), (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_bin_median_final(int F, void* workspace, long long ws_bytes, float* medians, void* stream) {
  if (F <= 0 || !workspace || !medians) { set_error("yabt_bin_median_final: bad arguments"); return YABT_ERR_ARG; }
  if (ws_bytes < yabt_bin_fit_workspace_bytes(1, F, 1)) {
    set_error("yabt_bin_median_final: workspace too small");
    return YABT_ERR_WORKSPACE;
  }
  BCUDA(median_final(F, carve_fit(workspace, F), medians, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_bin_median_bufs(int F, void* workspace, void** hist, long long* hist_words, void** nan_count) {
  if (F <= 0 || !workspace) { set_error("yabt_bin_median_bufs: bad arguments"); return YABT_ERR_ARG; }
  const FitWs w = carve_fit(workspace, F);
  if (hist) *hist = w.hist;
  if (hist_words) *hist_words = (long long)F * 2 * 2048;
  if (nan_count) *nan_count = w.nanc;
  return YABT_OK;
}

int yabt_bin_fit_edges(const float* Xs, long long nq, int F, int max_bins, void* workspace, long long ws_bytes,
                       float* edges, int32_t* edge_cnt, float* scales, void* stream) {
  if (!Xs || nq <= 0 || F <= 0 || max_bins < 2 || max_bins > 256 || !workspace || !edges || !edge_cnt ||
      !scales) {
    set_error("yabt_bin_fit_edges: bad arguments");
    return YABT_ERR_ARG;
  }
  if (ws_bytes < yabt_bin_fit_workspace_bytes(nq, F, nq)) {
    set_error("yabt_bin_fit_edges: workspace too small");
    return YABT_ERR_WORKSPACE;
  }
  BCUDA(fit_edges(Xs, nq, F, nullptr, nq, max_bins, carve_fit(workspace, F), edges, edge_cnt, scales,
                  (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_bin_transform(float* Xfm, long long n, int F, const float* medians, const float* edges,
                       const int32_t* edge_cnt, uint8_t* tiled, uint8_t* plain_out, uint8_t* fm_out,
                       void* stream) {
  if (n == 0 && F > 0) return YABT_OK;   // no rows: nothing is read (buffers may be NULL)
  if (!Xfm || n < 0 || F <= 0 || !medians || !edges || !edge_cnt || !tiled) {
    set_error("yabt_bin_transform: bad arguments");
    return YABT_ERR_ARG;
  }
  if (n == 0) return YABT_OK;
  cudaStream_t s = (cudaStream_t)stream;
  PhaseScope ph(PH_BINNING, s);
  long long bytes = 0;
  {
    std::vector<TileInfo> t(tile_count(F) + 1);
    bytes = make_tiles(F, n, t.data());
  }
  BCUDA(cudaMemsetAsync(tiled, 0, (size_t)bytes, s));
  dim3 grid((unsigned)((n + 63) / 64), (unsigned)((F + 31) / 32));
  k_transform<<<grid, 256, 0, s>>>(Xfm, n, F, medians, edges, edge_cnt, tiled, plain_out, fm_out);
  count_launches(1);
  BCUDA(cudaGetLastError());
  return YABT_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- allocation-free variant
// yabt_bin_fit_static: the same bin fit with its scratch in a fixed array that
// lives in the library's device image instead of a caller workspace. It is for
// callers that cannot allocate device memory at fit time -- for example a
// process whose GPU memory is reserved up front by another framework's caching
// allocator, or a latency-critical loop where cudaMalloc (which may
// synchronise the device and can fail under memory pressure) is not allowed.
// The array is BIN_FIT_STATIC_BYTES per GPU that loads the library, held until
// the process exits.
#include <mutex>

namespace yabt {

constexpr long long BIN_FIT_STATIC_BYTES = 8LL << 20;   // 8 MiB per device
static __device__ __align__(256) unsigned char g_bin_fit_scratch[BIN_FIT_STATIC_BYTES];

constexpr int MAX_DEVICES = 64;
static std::mutex g_static_mu;
static void* g_static_ptr[MAX_DEVICES] = {};

// Device address of the scratch array on the current device (host code must
// not pass the symbol itself: in host code its name is only a stand-in, not a
// device address). Outside stream capture the address is looked up on every
// call (a cheap host query), so it follows a device reset or a different
// context; during capture, where the lookup might not be allowed, the last
// address seen on this device is used -- so the first call on a device must
// come before any capture.
static int bin_fit_scratch_ptr(void** out, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) { set_error("yabt_bin_fit_static: cudaGetDevice: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  if (dev < 0 || dev >= MAX_DEVICES) { set_error("yabt_bin_fit_static: device %d out of range", dev); return YABT_ERR_ARG; }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(stream, &cap);
  if (e != cudaSuccess) { set_error("yabt_bin_fit_static: cudaStreamIsCapturing: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (cap == cudaStreamCaptureStatusNone || !g_static_ptr[dev]) {
    if (cap != cudaStreamCaptureStatusNone) {
      set_error("yabt_bin_fit_static: the first call on a device must come before stream capture");
      return YABT_ERR_ARG;
    }
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bin_fit_scratch);
    if (e != cudaSuccess || !p) {
      set_error("yabt_bin_fit_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return YABT_ERR_CUDA;
    }
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
  return YABT_OK;
}

}  // namespace yabt

extern "C" {

long long yabt_bin_fit_static_capacity(void) { return BIN_FIT_STATIC_BYTES; }

int yabt_bin_fit_static(const float* Xfm, long long n, int F, const int32_t* sample_idx, long long nq,
                        int max_bins, float* medians, float* edges, int32_t* edge_cnt, float* scales,
                        void* stream) {
  // every argument is checked before any size arithmetic or device query
  if (!Xfm || n <= 0 || F <= 0 || nq <= 0 || max_bins < 2 || max_bins > 256 || !medians || !edges || !edge_cnt ||
      !scales) {
    set_error("yabt_bin_fit_static: bad arguments");
    return YABT_ERR_ARG;
  }
  // the sorted sample alone takes 4 F nq bytes: anything larger cannot fit
  if (nq > BIN_FIT_STATIC_BYTES / (4LL * F) || n > (1LL << 40)) {
    set_error("yabt_bin_fit_static: %lld sample rows x %d features exceed the static buffer of %lld bytes; "
              "use yabt_bin_fit with a caller workspace", nq, F, BIN_FIT_STATIC_BYTES);
    return YABT_ERR_UNSUPPORTED;
  }
  const long long need = yabt_bin_fit_workspace_bytes(n, F, nq);
  if (need > BIN_FIT_STATIC_BYTES) {
    set_error("yabt_bin_fit_static: this fit needs %lld bytes of scratch but the static buffer holds %lld "
              "(F=%d, sample rows=%lld); use yabt_bin_fit with a caller workspace",
              need, BIN_FIT_STATIC_BYTES, F, nq);
    return YABT_ERR_UNSUPPORTED;
  }
  void* ws = nullptr;
  int rc = bin_fit_scratch_ptr(&ws, (cudaStream_t)stream);
  if (rc) return rc;
  // yabt_bin_fit clears every scratch region it accumulates into before use
  // (NaN counts, digit histograms) and fully writes the rest, so the contents
  // left by an earlier call do not matter.
  return yabt_bin_fit(Xfm, n, F, sample_idx, nq, max_bins, ws, BIN_FIT_STATIC_BYTES, medians, edges,
                      edge_cnt, scales, stream);
}

}  // extern "C"
