// Histogram of a plain row-major (n, F) uint8 bin matrix with an arbitrary
// node slot per row: the reference's build_hist FFI (yabt/cuda_hist.py:79-89,
// yabt/_cuda/hist.cu:27-133). Row i adds (g[i], h[i], w[i]) into bin
// binned[i, f] of slot slot[i] for every feature f; the result is the
// (3, K, F, B) float32 histogram.
//
// The reference adds float32 values with global (or, for K == 1, shared)
// atomics, so its sums depend on the order the atomics land in. Here every
// value is quantised once per call to a fixed-point integer (the same scheme
// as the grower's histograms), the sums are exact int64 and each bin is
// rounded to float32 once: the result is deterministic and at least as
// accurate as an in-order float32 sum.
//
// Kernel sequence (no host synchronisation):
//   k_hp_prep   slot range check, per-slot row counts (warp-aggregated
//               atomics), max |g|, |h|, |w|, non-finite check
//   k_hp_plan   one block: quantisation exponents, slot row offsets, the work
//               items (<= ITEM_ROWS rows of one slot each)
//   k_hp_place  row ids grouped by slot (order within a slot is irrelevant:
//               the sums are exact)
//   k_hp_hist   persistent, one 1024-thread block per SM; a unit is (item,
//               group of 32 features): warp = row, lane = feature, six u32
//               limb planes in shared memory (bank = lane), flushed as int64
//               global atomics
//   k_hp_out    int64 -> float32 (one rounding)
#include <algorithm>
#include <climits>

#include "../../include/yabt_b200.h"
#include "common.cuh"

namespace yabt {
namespace {

constexpr int ITEM_ROWS = 8192;        // limb bound: ITEM_ROWS * 65535 < 2^32
constexpr int HP_THREADS = 1024;
constexpr int HP_LIMBS = 6;            // g lo/hi, h lo/hi, w lo/hi
constexpr int HP_PLANE = YABT_NB * 32; // u32 words per limb plane ([bin][lane])
constexpr int HP_SMEM = HP_LIMBS * HP_PLANE * 4;

struct HpItem {
  int slot, begin, count;
};

struct HpState {
  unsigned amax[3];   // bit patterns of max |g|, |h|, |w| (non-negative floats order as u32)
  unsigned err;       // DERR_* bits
  int n_items;
  int unit_counter;
  float scale[3];     // 2^qe per channel
  float inv[3];       // 2^-qe per channel
};

struct HpBufs {
  HpState* st;
  int* cursor;        // [K] per-slot row counts, then row cursors (k_hp_place)
  int* seg;           // [K+1] row offset of each slot
  int* ioff;          // [K+1] item offset of each slot
  HpItem* items;      // [max_items]
  int* rows;          // [n] row ids grouped by slot
  unsigned long long* acc;   // [3][K][F][256] int64 sums
};

inline long long hp_max_items(long long n, long long K) { return n / ITEM_ROWS + K + 1; }

inline long long align256(long long x) { return (x + 255) & ~255LL; }

long long hp_carve(long long n, int K, int F, char* base, HpBufs* b) {
  long long off = 0;
  auto take = [&](long long bytes) { char* p = base ? base + off : nullptr; off += align256(bytes); return p; };
  HpBufs t;
  t.st = reinterpret_cast<HpState*>(take(sizeof(HpState)));
  t.cursor = reinterpret_cast<int*>(take(4LL * K));
  t.seg = reinterpret_cast<int*>(take(4LL * (K + 1)));
  t.ioff = reinterpret_cast<int*>(take(4LL * (K + 1)));
  t.items = reinterpret_cast<HpItem*>(take((long long)sizeof(HpItem) * hp_max_items(n, K)));
  t.rows = reinterpret_cast<int*>(take(4LL * n));
  t.acc = reinterpret_cast<unsigned long long*>(take(8LL * 3 * K * F * YABT_NB));
  if (b) *b = t;
  return off;
}

__device__ __forceinline__ bool finite_f(float x) { return (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u; }

// -------------------------------------------------------------- k_hp_prep
__global__ void __launch_bounds__(256) k_hp_prep(const int64_t* __restrict__ slot, const float* __restrict__ g,
                                                 const float* __restrict__ h, const float* __restrict__ w,
                                                 long long n, int K, HpState* st, int* __restrict__ counts) {
  const int lane = threadIdx.x & 31;
  unsigned mg = 0, mh = 0, mw = 0;
  bool bad_slot = false, bad_val = false;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long base = (long long)blockIdx.x * blockDim.x; base < n; base += stride) {
    const long long i = base + threadIdx.x;
    const bool valid = i < n;
    long long s = 0;
    if (valid) {
      s = slot[i];
      const float gv = g[i], hv = h[i], wv = w[i];
      const bool fin = finite_f(gv) && finite_f(hv) && finite_f(wv);
      bad_val |= !fin;
      if (fin) {
        mg = max(mg, __float_as_uint(fabsf(gv)));
        mh = max(mh, __float_as_uint(fabsf(hv)));
        mw = max(mw, __float_as_uint(fabsf(wv)));
      }
    }
    const bool ok = valid && s >= 0 && s < K;
    bad_slot |= valid && !ok;
    const int key = ok ? (int)s : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    if (ok && lane == __ffs(peers) - 1) atomicAdd(&counts[key], __popc(peers));
  }
  mg = __reduce_max_sync(0xffffffffu, mg);
  mh = __reduce_max_sync(0xffffffffu, mh);
  mw = __reduce_max_sync(0xffffffffu, mw);
  const bool any_slot = __any_sync(0xffffffffu, bad_slot), any_val = __any_sync(0xffffffffu, bad_val);
  if (lane == 0) {
    if (mg) atomicMax(&st->amax[0], mg);
    if (mh) atomicMax(&st->amax[1], mh);
    if (mw) atomicMax(&st->amax[2], mw);
    if (any_slot) atomicOr(&st->err, DERR_BAD_INDEX);
    if (any_val) atomicOr(&st->err, DERR_NONFINITE);
  }
}

// -------------------------------------------------------------- k_hp_plan
// One block: exponents, exclusive scans of rows and items over the K slots
// (chunks of 1024 slots with a running carry), then the item list.
__global__ void __launch_bounds__(HP_THREADS) k_hp_plan(int K, HpBufs b) {
  __shared__ long long s_rows[HP_THREADS / 32], s_items[HP_THREADS / 32];
  __shared__ long long s_carry_rows, s_carry_items;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  HpState* st = b.st;
  if (tid < 3) {
    const float a = __uint_as_float(st->amax[tid]);
    const int q = max(-100, min(30 - exp_bound(a), 100));
    st->scale[tid] = ldexpf(1.f, q);
    st->inv[tid] = ldexpf(1.f, -q);
  }
  if (tid == 0) { s_carry_rows = 0; s_carry_items = 0; }
  __syncthreads();
  for (int k0 = 0; k0 < K; k0 += HP_THREADS) {
    const int k = k0 + tid;
    const long long c = k < K ? b.cursor[k] : 0;      // row count of slot k
    const long long ni = (c + ITEM_ROWS - 1) / ITEM_ROWS;
    long long vr = c, vi = ni;                        // inclusive warp scans
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const long long tr = __shfl_up_sync(0xffffffffu, vr, d), ti = __shfl_up_sync(0xffffffffu, vi, d);
      if (lane >= d) { vr += tr; vi += ti; }
    }
    if (lane == 31) { s_rows[warp] = vr; s_items[warp] = vi; }
    __syncthreads();
    if (warp == 0) {
      long long wr = s_rows[lane], wi = s_items[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const long long tr = __shfl_up_sync(0xffffffffu, wr, d), ti = __shfl_up_sync(0xffffffffu, wi, d);
        if (lane >= d) { wr += tr; wi += ti; }
      }
      s_rows[lane] = wr;   // inclusive over warps
      s_items[lane] = wi;
    }
    __syncthreads();
    const long long pr = (warp ? s_rows[warp - 1] : 0) + vr - c + s_carry_rows;
    const long long pi = (warp ? s_items[warp - 1] : 0) + vi - ni + s_carry_items;
    if (k < K) {           // each thread reads and rewrites only its own slot k
      b.seg[k] = (int)pr;
      b.cursor[k] = (int)pr;
      b.ioff[k] = (int)pi;
    }
    __syncthreads();
    if (tid == 0) { s_carry_rows += s_rows[31]; s_carry_items += s_items[31]; }
    __syncthreads();
  }
  if (tid == 0) {
    b.seg[K] = (int)s_carry_rows;
    b.ioff[K] = (int)s_carry_items;
    st->n_items = (int)s_carry_items;
    st->unit_counter = 0;
  }
  __syncthreads();
  const int total = (int)s_carry_items;
  for (int it = tid; it < total; it += HP_THREADS) {
    // the slot k with ioff[k] <= it < ioff[k+1] (invariant: ioff[lo] <= it < ioff[hi])
    int lo = 0, hi = K;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (b.ioff[mid] <= it) lo = mid; else hi = mid;
    }
    const int j = it - b.ioff[lo];
    const int begin = b.seg[lo] + j * ITEM_ROWS;
    b.items[it] = HpItem{lo, begin, min(ITEM_ROWS, b.seg[lo + 1] - begin)};
  }
}

// -------------------------------------------------------------- k_hp_place
__global__ void __launch_bounds__(256) k_hp_place(const int64_t* __restrict__ slot, long long n, int K,
                                                  int* __restrict__ cursor, int* __restrict__ rows) {
  const int lane = threadIdx.x & 31;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long base = (long long)blockIdx.x * blockDim.x; base < n; base += stride) {
    const long long i = base + threadIdx.x;
    const long long s = i < n ? slot[i] : -1;
    const bool ok = s >= 0 && s < K;
    const int key = ok ? (int)s : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const int leader = __ffs(peers) - 1;
    int pos = 0;
    if (ok && lane == leader) pos = atomicAdd(&cursor[key], __popc(peers));
    pos = __shfl_sync(0xffffffffu, pos, leader);
    if (ok) rows[pos + __popc(peers & ((1u << lane) - 1u))] = (int)i;
  }
}

// -------------------------------------------------------------- k_hp_hist
__device__ __forceinline__ void red_u32(unsigned addr, unsigned v) {
  asm volatile("red.shared.add.u32 [%0], %1;\n" ::"r"(addr), "r"(v) : "memory");
}

constexpr int HP_RPW = 4;   // rows in flight per warp

__global__ void __launch_bounds__(HP_THREADS, 1)
k_hp_hist(const uint8_t* __restrict__ bins, const float* __restrict__ g, const float* __restrict__ h,
          const float* __restrict__ w, int K, int F, int B, HpBufs b) {
  extern __shared__ __align__(16) unsigned sh[];
  __shared__ int s_unit;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  HpState* st = b.st;
  const int G = (F + 31) >> 5;
  const long long units = (long long)st->n_items * G;
  const float sg = st->scale[0], shs = st->scale[1], sw = st->scale[2];
  const unsigned sbase = (unsigned)__cvta_generic_to_shared(sh) + lane * 4;
  bool bad_bin = false;
  for (;;) {
    if (threadIdx.x == 0) s_unit = atomicAdd(&st->unit_counter, 1);
    __syncthreads();
    const int u = s_unit;
    if (u >= units) break;
    const HpItem item = b.items[u / G];
    const int fg = u % G;
    for (int i = threadIdx.x * 4; i < HP_LIMBS * HP_PLANE; i += HP_THREADS * 4)
      *reinterpret_cast<uint4*>(sh + i) = make_uint4(0, 0, 0, 0);
    __syncthreads();
    const int f = fg * 32 + lane;
    const bool fok = f < F;
    const int* lst = b.rows + item.begin;
    for (int r0 = warp * HP_RPW; r0 < item.count; r0 += 32 * HP_RPW) {
      int row[HP_RPW];
      unsigned bin[HP_RPW];
      float gv[HP_RPW], hv[HP_RPW], wv[HP_RPW];
#pragma unroll
      for (int q = 0; q < HP_RPW; ++q) row[q] = r0 + q < item.count ? lst[r0 + q] : -1;
#pragma unroll
      for (int q = 0; q < HP_RPW; ++q) {
        const bool ok = row[q] >= 0;
        bin[q] = (ok && fok) ? bins[(long long)row[q] * F + f] : 0u;
        gv[q] = ok ? g[row[q]] : 0.f;
        hv[q] = ok ? h[row[q]] : 0.f;
        wv[q] = ok ? w[row[q]] : 0.f;
      }
#pragma unroll
      for (int q = 0; q < HP_RPW; ++q) {
        if (row[q] < 0 || !fok) continue;
        if (bin[q] >= (unsigned)B) { bad_bin = true; continue; }
        const int vg = __float2int_rn(gv[q] * sg), vh = __float2int_rn(hv[q] * shs),
                  vw = __float2int_rn(wv[q] * sw);
        const unsigned a = sbase + bin[q] * 128u;
        red_u32(a, (unsigned)vg & 0xFFFFu);
        red_u32(a + HP_PLANE * 4, (unsigned)(vg >> 16));
        red_u32(a + 2 * HP_PLANE * 4, (unsigned)vh & 0xFFFFu);
        red_u32(a + 3 * HP_PLANE * 4, (unsigned)(vh >> 16));
        red_u32(a + 4 * HP_PLANE * 4, (unsigned)vw & 0xFFFFu);
        red_u32(a + 5 * HP_PLANE * 4, (unsigned)(vw >> 16));
      }
    }
    __syncthreads();
    // flush: word idx = bin * 32 + lane of each plane (conflict-free reads)
    for (int idx = threadIdx.x; idx < HP_PLANE; idx += HP_THREADS) {
      const int ff = fg * 32 + (idx & 31), bb = idx >> 5;
      if (ff >= F || bb >= B) continue;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const unsigned lo = sh[(2 * c) * HP_PLANE + idx];
        const int hi = (int)sh[(2 * c + 1) * HP_PLANE + idx];
        const long long v = (long long)hi * 65536LL + (long long)lo;
        if (v != 0)
          atomicAdd(&b.acc[(((long long)c * K + item.slot) * F + ff) * YABT_NB + bb], (unsigned long long)v);
      }
    }
    __syncthreads();
  }
  if (__any_sync(0xffffffffu, bad_bin) && lane == 0) atomicOr(&st->err, DERR_BAD_INDEX);
}

// -------------------------------------------------------------- k_hp_out
__global__ void __launch_bounds__(256) k_hp_out(const unsigned long long* __restrict__ acc, const HpState* st,
                                                int K, int F, int B, float* __restrict__ out) {
  const long long total = 3LL * K * F * B;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += stride) {
    const long long cf = e / B;                 // (c * K + k) * F + f
    const int bb = (int)(e - cf * B);
    const int c = (int)(cf / ((long long)K * F));
    const long long v = (long long)acc[cf * YABT_NB + bb];
    out[e] = __fmul_rn(__ll2float_rn(v), st->inv[c]);
  }
}

int hp_sms() {
  int dev = 0, nsm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || nsm <= 0)
    nsm = YABT_SMS_HINT;
  return nsm;
}

}  // namespace
}  // namespace yabt

using namespace yabt;

extern "C" {

long long yabt_hist_build_workspace_bytes(long long n, int K, int F) {
  if (n < 0 || K <= 0 || F <= 0) return -1;
  return hp_carve(n, K, F, nullptr, nullptr);
}

int yabt_hist_build(const uint8_t* binned, const int64_t* slot, const float* g, const float* h,
                    const float* w, long long n, int K, int F, int B, float* out, int32_t* err_out,
                    void* workspace, long long ws_bytes, void* stream) {
  if (n < 0 || n > INT_MAX || K <= 0 || F <= 0 || B <= 0 || B > YABT_NB || !out ||
      (n > 0 && (!binned || !slot || !g || !h || !w))) {
    set_error("yabt_hist_build: bad arguments (n=%lld K=%d F=%d B=%d)", n, K, F, B);
    return YABT_ERR_ARG;
  }
  const long long need = hp_carve(n, K, F, nullptr, nullptr);
  if (!workspace || ws_bytes < need) {
    set_error("yabt_hist_build: workspace of %lld bytes, %lld needed", ws_bytes, need);
    return YABT_ERR_WORKSPACE;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PhaseScope ph(PH_HIST, s);
  HpBufs b;
  hp_carve(n, K, F, static_cast<char*>(workspace), &b);
  cudaError_t e = cudaFuncSetAttribute(k_hp_hist, cudaFuncAttributeMaxDynamicSharedMemorySize, HP_SMEM);
  if (e != cudaSuccess) { set_error("yabt_hist_build: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  const int nsm = hp_sms();
  const long long front = reinterpret_cast<char*>(b.rows) - reinterpret_cast<char*>(b.st);
  e = cudaMemsetAsync(b.st, 0, front, s);                       // state, counts, offsets, items
  if (e == cudaSuccess) e = cudaMemsetAsync(b.acc, 0, 8LL * 3 * K * F * YABT_NB, s);
  if (e == cudaSuccess && n > 0) {
    const int blocks = (int)std::min<long long>((n + 255) / 256, 4LL * nsm);
    k_hp_prep<<<blocks, 256, 0, s>>>(slot, g, h, w, n, K, b.st, b.cursor);
    k_hp_plan<<<1, HP_THREADS, 0, s>>>(K, b);
    k_hp_place<<<blocks, 256, 0, s>>>(slot, n, K, b.cursor, b.rows);
    k_hp_hist<<<nsm, HP_THREADS, HP_SMEM, s>>>(binned, g, h, w, K, F, B, b);
    count_launches(4);
  }
  if (e == cudaSuccess) {
    const long long total = 3LL * K * F * B;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 8LL * nsm);
    k_hp_out<<<blocks, 256, 0, s>>>(b.acc, b.st, K, F, B, out);
    count_launches(1);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && err_out) e = cudaMemcpyAsync(err_out, &b.st->err, 4, cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) {
    set_error("yabt_hist_build: %s", cudaGetErrorString(e));
    return YABT_ERR_CUDA;
  }
  return YABT_OK;
}

}  // extern "C"
