// Histogram kernels of the level-wise grower.
//
// Replaces the reference's histogram build (yabt/_cuda/hist.cu:27-133 and the
// torch scatter of yabt/tree.py:425-452) with a two-stage exact scheme:
//
// k_hist    persistent, one 1024-thread block per SM. A block takes work items
//           (rows [begin, begin+count) of one node's row list, one column unit)
//           and accumulates a private shared-memory histogram: warp = row,
//           lane = feature, so the 32 lanes of an atomic always hit 32
//           different banks. Values are fixed-point u32 limbs (u32 shared
//           atomics are several times faster than f32 ones on sm_100), and each
//           item's histogram is flushed as a plain coalesced copy into its own
//           partial slot -- no global atomics.
// k_reduce  one block per (job, unit, sub): sums the item partials of a node
//           into exact int64 totals and writes them feature-major
//           [job][channel][feature][bin] through a shared-memory transpose.
//
// Algorithmic traffic of k_hist per item: count * (tile width bytes + 4 B row
// id + 4 B g [+ 4 B h]) read, LIMBS*S*32 KB partial written.
#include "grow.cuh"

namespace yabt {

template <int S, int LIMBS>
struct HistCfg {
  static_assert((S == 2 && LIMBS == 3) || (S == 1 && LIMBS == 5), "supported (S, LIMBS) pairs");
  static constexpr int WORDS = LIMBS * S * YABT_NB * 32;   // u32 words per histogram
  static constexpr int LIMB_STRIDE = S * YABT_NB * 32;      // words between limbs
  static constexpr int SMEM = WORDS * 4;
};

__device__ __forceinline__ void red_add(unsigned* p, unsigned v) {
  atomicAdd(p, v);   // result unused -> shared-memory reduction (RED)
}

template <int S, int LIMBS>
__device__ __forceinline__ void acc_row(unsigned* sh, unsigned b0, unsigned b1, bool ok0, bool ok1,
                                        int lane, int vg, int vh) {
  using Cfg = HistCfg<S, LIMBS>;
  const unsigned glo = (unsigned)vg & 0xFFFFu, ghi = (unsigned)(vg >> 16);
  if (ok0) {
    unsigned* w = sh + ((b0 << 5) | lane);
    red_add(w, glo);
    red_add(w + Cfg::LIMB_STRIDE, ghi);
    if constexpr (LIMBS == 5) {
      red_add(w + 2 * Cfg::LIMB_STRIDE, (unsigned)vh & 0xFFFFu);
      red_add(w + 3 * Cfg::LIMB_STRIDE, (unsigned)(vh >> 16));
    }
    red_add(w + (LIMBS - 1) * Cfg::LIMB_STRIDE, 1u);
  }
  if constexpr (S == 2) {
    if (ok1) {
      unsigned* w = sh + (((YABT_NB + b1) << 5) | lane);
      red_add(w, glo);
      red_add(w + Cfg::LIMB_STRIDE, ghi);
      red_add(w + (LIMBS - 1) * Cfg::LIMB_STRIDE, 1u);
    }
  }
}

// rows: the active row list (nullptr = identity, row = begin + i)
template <int S, int LIMBS>
__global__ void __launch_bounds__(HIST_THREADS, 1)
k_hist(const uint8_t* __restrict__ bins, const int* __restrict__ rows,
       const float* __restrict__ g, const float* __restrict__ h,
       const HistItem* __restrict__ items, const UnitDesc* __restrict__ units,
       GrowState* st, unsigned* __restrict__ partials, int level_gate) {
  using Cfg = HistCfg<S, LIMBS>;
  extern __shared__ __align__(16) unsigned sh[];
  __shared__ int s_item;
  if (st->level != level_gate || !st->active) return;
  const int nitems = st->n_items;
  const float gs = st->gscale, hs = st->hscale;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  constexpr int UNR = 8;
  for (;;) {
    if (threadIdx.x == 0) s_item = atomicAdd(&st->item_counter, 1);
    __syncthreads();
    const int it = s_item;
    if (it >= nitems) break;
    const HistItem item = items[it];
    const UnitDesc& ud = units[item.unit];
    for (int i = threadIdx.x * 4; i < Cfg::WORDS; i += blockDim.x * 4)
      *reinterpret_cast<uint4*>(sh + i) = make_uint4(0, 0, 0, 0);
    __syncthreads();

    const uint8_t* tb = bins + ud.off;
    const int width = ud.width;
    const bool wide = ud.wide;
    const int k0 = ud.k0;
    const bool ok0 = ud.feat[0][lane] >= 0;
    const bool ok1 = (S == 2) && ud.nsub > 1 && ud.feat[S == 2 ? 1 : 0][lane] >= 0;
    const int* lst = rows ? rows + item.begin : nullptr;
    const int cnt = item.count;
    for (int base = warp * 32; base < cnt; base += nw * 32) {
      const int k = base + lane;
      const bool okr = k < cnt;
      int r = 0, vg = 0, vh = 0;
      if (okr) {
        r = lst ? __ldg(lst + k) : item.begin + k;
        vg = __float2int_rn(__ldg(g + r) * gs);
        if constexpr (LIMBS == 5) vh = __float2int_rn(__ldg(h + r) * hs);
      }
      const int nr = min(32, cnt - base);
      for (int u0 = 0; u0 < nr; u0 += UNR) {
        unsigned wv[UNR];
        int gv[UNR], hv[UNR];
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
          const int rr = __shfl_sync(0xffffffffu, r, u0 + u);
          gv[u] = __shfl_sync(0xffffffffu, vg, u0 + u);
          if constexpr (LIMBS == 5) hv[u] = __shfl_sync(0xffffffffu, vh, u0 + u);
          else hv[u] = 0;
          wv[u] = 0;
          if (u0 + u < nr) {
            const uint8_t* rp = tb + (size_t)rr * width;
            if (wide) {
              if constexpr (S == 2) wv[u] = __ldg(reinterpret_cast<const unsigned short*>(rp) + lane);
              else wv[u] = __ldg(rp + 2 * lane + k0);
            } else if (ok0) {
              wv[u] = __ldg(rp + lane);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
          if (u0 + u < nr)
            acc_row<S, LIMBS>(sh, wv[u] & 0xFFu, (wv[u] >> 8) & 0xFFu, ok0, ok1, lane, gv[u], hv[u]);
        }
      }
    }
    __syncthreads();
    unsigned* dst = partials + (size_t)item.slot * Cfg::WORDS;
    for (int i = threadIdx.x * 4; i < Cfg::WORDS; i += blockDim.x * 4)
      *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(sh + i);
  }
}

// One block per (job, unit, sub, bin-part): sums the u32-limb partials of the
// job's items for 32 bins x 32 lanes into exact int64 and writes
// [job][c][f][bin] (c = 0 g, 1 h (general path), last = count) through a small
// shared-memory transpose.
constexpr int RED_PARTS = 8;   // bins are split into 8 parts of 32
template <int S, int LIMBS>
__global__ void __launch_bounds__(512)
k_reduce(const unsigned* __restrict__ partials, const int* __restrict__ job_first,
         const int* __restrict__ job_nitems, const HistItem* __restrict__ items,
         const UnitDesc* __restrict__ units, GrowState* st, long long* __restrict__ out,
         int F, int U, int level_gate) {
  using Cfg = HistCfg<S, LIMBS>;
  constexpr int C = (LIMBS == 5) ? 3 : 2;
  __shared__ long long tsm[C][32][33];
  if (st->level != level_gate || !st->active) return;
  const int njobs = (level_gate == 0) ? 1 : st->P;
  int b = blockIdx.x;
  const int part = b % RED_PARTS; b /= RED_PARTS;
  const int sub = b % S; b /= S;
  const int unit = b % U;
  const int job = b / U;
  if (job >= njobs) return;
  const UnitDesc& ud = units[unit];
  if (sub >= ud.nsub) return;
  const int first = job_first[job * U + unit];
  const int nit = job_nitems[job * U + unit];
  // 1024 words (32 bins x 32 lanes) per block; thread t handles words t and t+512
  for (int w = threadIdx.x; w < 32 * 32; w += blockDim.x) {
    const int word = part * 32 * 32 + w;      // (bin, j) word inside the sub
    long long ag = 0, ah = 0;
    unsigned long long ac = 0;
    for (int q = 0; q < nit; ++q) {
      const unsigned* p = partials + (size_t)items[first + q].slot * Cfg::WORDS + sub * YABT_NB * 32 + word;
      const unsigned glo = __ldg(p), ghi = __ldg(p + Cfg::LIMB_STRIDE);
      ag += (long long)(int)ghi * 65536LL + (long long)glo;
      if constexpr (LIMBS == 5) {
        const unsigned hlo = __ldg(p + 2 * Cfg::LIMB_STRIDE), hhi = __ldg(p + 3 * Cfg::LIMB_STRIDE);
        ah += (long long)(int)hhi * 65536LL + (long long)hlo;
      }
      ac += __ldg(p + (LIMBS - 1) * Cfg::LIMB_STRIDE);
    }
    const int bl = w >> 5, j = w & 31;
    tsm[0][j][bl] = ag;
    if constexpr (C == 3) tsm[1][j][bl] = ah;
    tsm[C - 1][j][bl] = (long long)ac;
  }
  __syncthreads();
  const long long job_base = (long long)job * C * F * YABT_NB;
  for (int e = threadIdx.x; e < C * 32 * 32; e += blockDim.x) {
    const int bl = e & 31, j = (e >> 5) & 31, c = e >> 10;
    const int f = ud.feat[sub][j];
    if (f < 0) continue;
    out[job_base + ((long long)c * F + f) * YABT_NB + part * 32 + bl] = tsm[c][j][bl];
  }
}

cudaError_t launch_hist_kernels(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int d,
                                int jobs, int nsm, cudaStream_t s) {
  const int* rows = d == 0 ? nullptr : b.rows[d & 1];
  if (!p.general) {
    using Cfg = HistCfg<2, 3>;
    k_hist<2, 3><<<nsm, HIST_THREADS, Cfg::SMEM, s>>>(io.bins, rows, io.g, io.h, b.items, b.units,
                                                      b.st, b.partials, d);
    k_reduce<2, 3><<<jobs * p.U * 2 * RED_PARTS, 512, 0, s>>>(b.partials, b.job_first, b.job_nitems,
                                                              b.items, b.units, b.st, b.small, p.F, p.U, d);
  } else {
    using Cfg = HistCfg<1, 5>;
    k_hist<1, 5><<<nsm, HIST_THREADS, Cfg::SMEM, s>>>(io.bins, rows, io.g, io.h, b.items, b.units,
                                                      b.st, b.partials, d);
    k_reduce<1, 5><<<jobs * p.U * 1 * RED_PARTS, 512, 0, s>>>(b.partials, b.job_first, b.job_nitems,
                                                              b.items, b.units, b.st, b.small, p.F, p.U, d);
  }
  return cudaGetLastError();
}

cudaError_t set_hist_smem_attrs() {
  cudaError_t e = cudaFuncSetAttribute(k_hist<2, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       HistCfg<2, 3>::SMEM);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_hist<1, 5>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              HistCfg<1, 5>::SMEM);
}

}  // namespace yabt
