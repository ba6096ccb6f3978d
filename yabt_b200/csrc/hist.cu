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

// LIMBS: 3 (g low, g high, count; two subs per lane) or 5 (g, h low / high,
// count; one sub); 2 and 4 are the same without the count limb, for a root
// level whose per-bin row counts are cached (the counts of all rows do not
// change between the trees of a fit).
template <int S, int LIMBS>
struct HistCfg {
  static_assert((S == 2 && (LIMBS == 3 || LIMBS == 2)) || (S == 1 && (LIMBS == 5 || LIMBS == 4)),
                "supported (S, LIMBS) pairs");
  static constexpr bool HAS_H = LIMBS >= 4;                 // hessian limbs present
  static constexpr bool HAS_CNT = (LIMBS & 1) != 0;         // count limb present (the last one)
  static constexpr int WORDS = LIMBS * S * YABT_NB * 32;   // u32 words per histogram
  static constexpr int LIMB_STRIDE = S * YABT_NB * 32;      // words between limbs
  static constexpr int SMEM = WORDS * 4;
};

// Shared-memory reductions with explicit 32-bit shared addresses; the limb
// offsets are immediates, so each update is one red instruction.
template <int OFF>
__device__ __forceinline__ void red_s(unsigned addr, unsigned v) {
  asm volatile("red.shared.add.u32 [%0+%1], %2;\n" ::"r"(addr), "n"(OFF), "r"(v) : "memory");
}

// Row contribution of one lane: feature sub 0 at bin b0, sub 1 at bin b1.
// lb is the shared address of word (bin 0, lane) of limb 0. FULL: every lane
// owns a feature of every sub (no per-lane predicates).
template <int S, int LIMBS, bool FULL>
__device__ __forceinline__ void acc_row(unsigned lb, unsigned b0, unsigned b1, bool ok0, bool ok1,
                                        int vg, int vh) {
  constexpr int LS = HistCfg<S, LIMBS>::LIMB_STRIDE * 4;   // bytes between limbs
  const unsigned glo = (unsigned)vg & 0xFFFFu, ghi = (unsigned)(vg >> 16);
  if (FULL || ok0) {
    const unsigned a0 = lb + (b0 << 7);
    red_s<0>(a0, glo);
    red_s<LS>(a0, ghi);
    if constexpr (HistCfg<S, LIMBS>::HAS_H) {
      red_s<2 * LS>(a0, (unsigned)vh & 0xFFFFu);
      red_s<3 * LS>(a0, (unsigned)(vh >> 16));
    }
    if constexpr (HistCfg<S, LIMBS>::HAS_CNT) red_s<(LIMBS - 1) * LS>(a0, 1u);
  }
  if constexpr (S == 2) {
    if (FULL || ok1) {
      const unsigned a1 = lb + (b1 << 7) + YABT_NB * 32 * 4;
      red_s<0>(a1, glo);
      red_s<LS>(a1, ghi);
      if constexpr (HistCfg<S, LIMBS>::HAS_CNT) red_s<(LIMBS - 1) * LS>(a1, 1u);
    }
  }
}

// ---------------------------------------------------------------- async copy / shared helpers
__device__ __forceinline__ void cp_async16s(unsigned saddr, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(gmem));
}
__device__ __forceinline__ unsigned lds_u16(unsigned a) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ unsigned lds_u8(unsigned a) {
  unsigned short v;
  asm volatile("ld.shared.u8 %0, [%1];\n" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts_u32(unsigned a, int v) {
  asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void lds_v4(unsigned a, int& x, int& y, int& z, int& w) {
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n" : "=r"(x), "=r"(y), "=r"(z), "=r"(w) : "r"(a) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Block geometry and shared-memory budget of k_hist: the histogram plus a
// per-warp ring of STG stages of RPS row slots (64 bytes each). Eight rows per
// stage let every lane of a 64-wide tile copy 16 bytes and halve the per-row
// share of the stage bookkeeping (row ids, gradients, copy issue, waits); two
// stages (one in flight while one is consumed) keep the ring at 32 KB.
template <int S, int LIMBS>
struct HistPipe {
  static constexpr int WARPS = 32;
  static constexpr int THREADS = WARPS * 32;
  static constexpr int STG = 2;
  static constexpr int RPS = 8;                         // rows per stage
  static constexpr int STAGE_BYTES = RPS * 64;
  static constexpr int VSLOT = 64;                      // per warp: a stage's quantised g (and h) values
  static constexpr int SMEM = HistCfg<S, LIMBS>::SMEM + WARPS * STG * STAGE_BYTES + WARPS * VSLOT;
  static_assert(RPS == 8, "a stage's values are read back as two 16-byte loads");
};

// One work item of one warp: rows [0, nrow) of its share (positions in the row
// list), tile rows of TW bytes. Stage s holds RPS rows; the first RPS*LPR lanes
// copy 16 bytes each (row lane/LPR, piece lane%LPR) with cp.async; the row's
// gradient is loaded with the copy. Row ids are loaded one iteration ahead of
// their copy, so a warp keeps STG-1 stages in flight while it consumes one.
// The loads and shuffles of a stage's rows are issued before their shared-
// memory reductions, and full stages need no per-row bounds checks.
template <int S, int LIMBS, int TW, bool FULL>
__device__ __forceinline__ void hist_warp(unsigned lb, unsigned ring, unsigned vslot, const uint8_t* __restrict__ tb,
                                          const int* __restrict__ lst, int base, int nrow,
                                          const float* __restrict__ g, const float* __restrict__ h,
                                          float gs, float hs, int k0, bool ok0, bool ok1, int lane) {
  using Pipe = HistPipe<S, LIMBS>;
  constexpr int LPR = TW / 16;
  constexpr int SB = Pipe::STAGE_BYTES;
  constexpr int RPS = Pipe::RPS;
  constexpr int STG = Pipe::STG;
  constexpr int CL = RPS * LPR;                 // copying lanes (<= 32)
  static_assert(CL <= 32, "stage geometry");
  const int rr = lane / LPR, piece = lane % LPR;
  const bool copier = lane < CL;
  const int nst = (nrow + RPS - 1) / RPS;
  auto rid_of = [&](int s) -> int {
    const int k = s * RPS + rr;
    if (!copier || k >= nrow) return -1;
    return lst ? __ldg(lst + base + k) : base + k;
  };
  auto copy = [&](int s, int r) {
    if (r >= 0) cp_async16s(ring + (s % STG) * SB + rr * 64 + piece * 16, tb + (size_t)r * TW + piece * 16);
  };
  float gq[STG], hq[STG];
#pragma unroll
  for (int s = 0; s < STG - 1; ++s) {
    const int r = rid_of(s);
    gq[s] = r >= 0 ? __ldg(g + r) : 0.f;
    hq[s] = (HistCfg<S, LIMBS>::HAS_H && r >= 0) ? __ldg(h + r) : 0.f;
    if (s < nst) copy(s, r);
    cp_commit();
  }
  int rnext = rid_of(STG - 1);
  // byte offset of this lane's bin(s) inside a row slot
  const unsigned boff = (TW == 64) ? (S == 2 ? 2u * lane : 2u * lane + k0) : (unsigned)(lane & (TW - 1));
  for (int s = 0; s < nst; ++s) {
    const int r = rnext;
    rnext = rid_of(s + STG);
    gq[STG - 1] = r >= 0 ? __ldg(g + r) : 0.f;
    hq[STG - 1] = (HistCfg<S, LIMBS>::HAS_H && r >= 0) ? __ldg(h + r) : 0.f;
    if (s + STG - 1 < nst) copy(s + STG - 1, r);
    cp_commit();
    // the first lane of each stage row publishes the row's quantised values;
    // every lane reads all of them back with 16-byte loads (no per-row shuffle)
    if (lane % LPR == 0 && rr < RPS) {
      sts_u32(vslot + rr * 4, __float2int_rn(gq[0] * gs));
      if (HistCfg<S, LIMBS>::HAS_H) sts_u32(vslot + 32 + rr * 4, __float2int_rn(hq[0] * hs));
    }
    cp_wait<STG - 1>();
    __syncwarp();
    const unsigned stg = ring + (s % STG) * SB;   // row q at stg + 64 q
    const int nr = min(RPS, nrow - s * RPS);
    unsigned wv[RPS];
    int vg[RPS], vh[RPS];
    lds_v4(vslot, vg[0], vg[1], vg[2], vg[3]);
    lds_v4(vslot + 16, vg[4], vg[5], vg[6], vg[7]);
    if (HistCfg<S, LIMBS>::HAS_H) {
      lds_v4(vslot + 32, vh[0], vh[1], vh[2], vh[3]);
      lds_v4(vslot + 48, vh[4], vh[5], vh[6], vh[7]);
    } else {
#pragma unroll
      for (int q = 0; q < RPS; ++q) vh[q] = 0;
    }
#pragma unroll
    for (int q = 0; q < RPS; ++q) {
      if constexpr (TW == 64 && S == 2) wv[q] = lds_u16(stg + q * 64 + boff);
      else wv[q] = lds_u8(stg + q * 64 + boff);
    }
    if (nr == RPS) {
#pragma unroll
      for (int q = 0; q < RPS; ++q)
        acc_row<S, LIMBS, FULL>(lb, wv[q] & 0xFFu, wv[q] >> 8, ok0, ok1, vg[q], vh[q]);
    } else {
#pragma unroll
      for (int q = 0; q < RPS; ++q)
        if (q < nr) acc_row<S, LIMBS, FULL>(lb, wv[q] & 0xFFu, wv[q] >> 8, ok0, ok1, vg[q], vh[q]);
    }
    __syncwarp();
#pragma unroll
    for (int t = 0; t < STG - 1; ++t) { gq[t] = gq[t + 1]; hq[t] = hq[t + 1]; }
  }
  cp_wait<0>();
}

// A 16-wide tail tile with at most 16 real features: lane l takes feature
// l % LW of row l / LW, so one shared-memory reduction covers REP = 32 / LW
// rows of the stage (the tile's histogram is kept REP times, one copy per
// lane group, and k_reduce adds the copies). Same staging as hist_warp.
template <int S, int LIMBS, int REP>
__device__ __forceinline__ void hist_warp_narrow(unsigned lb, unsigned ring, const uint8_t* __restrict__ tb,
                                                 const int* __restrict__ lst, int base, int nrow,
                                                 const float* __restrict__ g, const float* __restrict__ h,
                                                 float gs, float hs, bool okf, int lane) {
  using Pipe = HistPipe<S, LIMBS>;
  constexpr int TW = 16, SB = Pipe::STAGE_BYTES, RPS = Pipe::RPS, STG = Pipe::STG;
  constexpr int LW = 32 / REP;
  static_assert(RPS % REP == 0, "stage rows");
  const bool copier = lane < RPS;
  const int nst = (nrow + RPS - 1) / RPS;
  auto rid_of = [&](int s) -> int {
    const int k = s * RPS + lane;
    if (!copier || k >= nrow) return -1;
    return lst ? __ldg(lst + base + k) : base + k;
  };
  auto copy = [&](int s, int r) {
    if (r >= 0) cp_async16s(ring + (s % STG) * SB + lane * 64, tb + (size_t)r * TW);
  };
  float gq[STG], hq[STG];
#pragma unroll
  for (int s = 0; s < STG - 1; ++s) {
    const int r = rid_of(s);
    gq[s] = r >= 0 ? __ldg(g + r) : 0.f;
    hq[s] = (HistCfg<S, LIMBS>::HAS_H && r >= 0) ? __ldg(h + r) : 0.f;
    if (s < nst) copy(s, r);
    cp_commit();
  }
  int rnext = rid_of(STG - 1);
  const int rsub = lane / LW, byte = lane % LW;
  for (int s = 0; s < nst; ++s) {
    const int r = rnext;
    rnext = rid_of(s + STG);
    gq[STG - 1] = r >= 0 ? __ldg(g + r) : 0.f;
    hq[STG - 1] = (HistCfg<S, LIMBS>::HAS_H && r >= 0) ? __ldg(h + r) : 0.f;
    if (s + STG - 1 < nst) copy(s + STG - 1, r);
    cp_commit();
    cp_wait<STG - 1>();
    __syncwarp();
    const int vgl = __float2int_rn(gq[0] * gs);
    const int vhl = HistCfg<S, LIMBS>::HAS_H ? __float2int_rn(hq[0] * hs) : 0;
    const unsigned stg = ring + (s % STG) * SB;
    const int nr = min(RPS, nrow - s * RPS);
#pragma unroll
    for (int it = 0; it < RPS / REP; ++it) {
      const int q = it * REP + rsub;                   // stage row of this lane
      const int vg = __shfl_sync(0xffffffffu, vgl, q);
      const int vh = HistCfg<S, LIMBS>::HAS_H ? __shfl_sync(0xffffffffu, vhl, q) : 0;
      const unsigned b = lds_u8(stg + q * 64 + byte);
      acc_row<S, LIMBS, false>(lb, b, 0u, okf && q < nr, false, vg, vh);
    }
    __syncwarp();
#pragma unroll
    for (int t = 0; t < STG - 1; ++t) { gq[t] = gq[t + 1]; hq[t] = hq[t + 1]; }
  }
  cp_wait<0>();
}

// rows: the active row list (nullptr = identity, row = begin + i)
// Persistent: one block per SM claims runs of consecutive work items from a
// device counter; the warps stream contiguous shares of each item's rows into
// a shared histogram that is flushed once per (job, unit) segment of the run.
// level_gate == LEVEL_DYN (device-side level loop): the level is the state's,
// the inputs are the tree's (io_dev) and the row list is rows (even levels) or
// rows_odd (odd levels).
template <int S, int LIMBS>
__global__ void __launch_bounds__(HistPipe<S, LIMBS>::THREADS, 1)
k_hist(const uint8_t* __restrict__ bins, const int* __restrict__ rows,
       const float* __restrict__ g, const float* __restrict__ h,
       HistItem* __restrict__ items, const UnitDesc* __restrict__ units,
       GrowState* st, unsigned* __restrict__ partials, int level_gate,
       const TreeIO* __restrict__ io_dev, const int* __restrict__ rows_odd) {
  using Cfg = HistCfg<S, LIMBS>;
  using Pipe = HistPipe<S, LIMBS>;
  extern __shared__ __align__(16) unsigned sh[];
  __shared__ int s_a, s_e;
  pdl_wait();
  if (level_gate == LEVEL_DYN) {
    level_gate = st->level;
    if (level_gate < 1) return;
    bins = io_dev->bins; g = io_dev->g; h = io_dev->h;
    if (level_gate & 1) rows = rows_odd;
  }
  if (st->level != level_gate || !st->active) return;
  const int nitems = st->n_items;
  const float gs = st->gscale, hs = st->hscale;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const unsigned sh_s = (unsigned)__cvta_generic_to_shared(sh);
  const unsigned lb = sh_s + lane * 4;                       // word (bin 0, lane) of limb 0
  const unsigned ring = sh_s + Cfg::WORDS * 4 + warp * Pipe::STG * Pipe::STAGE_BYTES;
  const unsigned vslot = sh_s + Cfg::WORDS * 4 + Pipe::WARPS * Pipe::STG * Pipe::STAGE_BYTES + warp * Pipe::VSLOT;
  auto flush = [&](int seg_item) {
    __syncthreads();
    unsigned* dst = partials + (size_t)items[seg_item].slot * Cfg::WORDS;
    for (int i = threadIdx.x * 4; i < Cfg::WORDS; i += blockDim.x * 4)
      *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(sh + i);
    __syncthreads();
  };
  for (;;) {
    // guided runs: a claim of up to RUN_MAX consecutive items, shrinking as the
    // level's work runs out so that the blocks finish together
    if (threadIdx.x == 0) {
      const int cur = *(volatile int*)&st->item_counter;
      const int k = max(1, min(RUN_MAX, (nitems - cur) / (int)gridDim.x));
      const int a = atomicAdd(&st->item_counter, k);
      s_a = a;
      s_e = min(a + k, nitems);
    }
    __syncthreads();
    const int a = s_a, e = s_e;
    if (a >= nitems) break;
    // consecutive items of one (job, unit) accumulate into one shared histogram
    // (at most CHUNK_MAX rows, the limb bound) and are flushed once, into the
    // partial slot of the segment's first item; `used` marks those slots
    int seg = -1, seg_rows = 0, seg_job = -1, seg_unit = -1;
    for (int it = a; it < e; ++it) {
      const HistItem item = items[it];
      const bool cont = seg >= 0 && item.job == seg_job && item.unit == seg_unit &&
                        seg_rows + item.count <= CHUNK_MAX;
      if (!cont) {
        if (seg >= 0) flush(seg);
        for (int i = threadIdx.x * 4; i < Cfg::WORDS; i += blockDim.x * 4)
          *reinterpret_cast<uint4*>(sh + i) = make_uint4(0, 0, 0, 0);
        __syncthreads();
        seg = it; seg_rows = 0; seg_job = item.job; seg_unit = item.unit;
      }
      if (threadIdx.x == 0) items[it].used = cont ? 0 : 1;
      seg_rows += item.count;
      const UnitDesc& ud = units[item.unit];
      const uint8_t* tb = bins + ud.off;
      const bool ok0 = ud.feat[0][lane] >= 0 && (ud.width != 16 || lane < 16);
      const bool ok1 = (S == 2) && ud.nsub > 1 && ud.feat[S == 2 ? 1 : 0][lane] >= 0;
      const int per = (item.count + nw - 1) / nw;
      const int w0 = min(item.count, warp * per), w1 = min(item.count, w0 + per);
      const int* lst = rows ? rows + item.begin : nullptr;
      const int base = rows ? w0 : item.begin + w0;
      if (YABT_BOUNDS_CHECKED) {
        // every row of this warp's share must be a row of the matrix
        bool bad = false;
        if (lst) {
          for (int k = lane; k < w1 - w0; k += 32) {
            const int r = lst[base + k];
            bad |= r < 0 || r >= st->n_rows;
          }
        } else {
          bad = base < 0 || base + (w1 - w0) > st->n_rows;
        }
        if (__any_sync(0xffffffffu, bad)) {
          if (lane == 0) atomicOr(&st->err, DERR_BOUNDS);
          continue;
        }
      }
      const bool full = ud.width == 64 && (S == 1 || ud.nsub == 2);
      if (full)
        hist_warp<S, LIMBS, 64, true>(lb, ring, vslot, tb, lst, base, w1 - w0, g, h, gs, hs, ud.k0, ok0, ok1, lane);
      else if (ud.width == 64)
        hist_warp<S, LIMBS, 64, false>(lb, ring, vslot, tb, lst, base, w1 - w0, g, h, gs, hs, ud.k0, ok0, ok1, lane);
      else if (ud.width == 32)
        hist_warp<S, LIMBS, 32, false>(lb, ring, vslot, tb, lst, base, w1 - w0, g, h, gs, hs, 0, ok0, false, lane);
      else if (ud.rep == 4)
        hist_warp_narrow<S, LIMBS, 4>(lb, ring, tb, lst, base, w1 - w0, g, h, gs, hs, ud.feat[0][lane] >= 0, lane);
      else if (ud.rep == 2)
        hist_warp_narrow<S, LIMBS, 2>(lb, ring, tb, lst, base, w1 - w0, g, h, gs, hs, ud.feat[0][lane] >= 0, lane);
      else
        hist_warp<S, LIMBS, 16, false>(lb, ring, vslot, tb, lst, base, w1 - w0, g, h, gs, hs, 0, ok0, false, lane);
    }
    flush(seg);
  }
}

// One block per (job, unit, sub, bin-part): sums the u32-limb partials of the
// job's items for 16 bins x 32 lanes (one word per thread) into exact int64
// and writes [job][c][f][bin] (c = 0 g, 1 h (general path), last = count)
// through a small shared-memory transpose. The item loop is unrolled so that
// 8 items' limbs are in flight per thread.
constexpr int RED_PARTS = 16;   // bins are split into 16 parts of 16
constexpr int RED_THREADS = 512;
template <int S, int LIMBS>
__global__ void __launch_bounds__(RED_THREADS)
k_reduce(const unsigned* __restrict__ partials, const int* __restrict__ job_first,
         const int* __restrict__ job_nitems, const HistItem* __restrict__ items,
         const UnitDesc* __restrict__ units, GrowState* st, long long* __restrict__ out,
         int F, int U, int level_gate, int igroups) {
  pdl_wait();
  using Cfg = HistCfg<S, LIMBS>;
  constexpr int C = Cfg::HAS_H ? 3 : 2;       // output channels (counts last)
  constexpr int CW = Cfg::HAS_CNT ? C : C - 1; // channels written here (cached counts are copied in)
  constexpr int BPP = YABT_NB / RED_PARTS;     // bins per part (16)
  __shared__ long long tsm[C][32][BPP + 1];
  if (level_gate == LEVEL_DYN && (level_gate = st->level) < 1) return;
  if (st->level != level_gate || !st->active) return;
  const int njobs = (level_gate == 0) ? 1 : st->P;
  int b = blockIdx.x;
  const int grp = b % igroups; b /= igroups;
  const int part = b % RED_PARTS; b /= RED_PARTS;
  const int sub = b % S; b /= S;
  const int unit = b % U;
  const int job = b / U;
  if (job >= njobs) return;
  const UnitDesc& ud = units[unit];
  if (sub >= ud.nsub) return;
  // item group grp of igroups (levels with few jobs split their items so that
  // enough blocks run; the groups' sums meet in int64 atomics)
  const int nall = job_nitems[job * U + unit];
  const int per = (nall + igroups - 1) / igroups;
  const int first = job_first[job * U + unit] + grp * per;
  const int nit = max(0, min(nall - grp * per, per));
  if (nit == 0 && igroups > 1) return;   // nothing to add
  const int w = threadIdx.x;                               // (bin-in-part, lane)
  const size_t woff = (size_t)sub * YABT_NB * 32 + (size_t)part * BPP * 32 + w;
  long long ag = 0, ah = 0;
  unsigned long long ac = 0;
  constexpr int UNR = 8;
  int q = 0;
  // only slots that received a flush (`used`) hold partials; merged items' slots are skipped
  for (; q + UNR <= nit; q += UNR) {
    unsigned lo[UNR], hi[UNR], cn[UNR], hlo[UNR], hhi[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const HistItem* ip = items + first + q + u;
      const bool used = __ldg(&ip->used) != 0;
      const unsigned* p = partials + (size_t)__ldg(&ip->slot) * Cfg::WORDS + woff;
      lo[u] = used ? __ldg(p) : 0u;
      hi[u] = used ? __ldg(p + Cfg::LIMB_STRIDE) : 0u;
      if constexpr (Cfg::HAS_H) {
        hlo[u] = used ? __ldg(p + 2 * Cfg::LIMB_STRIDE) : 0u;
        hhi[u] = used ? __ldg(p + 3 * Cfg::LIMB_STRIDE) : 0u;
      }
      cn[u] = (Cfg::HAS_CNT && used) ? __ldg(p + (LIMBS - 1) * Cfg::LIMB_STRIDE) : 0u;
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      ag += (long long)(int)hi[u] * 65536LL + (long long)lo[u];
      if constexpr (Cfg::HAS_H) ah += (long long)(int)hhi[u] * 65536LL + (long long)hlo[u];
      ac += cn[u];
    }
  }
  for (; q < nit; ++q) {
    const HistItem* ip = items + first + q;
    if (__ldg(&ip->used) == 0) continue;
    const unsigned* p = partials + (size_t)__ldg(&ip->slot) * Cfg::WORDS + woff;
    ag += (long long)(int)__ldg(p + Cfg::LIMB_STRIDE) * 65536LL + (long long)__ldg(p);
    if constexpr (Cfg::HAS_H)
      ah += (long long)(int)__ldg(p + 3 * Cfg::LIMB_STRIDE) * 65536LL + (long long)__ldg(p + 2 * Cfg::LIMB_STRIDE);
    if constexpr (Cfg::HAS_CNT) ac += __ldg(p + (LIMBS - 1) * Cfg::LIMB_STRIDE);
  }
  {
    const int bl = w >> 5, j = w & 31;
    tsm[0][j][bl] = ag;
    if constexpr (C == 3) tsm[1][j][bl] = ah;
    tsm[C - 1][j][bl] = (long long)ac;
  }
  __syncthreads();
  const long long job_base = (long long)job * small_job_words(C, F);
  for (int e = threadIdx.x; e < CW * 32 * BPP; e += blockDim.x) {
    const int bl = e % BPP, j = (e / BPP) & 31, c = e / (BPP * 32);
    const int f = ud.feat[sub][j];
    if (f < 0 || j >= ud.lw) continue;   // narrow tiles: lanes j, j+lw, ... are copies of one feature
    long long* dst;
    long long v;
    auto val = [&](int bb) {          // sum of the lane copies of feature f
      long long t = 0;
      for (int k = j; k < 32; k += ud.lw) t += tsm[c][k][bb];
      return t;
    };
    if (c < C - 1) {
      dst = out + job_base + ((long long)c * F + f) * YABT_NB + part * BPP + bl;
      v = val(bl);
    } else if ((bl & 1) == 0) {   // counts: bins 2k, 2k+1 in one word (no carry between the halves)
      const unsigned long long lo = (unsigned long long)val(bl) & 0xffffffffULL;
      const unsigned long long hi = (unsigned long long)val(bl + 1) << 32;
      dst = out + job_base + (long long)(C - 1) * F * YABT_NB + (long long)f * (YABT_NB / 2) + (part * BPP + bl) / 2;
      v = (long long)(lo | hi);
    } else {
      continue;
    }
    if (igroups == 1) *dst = v;
    else atomicAdd(reinterpret_cast<unsigned long long*>(dst), (unsigned long long)v);
  }
}

// root_counts (level 0 over all rows only): 0 as usual; 1 as usual and keep a
// copy of the per-bin row counts in b.root_cnt; 2 the kernels without the
// count limb, the counts copied in from b.root_cnt.
cudaError_t launch_hist_kernels(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int d,
                                int jobs, int nsm, cudaStream_t s, cudaEvent_t after_hist, int root_counts) {
  // nullptr: identity; a device-side loop level picks rows[0] / rows[1] by its parity
  const int* rows = d == 0 ? io.root_rows : d == LEVEL_DYN ? b.rows[0] : b.rows[d & 1];
  if (d != 0 || io.root_rows) root_counts = 0;
  const size_t cnt_off = (size_t)(p.C - 1) * p.F * YABT_NB;      // count words of job 0 in `small`
  const size_t cnt_bytes = (size_t)p.F * (YABT_NB / 2) * 8;
  // levels with at most a few jobs split each job's items over several reduce
  // blocks, which add into a zeroed histogram
  const int igroups = std::max(1, 8 / jobs);
  if (igroups > 1) {
    const cudaError_t e = cudaMemsetAsync(b.small, 0, (size_t)jobs * small_job_words(p.C, p.F) * 8, s);
    if (e != cudaSuccess) return e;
  }
  cudaError_t le = cudaSuccess;
  if (!p.general && root_counts != 2) {
    { PhaseScope ph(PH_HIST, s); le = launch_pdl(k_hist<2, 3>, dim3(nsm), dim3(HistPipe<2, 3>::THREADS), HistPipe<2, 3>::SMEM, s, io.bins, rows, io.g, io.h, b.items, b.units,
                                                      b.st, b.partials, d, b.io_dev, b.rows[1]); }
    if (le != cudaSuccess) return le;
    if (after_hist) cudaEventRecord(after_hist, s);
    { PhaseScope ph(PH_REDUCE, s); le = launch_pdl(k_reduce<2, 3>, dim3(jobs * p.U * 2 * RED_PARTS * igroups), dim3(RED_THREADS), 0, s, 
        b.partials, b.job_first, b.job_nitems, b.items, b.units, b.st, b.small, p.F, p.U, d, igroups); }
    if (le != cudaSuccess) return le;
  } else if (!p.general) {
    { PhaseScope ph(PH_HIST, s); le = launch_pdl(k_hist<2, 2>, dim3(nsm), dim3(HistPipe<2, 2>::THREADS), HistPipe<2, 2>::SMEM, s, io.bins, rows, io.g, io.h, b.items, b.units,
                                                      b.st, b.partials, d, b.io_dev, b.rows[1]); }
    if (le != cudaSuccess) return le;
    if (after_hist) cudaEventRecord(after_hist, s);
    { PhaseScope ph(PH_REDUCE, s); le = launch_pdl(k_reduce<2, 2>, dim3(jobs * p.U * 2 * RED_PARTS * igroups), dim3(RED_THREADS), 0, s, 
        b.partials, b.job_first, b.job_nitems, b.items, b.units, b.st, b.small, p.F, p.U, d, igroups); }
    if (le != cudaSuccess) return le;
  } else if (root_counts != 2) {
    { PhaseScope ph(PH_HIST, s); le = launch_pdl(k_hist<1, 5>, dim3(nsm), dim3(HistPipe<1, 5>::THREADS), HistPipe<1, 5>::SMEM, s, io.bins, rows, io.g, io.h, b.items, b.units,
                                                      b.st, b.partials, d, b.io_dev, b.rows[1]); }
    if (le != cudaSuccess) return le;
    if (after_hist) cudaEventRecord(after_hist, s);
    { PhaseScope ph(PH_REDUCE, s); le = launch_pdl(k_reduce<1, 5>, dim3(jobs * p.U * 1 * RED_PARTS * igroups), dim3(RED_THREADS), 0, s, 
        b.partials, b.job_first, b.job_nitems, b.items, b.units, b.st, b.small, p.F, p.U, d, igroups); }
    if (le != cudaSuccess) return le;
  } else {
    { PhaseScope ph(PH_HIST, s); le = launch_pdl(k_hist<1, 4>, dim3(nsm), dim3(HistPipe<1, 4>::THREADS), HistPipe<1, 4>::SMEM, s, io.bins, rows, io.g, io.h, b.items, b.units,
                                                      b.st, b.partials, d, b.io_dev, b.rows[1]); }
    if (le != cudaSuccess) return le;
    if (after_hist) cudaEventRecord(after_hist, s);
    { PhaseScope ph(PH_REDUCE, s); le = launch_pdl(k_reduce<1, 4>, dim3(jobs * p.U * 1 * RED_PARTS * igroups), dim3(RED_THREADS), 0, s, 
        b.partials, b.job_first, b.job_nitems, b.items, b.units, b.st, b.small, p.F, p.U, d, igroups); }
    if (le != cudaSuccess) return le;
  }
  count_launches(2);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && root_counts == 1)
    e = cudaMemcpyAsync(b.root_cnt, b.small + cnt_off, cnt_bytes, cudaMemcpyDeviceToDevice, s);
  if (e == cudaSuccess && root_counts == 2)
    e = cudaMemcpyAsync(b.small + cnt_off, b.root_cnt, cnt_bytes, cudaMemcpyDeviceToDevice, s);
  return e;
}

// root_cnt [F][128] (bins 2k, 2k + 1 in the low, high 32 bits) -> out [F][256]
__global__ void k_unpack_counts(const long long* __restrict__ packed, long long F, long long* __restrict__ out) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < F * (YABT_NB / 2);
       i += (long long)gridDim.x * blockDim.x) {
    const unsigned long long w = (unsigned long long)packed[i];
    out[2 * i] = (long long)(w & 0xffffffffull);
    out[2 * i + 1] = (long long)(w >> 32);
  }
}

cudaError_t launch_unpack_counts(const GrowParams& p, const GrowBufs& b, long long* out, cudaStream_t s) {
  const long long words = (long long)p.F * (YABT_NB / 2);
  k_unpack_counts<<<(unsigned)std::min<long long>((words + 255) / 256, 4096), 256, 0, s>>>(b.root_cnt, p.F, out);
  count_launches(1);
  return cudaGetLastError();
}

cudaError_t set_hist_smem_attrs() {
  cudaError_t e = cudaFuncSetAttribute(k_hist<2, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       HistPipe<2, 3>::SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_hist<2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, HistPipe<2, 2>::SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_hist<1, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, HistPipe<1, 4>::SMEM);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(k_hist<1, 5>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              HistPipe<1, 5>::SMEM);
}

}  // namespace yabt
