// Cross-GPU sum of the level histograms over NVLink peer memory.
//
// Row-sharded growth needs, at every level, the sum over the ranks of each
// rank's smaller-child histograms (int64 words). The exchange buffers of all
// ranks are mapped into every rank's address space (CUDA IPC, plain peer
// loads and stores -- no multicast objects), and k_xreduce sums them in place
// with a two-shot scheme: rank r owns slice r of the words, reads that slice
// from every rank, adds the N values in rank order and stores the sum into
// every rank's buffer. The word count comes from the grower's device state
// (pairs split by the previous level), so the host neither waits for the
// level nor moves a byte more than the level's histograms: this replaces an
// NCCL all-reduce whose size the host would have to read back first.
//
// Ordering: (1) each rank's block 0 tells every rank "my histograms are
// written" (fence, then a flag store); every block waits for all N flags
// before reading peers; (2) after its stores, each block fences and counts
// itself done; the last block tells every rank "your slice r is written" and
// waits for all N of those flags, so the kernel ends only when this rank's
// buffer holds the full sums. Every wait is bounded: on timeout the kernel
// sets an error bit in the grower state and returns.
#include <cstdint>
#include <cstddef>
#include <cstring>

#include "../../include/yabt_b200.h"
#include "grow.cuh"

namespace yabt {

constexpr int XR_MAX = 8;                 // ranks
constexpr long long XCHG_HEADER = 256;    // bytes before the data words
constexpr long long XSPIN_LIMIT = 1LL << 24;   // polls of ~64 ns (about 1 s)

struct XHeader {                          // at the start of every rank's exchange buffer
  unsigned ready[XR_MAX];                 // epoch when rank q's histograms were written
  unsigned done[XR_MAX];                  // epoch when rank q's slice of this buffer was summed
  unsigned blocks;                        // blocks of this rank's kernel that finished their stores
  unsigned blocks2;                       // second-phase block count of k_xallreduce
  unsigned gready[XR_MAX];                // epoch when rank q's per-node best splits were written (k_xgather)
};
static_assert(sizeof(XHeader) <= XCHG_HEADER, "exchange header");

struct XArgs {
  char* buf[XR_MAX];                      // every rank's exchange buffer, mapped here
  int rank, nranks;
  unsigned epoch;
  int level;
  long long per_job;                      // int64 words per job
  int sliced;                             // 1: reduce-scatter of this rank's feature slice only
  int F, C;                               // features, histogram channels (the slice's word ranges)
  int loop_first;                         // level == LEVEL_DYN: first level of the device-side loop
};

// Exchange epochs of a device-side level loop: the host reserves two per loop
// level starting at st->xepoch0 (every rank the same numbers), the
// reduce-scatter of level d uses xepoch0 + 2 (d - first), the gather one more.
__device__ __forceinline__ unsigned loop_epoch(const GrowState* st, int level, int first, unsigned k) {
  return st->xepoch0 + 2u * (unsigned)(level - first) + k;
}

// Feature slice of rank r of N: [F r / N, F (r + 1) / N) (the same rule as
// yabt_b200.distributed's feature_slice).
__host__ __device__ inline int slice_lo(int F, int r, int N) { return (int)((long long)F * r / N); }

__device__ __forceinline__ void st_flag(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_flag(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Waits until flags[q] == epoch for every rank q; false on timeout.
__device__ bool wait_all(const unsigned* flags, int nranks, unsigned epoch) {
  for (int q = 0; q < nranks; ++q) {
    long long spins = 0;
    while (ld_flag(flags + q) != epoch) {
      if (++spins > XSPIN_LIMIT) return false;
      __nanosleep(64);
    }
  }
  return true;
}

__global__ void __launch_bounds__(512) k_xreduce(XArgs a, GrowState* st) {
  __shared__ int s_ok, s_last;
  if (a.level == LEVEL_DYN) {                        // inside a device-side level loop
    a.level = st->level;
    if (a.level < a.loop_first) return;
    a.epoch = loop_epoch(st, a.level, a.loop_first, 0u);
  }
  if (st->level != a.level || !st->active) return;   // the same on every rank
  const long long jobs = a.level == 0 ? 1 : st->P;
  const long long words = jobs * a.per_job;
  XHeader* mine = reinterpret_cast<XHeader*>(a.buf[a.rank]);
  if (blockIdx.x == 0 && threadIdx.x < a.nranks) {
    __threadfence_system();                          // this rank's histograms (k_reduce) first
    st_flag(&reinterpret_cast<XHeader*>(a.buf[threadIdx.x])->ready[a.rank], a.epoch);
  }
  if (threadIdx.x == 0) s_ok = wait_all(mine->ready, a.nranks, a.epoch) ? 1 : 0;
  __syncthreads();
  if (!s_ok) {
    if (threadIdx.x == 0) atomicOr(&st->err, DERR_XCHG_TIMEOUT);
    return;
  }
  if (a.sliced) {
    // reduce-scatter: this rank sums only the words of its feature slice, in
    // rank order, into its own buffer (its scan reads nothing else); per job
    // the value channels [C-1][F][256] and the packed counts [F][128]
    const int flo = slice_lo(a.F, a.rank, a.nranks), fhi = slice_lo(a.F, a.rank + 1, a.nranks);
    const long long nf = fhi - flo;
    const long long vw = (long long)(a.C - 1) * YABT_NB * nf;       // value words of the slice per job
    const long long per = vw + (YABT_NB / 2) * nf;                  // + count words
    long long* own = reinterpret_cast<long long*>(a.buf[a.rank] + XCHG_HEADER);
    for (long long t = 2 * ((long long)blockIdx.x * blockDim.x + threadIdx.x); t < jobs * per;
         t += 2LL * gridDim.x * blockDim.x) {
      const long long j = t / per, w = t - j * per;
      long long i;
      if (w < vw) {
        const long long c = w / (YABT_NB * nf), off = w - c * (YABT_NB * nf);
        i = j * a.per_job + c * (long long)a.F * YABT_NB + flo * YABT_NB + off;
      } else {
        i = j * a.per_job + (long long)(a.C - 1) * a.F * YABT_NB + flo * (YABT_NB / 2) + (w - vw);
      }
      long long s0 = 0, s1 = 0;
      for (int q = 0; q < a.nranks; ++q) {           // rank order
        const longlong2 v = __ldcv(reinterpret_cast<const longlong2*>(
            reinterpret_cast<const long long*>(a.buf[q] + XCHG_HEADER) + i));
        s0 += v.x; s1 += v.y;
      }
      *reinterpret_cast<longlong2*>(own + i) = make_longlong2(s0, s1);
    }
    // no done phase: a rank overwrites its buffer only after the level's best
    // splits were gathered (k_xgather), which every rank reaches after its reads
    return;
  }
  // slice of this rank: words [lo, hi), in pairs of int64
  const long long lo = words * a.rank / a.nranks & ~1LL;
  const long long hi = a.rank + 1 == a.nranks ? words : (words * (a.rank + 1) / a.nranks & ~1LL);
  for (long long i = lo + 2 * ((long long)blockIdx.x * blockDim.x + threadIdx.x); i < hi;
       i += 2LL * gridDim.x * blockDim.x) {
    const bool pair = i + 1 < hi;
    long long s0 = 0, s1 = 0;
    for (int q = 0; q < a.nranks; ++q) {             // rank order: the same sum everywhere
      const long long* src = reinterpret_cast<const long long*>(a.buf[q] + XCHG_HEADER) + i;
      if (pair) {
        const longlong2 v = __ldcv(reinterpret_cast<const longlong2*>(src));
        s0 += v.x; s1 += v.y;
      } else {
        s0 += __ldcv(src);
      }
    }
    for (int q = 0; q < a.nranks; ++q) {
      long long* dst = reinterpret_cast<long long*>(a.buf[q] + XCHG_HEADER) + i;
      if (pair) *reinterpret_cast<longlong2*>(dst) = make_longlong2(s0, s1);
      else *dst = s0;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&mine->blocks, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x == 0) mine->blocks = 0;
  if (threadIdx.x < a.nranks) {
    __threadfence_system();
    st_flag(&reinterpret_cast<XHeader*>(a.buf[threadIdx.x])->done[a.rank], a.epoch);
  }
  __syncthreads();
  if (threadIdx.x == 0 && !wait_all(mine->done, a.nranks, a.epoch)) atomicOr(&st->err, DERR_XCHG_TIMEOUT);
}

// Per-node best split of every rank (feature-sliced growth): after each rank
// scanned its slice of the features, the ranks exchange, per active node, the
// best of their slice (the ordered key of k_scan and its NodeBest), and every
// rank keeps the largest key -- the first maximum over all features, as one
// GPU would choose it -- so k_finalize sees the same node_key and best split
// everywhere. The node totals need no exchange: every slice's features sum to
// the same node total. One block; records of 64 bytes at rec_off.
struct XGArgs {
  char* buf[XR_MAX];
  int rank, nranks;
  unsigned epoch;
  int level;
  long long rec_off;                      // bytes from the data start to the records
  int F;
  int loop_first;                         // level == LEVEL_DYN: first level of the device-side loop
};

struct XRec {
  unsigned long long key;
  NodeBest nb;
  long long pad[3];
};
static_assert(sizeof(XRec) == 64, "exchange record");
static_assert(sizeof(NodeBest) % 8 == 0 && alignof(NodeBest) == 8 && offsetof(XRec, nb) % 8 == 0,
              "records are copied in 8-byte words");

__global__ void __launch_bounds__(256) k_xgather(XGArgs a, GrowState* st, unsigned long long* node_key,
                                                 NodeBest* best) {
  __shared__ int s_ok;
  if (a.level == LEVEL_DYN) {                        // inside a device-side level loop
    a.level = st->level;
    if (a.level < a.loop_first) return;
    a.epoch = loop_epoch(st, a.level, a.loop_first, 1u);
  }
  if (st->level != a.level || !st->active) return;   // the same on every rank
  const int M = st->M;
  XRec* mine_rec = reinterpret_cast<XRec*>(a.buf[a.rank] + XCHG_HEADER + a.rec_off);
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    const unsigned long long key = node_key[m];
    const int f = (int)(0xffffffffu - (unsigned)(key & 0xffffffffULL));
    XRec r;
    r.key = key;
    r.nb = best[(size_t)m * a.F + (f >= 0 && f < a.F ? f : 0)];
    r.pad[0] = r.pad[1] = r.pad[2] = 0;
    mine_rec[m] = r;
  }
  __threadfence_system();
  __syncthreads();
  XHeader* mine = reinterpret_cast<XHeader*>(a.buf[a.rank]);
  if (threadIdx.x < a.nranks) st_flag(&reinterpret_cast<XHeader*>(a.buf[threadIdx.x])->gready[a.rank], a.epoch);
  if (threadIdx.x == 0) s_ok = wait_all(mine->gready, a.nranks, a.epoch) ? 1 : 0;
  __syncthreads();
  if (!s_ok) {
    if (threadIdx.x == 0) atomicOr(&st->err, DERR_XCHG_TIMEOUT);
    return;
  }
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    unsigned long long bk = 0;
    int bq = a.rank;
    for (int q = 0; q < a.nranks; ++q) {             // largest key; equal keys cannot come from two slices
      const XRec* rq = reinterpret_cast<const XRec*>(a.buf[q] + XCHG_HEADER + a.rec_off) + m;
      const unsigned long long k = __ldcv(reinterpret_cast<const unsigned long long*>(&rq->key));
      if (k > bk) { bk = k; bq = q; }
    }
    const int f = (int)(0xffffffffu - (unsigned)(bk & 0xffffffffULL));
    if (bq != a.rank && f >= 0 && f < a.F) {
      // 8-byte words: a record's NodeBest sits 8 bytes into the record, so it
      // is 8-byte but not 16-byte aligned
      const XRec* rq = reinterpret_cast<const XRec*>(a.buf[bq] + XCHG_HEADER + a.rec_off) + m;
      const unsigned long long* src = reinterpret_cast<const unsigned long long*>(&rq->nb);
      unsigned long long* dst = reinterpret_cast<unsigned long long*>(&best[(size_t)m * a.F + f]);
#pragma unroll
      for (int k = 0; k < (int)(sizeof(NodeBest) / 8); ++k) dst[k] = __ldcv(src + k);
    }
    node_key[m] = bk;
  }
}

// Small-vector all-reduce over the same mapped buffers (the per-tree
// statistics a row-sharded fit reduces: quantisation words, leaf-model sums
// and envelopes). The same two-shot scheme as k_xreduce: each rank copies its
// vector into its own buffer and flags it; rank r reduces slice r over the
// ranks in rank order (the same result on every rank) and stores it into
// every buffer; the done flags complete it; each rank copies the result out.
// T: element type; MAX: max instead of sum. Timeouts set st->xerr.
struct XAllArgs {
  char* buf[XR_MAX];
  int rank, nranks;
  unsigned epoch;
  long long count;                        // elements
  const void* src;
  void* dst;
};

template <typename T, bool MAX>
__global__ void __launch_bounds__(512) k_xallreduce(XAllArgs a, GrowState* st) {
  __shared__ int s_ok, s_last;
  XHeader* mine = reinterpret_cast<XHeader*>(a.buf[a.rank]);
  T* own = reinterpret_cast<T*>(a.buf[a.rank] + XCHG_HEADER);
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  for (long long i = tid; i < a.count; i += stride) own[i] = static_cast<const T*>(a.src)[i];
  // every block's copy must land before any rank reads this buffer
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&mine->blocks, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) mine->blocks = 0;   // every block has counted itself
  if (s_last && threadIdx.x < a.nranks) {
    __threadfence_system();
    st_flag(&reinterpret_cast<XHeader*>(a.buf[threadIdx.x])->ready[a.rank], a.epoch);
  }
  if (threadIdx.x == 0) s_ok = wait_all(mine->ready, a.nranks, a.epoch) ? 1 : 0;
  __syncthreads();
  if (!s_ok) {
    if (threadIdx.x == 0) atomicOr(&st->xerr, DERR_XCHG_TIMEOUT);
    return;
  }
  const long long lo = a.count * a.rank / a.nranks;
  const long long hi = a.count * (a.rank + 1) / a.nranks;
  for (long long i = lo + tid; i < hi; i += stride) {
    T acc = __ldcv(reinterpret_cast<const T*>(a.buf[0] + XCHG_HEADER) + i);
    for (int q = 1; q < a.nranks; ++q) {              // rank order: the same value everywhere
      const T v = __ldcv(reinterpret_cast<const T*>(a.buf[q] + XCHG_HEADER) + i);
      if constexpr (MAX) acc = v > acc ? v : acc;
      else acc = acc + v;
    }
    for (int q = 0; q < a.nranks; ++q) reinterpret_cast<T*>(a.buf[q] + XCHG_HEADER)[i] = acc;
  }
  __threadfence_system();
  __syncthreads();
  // second phase: the done flags (a separate counter word: blocks was reset above)
  if (threadIdx.x == 0) s_last = atomicAdd(&mine->blocks2, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last) {
    if (threadIdx.x == 0) mine->blocks2 = 0;
    if (threadIdx.x < a.nranks) {
      __threadfence_system();
      st_flag(&reinterpret_cast<XHeader*>(a.buf[threadIdx.x])->done[a.rank], a.epoch);
    }
  }
  if (threadIdx.x == 0) s_ok = wait_all(mine->done, a.nranks, a.epoch) ? 1 : 0;
  __syncthreads();
  if (!s_ok) {
    if (threadIdx.x == 0) atomicOr(&st->xerr, DERR_XCHG_TIMEOUT);
    return;
  }
  for (long long i = tid; i < a.count; i += stride) static_cast<T*>(a.dst)[i] = __ldcv(own + i);
}

}  // namespace yabt

using namespace yabt;

namespace yabt {

// Launchers of the feature-sliced exchange (the C ABI below, and the capture of
// a sharded device-side level loop in abi.cu, which passes level = LEVEL_DYN
// and the loop's first level). They check the arguments and return a YABT
// status.
int xchg_sliced_launch(yabt_grower* g, void* const* bufs, int rank, int nranks, int level, unsigned epoch,
                       int loop_first, cudaStream_t s) {
  if (!g || !bufs || nranks < 1 || nranks > XR_MAX || rank < 0 || rank >= nranks ||
      (level < 0 && level != LEVEL_DYN)) {
    set_error("yabt_grow_xreduce_sliced: bad arguments (at most %d ranks)", XR_MAX);
    return YABT_ERR_ARG;
  }
  int F = 0, C = 0, flo = 0, fhi = 0;
  if (grower_slice(g, &F, &C, &flo, &fhi) || flo != slice_lo(F, rank, nranks) || fhi != slice_lo(F, rank + 1, nranks)) {
    set_error("yabt_grow_xreduce_sliced: the grower's feature slice must be [F r / N, F (r + 1) / N)");
    return YABT_ERR_ARG;
  }
  XArgs a;
  for (int q = 0; q < XR_MAX; ++q) a.buf[q] = q < nranks ? static_cast<char*>(bufs[q]) : nullptr;
  for (int q = 0; q < nranks; ++q)
    if (!a.buf[q]) { set_error("yabt_grow_xreduce_sliced: missing buffer of rank %d", q); return YABT_ERR_ARG; }
  a.rank = rank; a.nranks = nranks; a.epoch = epoch; a.level = level;
  a.per_job = yabt_grow_small_count(g, 0);
  a.sliced = 1; a.F = F; a.C = C; a.loop_first = loop_first;
  GrowState* st = grower_state(g);
  if (!st) { set_error("yabt_grow_xreduce_sliced: grower not bound"); return YABT_ERR_ARG; }
  int dev = 0, nsm = YABT_SMS_HINT;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  {
    PhaseScope ph(PH_XCHG, s);
    k_xreduce<<<nsm, 512, 0, s>>>(a, st);
  }
  count_launches(1);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { set_error("yabt_grow_xreduce_sliced: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

int xchg_gather_launch(yabt_grower* g, void* const* bufs, int rank, int nranks, int level, unsigned epoch,
                       long long rec_offset, int loop_first, cudaStream_t s) {
  if (!g || !bufs || nranks < 1 || nranks > XR_MAX || rank < 0 || rank >= nranks ||
      (level < 0 && level != LEVEL_DYN) || rec_offset < 0 || (rec_offset & 255)) {
    set_error("yabt_grow_xgather: bad arguments (at most %d ranks, 256-byte aligned record offset)", XR_MAX);
    return YABT_ERR_ARG;
  }
  int F = 0, C = 0, flo = 0, fhi = 0;
  if (grower_slice(g, &F, &C, &flo, &fhi)) { set_error("yabt_grow_xgather: grower not bound"); return YABT_ERR_ARG; }
  XGArgs a;
  for (int q = 0; q < XR_MAX; ++q) a.buf[q] = q < nranks ? static_cast<char*>(bufs[q]) : nullptr;
  for (int q = 0; q < nranks; ++q)
    if (!a.buf[q]) { set_error("yabt_grow_xgather: missing buffer of rank %d", q); return YABT_ERR_ARG; }
  a.rank = rank; a.nranks = nranks; a.epoch = epoch; a.level = level; a.rec_off = rec_offset; a.F = F;
  a.loop_first = loop_first;
  GrowState* st = grower_state(g);
  unsigned long long* key = nullptr;
  NodeBest* best = nullptr;
  grower_best_bufs(g, &key, &best);
  if (!st || !key || !best) { set_error("yabt_grow_xgather: grower not bound"); return YABT_ERR_ARG; }
  {
    PhaseScope ph(PH_XCHG, s);
    k_xgather<<<1, 256, 0, s>>>(a, st, key, best);
  }
  count_launches(1);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { set_error("yabt_grow_xgather: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

__global__ void k_set_loop_epoch(GrowState* st, unsigned epoch0) { st->xepoch0 = epoch0; }

// The first exchange epoch of the next device-side level loop, in stream order.
int xchg_set_loop_epoch(yabt_grower* g, unsigned epoch0, cudaStream_t s) {
  GrowState* st = grower_state(g);
  if (!st) { set_error("grower not bound"); return YABT_ERR_ARG; }
  k_set_loop_epoch<<<1, 1, 0, s>>>(st, epoch0);
  count_launches(1);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { set_error("xchg_set_loop_epoch: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

}  // namespace yabt

extern "C" {

long long yabt_xchg_header_bytes(void) { return XCHG_HEADER; }

int yabt_xchg_alloc(long long bytes, void** ptr, void* ipc_handle) {
  if (bytes <= 0 || !ptr || !ipc_handle) { set_error("yabt_xchg_alloc: bad arguments"); return YABT_ERR_ARG; }
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)(bytes + XCHG_HEADER));
  if (e == cudaSuccess) e = cudaMemset(p, 0, (size_t)(bytes + XCHG_HEADER));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    set_error("yabt_xchg_alloc: %s", cudaGetErrorString(e));
    return YABT_ERR_CUDA;
  }
  *ptr = p;
  return YABT_OK;
}

int yabt_xchg_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) { set_error("yabt_xchg_open: bad arguments"); return YABT_ERR_ARG; }
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) { set_error("yabt_xchg_open: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

int yabt_xchg_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) { set_error("yabt_xchg_close: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

int yabt_xchg_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) { set_error("yabt_xchg_free: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

int yabt_grow_xreduce(yabt_grower* g, void* const* bufs, int rank, int nranks, int level, unsigned epoch,
                      void* stream) {
  if (!g || !bufs || nranks < 1 || nranks > XR_MAX || rank < 0 || rank >= nranks || level < 0) {
    set_error("yabt_grow_xreduce: bad arguments (at most %d ranks)", XR_MAX);
    return YABT_ERR_ARG;
  }
  XArgs a;
  for (int q = 0; q < XR_MAX; ++q) a.buf[q] = q < nranks ? static_cast<char*>(bufs[q]) : nullptr;
  for (int q = 0; q < nranks; ++q)
    if (!a.buf[q]) { set_error("yabt_grow_xreduce: missing buffer of rank %d", q); return YABT_ERR_ARG; }
  a.rank = rank; a.nranks = nranks; a.epoch = epoch; a.level = level;
  a.per_job = yabt_grow_small_count(g, 0);
  a.sliced = 0; a.F = 0; a.C = 0; a.loop_first = 0;
  GrowState* st = grower_state(g);
  if (!st) { set_error("yabt_grow_xreduce: grower not bound"); return YABT_ERR_ARG; }
  int dev = 0, nsm = YABT_SMS_HINT;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  // one block per SM: every block waits on the flags, so all must be resident
  {
    PhaseScope ph(PH_XCHG, static_cast<cudaStream_t>(stream));
    k_xreduce<<<nsm, 512, 0, static_cast<cudaStream_t>(stream)>>>(a, st);
  }
  count_launches(1);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { set_error("yabt_grow_xreduce: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

int yabt_grow_xallreduce(yabt_grower* g, void* const* bufs, long long buf_bytes, int rank, int nranks,
                         const void* src, void* dst, long long count, int kind, unsigned epoch, void* stream) {
  if (!g || !bufs || nranks < 1 || nranks > XR_MAX || rank < 0 || rank >= nranks || count < 0 ||
      (count > 0 && (!src || !dst)) || kind < 0 || kind > 3) {
    set_error("yabt_grow_xallreduce: bad arguments (at most %d ranks, kind 0..3)", XR_MAX);
    return YABT_ERR_ARG;
  }
  const long long esize = kind < 2 ? 8 : 4;
  if (count * esize > buf_bytes) {
    set_error("yabt_grow_xallreduce: %lld bytes exceed the exchange buffers' %lld", count * esize, buf_bytes);
    return YABT_ERR_ARG;
  }
  if (count == 0) return YABT_OK;
  XAllArgs a;
  for (int q = 0; q < XR_MAX; ++q) a.buf[q] = q < nranks ? static_cast<char*>(bufs[q]) : nullptr;
  for (int q = 0; q < nranks; ++q)
    if (!a.buf[q]) { set_error("yabt_grow_xallreduce: missing buffer of rank %d", q); return YABT_ERR_ARG; }
  a.rank = rank; a.nranks = nranks; a.epoch = epoch; a.count = count; a.src = src; a.dst = dst;
  GrowState* st = grower_state(g);
  if (!st) { set_error("yabt_grow_xallreduce: grower not bound"); return YABT_ERR_ARG; }
  // few blocks (all resident: every block waits on the flags)
  const unsigned grid = (unsigned)std::min<long long>(8, std::max<long long>(1, (count + 4095) / 4096));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  {
    PhaseScope ph(PH_XCHG, s);
    switch (kind) {
      case 0: k_xallreduce<long long, false><<<grid, 512, 0, s>>>(a, st); break;
      case 1: k_xallreduce<double, false><<<grid, 512, 0, s>>>(a, st); break;
      case 2: k_xallreduce<int, true><<<grid, 512, 0, s>>>(a, st); break;
      default: k_xallreduce<float, true><<<grid, 512, 0, s>>>(a, st); break;
    }
  }
  count_launches(1);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) { set_error("yabt_grow_xallreduce: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

int yabt_grow_xerr(yabt_grower* g, unsigned* bits) {
  GrowState* st = grower_state(g);
  if (!st || !bits) { set_error("yabt_grow_xerr: grower not bound"); return YABT_ERR_ARG; }
  const cudaError_t e = cudaMemcpy(bits, &st->xerr, sizeof(unsigned), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) { set_error("yabt_grow_xerr: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  return YABT_OK;
}

int yabt_grow_xreduce_sliced(yabt_grower* g, void* const* bufs, int rank, int nranks, int level, unsigned epoch,
                             void* stream) {
  if (level < 0) { set_error("yabt_grow_xreduce_sliced: bad level"); return YABT_ERR_ARG; }
  return xchg_sliced_launch(g, bufs, rank, nranks, level, epoch, 0, static_cast<cudaStream_t>(stream));
}

int yabt_grow_xgather(yabt_grower* g, void* const* bufs, int rank, int nranks, int level, unsigned epoch,
                      long long rec_offset, void* stream) {
  if (level < 0) { set_error("yabt_grow_xgather: bad level"); return YABT_ERR_ARG; }
  return xchg_gather_launch(g, bufs, rank, nranks, level, epoch, rec_offset, 0, static_cast<cudaStream_t>(stream));
}

long long yabt_grow_xgather_bytes(const yabt_grower* g) {
  return g ? ((long long)grower_maxa(g) * 64 + 255) / 256 * 256 : -1;
}

}  // extern "C"
