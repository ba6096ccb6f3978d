// Measurement only: the shared-memory reduction throughput that bounds k_hist.
//
// k_hist adds every (row, feature) into exact u32 limbs of a shared histogram
// laid out [limb][sub][bin][lane] (lane = feature, so the 32 lanes of one
// reduction hit 32 different banks): 3 reductions per (row, feature) on the
// unit-hessian path (g low, g high, count; two 32-feature subs per lane),
// 5 on the general path (g, h low / high, count; one sub). This kernel issues
// the same reductions with the same layout, grid (one 1024-thread block per
// SM) and pseudo-random bins, and nothing else, so its rate of (row, feature)
// updates is the ceiling k_hist's own rate is compared with. Every address
// stays inside the block's histogram; there are no waits. Limbs 2 and 4 are
// the root levels whose counts come from the fit's cache (no count limb).
#include "../../include/yabt_b200.h"
#include "common.cuh"

namespace yabt {
namespace {

constexpr int PROBE_THREADS = 1024;

// active < 32: each lane issues a (row, feature)'s reductions only with
// probability active/32 (a hash of the row and lane), the rest predicated off,
// as a sparse-bin histogram skipping the default bin would issue them.
template <int LIMBS, int S, bool MASKED>
__global__ void __launch_bounds__(PROBE_THREADS, 1) k_probe_red(int iters, unsigned long long* sink, int active) {
  extern __shared__ __align__(16) unsigned psh[];
  constexpr int WORDS = LIMBS * S * YABT_NB * 32;
  constexpr int LS = S * YABT_NB * 32 * 4;       // bytes between limbs
  for (int i = threadIdx.x; i < WORDS; i += blockDim.x) psh[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const unsigned lb = (unsigned)__cvta_generic_to_shared(psh) + lane * 4;
  unsigned seed = blockIdx.x * 977u + threadIdx.x * 131u + 1u;
  for (int it = 0; it < iters; ++it) {
#pragma unroll 4
    for (int r = 0; r < 64; ++r) {
      seed = seed * 1664525u + 1013904223u;                 // LCG: bins of this lane's features
      const unsigned v = seed >> 8;
#pragma unroll
      for (int s = 0; s < S; ++s) {
        const unsigned bin = (seed >> (24 - 8 * s)) & 0xFFu;
        const unsigned a = lb + (bin << 7) + s * YABT_NB * 32 * 4;
        if (MASKED && ((seed >> (3 + 5 * s)) & 31u) >= (unsigned)active) continue;
#pragma unroll
        for (int l = 0; l < LIMBS; ++l)
          asm volatile("red.shared.add.u32 [%0], %1;\n" ::"r"(a + l * LS), "r"(l == LIMBS - 1 ? 1u : v & 0xFFFFu)
                       : "memory");
      }
    }
  }
  __syncthreads();
  unsigned long long acc = 0;
  for (int i = threadIdx.x; i < WORDS; i += blockDim.x) acc += psh[i];
  atomicAdd(sink, acc);      // keeps the reductions observable
}

template <int LIMBS, int S, bool MASKED>
int run_probe(int iters, unsigned long long* sink, cudaStream_t s, float* ms, long long* updates, int active) {
  constexpr int SMEM = LIMBS * S * YABT_NB * 32 * 4;
  int dev = 0, nsm = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_probe_red<LIMBS, S, MASKED>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  cudaEvent_t a = nullptr, b = nullptr;
  if (e == cudaSuccess) e = cudaEventCreate(&a);
  if (e == cudaSuccess) e = cudaEventCreate(&b);
  if (e == cudaSuccess) {
    k_probe_red<LIMBS, S, MASKED><<<nsm, PROBE_THREADS, SMEM, s>>>(iters, sink, active);        // warm-up
    cudaEventRecord(a, s);
    k_probe_red<LIMBS, S, MASKED><<<nsm, PROBE_THREADS, SMEM, s>>>(iters, sink, active);
    cudaEventRecord(b, s);
    e = cudaEventSynchronize(b);
  }
  if (e == cudaSuccess) e = cudaEventElapsedTime(ms, a, b);
  if (a) cudaEventDestroy(a);
  if (b) cudaEventDestroy(b);
  if (e != cudaSuccess) { set_error("yabt_probe_shared_red: %s", cudaGetErrorString(e)); return YABT_ERR_CUDA; }
  *updates = (long long)nsm * PROBE_THREADS * iters * 64 * S;
  return YABT_OK;
}

}  // namespace
}  // namespace yabt

using namespace yabt;

static int probe(int limbs, int iters, void* sink, void* stream, float* ms, long long* updates, int active) {
  if (limbs < 2 || limbs > 5) {
    set_error("yabt_probe_shared_red: limbs must be 2 or 3 (two 32-feature subs per lane), 4 or 5 (one sub)");
    return YABT_ERR_ARG;
  }
  if (iters <= 0 || !sink || !ms || !updates || active < 0 || active > 32) {
    set_error("yabt_probe_shared_red: iters > 0, 0 <= active <= 32 and non-null outputs required");
    return YABT_ERR_ARG;
  }
  auto* k = static_cast<unsigned long long*>(sink);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the unmasked form is a kernel of its own: no per-lane test in its loop
  if (active >= 32) {
    switch (limbs) {
      case 2: return run_probe<2, 2, false>(iters, k, s, ms, updates, 32);
      case 3: return run_probe<3, 2, false>(iters, k, s, ms, updates, 32);
      case 4: return run_probe<4, 1, false>(iters, k, s, ms, updates, 32);
      default: return run_probe<5, 1, false>(iters, k, s, ms, updates, 32);
    }
  }
  switch (limbs) {
    case 2: return run_probe<2, 2, true>(iters, k, s, ms, updates, active);
    case 3: return run_probe<3, 2, true>(iters, k, s, ms, updates, active);
    case 4: return run_probe<4, 1, true>(iters, k, s, ms, updates, active);
    default: return run_probe<5, 1, true>(iters, k, s, ms, updates, active);
  }
}

extern "C" int yabt_probe_shared_red(int limbs, int iters, void* sink, void* stream, float* ms, long long* updates) {
  return probe(limbs, iters, sink, stream, ms, updates, 32);
}

extern "C" int yabt_probe_shared_red_masked(int limbs, int iters, int active, void* sink, void* stream, float* ms,
                                            long long* updates) {
  return probe(limbs, iters, sink, stream, ms, updates, active);
}
