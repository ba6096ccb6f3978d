// Shared definitions for the yabt_b200 CUDA kernels (sm_100a).
//
// Layout conventions used across the library
// -------------------------------------------
// * Bin matrix ("tiled layout"): features are grouped into column tiles. A
//   full tile holds 64 features; the remainder of F mod 64 becomes a 32-wide
//   tile (if >= 32 features remain) and then a tile of width 32 (more than
//   16 features left) or 16, padded. Each tile is its own (n x width) row-major uint8 block, the
//   blocks stored one after another (each starting on a 256-byte boundary).
//   Within a 64-wide tile, byte 2*j + k of a row holds feature f0 + j + 32*k,
//   so lane j of a warp loads one u16 and receives features j and j+32: the
//   warp covers 64 features with one 64-byte load, and every lane owns a
//   distinct feature, which makes the shared-memory histogram bank-conflict
//   free (bank = lane). In 32-wide and narrow tiles byte j holds feature f0+j.
// * Histograms: exact fixed-point integers. A row's gradient g is quantised as
//   V = rint(g * 2^qe) with 2^qe chosen per tree so |V| <= 2^30; shared
//   memory accumulates V as two u32 limbs (low 16 bits, high signed part) plus
//   a u32 row count; node totals are int64. Sums are therefore exact and
//   independent of accumulation order.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#define YABT_NB 256                 // bins per feature (uint8 codes)
#define YABT_TILE 64                // features per full tile
#define YABT_SMS_HINT 148           // SMs of a B200: sizes grid-stride grids and per-level work targets

namespace yabt {

// error codes returned through the C ABI
enum : int {
  OK = 0,
  ERR_ARG = 1,
  ERR_CUDA = 2,
  ERR_WORKSPACE = 3,
  ERR_DEVICE = 4,      // device-side check failed (see error word)
  ERR_UNSUPPORTED = 5,
};

// device-side error word bits (written with atomicOr, read by the host)
enum : unsigned {
  DERR_LOOKBACK_TIMEOUT = 1u << 0,
  DERR_SEGMENT_OVERFLOW = 1u << 1,
  DERR_ITEM_OVERFLOW = 1u << 2,
  DERR_TILE_OVERFLOW = 1u << 3,
  DERR_BAD_INDEX = 1u << 4,
  DERR_NODE_OVERFLOW = 1u << 5,
  DERR_NONFINITE = 1u << 6,
  DERR_XCHG_TIMEOUT = 1u << 7,    // a cross-GPU exchange gave up waiting for a peer
  DERR_BOUNDS = 1u << 8,          // bounds-checked build: an index outside its array (access skipped)
};

// Bounds-checked build (-DYABT_BOUNDS_CHECK, libyabt_b200_checked.so): the
// index checks below run before the accesses they guard; a failing one sets
// DERR_BOUNDS in the kernel's error word and the access is skipped. In the
// ordinary build they compile to nothing.
#ifdef YABT_BOUNDS_CHECK
#define YABT_BOUNDS_CHECKED 1
#else
#define YABT_BOUNDS_CHECKED 0
#endif

void set_error(const char* fmt, ...);
// host-side count of kernel launches issued by the library (gpu_launches)
void count_launches(int k);

// ---------------------------------------------------------------- dependent launches
// Programmatic dependent launch (sm_90 and later): a kernel launched with
// launch_pdl may begin while its predecessor in the stream finishes, hiding
// the launch latency between the short kernels of a tree level. Such a kernel
// calls pdl_wait() first, unconditionally, before it reads or writes anything
// (it returns once the predecessor grid has completed and its memory is
// visible; without a predecessor launched this way it returns at once).
// Single-block kernels call pdl_trigger() after it, so their successor's
// blocks are scheduled while they run. YABT_NO_PDL=1 in the environment
// launches everything the ordinary way.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

bool pdl_enabled();

// ---------------------------------------------------------------- device-side level loop
// A level kernel launched with level_gate == LEVEL_DYN takes its level from the
// grower's device state instead of the launch (kernels inside the CUDA graph of
// a device-side level loop, abi.cu). While the calling thread captures that
// graph, launches go in without PDL, phase events or host launch counts.
constexpr int LEVEL_DYN = -1;
bool capturing_level_loop();
void set_capturing_level_loop(bool on);

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() && !capturing_level_loop() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// ---------------------------------------------------------------- phases
// Launch groups by phase (phase.cu): an NVTX range always, CUDA events on the
// launching stream while phase timing is on (yabt_phase_timing).
enum Phase : int {
  PH_BEGIN = 0,    // per-tree set-up: gradient quantisation scale, tree init
  PH_HIST,         // k_hist (and the build_hist drop-in)
  PH_REDUCE,       // k_reduce
  PH_XCHG,         // cross-GPU level-histogram exchange kernel
  PH_SCAN,         // split-gain scan
  PH_FINALIZE,     // per-level split choice / best-first pick
  PH_PARTITION,    // row partition
  PH_PLAN,         // next level's histogram work items
  PH_FINISH,       // tree finish, leaf of every row
  PH_LEAFNET,      // ridge-linear leaf models
  PH_INTERACT,     // interaction detector
  PH_UPDATE,       // margin update and next gradients
  PH_BINNING,      // binning (once per fit)
  PH_COLLECTIVE,   // host-issued collectives (yabt_phase_push from the host)
  PH_OTHER,
  PH_COUNT
};

bool phase_timing_on();     // yabt_phase_timing is recording

class PhaseScope {
 public:
  PhaseScope(int phase, cudaStream_t s);
  ~PhaseScope();
  PhaseScope(const PhaseScope&) = delete;
  PhaseScope& operator=(const PhaseScope&) = delete;

 private:
  int slot_;
  cudaStream_t s_;
};

// ---------------------------------------------------------------- layout
struct TileInfo {
  int f0;        // first feature
  int nfeat;     // features in the tile
  int width;     // bytes per row in the tile
  int wide;      // 1: 64-wide interleaved tile (u16 per lane), 0: byte j = feature f0+j
  long long off; // byte offset of the tile block in the bin matrix
};

// Host-side description of the bin-matrix layout (also copied to device).
struct BinLayout {
  int F;
  int ntiles;
  long long n;
  long long bytes;
  TileInfo tiles[1];   // variable length (allocated with ntiles entries)
};

// Per-feature address helpers (device arrays, F entries)
struct FeatAddr {
  long long off;  // tile block offset
  int width;      // tile row width
  int pos;        // byte position within the tile row
};

// Tile plan of F features: full 64-wide tiles; a remainder r >= 32 becomes a
// 32-wide tile (r -= 32); a remaining r' > 16 a 32-wide tile padded with
// zero bytes, r' in 1..16 a 16-wide padded tile. Every tile row is 64, 32 or
// 16 bytes, so rows are always moved with 16-byte copies.
__host__ __device__ inline int tile_count(int F) {
  int t = F / YABT_TILE, r = F % YABT_TILE;
  if (r >= 32) { t += 1; r -= 32; }
  if (r > 0) t += 1;
  return t;
}

__host__ __device__ inline long long tile_block_bytes(long long n, int width) {
  return (n * width + 255) & ~255LL;
}

// fill tiles[0..ntiles) for F features and n rows; returns total bytes
inline long long make_tiles(int F, long long n, TileInfo* tiles) {
  int t = 0, f = 0;
  long long off = 0;
  for (; f + YABT_TILE <= F; f += YABT_TILE) {
    tiles[t] = TileInfo{f, YABT_TILE, YABT_TILE, 1, off};
    off += tile_block_bytes(n, YABT_TILE); ++t;
  }
  int r = F - f;
  if (r >= 32) {
    tiles[t] = TileInfo{f, 32, 32, 0, off};
    off += tile_block_bytes(n, 32); ++t; f += 32; r -= 32;
  }
  if (r > 0) {
    const int w = r > 16 ? 32 : 16;
    tiles[t] = TileInfo{f, r, w, 0, off};
    off += tile_block_bytes(n, w); ++t;
  }
  return off;
}

inline void feat_addrs(int F, const TileInfo* tiles, int ntiles, FeatAddr* out) {
  for (int t = 0; t < ntiles; ++t) {
    const TileInfo& ti = tiles[t];
    for (int i = 0; i < ti.nfeat; ++i) {
      int pos = ti.wide ? (2 * (i & 31) + (i >> 5)) : i;
      out[ti.f0 + i] = FeatAddr{ti.off, ti.width, pos};
    }
  }
}

// Address of feature f in the tiled layout, computed analytically (matches
// make_tiles / feat_addrs).
__host__ __device__ inline FeatAddr feat_addr(int F, long long n, int f) {
  const long long a64 = tile_block_bytes(n, YABT_TILE);
  const int nfull = F / YABT_TILE;
  if (f < nfull * YABT_TILE) {
    const int t = f / YABT_TILE, i = f % YABT_TILE;
    return FeatAddr{t * a64, YABT_TILE, 2 * (i & 31) + (i >> 5)};
  }
  long long off = nfull * a64;
  int r = F - nfull * YABT_TILE, f0 = nfull * YABT_TILE;
  if (r >= 32) {
    if (f < f0 + 32) return FeatAddr{off, 32, f - f0};
    off += tile_block_bytes(n, 32); f0 += 32; r -= 32;
  }
  return FeatAddr{off, r > 16 ? 32 : 16, f - f0};
}

// ---------------------------------------------------------------- misc device helpers
__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31; }

// float <-> order-preserving unsigned (for atomic min/max of floats)
__device__ __forceinline__ unsigned f2ord(float x) {
  unsigned u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(unsigned u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// exponent e with |x| < 2^e for the largest |x| (x >= 0 finite), 0 for x == 0
__host__ __device__ inline int exp_bound(float amax) {
  if (!(amax > 0.f)) return 0;
  int e;
  frexpf(amax, &e);   // amax = m * 2^e, m in [0.5, 1)
  return e;
}

}  // namespace yabt
