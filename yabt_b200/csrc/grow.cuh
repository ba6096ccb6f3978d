// Device-side data structures of the level-wise grower (shared by the kernels
// in hist.cu / grow.cu). All per-tree state lives in device memory so that a
// whole tree is grown by a fixed sequence of launches with no host sync.
#pragma once
#include "common.cuh"

namespace yabt {

constexpr int HIST_THREADS = 1024;    // k_hist block size (one block per SM)
constexpr int PART_TILE = 4096;       // rows per partition tile
constexpr int PART_THREADS = 512;
constexpr int PART_RPT = PART_TILE / PART_THREADS;   // rows per thread (8)
static_assert(PART_TILE % PART_THREADS == 0, "partition tile");
constexpr int ITEM_TARGET = 4 * YABT_SMS_HINT;  // histogram work items per level (target)
constexpr int CHUNK_MIN = 4096;       // rows per histogram item (lower bound)
constexpr int CHUNK_MAX = 65536;      // rows per item and per flushed segment (u32 limb overflow bound)
constexpr int RUN_MAX = 16;          // items per claimed run (k_hist)

// int64 words of one job's small-child histogram: C-1 value channels of F x 256
// bins, then the count channel with two bins per word (per-bin counts stay
// below 2^32 even summed over ranks, so packed words add without carries)
__host__ __device__ constexpr long long small_job_words(int C, int F) {
  return (long long)(C - 1) * F * YABT_NB + (long long)F * (YABT_NB / 2);
}
constexpr int SCAN_WARPS = 8;         // k_scan: one warp per feature
// kernels of one pass of a device-side level loop: k_hist, k_reduce, k_scan,
// k_finalize, k_partition, k_plan and the loop condition; a sharded loop adds
// the reduce-scatter and the best-split gather
constexpr int LEVEL_LOOP_BODY_KERNELS = 7;
constexpr int LEVEL_LOOP_BODY_KERNELS_SHARDED = 9;
constexpr int FIN_SMEM_NODES = 2048;  // k_finalize: active nodes whose gains / tile prefixes fit shared memory

// leaf row sources
enum : int { SRC_FIN = 0, SRC_LIST0 = 1, SRC_LIST1 = 2, SRC_IDENTITY = 3 };

// A column unit = the features one histogram block accumulates: up to S
// sub-groups ("subs") of 32 features, lane j of sub s <-> feature feat[s][j].
struct UnitDesc {
  long long off;  // tile block byte offset in the bin matrix
  int width;      // tile row width in bytes
  int wide;       // 64-wide interleaved tile
  int k0;         // byte (0/1) of a wide tile handled by this unit when S == 1
  int nsub;       // subs actually present (1 or 2)
  int rep;        // narrow 16-wide tiles: rows per shared-memory reduction (1, 2 or 4);
  int lw;         //   lanes per row (32 / rep); lane l handles feature l % lw of row l / lw
  int feat[2][32];
};

struct HistItem {       // one histogram work item: rows [begin, begin+count) of a list
  int begin;
  int count;
  int unit;
  int job;              // pair index (or 0 for the root)
  int slot;             // partial-histogram slot
  int used;             // set by k_hist: 1 if the slot holds a flushed partial
  int pad[2];
};

struct PartTile {       // one partition tile: rows [begin, end) of active node `pos`
  int pos;
  int begin;
  int end;
  int last;             // 1 if this is the node's last tile
  int t_in_node;
  int pad[3];
};

struct NodeBest {       // best split of one (node, feature)
  float sel;            // selection score (gain * boost)
  float gain;           // true gain
  float GL, HL, CL;     // left sums at the chosen bin (float32 of exact sums)
  int bin;
  long long cl;         // exact left row count (global)
};

struct BfCand {         // best-first: a node's chosen split with exact sums
  double sel;           // selection score (gain * boost); float64 mode: of the float64 gain
  float gain;           // true gain (-inf: no valid split)
  int f, bin;           // bin -1: the feature has no valid split (float64 mode)
  int flag;             // 1: a candidate (gain > 0, depth < max_depth, still a leaf)
  long long gl, hl, cl; // exact left sums at the split (hl = cl on the unit-hessian path)
  long long g, h, c;    // exact node totals
};

struct NodeTot {        // node totals
  float G, H, C;
  int pad;
  long long c;          // exact row count (global)
};

struct GrowState {
  int level;            // level the next level-kernels will process
  int active;           // 1 while the level loop continues
  int M;                // active nodes at `level`
  int P;                // pairs produced by the last finalize
  int n_nodes;          // nodes in the tree so far
  int remaining;        // leaf budget: splits still allowed
  int part_level;       // level whose partition is pending (-1 none)
  int plan_level;       // level whose plan is pending (-1 none)
  int n_items;
  int item_counter;
  int n_tiles;
  int tile_counter;
  unsigned epoch;       // look-back epoch, bumped by every partition launch
  unsigned err;         // device error bits
  int qe_g, qe_h;       // quantisation exponents
  float gscale, hscale; // 2^qe
  float ginv, hinv;     // 2^-qe
  int depth_max;        // deepest node depth so far
  unsigned amax_g, amax_h;  // bit patterns of max |g| and max |h|
  int n_leaves;
  int bf_split;         // best-first: node split by the current step (-2: root scanned, -1: none)
  int bf_next_slot;     // best-first: next free histogram slot
  int bf_scan;          // best-first: 1 if the children of bf_split are histogrammed and scanned
  long long hist_rows[64];   // rows histogrammed at each level (algorithmic-traffic accounting)
  long long acc_root_rows;   // accumulated since the last yabt_grower_acc_reset: root-level rows,
  long long acc_child_rows;  // smaller-child rows of deeper levels,
  long long acc_launches;    // histogram levels that did work
  unsigned xerr;             // persistent error bits of the per-tree peer all-reduces (not reset per tree)
  unsigned xepoch0;          // first exchange epoch of the tree's device-side level loop (sharded trees)
  long long n_rows;          // rows of the bin matrix (bounds-checked build)
};

// Per-call grower parameters (copied by value into kernels).
struct GrowParams {
  long long n;
  int F, U, S, C;       // features, units, subs per unit, hist channels (2 or 3)
  int general;          // 1: hessian channel present (else hessian == 1 for every row)
  int maxa;             // max active nodes per level (= max_leaves)
  int maxn;             // max nodes
  int max_pairs;
  int max_items;
  int max_tiles;
  int max_leaves, max_depth;
  int levels_max;
  float lam, gamma, mcw, lr, ib;
  int msl;
  int use_imat;
  int use_fmask;
  int bf_f64;           // best-first in the C / Numba grower's arithmetic (float64 scan, slot tie order)
  int f_lo, f_hi;       // level-wise scan: features [f_lo, f_hi) (a rank's slice in feature-sliced sharding)
};

// Device pointers of one grower workspace.
struct TreeIO;

struct GrowBufs {
  GrowState* st;
  TreeIO* io_dev;        // the current tree's TreeIO (written by k_tree_init)
  int* rows[2];          // active row lists (ping-pong by level parity)
  int* fin;              // rows of nodes that stopped (same offsets as the lists)
  int* seg_begin[2];     // [maxa] per level parity
  int* seg_count[2];
  int* act_gid[2];
  long long* hist[2];    // [maxa][C][F][256] int64 full histograms per level parity
  long long* root_cnt;   // [F][128] packed per-bin row counts of all rows (cached root level)
  long long* small;      // [max_pairs][small_job_words(C, F)] small-child (or root) histograms:
                         // value channels [C-1][F][256], then counts [F][128] with bins
                         // 2k, 2k+1 packed in the low / high 32 bits of one int64
  float* pathmax[2];     // [maxa][F] max over path features p of imat[p][f]
  NodeBest* best;        // [maxa][F]
  NodeBest* nbest;       // [maxa] chosen split per active node
  unsigned long long* node_key;   // [maxa] max over features of (ordered sel << 32 | ~feature)
  NodeTot* tot;          // [maxa]
  int* pair_pos;         // [max_pairs] active position of the parent of pair p
  int* pair_sil;         // [max_pairs] small child is the left one
  int* split_pair;       // [maxa] pair index of an active node, -1 if it stops
  int* split_f;          // [maxa]
  int* split_b;          // [maxa]
  int* node_tpre;        // [max(maxa, max_pairs) + 1] scratch for per-node / per-pair prefixes
  HistItem* items;       // [max_items]
  int* job_first;        // [max_pairs * U]
  int* job_nitems;       // [max_pairs * U]
  PartTile* tiles;       // [max_tiles]
  unsigned long long* tile_status;  // [max_tiles]
  unsigned* partials;    // [max_items][LIMBS][S][256][32]
  UnitDesc* units;       // [U]
  FeatAddr* faddr;       // [F]
  int* leaf_src;         // [maxn] SRC_*
  int* leaf_begin;       // [maxn]
  int* leaf_count;       // [maxn]
  int* node_depth;       // [maxn]
  int* node_bin;         // [maxn] split bin of internal nodes, -1 at leaves
  // best-first growth
  BfCand* bf_feat;       // [2][F] per child position and feature: best split of the feature
  BfCand* bf_cand;       // [maxn] per node: its best split
  int* node_slot;        // [maxn] histogram / path-max slot of a leaf (slots < maxa)
};

// Caller-owned inputs / outputs of one tree.
struct TreeIO {
  const uint8_t* bins;       // tiled bin matrix
  const float* g;
  const float* h;            // nullptr on the unit-hessian path
  const float* edges;        // concatenated per-feature interior edges
  const int* edge_off;       // [F]
  const int* edge_cnt;       // [F]
  const float* scales;       // [F]
  const unsigned char* fmask;  // [F] or nullptr
  const float* imat;         // [F][F] or nullptr
  long long* feature;        // [maxn]
  float* threshold;
  long long* left;
  long long* right;
  float* value;
  float* gate;
  int* leaf_of_row;          // [n]
  const uint8_t* bins_fm;    // feature-major (F, n) bins, or nullptr (partition reads the tiled matrix)
  const int* root_rows;      // rows the tree is grown on (row subsampling), or nullptr: all n rows
  long long n_root;          // number of root rows (n when root_rows is nullptr)
};

// Multi-task growth (shared structure, one leaf value per task).
constexpr int MT_MAX = 8;            // tasks per tree
struct MtRec {                       // per-task exact sums of a node's chosen split
  long long gl[MT_MAX];              // left gradient sums at the split bin
  long long g[MT_MAX];               // node gradient totals
};
struct MtBufs {
  int T, P;                 // tasks, task pairs (histogram passes)
  const float* grads;       // [T][n] task-major gradients
  const float* zeros;       // [n] zeros: the second channel of the last pass when T is odd
  long long* small;         // [2P][F][256] value channels, then counts [F][128] (two bins per word)
  long long* hist;          // [slot][T + 1][F][256]: per-task channels, then counts
  MtRec* feat;              // [2][F] per child position and feature
  MtRec* cand;              // [maxn] per node
  float* values;            // [maxn][T] leaf values (output)
  float* scratch_value;     // [maxn] scalar values the shared best-first kernels write (unused)
};

// the device state of a bound grower (C ABI handle), or nullptr
GrowState* grower_state(struct yabt_grower* g);
int grower_slice(struct yabt_grower* g, int* F, int* C, int* f_lo, int* f_hi);   // 0 if bound
// feature-sliced exchange launchers (xchg.cu); level may be LEVEL_DYN inside a
// device-side level loop whose first level is loop_first
int xchg_sliced_launch(struct yabt_grower* g, void* const* bufs, int rank, int nranks, int level, unsigned epoch,
                       int loop_first, cudaStream_t s);
int xchg_gather_launch(struct yabt_grower* g, void* const* bufs, int rank, int nranks, int level, unsigned epoch,
                       long long rec_offset, int loop_first, cudaStream_t s);
int xchg_set_loop_epoch(struct yabt_grower* g, unsigned epoch0, cudaStream_t s);
void grower_best_bufs(struct yabt_grower* g, unsigned long long** node_key, NodeBest** best);
int grower_maxa(const struct yabt_grower* g);

}  // namespace yabt
