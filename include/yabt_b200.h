/* yabt_b200 -- C ABI of the B200 tree-growth library (libyabt_b200.so).
 *
 * Every entry point returns 0 (YABT_OK) or an error code; yabt_last_error()
 * gives the message of the last failure on the calling thread. All device
 * buffers are caller-owned (e.g. torch tensors) and passed as plain pointers;
 * `stream` is a cudaStream_t (NULL = legacy default stream). No function
 * allocates device memory except where stated.
 *
 * Each declaration names the reference interface it replaces
 * (grafael/yabt, paths relative to the project root).
 */
#ifndef YABT_B200_H
#define YABT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  YABT_OK = 0,
  YABT_ERR_ARG = 1,
  YABT_ERR_CUDA = 2,
  YABT_ERR_WORKSPACE = 3,
  YABT_ERR_DEVICE = 4,
  YABT_ERR_UNSUPPORTED = 5
};

/* Library version (major*10000 + minor*100 + patch). */
int yabt_version(void);

/* Copy the last error message of this thread into buf (NUL-terminated). */
int yabt_last_error(char* buf, int len);

/* Number of kernels the library has launched so far in this process from the
 * host. Kernels that device-side level loops ran (yabt_grower_set_level_loop)
 * are counted on the device of the calling thread: yabt_launch_count_device
 * reads that counter (waits for the device; -1 on error) and
 * yabt_launch_count_device_reset zeroes it in stream order. */
long long yabt_launch_count(void);
long long yabt_launch_count_device(void);
int yabt_launch_count_device_reset(void* stream);

/* Measurement only (no reference counterpart): the shared-memory reduction
 * ceiling of the histogram kernel. Issues k_hist's u32 reductions (limbs = 3:
 * unit-hessian path, two 32-feature subs per lane; 5: general path; 2 and 4:
 * the same at a root whose counts come from the fit's cache) with its layout
 * and grid and pseudo-random bins, twice (warm-up, then timed); *ms = the
 * timed launch, *updates = its (row, feature) updates. sink: 8 bytes of
 * device memory the result is folded into. Synchronises the stream.       */
int yabt_probe_shared_red(int limbs, int iters, void* sink, void* stream, float* ms, long long* updates);
/* The same with each lane's reductions of a (row, feature) predicated off
 * with probability 1 - active/32 (0 <= active <= 32): what a sparse-bin
 * histogram that skips each feature's default bin issues
 * (yabt/grow_numba.py:42-87, yabt/_cgrow/grow.c:68-107). *updates still
 * counts every (row, feature), issued or not.                             */
int yabt_probe_shared_red_masked(int limbs, int iters, int active, void* sink, void* stream, float* ms,
                                 long long* updates);

/* Per-phase device timing (no reference counterpart; the reference's loop only
 * prints progress, yabt/boosting.py:329-342). Every launch group of the
 * library sits in a named phase (yabt_phase_name: begin, hist, reduce,
 * exchange, scan, finalize, partition, plan, finish, leafnet, interaction,
 * update, binning, collective, other), which always opens an NVTX range.
 * yabt_phase_timing(max) > 0 creates (or reuses) a pool of max event pairs
 * on the current device, clears it and records every phase range launched on
 * that device until the pool is full; 0 stops recording. yabt_phase_read
 * sums the recorded ranges per phase (ms[p], counts[p]; nphases >=
 * yabt_phase_count()), waiting for their events. yabt_phase_push/pop let
 * host code time its own stream work (collectives) as a phase.            */
int yabt_phase_count(void);
int yabt_phase_name(int phase, char* buf, int len);
int yabt_phase_timing(int max_ranges);
int yabt_phase_read(double* ms, long long* counts, int nphases);
int yabt_phase_push(int phase, void* stream);
int yabt_phase_pop(void);

/* ------------------------------------------------------------------ bin matrix
 * The tiled bin-matrix layout: features in column tiles (64-wide tiles, then
 * a 32-wide tile if >= 32 features remain, then a 16- or 32-wide padded
 * tile), each tile an (n x width) row-major uint8 block starting on a 256-byte
 * boundary; in a 64-wide tile byte 2j+k of a row holds feature f0+j+32k.
 * Size in bytes for n rows x F features, and the address of a feature: tile
 * block offset, tile row width and byte position within the tile row.     */
long long yabt_bin_matrix_bytes(long long n, int F);
int yabt_bin_address(long long n, int F, int feature, long long* tile_off, int* width, int* pos);

/* Pack a plain row-major (n, F) uint8 bin matrix into the tiled layout.
 * Replaces the layout contract of yabt/cuda_hist.py:79-89 (row-major (n, F)
 * uint8 input) for callers that hold plain bin matrices.                  */
int yabt_pack_bins(const uint8_t* plain, long long n, int F, uint8_t* tiled, void* stream);

/* ------------------------------------------------------------------ histogram FFI
 * Replaces the reference's fused histogram build, build_hist
 * (yabt/cuda_hist.py:79-89 -> hist_build in yabt/_cuda/hist.cu:105-133):
 * row i of the plain row-major (n, F) uint8 matrix `binned` adds
 * (g[i], h[i], w[i]) into bin binned[i, f] of node slot slot[i] (int64, in
 * [0, K)) for every feature f; `out` is the (3, K, F, B) float32 histogram
 * (channels g, h, w). Sums are exact fixed-point integers rounded once to
 * float32, so the result is deterministic. Rows with a slot outside [0, K) or
 * a bin >= B are skipped, and non-finite g/h/w values are rejected: each sets
 * a bit in the device word *err_out (0 = clean; may be NULL). No host
 * synchronisation; the workspace (yabt_hist_build_workspace_bytes) is
 * caller-owned.                                                            */
long long yabt_hist_build_workspace_bytes(long long n, int K, int F);
int yabt_hist_build(const uint8_t* binned, const int64_t* slot, const float* g, const float* h,
                    const float* w, long long n, int K, int F, int B, float* out, int32_t* err_out,
                    void* workspace, long long ws_bytes, void* stream);

/* ------------------------------------------------------------------ grower
 * Level-wise tree grower. Replaces grow_tree_levelwise
 * (yabt/tree.py:362-625) and, inside it, the CUDA histogram FFI
 * cuda_hist.build_hist (yabt/cuda_hist.py:79-89, yabt/_cuda/hist.cu:101-133).
 *
 * A grower is created for a problem shape; its scratch lives in one
 * caller-allocated device workspace of yabt_grower_workspace_bytes() bytes,
 * bound once with yabt_grower_bind(). One grower per device and stream; not
 * thread-safe.                                                           */
typedef struct yabt_grower yabt_grower;

/* general = 0: unit hessian (every hess == 1, squared loss), 2 histogram
 * channels; general = 1: arbitrary hessian, 3 channels.                  */
int yabt_grower_create(long long n, int F, int max_leaves, int max_depth, int general,
                       yabt_grower** out);
long long yabt_grower_workspace_bytes(const yabt_grower* g);
int yabt_grower_bind(yabt_grower* g, void* workspace, long long bytes, void* stream);
int yabt_grower_destroy(yabt_grower* g);
/* Max nodes a tree can have (length of the per-node output arrays). */
int yabt_grower_max_nodes(const yabt_grower* g);
/* Levels the host must drive (yabt_grow_hist / yabt_grow_split calls). */
int yabt_grower_levels(const yabt_grower* g);
/* Per-launch timing of the histogram kernel: record CUDA events around up to
 * max_launches histogram launches (0 disables); yabt_grower_hist_times returns
 * their durations in ms (synchronising) and resets the pool.              */
int yabt_grower_set_timing(yabt_grower* g, int max_launches);
int yabt_grower_hist_times(yabt_grower* g, float* ms, int cap, int* count);
/* Rows histogrammed at each level of the last tree (synchronising copy). */
int yabt_grower_hist_rows(yabt_grower* g, long long* rows, int cap);
/* Accumulators since the last reset: root-level rows, deeper-level smaller-
 * child rows, histogram levels that did work (reset is stream-ordered).    */
int yabt_grower_acc_reset(yabt_grower* g, void* stream);
int yabt_grower_acc_read(yabt_grower* g, long long* out3);

typedef struct {
  /* inputs (device) */
  const uint8_t* bins;            /* tiled bin matrix (yabt_pack_bins / yabt_bin_transform) */
  const float* grad;              /* [n] */
  const float* hess;              /* [n]; ignored when the grower was created with general = 0 */
  const float* edges;             /* concatenated interior edges of every feature */
  const int32_t* edge_off;        /* [F] offset of feature f's edges in `edges` */
  const int32_t* edge_cnt;        /* [F] number of edges of feature f (>= 1) */
  const float* scales;            /* [F] robust feature scales (gate_scale source) */
  const uint8_t* feature_mask;    /* [F] 1 = usable, or NULL */
  const float* interaction;       /* [F][F] normalised interaction matrix, or NULL */
  float reg_lambda, gamma, min_child_weight, learning_rate, interaction_boost;
  int32_t min_samples_leaf;
  /* outputs (device), max_nodes entries each: the Tree layout of yabt/tree.py:39-76 */
  int64_t* feature;               /* -1 at leaves */
  float* threshold;
  int64_t* left;
  int64_t* right;
  float* value;
  float* gate_scale;
  int32_t* leaf_of_row;           /* [n] final leaf (node id) of every row */
  int32_t* meta;                  /* [4] n_nodes, depth, device error bits, levels run */
  /* optional input (device): the feature-major (F, n) bin matrix
   * (yabt_bin_transform fm_out), or NULL; when given, the row partition reads
   * each row's split bin from it (one byte per row instead of a sector of
   * the tiled matrix)                                                      */
  const uint8_t* bins_fm;
  /* optional input (device): grow the tree on these rows only (row
   * subsampling, yabt/boosting.py:374-376), n_root of them, or NULL (all n
   * rows; n_root is then ignored). leaf_of_row is written for these rows;
   * yabt_grow_apply_all routes every row.                                  */
  const int32_t* root_rows;
  long long n_root;
} yabt_tree_args;

/* Grow one tree (single device). The host stops queuing levels once the tree
 * is complete: after each level's split the level state is copied to pinned
 * host memory and read three levels later, so the GPU keeps three levels
 * queued while the host waits. yabt_grower_set_level_wait(g, 0) queues the
 * levels without waiting instead (for callers that interleave several growers
 * on several streams from one host thread): every level, or the levels below
 * the device-side level loop's start and then the loop (below).           */
int yabt_grower_set_level_wait(yabt_grower* g, int wait);
/* Device-side level loop (on by default; no reference counterpart: the
 * reference's level loop is a host while loop, yabt/tree.py:484-625). Without level
 * wait, a tree whose levels may go far deeper than it grows (max_depth well
 * above log2(max_leaves)) would otherwise queue every possible level, most of
 * them device-side no-ops. With the loop, yabt_grow_tree launches levels
 * 0 .. L-1 as usual and then one CUDA graph whose conditional WHILE node
 * repeats one level's kernels while the tree is active; the graph is captured
 * on first use and again when the grower's parameters or workspace change.
 * yabt_grower_level_loop_start returns L, or -1 when the loop is off or would
 * not pay (level wait on, fewer than 9 leaves, fewer than two levels past L).
 * The loop is not used while histogram or phase timing records events, or
 * when the stream is being captured.                                       */
int yabt_grower_set_level_loop(yabt_grower* g, int on);
int yabt_grower_level_loop_start(const yabt_grower* g);
/* Root-level row counts cached across the trees of a fit: with on = 1, the
 * next root histogram over all rows (no root_rows) keeps its per-bin row
 * counts, and later root histograms over all rows skip the count channel and
 * copy them in (the same rows and bins give the same counts). The caller
 * turns it on only while the bin matrix stays the same (Booster.fit);
 * on = 0 turns it off and forgets the counts. Off by default.             */
int yabt_grower_set_root_count_cache(yabt_grower* g, int on);
/* The cached root counts, unpacked: out[f][b] (device, F x 256 int64) = the
 * number of this grower's rows whose bin of feature f is b, as recorded by
 * the last root histogram over all rows with the cache on; the count channel
 * of the root histogram of yabt/tree.py:425-452 (scatter_hist over every
 * row). YABT_ERR_ARG when nothing has been recorded yet.                  */
int yabt_grower_root_counts(yabt_grower* g, int64_t* out, void* stream);
/* After yabt_grow_tree: leaf_of_row for every row 0..n-1 (not only the root
 * rows), routed by the split bins through the feature-major bins (required);
 * Tree.apply of yabt/tree.py:82-116 on the training rows.                 */
int yabt_grow_apply_all(yabt_grower* g, const yabt_tree_args* a, void* stream);
/* Stable grouping of rows by leaf (node id < num_leaves <= 4096): rows[begin[l]
 * .. begin[l] + count[l]) = the rows i with leaf_of_row[i] == l, increasing;
 * the leaf-model ranges over every row after growth on a row sample
 * (yabt/boosting.py:486-497 fits leaf models on all rows). Rows with an
 * out-of-range leaf are skipped.                                           */
long long yabt_group_rows_workspace_bytes(long long n, int num_leaves);
int yabt_group_rows(const int32_t* leaf_of_row, long long n, int num_leaves, void* workspace, long long ws_bytes,
                    int32_t* begin, int32_t* count, int32_t* rows, void* stream);
int yabt_grow_tree(yabt_grower* g, const yabt_tree_args* a, void* stream);

/* Best-first (leaf-wise) growth, the heap grower of yabt/tree.py:206-360 that
 * Booster uses when levelwise is False, or "auto" with max_leaves < 16
 * (yabt/boosting.py:415-421): one split per step, the candidate leaf with the
 * largest gain first (ties: lower node id = earlier push), children become
 * candidates when depth < max_depth and gain > 0, at most max_leaves leaves.
 * Same arguments, outputs and node numbering as the reference (children get
 * the next two ids in split order). yabt_grow_tree_bestfirst runs the whole
 * tree (host stop as yabt_grow_tree); the step-wise form, for callers that
 * reduce the small-child histogram (one job) across ranks between the two
 * halves of a step like yabt_grow_hist / yabt_grow_split, is
 *   begin, init, bf_root_hist, [reduce], bf_scan(0),
 *   for step = 1 .. max(1, max_leaves - 1): bf_split(step), [reduce], bf_scan(step)
 *   end.                                                                    */
int yabt_grow_tree_bestfirst(yabt_grower* g, const yabt_tree_args* a, void* stream);
/* Arithmetic of best-first growth: 0 (default) that of the heap grower
 * yabt/tree.py:206-360 (float32 split scan, ties to the earlier push); 1 that
 * of the C / Numba grower cgrow (yabt/_cgrow/grow.c:243-427, wrapped by
 * grow_tree_c, yabt/grow_c.py:336-456): float64 split scan over bins below
 * min(edges + 1, 256), float64 leaf values, ties to the lower active-leaf
 * slot.                                                                   */
int yabt_grower_set_bestfirst_f64(yabt_grower* g, int on);

/* Multi-task trees: grow_multitask_tree (yabt/multitask.py:60-150) with
 * find_best_split_multi (yabt/histogram.py:143-188) for squared-loss tasks
 * (YABTMultiTaskRegressor): one best-first structure for `tasks` targets
 * (1..8), split on the sum of the per-task gains, validity from the shared
 * counts; values[node * tasks + t] = -lr * G_t / (count + lambda). The grower
 * must be created with general = 1; grads are task-major [tasks][n] (rows of
 * a->root_rows when given); a->grad / a->hess must be non-null (not read) and
 * a->value is scratch (scalar values are not meaningful here). The tree
 * arrays, leaf_of_row and meta are written as by yabt_grow_tree.
 * yabt_mt_update: margin[t][i] += values[leaf[i]][t] (values may be null),
 * then grad[t][i] = margin[t][i] - y[t][i] (grad may be null).            */
long long yabt_mt_workspace_bytes(const yabt_grower* g, int tasks);
int yabt_grow_tree_multitask(yabt_grower* g, const yabt_tree_args* a, int tasks, const float* grads, void* ws,
                             long long ws_bytes, float* values, void* stream);
int yabt_mt_update(const int32_t* leaf_of_row, const float* values, int tasks, long long n, float* margin,
                   const float* y, float* grad, void* stream);
int yabt_grow_bf_root_hist(yabt_grower* g, const yabt_tree_args* a, void* stream);
int yabt_grow_bf_split(yabt_grower* g, const yabt_tree_args* a, int step, void* stream);
int yabt_grow_bf_scan(yabt_grower* g, const yabt_tree_args* a, int step, void* stream);

/* Step-wise driving for row-sharded multi-GPU growth: the caller reduces
 * (max, as int32) the two words at yabt_grow_amax_ptr() -- bit patterns of
 * max |g| and max |h| -- after yabt_grow_begin, and sums (int64) the
 * small-child histograms at yabt_grow_small_ptr() between yabt_grow_hist and
 * yabt_grow_split of each level: at most yabt_grow_small_count(level) int64
 * words, exactly pairs * yabt_grow_small_count(0) (see yabt_grow_level_ptr).
 * Per job: the value channels, then the counts two bins per word (low / high
 * 32 bits; they add without carries while the total row count is < 2^32). */
int yabt_grow_begin(yabt_grower* g, const yabt_tree_args* a, void* stream);
int yabt_grow_init(yabt_grower* g, const yabt_tree_args* a, void* stream);
int yabt_grow_hist(yabt_grower* g, const yabt_tree_args* a, int level, void* stream);
int yabt_grow_split(yabt_grower* g, const yabt_tree_args* a, int level, void* stream);
int yabt_grow_end(yabt_grower* g, const yabt_tree_args* a, void* stream);
void* yabt_grow_amax_ptr(yabt_grower* g);
/* Device address of four int32 words of the level state: level, active,
 * active node count, pairs split by the last yabt_grow_split. After
 * yabt_grow_split(level d) the pairs count is the number of jobs of level d+1
 * (the small-child histograms to reduce are then pairs * small_count(0)
 * int64 values), and active = 0 means the tree is complete.              */
void* yabt_grow_level_ptr(yabt_grower* g);

/* Cross-GPU level reduction over NVLink peer memory for row-sharded growth,
 * instead of a host-driven all-reduce between yabt_grow_hist and
 * yabt_grow_split (replaces, like the hooks above, the single-process
 * histogram of yabt/tree.py:425-452 for sharded rows). Each rank allocates an
 * exchange buffer (yabt_xchg_alloc: cudaMalloc of bytes + header, zeroed, and
 * its 64-byte CUDA IPC handle), makes it the grower's small-child histogram
 * buffer (yabt_grower_set_small(g, buf + yabt_xchg_header_bytes(), bytes)),
 * shares the handle with the other ranks and maps theirs (yabt_xchg_open).
 * Then yabt_grow_xreduce(level) after yabt_grow_hist sums the level's
 * histograms of all ranks in place in every rank's buffer, sized from the
 * grower's device state (no host synchronisation). `bufs` are the exchange
 * buffers of ranks 0..nranks-1 as mapped in this process (this rank's own
 * pointer at index rank); `epoch` must differ between consecutive calls and
 * be the same on every rank. Ranks must be on distinct GPUs of one node (at
 * most 8); every wait is bounded, and a timeout sets a device error bit that
 * the tree's meta reports.                                                */
long long yabt_xchg_header_bytes(void);
int yabt_xchg_alloc(long long bytes, void** ptr, void* ipc_handle);
int yabt_xchg_open(const void* ipc_handle, void** ptr);
int yabt_xchg_close(void* ptr);
int yabt_xchg_free(void* ptr);
int yabt_grower_set_small(yabt_grower* g, void* ptr, long long bytes);
int yabt_grow_xreduce(yabt_grower* g, void* const* bufs, int rank, int nranks, int level, unsigned epoch,
                      void* stream);
/* Element-wise all-reduce of a small device vector over the same mapped
 * exchange buffers (the per-tree reductions of a row-sharded fit -- the
 * quantisation words, the leaf-model sums and envelopes -- that the reference
 * computes over all rows, yabt/tree.py:473, yabt/neural_leaves.py:147-184):
 * dst = reduce over ranks of src, count elements of kind 0 int64 sum, 1
 * float64 sum, 2 int32 max, 3 float32 max; summed in rank order, so every
 * rank gets the same result. src and dst may alias; count * element size must
 * fit buf_bytes (each exchange buffer's data bytes). Uses the buffers' data
 * region (nothing of a level's histograms may be pending there) and `epoch`
 * like yabt_grow_xreduce (one sequence shared by both). Timeouts set a
 * persistent error bit (yabt_grow_xerr; also OR-ed into later trees' meta).  */
int yabt_grow_xallreduce(yabt_grower* g, void* const* bufs, long long buf_bytes, int rank, int nranks,
                         const void* src, void* dst, long long count, int kind, unsigned epoch, void* stream);
int yabt_grow_xerr(yabt_grower* g, unsigned* bits);
/* Feature-sliced level-wise growth over sharded rows (the same split
 * decisions as yabt_grow_tree on one GPU over all rows, yabt/tree.py:504-560;
 * less scan work and half the exchange bytes per rank). Rank r of N scans only
 * features [F r / N, F (r + 1) / N) (yabt_grower_set_feature_slice, exactly
 * that range). Per level: yabt_grow_hist; yabt_grow_xreduce_sliced (every
 * rank sums only its slice's words over the ranks, into its own buffer);
 * yabt_grow_scan (the slice's split scan); yabt_grow_xgather (every rank's
 * best split per node exchanged through records at rec_offset bytes after the
 * data start of every exchange buffer, yabt_grow_xgather_bytes of room; the
 * largest key wins, the first maximum over all features); yabt_grow_choose
 * (k_finalize, partition, next level's plan). yabt_grow_scan + yabt_grow_choose
 * on one GPU are yabt_grow_split. epochs as for yabt_grow_xreduce.          */
int yabt_grower_set_feature_slice(yabt_grower* g, int f_lo, int f_hi);
int yabt_grow_scan(yabt_grower* g, const yabt_tree_args* a, int level, void* stream);
int yabt_grow_choose(yabt_grower* g, const yabt_tree_args* a, int level, void* stream);
int yabt_grow_xreduce_sliced(yabt_grower* g, void* const* bufs, int rank, int nranks, int level, unsigned epoch,
                             void* stream);
int yabt_grow_xgather(yabt_grower* g, void* const* bufs, int rank, int nranks, int level, unsigned epoch,
                      long long rec_offset, void* stream);
long long yabt_grow_xgather_bytes(const yabt_grower* g);
/* The device-side level loop of a feature-sliced sharded tree (no reference
 * counterpart; the reference's level loop is a host while loop,
 * yabt/tree.py:484-625): after the caller grew levels 0 .. L-1 with the calls
 * above (L = yabt_grower_level_loop_start), one CUDA graph runs the remaining
 * levels, each a histogram, reduce-scatter, slice scan, best-split gather and
 * choice, while the tree is active. The loop's level d uses exchange epochs
 * epoch0 + 2 (d - L) (reduce-scatter) and that + 1 (gather), so the caller
 * reserves 2 (levels - L) epochs from epoch0 on every rank alike. *used is 0
 * (nothing launched: the caller grows the levels itself) when the loop is off
 * or histogram / phase timing records events.                              */
int yabt_grow_level_loop_sharded(yabt_grower* g, const yabt_tree_args* a, void* const* bufs, int rank, int nranks,
                                 long long rec_offset, unsigned epoch0, int* used, void* stream);
void* yabt_grow_small_ptr(yabt_grower* g);
long long yabt_grow_small_count(const yabt_grower* g, int level);
/* Per-leaf row ranges of the last tree (device arrays inside the workspace):
 * src (0 fin, 1 list0, 2 list1, 3 identity), begin, count; plus list bases. */
int yabt_grow_leaf_rows(yabt_grower* g, void** src, void** begin, void** count,
                        void** fin, void** list0, void** list1);


/* ------------------------------------------------------------------ binning
 * Quantile binner, bit-exact with the numpy path of Binner.fit / transform
 * (yabt/binning.py:29-112).                                               */

/* X (n, F) row-major float32 -> Xfm (F, n) feature-major. */
int yabt_transpose(const float* X, long long n, int F, float* Xfm, void* stream);
/* A block of m rows into a larger feature-major matrix: Xfm[f * ld + r] =
 * X[r * F + f] for r < m (pass Xfm + first row; used to transpose host data
 * chunk by chunk while the next chunk is being copied in).                 */
int yabt_transpose_block(const float* X, long long m, int F, float* Xfm, long long ld, void* stream);
long long yabt_bin_fit_workspace_bytes(long long n, int F, long long nq);
/* Medians over all rows; edges / scales from the sample rows sample_idx[nq]
 * (NULL: rows 0..nq-1). edges is [F][255] (first edge_cnt[f] valid).
 * Replaces Binner.fit (yabt/binning.py:29-69).                           */
int yabt_bin_fit(const float* Xfm, long long n, int F, const int32_t* sample_idx, long long nq,
                 int max_bins, void* workspace, long long ws_bytes, float* medians, float* edges,
                 int32_t* edge_cnt, float* scales, void* stream);
/* yabt_bin_fit in steps, for a fit over rows sharded across GPUs
 * (yabt/binning.py:29-69 on the concatenation of every rank's rows). The
 * medians are a 3-pass radix selection: for pass = 0, 1, 2 each rank calls
 * yabt_bin_median_hist on its rows, the caller sums the digit histogram
 * (hist_words uint32 counts) and, after pass 0, the per-feature NaN counts
 * (F uint64) over the ranks in place (yabt_bin_median_bufs gives both
 * addresses), then every rank calls yabt_bin_median_pick with the total row
 * count; yabt_bin_median_final writes the medians. The workspace is sized by
 * yabt_bin_fit_workspace_bytes(n_local, F, 1). yabt_bin_fit_edges fits the
 * edges and scales on a gathered (F, nq) feature-major sample matrix
 * (workspace yabt_bin_fit_workspace_bytes(nq, F, nq)).                    */
int yabt_bin_median_hist(const float* Xfm, long long n, int F, int pass, void* workspace, long long ws_bytes,
                         void* stream);
int yabt_bin_median_pick(long long n_total, int F, int pass, void* workspace, long long ws_bytes, void* stream);
int yabt_bin_median_final(int F, void* workspace, long long ws_bytes, float* medians, void* stream);
int yabt_bin_median_bufs(int F, void* workspace, void** hist, long long* hist_words, void** nan_count);
int yabt_bin_fit_edges(const float* Xs, long long nq, int F, int max_bins, void* workspace, long long ws_bytes,
                       float* edges, int32_t* edge_cnt, float* scales, void* stream);
/* Allocation-free variant of yabt_bin_fit (no counterpart in the reference).
 * For callers that cannot allocate device memory when they fit -- e.g. a
 * process whose GPU memory is reserved up front by another framework's caching
 * allocator, or a latency-critical loop where cudaMalloc (which may
 * synchronise the device and can fail under memory pressure) is not allowed.
 * Same inputs, outputs and results as yabt_bin_fit; the scratch lives in a
 * fixed device array of yabt_bin_fit_static_capacity() bytes (8 MiB) that
 * every GPU loading the library holds until the process exits. Fits whose
 * scratch (yabt_bin_fit_workspace_bytes) exceeds it are rejected with
 * YABT_ERR_UNSUPPORTED (e.g. F = 64 features with up to 16384 sample rows fit,
 * the default 200000-row sample of 200 features does not). The first call on
 * each device looks up the array's device address; make that first call before
 * any stream capture. All calls on a device share the one array: calls whose
 * work overlaps on the GPU (different streams, or host threads) race and
 * corrupt each other's results -- serialise them. The function allocates
 * nothing.                                                                */
long long yabt_bin_fit_static_capacity(void);
int yabt_bin_fit_static(const float* Xfm, long long n, int F, const int32_t* sample_idx, long long nq,
                        int max_bins, float* medians, float* edges, int32_t* edge_cnt, float* scales,
                        void* stream);
/* NaN -> median in Xfm (in place), bins = #{edges < x} into the tiled layout
 * (and, if plain_out != NULL, the plain (n, F) matrix; if fm_out != NULL, a
 * feature-major (F, n) copy, which the grower's row partition reads).
 * Replaces Binner.transform / impute (yabt/binning.py:97-124).           */
int yabt_bin_transform(float* Xfm, long long n, int F, const float* medians, const float* edges,
                       const int32_t* edge_cnt, uint8_t* tiled, uint8_t* plain_out, uint8_t* fm_out,
                       void* stream);

/* ------------------------------------------------------------------ neural leaves
 * Ridge-linear leaf models of one grown tree (fit_leaf_networks with
 * leaf_net_hidden == 0, yabt/neural_leaves.py:131-184).                  */
typedef struct {
  const int64_t* feature;         /* [max_nodes] tree arrays from yabt_grow_* */
  float* value;                   /* [max_nodes] updated in place (folded bias) */
  int32_t max_nodes;
  const int32_t* meta;            /* grower meta (n_nodes first) */
  const int32_t* leaf_src;        /* leaf row ranges (yabt_grow_leaf_rows) */
  const int32_t* leaf_begin;
  const int32_t* leaf_count;
  const int32_t* fin;
  const int32_t* list0;
  const int32_t* list1;
  const int32_t* leaf_of_row;     /* [n] */
  const float* Xfm;               /* [F][n] imputed features */
  const float* col_mean;          /* [F] column means (yabt_column_stats) */
  const float* col_std;           /* [F] unbiased column std */
  const float* margin;            /* [n] ensemble margin excluding this tree */
  const float* y;                 /* [n] */
  long long n;
  int32_t F;
  int32_t K;                      /* min(leaf_net_features, F), 1..8 */
  int32_t loss;                   /* 0 squared error, 1 logistic */
  int32_t min_samples;            /* leaf_net_min_samples */
  float l2;                       /* leaf_net_l2 */
  float learning_rate;
  int64_t* feats;                 /* out [K] */
  float* linear;                  /* out [max_nodes][K] */
  float* lo;                      /* out [max_nodes][K] */
  float* hi;                      /* out [max_nodes][K] */
  int32_t* has_nets;              /* out [1]: 0 when no leaf is eligible */
} yabt_leafnet_args;

long long yabt_leafnet_workspace_bytes(long long n, int F, int max_nodes);
int yabt_leafnet_fit(const yabt_leafnet_args* a, void* workspace, long long ws_bytes, void* stream);
/* yabt_leafnet_fit in three stages for rows sharded across GPUs
 * (fit_leaf_networks over every rank's rows). Between the stages the caller
 * reduces over the ranks, in place:
 *   after stage 0: sum of stats (float64: X^T g, sum g, leaf row counts);
 *   after stage 1: sum of totals (float64 per-leaf normal equations) and max
 *                  of envelope (float32: -min x, max x per leaf input).
 * Stage 2 solves and folds. yabt_leafnet_bufs gives addresses and counts.  */
int yabt_leafnet_stage(const yabt_leafnet_args* a, int stage, void* workspace, long long ws_bytes, void* stream);
int yabt_leafnet_bufs(const yabt_leafnet_args* a, void* workspace, long long ws_bytes, void** stats,
                      long long* stats_count, void** totals, long long* totals_count, void** envelope,
                      long long* envelope_count);

/* Margin update of one tree and the next tree's gradients
 * (yabt/boosting.py:36-38,53-54,511-514; Tree.net_contribution yabt/tree.py:118-128). */
typedef struct {
  const int32_t* leaf_of_row;
  int32_t max_nodes;              /* length of the per-node tables */
  const float* value;
  const float* linear;            /* NULL: constant leaves */
  const float* lo;
  const float* hi;
  const int64_t* feats;
  const int32_t* has_nets;
  int32_t K;
  const float* Xfm;
  long long n;
  float* margin;                  /* in/out */
  const float* y;
  float* grad;                    /* out, or NULL */
  float* hess;                    /* out, or NULL (unit hessian) */
  int32_t loss;
} yabt_update_args;

int yabt_update_margin(const yabt_update_args* a, void* stream);
int yabt_grad_init(const float* margin, const float* y, long long n, int loss, float* grad, float* hess,
                   void* stream);
/* Column means and unbiased stds of Xfm (fp64 accumulation). */
int yabt_column_stats(const float* Xfm, long long n, int F, float* mean, float* std, void* stream);
/* The same moments over rows sharded across GPUs: pass 0 writes acc[f] = sum x
 * of this rank's rows; once acc[0..F) holds the sum over all ranks, pass 1
 * writes acc[F+f] = sum (x - mean)^2; once that is summed too,
 * yabt_column_finish writes mean and std. acc is [2F] float64.          */
int yabt_column_sums(const float* Xfm, long long n, long long n_total, int F, int pass, double* acc, void* stream);
int yabt_column_finish(const double* acc, long long n_total, int F, float* mean, float* std, void* stream);

/* ------------------------------------------------------------------ interaction steering
 * FeatureInteractionDetector.update_from_path_pairs / normalized_matrix
 * (yabt/adaptive_features.py:129-160) on the device.                     */
int yabt_interaction_update(const int64_t* feature, const int64_t* left, const int64_t* right,
                            const int32_t* meta, int F, int max_nodes, float* scores,
                            int32_t* parent_scratch, void* stream);
int yabt_interaction_normalize(const float* scores, int F, float* imat, void* stream);

/* ------------------------------------------------------------------ inference
 * Batched prediction of a packed forest (Booster._margin / Tree.predict,
 * yabt/boosting.py:542-550, yabt/tree.py:82-135). X is the imputed raw
 * (n, F) row-major matrix; node arrays of all trees are concatenated, tree t
 * starting at tree_off[t], child indices local to the tree. has_nets[t] = 0
 * (or has_nets == NULL) means constant leaves.                           */
int yabt_predict_forest(const float* X, long long n, int F, int ntrees, const int64_t* tree_off,
                        const int32_t* feature, const float* threshold, const int32_t* left,
                        const int32_t* right, const float* value, const int32_t* has_nets,
                        const int64_t* feats, int K, const float* linear, const float* lo, const float* hi,
                        float base, float* out, void* stream);
/* Leaf index per row for one tree (Tree.apply, yabt/tree.py:82-116; the
 * reference's C variant capply, yabt/_cgrow/grow.c:223-239).              */
int yabt_apply_tree(const float* X, long long n, int F, const int64_t* feature, const float* threshold,
                    const int64_t* left, const int64_t* right, int64_t* out, void* stream);
/* NaN -> medians[f] in a row-major (n, F) matrix (Binner.impute, yabt/binning.py:121-124). */
int yabt_impute_rows(float* X, long long n, int F, const float* medians, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* YABT_B200_H */
