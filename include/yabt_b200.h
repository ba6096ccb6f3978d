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

/* ------------------------------------------------------------------ bin matrix
 * The tiled bin-matrix layout (see DESIGN.md "Data layout"): size in bytes for
 * n rows x F features, and the byte address of (row, feature).            */
long long yabt_bin_matrix_bytes(long long n, int F);
int yabt_bin_address(long long n, int F, int feature, long long* tile_off, int* width, int* pos);

/* Pack a plain row-major (n, F) uint8 bin matrix into the tiled layout.
 * Replaces the layout contract of yabt/cuda_hist.py:79-89 (row-major (n, F)
 * uint8 input) for callers that hold plain bin matrices.                  */
int yabt_pack_bins(const uint8_t* plain, long long n, int F, uint8_t* tiled, void* stream);

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
} yabt_tree_args;

/* Grow one tree (single device): all levels, no host synchronisation. */
int yabt_grow_tree(yabt_grower* g, const yabt_tree_args* a, void* stream);

/* Step-wise driving for row-sharded multi-GPU growth: the caller may
 * all-reduce (max) the two words at yabt_grow_amax_ptr() after
 * yabt_grow_begin, and all-reduce (sum, int64) the small-child histograms at
 * yabt_grow_small_ptr() between yabt_grow_hist and yabt_grow_split of each
 * level (count = yabt_grow_small_count(level) int64 values).             */
int yabt_grow_begin(yabt_grower* g, const yabt_tree_args* a, void* stream);
int yabt_grow_init(yabt_grower* g, const yabt_tree_args* a, void* stream);
int yabt_grow_hist(yabt_grower* g, const yabt_tree_args* a, int level, void* stream);
int yabt_grow_split(yabt_grower* g, const yabt_tree_args* a, int level, void* stream);
int yabt_grow_end(yabt_grower* g, const yabt_tree_args* a, void* stream);
void* yabt_grow_amax_ptr(yabt_grower* g);
void* yabt_grow_small_ptr(yabt_grower* g);
long long yabt_grow_small_count(const yabt_grower* g, int level);
/* Per-leaf row ranges of the last tree (device arrays inside the workspace):
 * src (0 fin, 1 list0, 2 list1, 3 identity), begin, count; plus list bases. */
int yabt_grow_leaf_rows(yabt_grower* g, void** src, void** begin, void** count,
                        void** fin, void** list0, void** list1);

#ifdef __cplusplus
}
#endif
#endif /* YABT_B200_H */
