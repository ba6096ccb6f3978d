// C ABI of libyabt_b200.so: error reporting, bin-matrix layout helpers and the
// level-wise grower context (workspace carving + launch sequencing).
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "../../include/yabt_b200.h"
#include "grow.cuh"

namespace yabt {

static thread_local char g_err[512] = "";
static std::atomic<long long> g_launches{0};

void count_launches(int k) {
  if (!capturing_level_loop()) g_launches.fetch_add(k, std::memory_order_relaxed);   // graph loops count on the device
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

cudaError_t launch_level_hist(const GrowParams&, const GrowBufs&, const TreeIO&, int, int, cudaStream_t,
                              cudaEvent_t after_hist, int root_counts);
cudaError_t launch_level_split(const GrowParams&, const GrowBufs&, const TreeIO&, int, int, cudaStream_t);
cudaError_t launch_level_scan(const GrowParams&, const GrowBufs&, const TreeIO&, int, int, cudaStream_t);
cudaError_t launch_level_choose(const GrowParams&, const GrowBufs&, const TreeIO&, int, int, cudaStream_t);
cudaError_t launch_tree_begin(const GrowParams&, const GrowBufs&, const TreeIO&, int, cudaStream_t);
cudaError_t launch_tree_init(const GrowParams&, const GrowBufs&, const TreeIO&, cudaStream_t);
cudaError_t launch_tree_finish(const GrowParams&, const GrowBufs&, const TreeIO&, int*, int*, int, cudaStream_t);
cudaError_t launch_apply_all(const GrowParams&, const GrowBufs&, const TreeIO&, int, cudaStream_t);
cudaError_t launch_hist_kernels(const GrowParams&, const GrowBufs&, const TreeIO&, int, int, int, cudaStream_t,
                                cudaEvent_t, int);
cudaError_t launch_bf_root_scan(const GrowParams&, const GrowBufs&, const TreeIO&, cudaStream_t);
cudaError_t launch_bf_split(const GrowParams&, const GrowBufs&, const TreeIO&, int, int, cudaStream_t);
cudaError_t launch_bf_scan(const GrowParams&, const GrowBufs&, const TreeIO&, int, cudaStream_t);
cudaError_t launch_bf_pick_partition(const GrowParams&, const GrowBufs&, const TreeIO&, int, int, cudaStream_t);
cudaError_t launch_absmax_shared(const float* const*, int, long long, const int*, GrowState*, int, cudaStream_t);
cudaError_t launch_mt_scan(const GrowParams&, const GrowBufs&, const MtBufs&, const TreeIO&, int, int, cudaStream_t);
cudaError_t launch_mt_commit(const GrowParams&, const GrowBufs&, const MtBufs&, cudaStream_t);
cudaError_t launch_mt_values(const GrowParams&, const GrowBufs&, const MtBufs&, cudaStream_t);
cudaError_t launch_mt_update(const int*, const float*, int, long long, float*, const float*, float*, int, cudaStream_t);
cudaError_t set_hist_smem_attrs();
cudaError_t launch_unpack_counts(const GrowParams&, const GrowBufs&, long long*, cudaStream_t);
cudaError_t launch_level_loop_cond(const GrowParams&, const GrowBufs&, cudaGraphConditionalHandle, int, cudaStream_t);
cudaError_t loop_launches_reset(cudaStream_t);
cudaError_t loop_launches_read(long long*);

// ---------------------------------------------------------------- pack kernel
__global__ void k_pack_bins(const uint8_t* __restrict__ plain, long long n, int F,
                            uint8_t* __restrict__ tiled) {
  const long long total = n * F;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long r = e / F;
    const int f = (int)(e % F);
    const FeatAddr a = feat_addr(F, n, f);
    tiled[a.off + r * a.width + a.pos] = plain[e];
  }
}

}  // namespace yabt

using namespace yabt;

#define CUDA_TRY(x)                                                              \
  do {                                                                           \
    cudaError_t e__ = (x);                                                       \
    if (e__ != cudaSuccess) {                                                    \
      set_error("%s failed: %s (%s:%d)", #x, cudaGetErrorString(e__), __FILE__, __LINE__); \
      return YABT_ERR_CUDA;                                                      \
    }                                                                            \
  } while (0)

static std::vector<TileInfo> host_tiles(int F, long long n, long long* bytes) {
  std::vector<TileInfo> t(tile_count(F) + 1);
  long long b = make_tiles(F, n, t.data());
  t.resize(tile_count(F));
  if (bytes) *bytes = b;
  return t;
}

extern "C" {

int yabt_version(void) { return 100; }

long long yabt_launch_count(void) { return g_launches.load(); }

long long yabt_launch_count_device(void) {
  long long v = 0;
  if (loop_launches_read(&v) != cudaSuccess) {
    cudaGetLastError();
    set_error("yabt_launch_count_device: reading the device counter failed");
    return -1;
  }
  return v;
}

int yabt_launch_count_device_reset(void* stream) {
  CUDA_TRY(loop_launches_reset((cudaStream_t)stream));
  return YABT_OK;
}

int yabt_last_error(char* buf, int len) {
  if (!buf || len <= 0) return YABT_ERR_ARG;
  strncpy(buf, g_err, (size_t)len - 1);
  buf[len - 1] = 0;
  return YABT_OK;
}

long long yabt_bin_matrix_bytes(long long n, int F) {
  if (n < 0 || F <= 0) return -1;
  long long b = 0;
  host_tiles(F, n, &b);
  return b;
}

int yabt_bin_address(long long n, int F, int feature, long long* tile_off, int* width, int* pos) {
  if (n < 0 || F <= 0 || feature < 0 || feature >= F) { set_error("bad bin address query"); return YABT_ERR_ARG; }
  auto t = host_tiles(F, n, nullptr);
  std::vector<FeatAddr> fa(F);
  feat_addrs(F, t.data(), (int)t.size(), fa.data());
  if (tile_off) *tile_off = fa[feature].off;
  if (width) *width = fa[feature].width;
  if (pos) *pos = fa[feature].pos;
  return YABT_OK;
}

int yabt_pack_bins(const uint8_t* plain, long long n, int F, uint8_t* tiled, void* stream) {
  if (!plain || !tiled || n < 0 || F <= 0) { set_error("yabt_pack_bins: bad arguments"); return YABT_ERR_ARG; }
  if (n == 0) return YABT_OK;
  cudaStream_t s = (cudaStream_t)stream;
  long long bytes = 0;
  host_tiles(F, n, &bytes);
  CUDA_TRY(cudaMemsetAsync(tiled, 0, (size_t)bytes, s));
  const long long total = n * F;
  const int grid = (int)std::min<long long>((total + 255) / 256, (long long)YABT_SMS_HINT * 32);
  k_pack_bins<<<grid, 256, 0, s>>>(plain, n, F, tiled);
  count_launches(1);
  CUDA_TRY(cudaGetLastError());
  return YABT_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- grower
// The feature-sliced exchange of a sharded device-side level loop (all zero
// for a single-GPU loop).
struct LoopXchg {
  int on;
  int rank, nranks, first;
  long long rec_offset;
  void* bufs[8];
};

struct yabt_grower {
  GrowParams p;
  GrowBufs b;
  long long ws_bytes;
  int bound;
  int nsm;
  int LIMBS;
  std::vector<UnitDesc> units;
  std::vector<FeatAddr> faddr;
  // optional per-launch timing of the histogram kernel
  int timing = 0;
  std::vector<cudaEvent_t> ev;   // pairs (start, stop)
  int ev_used = 0;
  // carve offsets
  struct Off { const char* name; long long bytes; long long off; };
  std::vector<Off> offs;
  // yabt_grow_tree stops launching levels once a level reports the tree
  // complete: the level state is copied to pinned host memory after each
  // split and read LEVEL_LOOKAHEAD levels later (the GPU keeps that many
  // levels queued, so the read rarely waits on work it could be doing)
  int* host_state = nullptr;               // [LEVEL_SLOTS][4] pinned
  cudaEvent_t lvl_ev[8] = {};
  int level_wait = 1;                      // 0: queue every level without waiting
  // cached root-level counts (yabt_grower_set_root_count_cache): 0 off; 1 on,
  // recorded by the next root histogram over all rows and reused after that
  int rc_mode = 0, rc_valid = 0;
  // device-side level loop (yabt_grower_set_level_loop): yabt_grow_tree
  // launches the levels below level_loop_start() as usual, then one CUDA graph
  // whose WHILE node repeats a level's kernels while the tree is active, so a
  // tree that finishes early leaves no queued no-op levels behind. The graph
  // bakes in p and b; it is captured again when either changes.
  int level_loop = 1;
  cudaGraphExec_t loop_exec = nullptr;
  cudaStream_t loop_cap = nullptr;         // capture stream
  GrowParams loop_p;
  GrowBufs loop_b;
  LoopXchg loop_x = {};                    // the exchange the graph was captured with (sharded trees)
};

static constexpr int LEVEL_SLOTS = 8, LEVEL_LOOKAHEAD = 3;

static long long al(long long x) { return (x + 255) & ~255LL; }

namespace yabt {
GrowState* grower_state(yabt_grower* g) { return g && g->bound ? g->b.st : nullptr; }
int grower_slice(yabt_grower* g, int* F, int* C, int* f_lo, int* f_hi) {
  if (!g || !g->bound) return 1;
  *F = g->p.F; *C = g->p.C; *f_lo = g->p.f_lo; *f_hi = g->p.f_hi;
  return 0;
}
void grower_best_bufs(yabt_grower* g, unsigned long long** node_key, NodeBest** best) {
  *node_key = g && g->bound ? g->b.node_key : nullptr;
  *best = g && g->bound ? g->b.best : nullptr;
}
int grower_maxa(const yabt_grower* g) { return g ? g->p.maxa : 0; }
}  // namespace yabt

extern "C" {

int yabt_grower_create(long long n, int F, int max_leaves, int max_depth, int general,
                       yabt_grower** out) {
  if (!out || n <= 0 || n >= (1LL << 31) || F <= 0 || max_leaves < 1 || max_depth < 0) {
    set_error("yabt_grower_create: bad arguments (n=%lld F=%d max_leaves=%d max_depth=%d)", n, F,
              max_leaves, max_depth);
    return YABT_ERR_ARG;
  }
  yabt_grower* g = new yabt_grower();
  GrowParams& p = g->p;
  memset(&p, 0, sizeof(p));
  p.n = n; p.F = F; p.general = general ? 1 : 0;
  p.f_lo = 0; p.f_hi = F;
  p.S = general ? 1 : 2; g->LIMBS = general ? 5 : 3; p.C = general ? 3 : 2;
  p.max_leaves = max_leaves; p.max_depth = max_depth;
  p.maxa = max_leaves;
  p.maxn = 2 * max_leaves + 1;
  p.max_pairs = std::max(1, max_leaves - 1);
  p.levels_max = std::max(1, std::min(max_depth, max_leaves - 1));
  // units
  auto tiles = host_tiles(F, n, nullptr);
  for (auto& t : tiles) {
    if (t.wide && p.S == 1) {
      for (int k0 = 0; k0 < 2; ++k0) {
        UnitDesc u; memset(&u, 0, sizeof(u));
        u.off = t.off; u.width = t.width; u.wide = 1; u.k0 = k0; u.nsub = 1; u.rep = 1; u.lw = 32;
        for (int j = 0; j < 32; ++j) { u.feat[0][j] = t.f0 + 32 * k0 + j; u.feat[1][j] = -1; }
        g->units.push_back(u);
      }
    } else {
      UnitDesc u; memset(&u, 0, sizeof(u));
      u.off = t.off; u.width = t.width; u.wide = t.wide; u.k0 = 0;
      u.nsub = t.wide ? 2 : 1;
      u.rep = 1; u.lw = 32;
      if (t.width == 16) {            // 16-wide tail tile: several rows per reduction
        u.rep = t.nfeat <= 8 ? 4 : 2;
        u.lw = 32 / u.rep;
      }
      for (int j = 0; j < 32; ++j) {
        const int jj = j % u.lw;        // lanes of one row hold features 0 .. lw-1
        u.feat[0][j] = jj < std::min(t.nfeat, 32) ? t.f0 + jj : -1;
        u.feat[1][j] = (t.wide && 32 + j < t.nfeat) ? t.f0 + 32 + j : -1;
      }
      g->units.push_back(u);
    }
  }
  p.U = (int)g->units.size();
  g->faddr.resize(F);
  feat_addrs(F, tiles.data(), (int)tiles.size(), g->faddr.data());
  p.max_items = ITEM_TARGET + p.U * (int)(n / CHUNK_MAX + 1) + p.U * (p.max_pairs + 1);
  p.max_tiles = (int)((n + PART_TILE - 1) / PART_TILE) + p.maxa + 1;
  // workspace carve list
  const long long HN = (long long)p.C * F * YABT_NB * 8;
  const long long words = (long long)g->LIMBS * p.S * YABT_NB * 32;
  auto add = [&](const char* nm, long long bytes) { g->offs.push_back({nm, bytes, 0}); };
  add("st", sizeof(GrowState));
  add("io", sizeof(TreeIO));
  add("rows0", n * 4); add("rows1", n * 4); add("fin", n * 4);
  add("segb0", std::max(p.maxa, 2) * 4); add("segb1", std::max(p.maxa, 2) * 4);
  add("segc0", std::max(p.maxa, 2) * 4); add("segc1", std::max(p.maxa, 2) * 4);
  add("gid0", p.maxa * 4); add("gid1", p.maxa * 4);
  add("hist0", p.maxa * HN); add("hist1", p.maxa * HN);
  add("small", (long long)p.max_pairs * small_job_words(p.C, F) * 8);
  add("pm0", (long long)p.maxa * F * 4); add("pm1", (long long)p.maxa * F * 4);
  add("best", (long long)p.maxa * F * sizeof(NodeBest));
  add("nbest", (long long)p.maxa * sizeof(NodeBest));
  add("nkey", (long long)std::max(p.maxa, 2) * 8);   // best-first folds two children
  add("rootcnt", (long long)F * (YABT_NB / 2) * 8);
  add("bffeat", 2LL * F * sizeof(BfCand));
  add("bfcand", (long long)p.maxn * sizeof(BfCand));
  add("nslot", (long long)p.maxn * 4);
  add("tot", (long long)p.maxa * sizeof(NodeTot));
  add("pair_pos", p.max_pairs * 4); add("pair_sil", p.max_pairs * 4);
  add("split_pair", p.maxa * 4); add("split_f", p.maxa * 4); add("split_b", p.maxa * 4);
  add("tpre", (long long)(std::max(p.maxa, p.max_pairs) + 1) * 4);
  add("items", (long long)p.max_items * sizeof(HistItem));
  add("job_first", (long long)p.max_pairs * p.U * 4); add("job_nitems", (long long)p.max_pairs * p.U * 4);
  add("tiles", (long long)p.max_tiles * sizeof(PartTile));
  add("tile_status", (long long)p.max_tiles * 8);
  add("partials", (long long)p.max_items * words * 4);
  add("units", (long long)p.U * sizeof(UnitDesc));
  add("faddr", (long long)F * sizeof(FeatAddr));
  add("leaf_src", p.maxn * 4); add("leaf_begin", p.maxn * 4); add("leaf_count", p.maxn * 4);
  add("node_depth", p.maxn * 4); add("node_bin", p.maxn * 4);
  long long off = 0;
  for (auto& o : g->offs) { o.off = off; off = al(off + o.bytes); }
  g->ws_bytes = off;
  int dev = 0;
  cudaGetDevice(&dev);
  int nsm = YABT_SMS_HINT;
  if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) nsm = YABT_SMS_HINT;
  cudaGetLastError();
  g->nsm = nsm;
  *out = g;
  return YABT_OK;
}

long long yabt_grower_workspace_bytes(const yabt_grower* g) { return g ? g->ws_bytes : -1; }
int yabt_grower_max_nodes(const yabt_grower* g) { return g ? g->p.maxn : -1; }
int yabt_grower_levels(const yabt_grower* g) { return g ? g->p.levels_max : -1; }

int yabt_grower_bind(yabt_grower* g, void* ws, long long bytes, void* stream) {
  if (!g || !ws) { set_error("yabt_grower_bind: null argument"); return YABT_ERR_ARG; }
  if (bytes < g->ws_bytes) {
    set_error("yabt_grower_bind: workspace of %lld bytes < required %lld", bytes, g->ws_bytes);
    return YABT_ERR_WORKSPACE;
  }
  if (((uintptr_t)ws & 255) != 0) { set_error("yabt_grower_bind: workspace not 256-byte aligned"); return YABT_ERR_ARG; }
  char* base = (char*)ws;
  auto P = [&](const char* nm) -> char* {
    for (auto& o : g->offs) if (!strcmp(o.name, nm)) return base + o.off;
    return nullptr;
  };
  GrowBufs& b = g->b;
  b.st = (GrowState*)P("st");
  b.io_dev = (TreeIO*)P("io");
  b.rows[0] = (int*)P("rows0"); b.rows[1] = (int*)P("rows1"); b.fin = (int*)P("fin");
  b.seg_begin[0] = (int*)P("segb0"); b.seg_begin[1] = (int*)P("segb1");
  b.seg_count[0] = (int*)P("segc0"); b.seg_count[1] = (int*)P("segc1");
  b.act_gid[0] = (int*)P("gid0"); b.act_gid[1] = (int*)P("gid1");
  b.hist[0] = (long long*)P("hist0"); b.hist[1] = (long long*)P("hist1");
  b.small = (long long*)P("small");
  b.node_key = (unsigned long long*)P("nkey");
  b.root_cnt = (long long*)P("rootcnt");
  b.bf_feat = (BfCand*)P("bffeat"); b.bf_cand = (BfCand*)P("bfcand"); b.node_slot = (int*)P("nslot");
  b.pathmax[0] = (float*)P("pm0"); b.pathmax[1] = (float*)P("pm1");
  b.best = (NodeBest*)P("best"); b.nbest = (NodeBest*)P("nbest"); b.tot = (NodeTot*)P("tot");
  b.pair_pos = (int*)P("pair_pos"); b.pair_sil = (int*)P("pair_sil");
  b.split_pair = (int*)P("split_pair"); b.split_f = (int*)P("split_f"); b.split_b = (int*)P("split_b");
  b.node_tpre = (int*)P("tpre");
  b.items = (HistItem*)P("items");
  b.job_first = (int*)P("job_first"); b.job_nitems = (int*)P("job_nitems");
  b.tiles = (PartTile*)P("tiles"); b.tile_status = (unsigned long long*)P("tile_status");
  b.partials = (unsigned*)P("partials");
  b.units = (UnitDesc*)P("units"); b.faddr = (FeatAddr*)P("faddr");
  b.leaf_src = (int*)P("leaf_src"); b.leaf_begin = (int*)P("leaf_begin"); b.leaf_count = (int*)P("leaf_count");
  b.node_depth = (int*)P("node_depth"); b.node_bin = (int*)P("node_bin");
  cudaStream_t s = (cudaStream_t)stream;
  CUDA_TRY(set_hist_smem_attrs());
  CUDA_TRY(cudaMemsetAsync(b.st, 0, sizeof(GrowState), s));
  CUDA_TRY(cudaMemsetAsync(b.tile_status, 0, (size_t)g->p.max_tiles * 8, s));
  CUDA_TRY(cudaMemcpyAsync(b.units, g->units.data(), sizeof(UnitDesc) * g->units.size(), cudaMemcpyHostToDevice, s));
  CUDA_TRY(cudaMemcpyAsync(b.faddr, g->faddr.data(), sizeof(FeatAddr) * g->faddr.size(), cudaMemcpyHostToDevice, s));
  CUDA_TRY(cudaStreamSynchronize(s));
  g->bound = 1;
  return YABT_OK;
}

int yabt_grower_destroy(yabt_grower* g) {
  if (g) {
    if (g->loop_exec) cudaGraphExecDestroy(g->loop_exec);
    if (g->loop_cap) cudaStreamDestroy(g->loop_cap);
    for (auto e : g->ev) cudaEventDestroy(e);
    for (auto e : g->lvl_ev) if (e) cudaEventDestroy(e);
    if (g->host_state) cudaFreeHost(g->host_state);
  }
  delete g;
  return YABT_OK;
}

int yabt_grower_set_timing(yabt_grower* g, int max_launches) {
  if (!g) { set_error("null grower"); return YABT_ERR_ARG; }
  g->ev_used = 0;
  g->timing = max_launches > 0;
  while ((int)g->ev.size() < 2 * max_launches) {
    cudaEvent_t e;
    CUDA_TRY(cudaEventCreate(&e));
    g->ev.push_back(e);
  }
  return YABT_OK;
}

int yabt_grower_acc_reset(yabt_grower* g, void* stream) {
  if (!g || !g->bound) { set_error("grower not bound"); return YABT_ERR_ARG; }
  CUDA_TRY(cudaMemsetAsync(&g->b.st->acc_root_rows, 0, 3 * sizeof(long long), (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_grower_acc_read(yabt_grower* g, long long* out3) {
  if (!g || !g->bound || !out3) { set_error("grower not bound"); return YABT_ERR_ARG; }
  CUDA_TRY(cudaMemcpy(out3, &g->b.st->acc_root_rows, 3 * sizeof(long long), cudaMemcpyDeviceToHost));
  return YABT_OK;
}

int yabt_grower_hist_rows(yabt_grower* g, long long* rows, int cap) {
  if (!g || !g->bound || !rows) { set_error("null argument"); return YABT_ERR_ARG; }
  CUDA_TRY(cudaMemcpy(rows, g->b.st->hist_rows, sizeof(long long) * std::min(cap, 64), cudaMemcpyDeviceToHost));
  return YABT_OK;
}

int yabt_grower_hist_times(yabt_grower* g, float* ms, int cap, int* count) {
  if (!g || !count) { set_error("null argument"); return YABT_ERR_ARG; }
  const int k = g->ev_used / 2;
  for (int i = 0; i < k && i < cap; ++i) {
    CUDA_TRY(cudaEventSynchronize(g->ev[2 * i + 1]));
    CUDA_TRY(cudaEventElapsedTime(&ms[i], g->ev[2 * i], g->ev[2 * i + 1]));
  }
  *count = k;
  g->ev_used = 0;
  return YABT_OK;
}

}  // extern "C"

// the root-count mode of this tree's root histogram (see launch_hist_kernels)
static int root_count_mode(yabt_grower* g, const TreeIO& io) {
  if (!g->rc_mode || io.root_rows) return 0;
  if (g->rc_valid) return 2;
  g->rc_valid = 1;          // this launch records them
  return 1;
}

static int fill_io(yabt_grower* g, const yabt_tree_args* a, TreeIO* io) {
  if (!g || !a || !g->bound) { set_error("grower not created/bound"); return YABT_ERR_ARG; }
  if (!a->bins || !a->grad || (g->p.general && !a->hess) || !a->edges || !a->edge_off || !a->edge_cnt ||
      !a->scales || !a->feature || !a->threshold || !a->left || !a->right || !a->value ||
      !a->gate_scale || !a->leaf_of_row || !a->meta) {
    set_error("yabt_tree_args: null required pointer");
    return YABT_ERR_ARG;
  }
  GrowParams& p = g->p;
  p.lam = a->reg_lambda; p.gamma = a->gamma; p.mcw = a->min_child_weight; p.lr = a->learning_rate;
  p.ib = a->interaction_boost; p.msl = a->min_samples_leaf;
  p.use_imat = a->interaction != nullptr; p.use_fmask = a->feature_mask != nullptr;
  io->bins = a->bins; io->g = a->grad; io->h = g->p.general ? a->hess : nullptr;
  io->edges = a->edges; io->edge_off = a->edge_off; io->edge_cnt = a->edge_cnt; io->scales = a->scales;
  io->fmask = a->feature_mask; io->imat = a->interaction;
  io->feature = (long long*)a->feature; io->threshold = a->threshold;
  io->left = (long long*)a->left; io->right = (long long*)a->right;
  io->value = a->value; io->gate = a->gate_scale; io->leaf_of_row = a->leaf_of_row;
  io->bins_fm = a->bins_fm;
  io->root_rows = a->root_rows;
  io->n_root = a->root_rows ? a->n_root : p.n;
  if (io->n_root < 0 || io->n_root > p.n) { set_error("yabt_tree_args: n_root out of range"); return YABT_ERR_ARG; }
  return YABT_OK;
}

extern "C" {

int yabt_grow_begin(yabt_grower* g, const yabt_tree_args* a, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  CUDA_TRY(launch_tree_begin(g->p, g->b, io, g->nsm, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_grow_init(yabt_grower* g, const yabt_tree_args* a, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  CUDA_TRY(launch_tree_init(g->p, g->b, io, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_grow_hist(yabt_grower* g, const yabt_tree_args* a, int level, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  if (level < 0 || level >= g->p.levels_max) { set_error("level out of range"); return YABT_ERR_ARG; }
  cudaStream_t s = (cudaStream_t)stream;
  const bool tm = g->timing && g->ev_used + 2 <= (int)g->ev.size();
  if (tm) CUDA_TRY(cudaEventRecord(g->ev[g->ev_used], s));
  CUDA_TRY(launch_level_hist(g->p, g->b, io, level, g->nsm, s, tm ? g->ev[g->ev_used + 1] : nullptr,
                             level == 0 ? root_count_mode(g, io) : 0));
  if (tm) g->ev_used += 2;
  return YABT_OK;
}

int yabt_grow_split(yabt_grower* g, const yabt_tree_args* a, int level, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  if (level < 0 || level >= g->p.levels_max) { set_error("level out of range"); return YABT_ERR_ARG; }
  CUDA_TRY(launch_level_split(g->p, g->b, io, level, g->nsm, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_grow_scan(yabt_grower* g, const yabt_tree_args* a, int level, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  if (level < 0 || level >= g->p.levels_max) { set_error("level out of range"); return YABT_ERR_ARG; }
  CUDA_TRY(launch_level_scan(g->p, g->b, io, level, g->nsm, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_grow_choose(yabt_grower* g, const yabt_tree_args* a, int level, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  if (level < 0 || level >= g->p.levels_max) { set_error("level out of range"); return YABT_ERR_ARG; }
  CUDA_TRY(launch_level_choose(g->p, g->b, io, level, g->nsm, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_grower_set_feature_slice(yabt_grower* g, int f_lo, int f_hi) {
  if (!g || f_lo < 0 || f_hi > g->p.F || f_lo >= f_hi) {
    set_error("yabt_grower_set_feature_slice: need 0 <= f_lo < f_hi <= F");
    return YABT_ERR_ARG;
  }
  g->p.f_lo = f_lo;
  g->p.f_hi = f_hi;
  return YABT_OK;
}

int yabt_grow_end(yabt_grower* g, const yabt_tree_args* a, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  CUDA_TRY(launch_tree_finish(g->p, g->b, io, a->meta, a->leaf_of_row, g->nsm, (cudaStream_t)stream));
  return YABT_OK;
}

// First level of the device-side loop, or -1 when the loop would not pay: the
// loop's launches are sized for max_pairs jobs and need at least 8 of them
// (one reduce group per job), so it starts at the first level whose job bound
// reaches max_pairs, and only when at least two levels are left after it.
static int level_loop_first(const yabt_grower* g) {
  const GrowParams& p = g->p;
  if (!g->level_loop || g->level_wait || p.max_pairs < 8) return -1;
  int L = 4;
  while (L < 31 && (1LL << (L - 1)) < p.max_pairs) ++L;
  return p.levels_max - L >= 2 ? L : -1;
}

// Captures the loop graph: [condition] -> WHILE { level at the state's level;
// condition }. With x.on the level also reduce-scatters its histograms and
// gathers the best splits (the sharded feature-sliced level). Returns a YABT
// status; on failure nothing is kept.
static int build_level_loop(yabt_grower* g, const TreeIO& io, const LoopXchg& x) {
  if (g->loop_exec) { cudaGraphExecDestroy(g->loop_exec); g->loop_exec = nullptr; }
  cudaError_t e = cudaSuccess;
  auto cuda_fail = [&](cudaError_t err) {
    set_error("capturing the level-loop graph failed: %s", cudaGetErrorString(err));
    return YABT_ERR_CUDA;
  };
  if (!g->loop_cap && (e = cudaStreamCreateWithFlags(&g->loop_cap, cudaStreamNonBlocking)) != cudaSuccess)
    return cuda_fail(e);
  cudaGraph_t graph = nullptr;
  if ((e = cudaGraphCreate(&graph, 0)) != cudaSuccess) return cuda_fail(e);
  cudaGraphConditionalHandle h;
  cudaGraphNode_t pre = nullptr;
  size_t npre = 1;
  cudaGraphNodeParams cp = {};
  bool capturing = false;
  auto fail = [&](int rc) {
    if (capturing) {
      cudaGraph_t partial = nullptr;
      cudaStreamEndCapture(g->loop_cap, &partial);
    }
    set_capturing_level_loop(false);
    cudaGraphDestroy(graph);
    cudaGetLastError();
    return rc;
  };
  auto fail_cuda = [&](cudaError_t err) { return fail(cuda_fail(err)); };
  if ((e = cudaGraphConditionalHandleCreate(&h, graph, 0, 0)) != cudaSuccess) return fail_cuda(e);
  set_capturing_level_loop(true);
  if ((e = cudaStreamBeginCaptureToGraph(g->loop_cap, graph, nullptr, nullptr, 0, cudaStreamCaptureModeRelaxed)) !=
      cudaSuccess)
    return fail_cuda(e);
  capturing = true;
  if ((e = launch_level_loop_cond(g->p, g->b, h, 0, g->loop_cap)) != cudaSuccess) return fail_cuda(e);
  capturing = false;
  if ((e = cudaStreamEndCapture(g->loop_cap, &graph)) != cudaSuccess) return fail_cuda(e);
  if ((e = cudaGraphGetNodes(graph, &pre, &npre)) != cudaSuccess || npre != 1)
    return fail_cuda(e != cudaSuccess ? e : cudaErrorInvalidValue);
  cp.type = cudaGraphNodeTypeConditional;
  cp.conditional.handle = h;
  cp.conditional.type = cudaGraphCondTypeWhile;
  cp.conditional.size = 1;
  cudaGraphNode_t cond = nullptr;
  if ((e = cudaGraphAddNode(&cond, graph, &pre, 1, &cp)) != cudaSuccess) return fail_cuda(e);
  cudaGraph_t body = cp.conditional.phGraph_out[0];
  if ((e = cudaStreamBeginCaptureToGraph(g->loop_cap, body, nullptr, nullptr, 0, cudaStreamCaptureModeRelaxed)) !=
      cudaSuccess)
    return fail_cuda(e);
  capturing = true;
  // one level at the state's level (LEVEL_DYN launches, grids sized for max_pairs jobs)
  if ((e = launch_level_hist(g->p, g->b, io, LEVEL_DYN, g->nsm, g->loop_cap, nullptr, 0)) != cudaSuccess)
    return fail_cuda(e);
  if (x.on) {
    int rc = xchg_sliced_launch(g, x.bufs, x.rank, x.nranks, LEVEL_DYN, 0u, x.first, g->loop_cap);
    if (rc) return fail(rc);
    if ((e = launch_level_scan(g->p, g->b, io, LEVEL_DYN, g->nsm, g->loop_cap)) != cudaSuccess) return fail_cuda(e);
    rc = xchg_gather_launch(g, x.bufs, x.rank, x.nranks, LEVEL_DYN, 0u, x.rec_offset, x.first, g->loop_cap);
    if (rc) return fail(rc);
    if ((e = launch_level_choose(g->p, g->b, io, LEVEL_DYN, g->nsm, g->loop_cap)) != cudaSuccess) return fail_cuda(e);
  } else if ((e = launch_level_split(g->p, g->b, io, LEVEL_DYN, g->nsm, g->loop_cap)) != cudaSuccess) {
    return fail_cuda(e);
  }
  const int body_kernels = x.on ? LEVEL_LOOP_BODY_KERNELS_SHARDED : LEVEL_LOOP_BODY_KERNELS;
  if ((e = launch_level_loop_cond(g->p, g->b, h, body_kernels, g->loop_cap)) != cudaSuccess) return fail_cuda(e);
  capturing = false;
  if ((e = cudaStreamEndCapture(g->loop_cap, &body)) != cudaSuccess) return fail_cuda(e);
  set_capturing_level_loop(false);
  e = cudaGraphInstantiate(&g->loop_exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) { g->loop_exec = nullptr; cudaGetLastError(); return cuda_fail(e); }
  memcpy(&g->loop_p, &g->p, sizeof(GrowParams));
  memcpy(&g->loop_b, &g->b, sizeof(GrowBufs));
  memcpy(&g->loop_x, &x, sizeof(LoopXchg));
  return YABT_OK;
}

// Whether a tree's levels from level_loop_first() on can run in the loop graph
// now: no event timing (event nodes cannot sit in a conditional body) and no
// capture of the caller's stream in progress.
static bool level_loop_usable(yabt_grower* g, cudaStream_t s) {
  cudaStreamCaptureStatus cst = cudaStreamCaptureStatusNone;
  const bool ok = level_loop_first(g) > 0 && !g->timing && !phase_timing_on() &&
                  cudaStreamIsCapturing(s, &cst) == cudaSuccess && cst == cudaStreamCaptureStatusNone;
  cudaGetLastError();
  return ok;
}

// Launches the loop graph, capturing it first when it is missing or was
// captured with other parameters, buffers or exchange.
static int launch_level_loop(yabt_grower* g, const yabt_tree_args* a, const LoopXchg& x, cudaStream_t s) {
  if (!g->loop_exec || memcmp(&g->loop_p, &g->p, sizeof(GrowParams)) ||
      memcmp(&g->loop_b, &g->b, sizeof(GrowBufs)) || memcmp(&g->loop_x, &x, sizeof(LoopXchg))) {
    TreeIO io;
    int rc = fill_io(g, a, &io);
    if (rc) return rc;
    if ((rc = build_level_loop(g, io, x))) return rc;
  }
  CUDA_TRY(cudaGraphLaunch(g->loop_exec, s));
  count_launches(1);                       // the condition before the loop; the loop counts on the device
  return YABT_OK;
}

int yabt_grow_level_loop_sharded(yabt_grower* g, const yabt_tree_args* a, void* const* bufs, int rank, int nranks,
                                 long long rec_offset, unsigned epoch0, int* used, void* stream) {
  if (!g || !a || !bufs || !used || nranks < 2 || nranks > 8 || rank < 0 || rank >= nranks) {
    set_error("yabt_grow_level_loop_sharded: bad arguments (2 to 8 ranks)");
    return YABT_ERR_ARG;
  }
  *used = 0;
  cudaStream_t s = (cudaStream_t)stream;
  TreeIO io;
  int rc = fill_io(g, a, &io);               // also refreshes the per-call parameters
  if (rc) return rc;
  if (!level_loop_usable(g, s)) return YABT_OK;
  LoopXchg x = {};
  x.on = 1; x.rank = rank; x.nranks = nranks; x.first = level_loop_first(g); x.rec_offset = rec_offset;
  for (int q = 0; q < nranks; ++q) x.bufs[q] = bufs[q];
  if ((rc = xchg_set_loop_epoch(g, epoch0, s))) return rc;
  if ((rc = launch_level_loop(g, a, x, s))) return rc;
  *used = 1;
  return YABT_OK;
}

int yabt_grow_tree(yabt_grower* g, const yabt_tree_args* a, void* stream) {
  int rc;
  if ((rc = yabt_grow_begin(g, a, stream))) return rc;
  if ((rc = yabt_grow_init(g, a, stream))) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (level_loop_usable(g, s)) {
    const int L = level_loop_first(g);
    for (int d = 0; d < L; ++d) {
      if ((rc = yabt_grow_hist(g, a, d, stream))) return rc;
      if ((rc = yabt_grow_split(g, a, d, stream))) return rc;
    }
    const LoopXchg none = {};
    if ((rc = launch_level_loop(g, a, none, s))) return rc;
    return yabt_grow_end(g, a, stream);
  }
  if (!g->host_state) {
    CUDA_TRY(cudaHostAlloc((void**)&g->host_state, sizeof(int) * 4 * LEVEL_SLOTS, cudaHostAllocDefault));
    for (auto& e : g->lvl_ev) CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  for (int d = 0; d < g->p.levels_max; ++d) {
    if ((rc = yabt_grow_hist(g, a, d, stream))) return rc;
    if ((rc = yabt_grow_split(g, a, d, stream))) return rc;
    if (!g->level_wait) continue;
    const int slot = d % LEVEL_SLOTS;
    CUDA_TRY(cudaMemcpyAsync(g->host_state + 4 * slot, &g->b.st->level, 4 * sizeof(int), cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaEventRecord(g->lvl_ev[slot], s));
    if (d >= LEVEL_LOOKAHEAD) {
      const int old = (d - LEVEL_LOOKAHEAD) % LEVEL_SLOTS;
      CUDA_TRY(cudaEventSynchronize(g->lvl_ev[old]));
      if (!g->host_state[4 * old + 1]) break;     // active == 0: later levels would be no-ops
    }
  }
  return yabt_grow_end(g, a, stream);
}

int yabt_grow_bf_root_hist(yabt_grower* g, const yabt_tree_args* a, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  CUDA_TRY(launch_hist_kernels(g->p, g->b, io, 0, 1, g->nsm, (cudaStream_t)stream, nullptr, root_count_mode(g, io)));
  return YABT_OK;
}

int yabt_grow_bf_split(yabt_grower* g, const yabt_tree_args* a, int step, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  if (step < 1 || step > std::max(1, g->p.max_leaves - 1)) { set_error("step out of range"); return YABT_ERR_ARG; }
  CUDA_TRY(launch_bf_split(g->p, g->b, io, step, g->nsm, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_grow_bf_scan(yabt_grower* g, const yabt_tree_args* a, int step, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  if (step < 0 || step > std::max(1, g->p.max_leaves - 1)) { set_error("step out of range"); return YABT_ERR_ARG; }
  if (step == 0) CUDA_TRY(launch_bf_root_scan(g->p, g->b, io, (cudaStream_t)stream));
  else CUDA_TRY(launch_bf_scan(g->p, g->b, io, g->nsm, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_grow_tree_bestfirst(yabt_grower* g, const yabt_tree_args* a, void* stream) {
  int rc;
  if ((rc = yabt_grow_begin(g, a, stream))) return rc;
  if ((rc = yabt_grow_init(g, a, stream))) return rc;
  if ((rc = yabt_grow_bf_root_hist(g, a, stream))) return rc;
  if ((rc = yabt_grow_bf_scan(g, a, 0, stream))) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  if (g->level_wait && !g->host_state) {
    CUDA_TRY(cudaHostAlloc((void**)&g->host_state, sizeof(int) * 4 * LEVEL_SLOTS, cudaHostAllocDefault));
    for (auto& e : g->lvl_ev) CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  const int steps = std::max(1, g->p.max_leaves - 1);
  for (int k = 1; k <= steps; ++k) {
    if ((rc = yabt_grow_bf_split(g, a, k, stream))) return rc;
    if ((rc = yabt_grow_bf_scan(g, a, k, stream))) return rc;
    if (!g->level_wait) continue;
    const int slot = k % LEVEL_SLOTS;
    CUDA_TRY(cudaMemcpyAsync(g->host_state + 4 * slot, &g->b.st->level, 4 * sizeof(int), cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaEventRecord(g->lvl_ev[slot], s));
    if (k > LEVEL_LOOKAHEAD) {
      const int old = (k - LEVEL_LOOKAHEAD) % LEVEL_SLOTS;
      CUDA_TRY(cudaEventSynchronize(g->lvl_ev[old]));
      if (!g->host_state[4 * old + 1]) break;     // active == 0: later steps would be no-ops
    }
  }
  return yabt_grow_end(g, a, stream);
}

}  // extern "C"

// multi-task workspace: small-child channels, per-slot histograms, records, zeros
static long long mt_carve(const yabt_grower* g, int T, char* base, MtBufs* mb) {
  const GrowParams& p = g->p;
  const int P = (T + 1) / 2;
  const long long FB = (long long)p.F * YABT_NB;
  long long o = 0;
  auto take = [&](long long bytes) { const long long at = o; o += al(bytes); return base ? base + at : nullptr; };
  char* small = take((2LL * P * FB + (long long)p.F * (YABT_NB / 2)) * 8);
  char* hist = take((long long)p.maxa * (T + 1) * FB * 8);
  char* feat = take(2LL * p.F * sizeof(MtRec));
  char* cand = take((long long)p.maxn * sizeof(MtRec));
  char* zeros = take(p.n * 4);
  if (mb) {
    mb->T = T; mb->P = P;
    mb->small = (long long*)small; mb->hist = (long long*)hist;
    mb->feat = (MtRec*)feat; mb->cand = (MtRec*)cand; mb->zeros = (const float*)zeros;
  }
  return o;
}

// the histogram of this level's smaller child for every task: ceil(T/2) passes
// of the two-channel kernel into the channel pairs of mb.small
static cudaError_t mt_hist_passes(yabt_grower* g, const TreeIO& io, const MtBufs& mb, int level, cudaStream_t s) {
  const long long FB = (long long)g->p.F * YABT_NB;
  for (int i = 0; i < mb.P; ++i) {
    if (i > 0) {
      const cudaError_t e = cudaMemsetAsync(&g->b.st->item_counter, 0, sizeof(int), s);
      if (e != cudaSuccess) return e;
    }
    GrowBufs b = g->b;
    b.small = mb.small + 2LL * i * FB;
    TreeIO io2 = io;
    io2.g = mb.grads + 2LL * i * g->p.n;
    io2.h = 2 * i + 1 < mb.T ? mb.grads + (2LL * i + 1) * g->p.n : mb.zeros;
    const cudaError_t e = launch_hist_kernels(g->p, b, io2, level, 1, g->nsm, s, nullptr, 0);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

extern "C" {

long long yabt_mt_workspace_bytes(const yabt_grower* g, int tasks) {
  if (!g || tasks < 1 || tasks > MT_MAX) return -1;
  return mt_carve(g, tasks, nullptr, nullptr);
}

int yabt_grow_tree_multitask(yabt_grower* g, const yabt_tree_args* a, int tasks, const float* grads, void* ws,
                             long long ws_bytes, float* values, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  if (!g->p.general || tasks < 1 || tasks > MT_MAX || !grads || !ws || !values || ((uintptr_t)ws & 255)) {
    set_error("yabt_grow_tree_multitask: needs a grower created with general=1, 1 <= tasks <= %d, "
              "gradients, values and a 256-byte aligned workspace", MT_MAX);
    return YABT_ERR_ARG;
  }
  if (ws_bytes < yabt_mt_workspace_bytes(g, tasks)) { set_error("yabt_grow_tree_multitask: workspace too small"); return YABT_ERR_WORKSPACE; }
  if (g->p.bf_f64) { set_error("yabt_grow_tree_multitask: the float64 best-first mode does not apply"); return YABT_ERR_ARG; }
  MtBufs mb;
  mt_carve(g, tasks, static_cast<char*>(ws), &mb);
  mb.grads = grads; mb.values = values; mb.scratch_value = nullptr;
  cudaStream_t s = (cudaStream_t)stream;
  const GrowParams& p = g->p;
  if (tasks % 2) CUDA_TRY(cudaMemsetAsync((void*)mb.zeros, 0, p.n * 4, s));
  std::vector<const float*> arrays(tasks);
  for (int t = 0; t < tasks; ++t) arrays[t] = grads + (long long)t * p.n;
  CUDA_TRY(launch_absmax_shared(arrays.data(), tasks, io.n_root, io.root_rows, g->b.st, g->nsm, s));
  CUDA_TRY(launch_tree_init(p, g->b, io, s));
  CUDA_TRY(mt_hist_passes(g, io, mb, 0, s));
  CUDA_TRY(launch_mt_scan(p, g->b, mb, io, 1, g->nsm, s));
  if (g->level_wait && !g->host_state) {
    CUDA_TRY(cudaHostAlloc((void**)&g->host_state, sizeof(int) * 4 * LEVEL_SLOTS, cudaHostAllocDefault));
    for (auto& e : g->lvl_ev) CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  const int steps = std::max(1, p.max_leaves - 1);
  for (int k = 1; k <= steps; ++k) {
    CUDA_TRY(launch_mt_commit(p, g->b, mb, s));
    CUDA_TRY(launch_bf_pick_partition(p, g->b, io, k, g->nsm, s));
    CUDA_TRY(launch_mt_values(p, g->b, mb, s));
    CUDA_TRY(mt_hist_passes(g, io, mb, 1, s));
    CUDA_TRY(launch_mt_scan(p, g->b, mb, io, 0, g->nsm, s));
    if (!g->level_wait) continue;
    const int slot = k % LEVEL_SLOTS;
    CUDA_TRY(cudaMemcpyAsync(g->host_state + 4 * slot, &g->b.st->level, 4 * sizeof(int), cudaMemcpyDeviceToHost, s));
    CUDA_TRY(cudaEventRecord(g->lvl_ev[slot], s));
    if (k > LEVEL_LOOKAHEAD) {
      const int old = (k - LEVEL_LOOKAHEAD) % LEVEL_SLOTS;
      CUDA_TRY(cudaEventSynchronize(g->lvl_ev[old]));
      if (!g->host_state[4 * old + 1]) break;
    }
  }
  CUDA_TRY(launch_tree_finish(p, g->b, io, a->meta, a->leaf_of_row, g->nsm, s));
  return YABT_OK;
}

int yabt_mt_update(const int32_t* leaf_of_row, const float* values, int tasks, long long n, float* margin,
                   const float* y, float* grad, void* stream) {
  if (n == 0 && tasks >= 1) return YABT_OK;   // no rows: nothing is read (buffers may be NULL)
  if (tasks < 1 || n < 0 || !margin || (values && !leaf_of_row) || (grad && !y)) {
    set_error("yabt_mt_update: bad arguments");
    return YABT_ERR_ARG;
  }
  int dev = 0, nsm = 0;
  CUDA_TRY(cudaGetDevice(&dev));
  CUDA_TRY(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  CUDA_TRY(launch_mt_update(leaf_of_row, values, tasks, n, margin, y, grad, nsm, (cudaStream_t)stream));
  return YABT_OK;
}

void* yabt_grow_amax_ptr(yabt_grower* g) { return g && g->bound ? (void*)&g->b.st->amax_g : nullptr; }
void* yabt_grow_small_ptr(yabt_grower* g) { return g && g->bound ? (void*)g->b.small : nullptr; }
void* yabt_grow_level_ptr(yabt_grower* g) { return g && g->bound ? (void*)&g->b.st->level : nullptr; }

int yabt_grow_apply_all(yabt_grower* g, const yabt_tree_args* a, void* stream) {
  TreeIO io;
  int rc = fill_io(g, a, &io);
  if (rc) return rc;
  if (!io.bins_fm) { set_error("yabt_grow_apply_all: needs the feature-major bins (bins_fm)"); return YABT_ERR_ARG; }
  CUDA_TRY(launch_apply_all(g->p, g->b, io, g->nsm, (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_grower_set_root_count_cache(yabt_grower* g, int on) {
  if (!g) { set_error("null grower"); return YABT_ERR_ARG; }
  g->rc_mode = on ? 1 : 0;
  g->rc_valid = 0;
  return YABT_OK;
}

int yabt_grower_root_counts(yabt_grower* g, int64_t* out, void* stream) {
  if (!g || !g->bound || !out) { set_error("yabt_grower_root_counts: needs a bound grower and an output"); return YABT_ERR_ARG; }
  if (!g->rc_mode || !g->rc_valid) {
    set_error("yabt_grower_root_counts: no root counts recorded (cache off, or no root histogram over all rows yet)");
    return YABT_ERR_ARG;
  }
  CUDA_TRY(launch_unpack_counts(g->p, g->b, reinterpret_cast<long long*>(out), (cudaStream_t)stream));
  return YABT_OK;
}

int yabt_grower_set_bestfirst_f64(yabt_grower* g, int on) {
  if (!g) { set_error("null grower"); return YABT_ERR_ARG; }
  g->p.bf_f64 = on ? 1 : 0;
  return YABT_OK;
}

int yabt_grower_set_level_wait(yabt_grower* g, int wait) {
  if (!g) { set_error("null grower"); return YABT_ERR_ARG; }
  g->level_wait = wait ? 1 : 0;
  return YABT_OK;
}

int yabt_grower_set_level_loop(yabt_grower* g, int on) {
  if (!g) { set_error("null grower"); return YABT_ERR_ARG; }
  g->level_loop = on ? 1 : 0;
  return YABT_OK;
}

int yabt_grower_level_loop_start(const yabt_grower* g) { return g ? level_loop_first(g) : -1; }

int yabt_grower_set_small(yabt_grower* g, void* ptr, long long bytes) {
  if (!g || !g->bound || !ptr || ((uintptr_t)ptr & 255)) {
    set_error("yabt_grower_set_small: needs a bound grower and a 256-byte aligned buffer");
    return YABT_ERR_ARG;
  }
  const long long need = (long long)g->p.max_pairs * small_job_words(g->p.C, g->p.F) * 8;
  if (bytes < need) { set_error("yabt_grower_set_small: %lld bytes, %lld needed", bytes, need); return YABT_ERR_ARG; }
  g->b.small = static_cast<long long*>(ptr);
  return YABT_OK;
}

long long yabt_grow_small_count(const yabt_grower* g, int level) {
  if (!g) return -1;
  long long jobs = level == 0 ? 1 : std::min<long long>(1LL << std::min(level - 1, 30), g->p.max_pairs);
  return jobs * small_job_words(g->p.C, g->p.F);
}

int yabt_grow_leaf_rows(yabt_grower* g, void** src, void** begin, void** count, void** fin,
                        void** list0, void** list1) {
  if (!g || !g->bound) { set_error("grower not bound"); return YABT_ERR_ARG; }
  if (src) *src = g->b.leaf_src;
  if (begin) *begin = g->b.leaf_begin;
  if (count) *count = g->b.leaf_count;
  if (fin) *fin = g->b.fin;
  if (list0) *list0 = g->b.rows[0];
  if (list1) *list1 = g->b.rows[1];
  return YABT_OK;
}

}  // extern "C"
