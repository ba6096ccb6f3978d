// Level-wise tree growth on the device: split scan, level finalisation (split
// choice, leaf budget, node ids), stable row partition and next-level planning.
//
// Restates yabt/tree.py:362-625 (grow_tree_levelwise). Per level the host
// launches a fixed sequence
//     k_hist -> k_reduce -> [all-reduce hook] -> k_scan -> k_finalize -> k_partition -> k_plan
// and every kernel reads what it has to do from the device-resident
// GrowState, so a whole tree needs no host synchronisation.
//
// Floating-point semantics of the split scan match the reference CPU
// execution: left sums are the float32 rounding of exact prefix sums (the
// reference accumulates cumsum in float64, yabt/tree.py:504), and the gain,
// validity, boost and leaf values use float32 operations in the reference's
// operand order with round-to-nearest intrinsics (no FMA contraction).
#include "grow.cuh"

namespace yabt {

cudaError_t launch_hist_kernels(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int d,
                                int jobs, int nsm, cudaStream_t s, cudaEvent_t after_hist, int root_counts);

__device__ __forceinline__ int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

// Exclusive prefix sum of n ints by one warp (all 32 lanes must call it).
// `in` and `out` may alias. Returns the total.
__device__ int warp_excl_scan(const int* in, int* out, int n) {
  const int lane = threadIdx.x & 31;
  int carry = 0;
  for (int base = 0; base < n; base += 32) {
    const int v = base + lane < n ? in[base + lane] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (base + lane < n) out[base + lane] = carry + x - v;
    carry += __shfl_sync(0xffffffffu, x, 31);
  }
  return carry;
}

// ------------------------------------------------------------------ per-tree setup
__global__ void k_absmax(const float* __restrict__ g, const float* __restrict__ h, long long n,
                         const int* __restrict__ root, GrowState* st) {
  pdl_wait();
  unsigned mg = 0, mh = 0;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = root ? root[i] : i;
    // bit patterns of non-negative floats order like the values, as signed and
    // as unsigned 32-bit integers (so ranks can combine them with an int max)
    mg = max(mg, __float_as_uint(fabsf(g[r])));
    if (h) mh = max(mh, __float_as_uint(fabsf(h[r])));
  }
  for (int o = 16; o; o >>= 1) {
    mg = max(mg, __shfl_xor_sync(0xffffffffu, mg, o));
    mh = max(mh, __shfl_xor_sync(0xffffffffu, mh, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMax(&st->amax_g, mg);
    if (h) atomicMax(&st->amax_h, mh);
  }
}

__device__ void quant_scale(unsigned amax_bits, int* qe, float* scale, float* inv) {
  float a = __uint_as_float(amax_bits);
  int e = exp_bound(a);
  int q = 30 - e;
  q = max(-100, min(q, 100));
  *qe = q;
  *scale = ldexpf(1.f, q);
  *inv = ldexpf(1.f, -q);
}

// chunk size (rows per histogram item) for R rows spread over U units
__device__ __forceinline__ int item_chunk(long long R, int U) {
  long long c = (R * U + ITEM_TARGET - 1) / ITEM_TARGET;
  c = max((long long)CHUNK_MIN, min((long long)CHUNK_MAX, c));
  return (int)c;
}

__global__ void k_tree_init(GrowParams p, GrowBufs b, TreeIO io) {
  pdl_wait();
  pdl_trigger();
  GrowState* st = b.st;
  for (int m = threadIdx.x; m < p.maxa; m += blockDim.x) b.node_key[m] = 0ULL;
  if (threadIdx.x == 0) {
    *b.io_dev = io;                    // the tree's inputs for launches of a device-side level loop
    st->level = 0; st->active = 1; st->M = 1; st->P = 0; st->n_nodes = 1; st->n_rows = p.n;
    st->remaining = p.max_leaves - 1; st->part_level = -1; st->plan_level = -1;
    st->depth_max = 0; st->n_leaves = 0; st->err = 0; st->tile_counter = 0; st->n_tiles = 0;
    quant_scale(st->amax_g, &st->qe_g, &st->gscale, &st->ginv);
    if (p.general) quant_scale(st->amax_h, &st->qe_h, &st->hscale, &st->hinv);
    else { st->qe_h = 0; st->hscale = 1.f; st->hinv = 1.f; }
    b.act_gid[0][0] = 0; b.seg_begin[0][0] = 0; b.seg_count[0][0] = (int)io.n_root;
    io.feature[0] = -1; io.threshold[0] = 0.f; io.left[0] = -1; io.right[0] = -1;
    io.value[0] = 0.f; io.gate[0] = 1.f; b.node_depth[0] = 0; b.node_bin[0] = -1;
    // root histogram items: the root rows (positions into io.root_rows, or rows)
    const int chunk = item_chunk(io.n_root, p.U);
    const int nch = (int)((io.n_root + chunk - 1) / chunk);
    int slot = 0;
    for (int u = 0; u < p.U; ++u) {
      b.job_first[u] = slot;
      b.job_nitems[u] = nch;
      slot += nch;
    }
    if (slot > p.max_items) { atomicOr(&st->err, DERR_ITEM_OVERFLOW); slot = 0; }
    st->n_items = slot; st->item_counter = 0;
    for (int l = 0; l < 64; ++l) st->hist_rows[l] = 0;
    st->hist_rows[0] = io.n_root;
    st->acc_root_rows += io.n_root;
    st->acc_launches += 1;
  }
  __syncthreads();
  const int chunk = item_chunk(io.n_root, p.U);
  const int nch = (int)((io.n_root + chunk - 1) / chunk);
  if (nch * p.U <= p.max_items) {
    for (int i = threadIdx.x; i < nch * p.U; i += blockDim.x) {
      const int u = i / nch, c = i % nch;
      HistItem it;
      it.begin = c * chunk;
      it.count = (int)min((long long)chunk, io.n_root - (long long)c * chunk);
      it.unit = u; it.job = 0; it.slot = i;
      it.used = 0; it.pad[0] = it.pad[1] = 0;
      b.items[i] = it;
    }
  }
  for (int f = threadIdx.x; f < p.F; f += blockDim.x) b.pathmax[0][f] = 0.f;
}

// ------------------------------------------------------------------ split scan
// grid: jobs x ceil(F / SCAN_WARPS); one warp per feature, lane L owns bins 8L..8L+7.
// The unit-hessian form is held to 3 resident blocks per SM (at most 80
// registers; 89 otherwise, 2 blocks): the kernel waits on its histogram loads,
// and the extra warps cut its time per tree by 8-9% (C4, 10M and 1.25M rows).
template <int C>
__global__ void __launch_bounds__(SCAN_WARPS * 32, C == 2 ? 3 : 2)
k_scan(GrowParams p, GrowBufs b, TreeIO io, int level_gate) {
  pdl_wait();
  GrowState* st = b.st;
  if (level_gate == LEVEL_DYN) {
    if ((level_gate = st->level) < 1) return;
    io = *b.io_dev;
  }
  if (st->level != level_gate || !st->active) return;
  const int d = level_gate;
  const int njobs = d == 0 ? 1 : st->P;
  const int fblocks = (p.f_hi - p.f_lo + SCAN_WARPS - 1) / SCAN_WARPS;
  const int job = blockIdx.x / fblocks;
  if (job >= njobs) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int f = p.f_lo + (blockIdx.x % fblocks) * SCAN_WARPS + warp;
  if (f >= p.f_hi) return;
  const int cur = d & 1, prv = cur ^ 1;
  const bool write_hist = d + 1 < p.levels_max;
  const float ginv = st->ginv, hinv = st->hinv;
  const float lam = p.lam, gam = p.gamma, mcw = p.mcw, fmsl = (float)p.msl;
  const bool fok = !(p.use_fmask && io.fmask && !io.fmask[f]);
  const size_t FB = (size_t)p.F * YABT_NB;
  const size_t HN = (size_t)C * FB;           // int64 per node histogram
  const long long* sjob = b.small + (size_t)job * small_job_words(C, p.F);
  const long long* sm = sjob + (size_t)f * YABT_NB + lane * 8;
  const long long* scnt = sjob + (size_t)(C - 1) * FB + (size_t)f * (YABT_NB / 2) + lane * 4;

  int nchild, pos_small, pos_other = -1;
  const long long* par = nullptr;
  // interaction steering: max over the node's path features p of imat[p][f];
  // both children of a pair share it: max(parent's, imat[parent's split feature][f])
  float pm = 0.f;
  if (d == 0) {
    nchild = 1; pos_small = 0;
    if (p.use_imat) pm = b.pathmax[0][f];
  } else {
    nchild = 2;
    const int sil = b.pair_sil[job];
    pos_small = sil ? 2 * job : 2 * job + 1;
    pos_other = sil ? 2 * job + 1 : 2 * job;
    const int m = b.pair_pos[job];
    par = b.hist[prv] + (size_t)m * HN + (size_t)f * YABT_NB + lane * 8;
    if (p.use_imat) {
      pm = fmaxf(b.pathmax[prv][(size_t)m * p.F + f], io.imat[(size_t)b.split_f[m] * p.F + f]);
      if (lane == 0) {     // the children's own path max, read by their children's scan
        b.pathmax[cur][(size_t)(2 * job) * p.F + f] = pm;
        b.pathmax[cur][(size_t)(2 * job + 1) * p.F + f] = pm;
      }
    }
  }
  long long vs[C][8];
#pragma unroll
  for (int c = 0; c < C - 1; ++c) {
    const longlong2* q = reinterpret_cast<const longlong2*>(sm + c * FB);
#pragma unroll
    for (int i = 0; i < 4; ++i) { longlong2 t = q[i]; vs[c][2 * i] = t.x; vs[c][2 * i + 1] = t.y; }
  }
  {
    const longlong2* q = reinterpret_cast<const longlong2*>(scnt);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const longlong2 t = q[i];
      vs[C - 1][4 * i + 0] = (long long)((unsigned long long)t.x & 0xffffffffULL);
      vs[C - 1][4 * i + 1] = (long long)((unsigned long long)t.x >> 32);
      vs[C - 1][4 * i + 2] = (long long)((unsigned long long)t.y & 0xffffffffULL);
      vs[C - 1][4 * i + 3] = (long long)((unsigned long long)t.y >> 32);
    }
  }
  for (int ch = 0; ch < nchild; ++ch) {
    long long v[C][8];
    const int pos = ch == 0 ? pos_small : pos_other;
    if (ch == 0) {
#pragma unroll
      for (int c = 0; c < C; ++c)
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] = vs[c][i];
    } else {
#pragma unroll
      for (int c = 0; c < C; ++c) {
        const longlong2* q = reinterpret_cast<const longlong2*>(par + c * FB);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          longlong2 t = q[i];
          v[c][2 * i] = t.x - vs[c][2 * i];
          v[c][2 * i + 1] = t.y - vs[c][2 * i + 1];
        }
      }
    }
    if (write_hist) {
      long long* dst = b.hist[cur] + (size_t)pos * HN + (size_t)f * YABT_NB + lane * 8;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        longlong2* q = reinterpret_cast<longlong2*>(dst + c * FB);
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = make_longlong2(v[c][2 * i], v[c][2 * i + 1]);
      }
    }
    // inclusive prefix inside the lane, then exclusive scan of lane totals
    long long lt[C];
#pragma unroll
    for (int c = 0; c < C; ++c) {
#pragma unroll
      for (int i = 1; i < 8; ++i) v[c][i] += v[c][i - 1];
      long long x = v[c][7];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        long long y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      long long total = __shfl_sync(0xffffffffu, x, 31);
      long long excl = x - v[c][7];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] += excl;
      lt[c] = total;
    }
    const float G = __fmul_rn(__ll2float_rn(lt[0]), ginv);
    const float H = (C == 3) ? __fmul_rn(__ll2float_rn(lt[1]), hinv) : __ll2float_rn(lt[C - 1]);
    const float Cn = __ll2float_rn(lt[C - 1]);
    const float t3 = __fdiv_rn(__fmul_rn(G, G), __fadd_rn(H, lam));
    float boost = 1.f;
    if (p.use_imat) boost = __fadd_rn(1.f, __fmul_rn(p.ib, pm));
    float bsel = -INFINITY, bgain = -INFINITY, bGL = 0.f, bHL = 0.f, bCL = 0.f;
    int bbin = 0;
    long long bcl = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int bin = lane * 8 + i;
      const float GL = __fmul_rn(__ll2float_rn(v[0][i]), ginv);
      const float CL = __ll2float_rn(v[C - 1][i]);
      const float HL = (C == 3) ? __fmul_rn(__ll2float_rn(v[1][i]), hinv) : CL;
      const float GR = __fsub_rn(G, GL), HR = __fsub_rn(H, HL), CR = __fsub_rn(Cn, CL);
      const float t1 = __fdiv_rn(__fmul_rn(GL, GL), __fadd_rn(HL, lam));
      const float t2 = __fdiv_rn(__fmul_rn(GR, GR), __fadd_rn(HR, lam));
      float gain = __fsub_rn(__fmul_rn(0.5f, __fsub_rn(__fadd_rn(t1, t2), t3)), gam);
      const bool valid = fok && bin != YABT_NB - 1 && CL >= fmsl && CR >= fmsl && HL >= mcw && HR >= mcw;
      if (!valid) gain = -INFINITY;
      const float sel = p.use_imat ? __fmul_rn(gain, boost) : gain;
      if (i == 0 || sel > bsel) {
        bsel = sel; bgain = gain; bGL = GL; bHL = HL; bCL = CL; bbin = bin; bcl = v[C - 1][i];
      }
    }
    // warp argmax: larger sel wins, ties -> lower bin
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float os = __shfl_xor_sync(0xffffffffu, bsel, o);
      const int ob = __shfl_xor_sync(0xffffffffu, bbin, o);
      const float og = __shfl_xor_sync(0xffffffffu, bgain, o);
      const float oGL = __shfl_xor_sync(0xffffffffu, bGL, o);
      const float oHL = __shfl_xor_sync(0xffffffffu, bHL, o);
      const float oCL = __shfl_xor_sync(0xffffffffu, bCL, o);
      const long long ocl = __shfl_xor_sync(0xffffffffu, bcl, o);
      if (os > bsel || (os == bsel && ob < bbin)) {
        bsel = os; bbin = ob; bgain = og; bGL = oGL; bHL = oHL; bCL = oCL; bcl = ocl;
      }
    }
    if (lane == 0) {
      NodeBest nb;
      nb.sel = bsel; nb.gain = bgain; nb.GL = bGL; nb.HL = bHL; nb.CL = bCL; nb.bin = bbin; nb.cl = bcl;
      b.best[(size_t)pos * p.F + f] = nb;
      // node argmax over features: larger sel, ties -> lower feature
      atomicMax(&b.node_key[pos], ((unsigned long long)f2ord(bsel) << 32) | (0xffffffffu - (unsigned)f));
      if (f == p.f_lo) {      // every feature's bins sum to the node total; the slice's first one records it
        NodeTot t; t.G = G; t.H = H; t.C = Cn; t.pad = 0; t.c = lt[C - 1];
        b.tot[pos] = t;
      }
    }
  }
}

// ------------------------------------------------------------------ finalize
// One block. Picks each node's split (first max over features), applies the
// leaf budget (highest gains, ties -> lower position), numbers the children
// (ascending position, left then right), writes the tree arrays and plans the
// partition of this level.
__global__ void __launch_bounds__(1024)
k_finalize(GrowParams p, GrowBufs b, TreeIO io, int level_gate) {
  pdl_wait();
  pdl_trigger();
  GrowState* st = b.st;
  if (level_gate == LEVEL_DYN) {
    if ((level_gate = st->level) < 1) return;
    io = *b.io_dev;
  }
  if (st->level != level_gate || !st->active) return;
  const int d = level_gate, cur = d & 1, nxt = cur ^ 1;
  const int M = st->M;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ int s_P, s_ntiles, s_remaining, s_nnodes;
  // per-node gains and tile prefixes staged in shared memory (the rank loop and
  // the tile search read them many times); larger levels read global memory
  __shared__ float s_gain[FIN_SMEM_NODES];
  __shared__ int s_tpre[FIN_SMEM_NODES + 1];
  const bool staged = M <= FIN_SMEM_NODES;
  // A: per node argmax over features (k_scan left the winner in node_key)
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    const int bf = (int)(0xffffffffu - (unsigned)(b.node_key[m] & 0xffffffffULL));
    const NodeBest nb = b.best[(size_t)m * p.F + bf];
    b.nbest[m] = nb;
    b.split_f[m] = bf;
    b.split_b[m] = nb.bin;
    if (staged) s_gain[m] = nb.gain;
  }
  __syncthreads();
  // the next level's scan accumulates into node_key again
  for (int m = threadIdx.x; m < p.maxa; m += blockDim.x) b.node_key[m] = 0ULL;
  const bool loop_ok = d < p.max_depth && st->remaining > 0;
  const int remaining = st->remaining;
  // B: budget rank (parallel) -> split_pair = 1 tentatively
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    const float gm = staged ? s_gain[m] : b.nbest[m].gain;
    int keep = loop_ok && gm > 0.f;
    if (keep) {
      int rank = 0;
      for (int q = 0; q < M; ++q) {
        const float gq = staged ? s_gain[q] : b.nbest[q].gain;
        if (gq > 0.f && (gq > gm || (gq == gm && q < m))) ++rank;
      }
      keep = rank < remaining;
    }
    b.split_pair[m] = keep ? 1 : -1;
  }
  __syncthreads();
  if (warp == 0) {
    // split_pair holds 1 (keep) / -1; number the kept nodes in ascending position
    int P = 0;
    for (int base = 0; base < M; base += 32) {
      const int m = base + lane;
      const bool k = m < M && b.split_pair[m] > 0;
      const unsigned bal = __ballot_sync(0xffffffffu, k);
      if (m < M) {
        if (k) { const int q = P + __popc(bal & ((1u << lane) - 1u)); b.split_pair[m] = q; b.pair_pos[q] = m; }
        else b.split_pair[m] = -1;
      }
      P += __popc(bal);
    }
    if (lane == 0) {
      s_P = P;
      s_nnodes = st->n_nodes;
      s_remaining = remaining - P;
      if (s_nnodes + 2 * P > p.maxn) atomicOr(&st->err, DERR_NODE_OVERFLOW);
    }
  }
  __syncthreads();
  const int P = s_P, n0 = s_nnodes;
  const float lr = p.lr, lam = p.lam;
  // C: tree arrays, pairs, children, leaf ranges of stopping nodes
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    const int gid = b.act_gid[cur][m];
    const int pr = b.split_pair[m];
    const NodeTot t = b.tot[m];
    if (d == 0) {
      // root value, yabt/tree.py:473 (double arithmetic on the float32 sums)
      io.value[0] = pr >= 0 ? 0.f : (float)(-(double)lr * (double)t.G / ((double)t.H + (double)lam));
    }
    if (pr < 0) {
      b.leaf_src[gid] = SRC_FIN;
      b.leaf_begin[gid] = b.seg_begin[cur][m];
      b.leaf_count[gid] = b.seg_count[cur][m];
      continue;
    }
    const NodeBest nb = b.nbest[m];
    const int f = b.split_f[m], bin = nb.bin;
    const int ne = io.edge_cnt[f];
    io.feature[gid] = f;
    io.threshold[gid] = io.edges[io.edge_off[f] + min(bin, ne - 1)];
    io.gate[gid] = fmaxf(io.scales[f], 1e-12f);
    io.value[gid] = 0.f;
    b.node_bin[gid] = bin;
    const int nl = n0 + 2 * pr, nr = nl + 1;
    io.left[gid] = nl; io.right[gid] = nr;
    const float nlr = -lr;
    const float vL = __fdiv_rn(__fmul_rn(nlr, nb.GL), __fadd_rn(nb.HL, lam));
    const float vR = __fdiv_rn(__fmul_rn(nlr, __fsub_rn(t.G, nb.GL)), __fadd_rn(__fsub_rn(t.H, nb.HL), lam));
    io.feature[nl] = -1; io.threshold[nl] = 0.f; io.left[nl] = -1; io.right[nl] = -1;
    io.value[nl] = vL; io.gate[nl] = 1.f; b.node_depth[nl] = d + 1; b.node_bin[nl] = -1;
    io.feature[nr] = -1; io.threshold[nr] = 0.f; io.left[nr] = -1; io.right[nr] = -1;
    io.value[nr] = vR; io.gate[nr] = 1.f; b.node_depth[nr] = d + 1; b.node_bin[nr] = -1;
    b.pair_sil[pr] = nb.cl <= t.c - nb.cl;   // smaller child by (global) row count
    b.act_gid[nxt][2 * pr] = nl;
    b.act_gid[nxt][2 * pr + 1] = nr;
    // child segments: inherit the parent's region; the partition fills in the split point
    const int B = b.seg_begin[cur][m], cnt = b.seg_count[cur][m];
    b.seg_begin[nxt][2 * pr] = B; b.seg_count[nxt][2 * pr] = 0;
    b.seg_begin[nxt][2 * pr + 1] = B; b.seg_count[nxt][2 * pr + 1] = cnt;
  }
  // (the children's interaction path max is formed by the next level's scan)
  // D: partition tiles over every active node's rows (stopping nodes move to fin)
  int* tpre = staged ? s_tpre : b.node_tpre;
  for (int m = threadIdx.x; m < M; m += blockDim.x)
    tpre[m] = P > 0 ? (b.seg_count[cur][m] + PART_TILE - 1) / PART_TILE : 0;
  __syncthreads();
  if (warp == 0) {
    const int nt = warp_excl_scan(tpre, tpre, M);
    if (lane == 0) { tpre[M] = nt; s_ntiles = nt <= p.max_tiles ? nt : 0; }
    if (lane == 0 && nt > p.max_tiles) atomicOr(&st->err, DERR_TILE_OVERFLOW);
  }
  __syncthreads();
  const int ntl = s_ntiles;
  for (int e = threadIdx.x; e < ntl; e += blockDim.x) {
    int lo = 0, hi = M - 1;            // last node with tpre <= e
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tpre[mid] <= e) lo = mid; else hi = mid - 1;
    }
    const int m = lo, q = e - tpre[m];
    const int k = tpre[m + 1] - tpre[m];
    const int B = b.seg_begin[cur][m], cnt = b.seg_count[cur][m];
    PartTile t;
    t.pos = m; t.begin = B + q * PART_TILE; t.end = min(B + cnt, t.begin + PART_TILE);
    t.last = q == k - 1; t.t_in_node = q;
    t.pad[0] = t.pad[1] = t.pad[2] = 0;
    b.tiles[e] = t;
  }
  if (P == 0) {
    // nothing splits: every active node is a final leaf and keeps its rows in place
    const int src = d == 0 ? SRC_IDENTITY : (cur == 0 ? SRC_LIST0 : SRC_LIST1);
    for (int m = threadIdx.x; m < M; m += blockDim.x) b.leaf_src[b.act_gid[cur][m]] = src;
  }
  if (threadIdx.x == 0) {
    const int nt = ntl;
    st->n_tiles = nt; st->tile_counter = 0;
    st->epoch = st->epoch + 1;
    st->part_level = P > 0 ? d : -1;
    st->plan_level = P > 0 ? d : -1;
    st->P = P;
    st->n_nodes = n0 + 2 * P;
    st->remaining = s_remaining;
    st->M = 2 * P;
    st->level = d + 1;
    st->active = (P > 0 && d + 1 < p.max_depth && s_remaining > 0) ? 1 : 0;
    if (P > 0) st->depth_max = max(st->depth_max, d + 1);
  }
}

// ------------------------------------------------------------------ partition
// Stable partition of each splitting node's rows: left rows ascending from the
// region start, right rows descending from the region end, with a decoupled
// look-back over the node's tiles for the running left count. Rows of nodes
// that stop are copied to `fin` at the same offsets.
__device__ __forceinline__ unsigned long long lb_word(unsigned epoch, unsigned flag, unsigned v) {
  return ((unsigned long long)(epoch & 0x3fffffffu) << 34) | ((unsigned long long)flag << 32) | v;
}

__global__ void __launch_bounds__(PART_THREADS)
k_partition(GrowParams p, GrowBufs b, TreeIO io, int level_gate) {
  pdl_wait();
  GrowState* st = b.st;
  if (level_gate == LEVEL_DYN) {
    if ((level_gate = st->part_level) < 1) return;
    io = *b.io_dev;
  }
  if (st->part_level != level_gate) return;
  const int d = level_gate, cur = d & 1, nxt = cur ^ 1;
  const int ntiles = st->n_tiles;
  const unsigned epoch = st->epoch;
  const int* src = d == 0 ? io.root_rows : b.rows[cur];   // nullptr: identity
  int* dst = b.rows[nxt];
  __shared__ int s_tile, s_excl;
  __shared__ int s_wc[PART_RPT][PART_THREADS / 32];
  __shared__ int s_wpre[PART_RPT][PART_THREADS / 32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  constexpr int NW = PART_THREADS / 32;
  for (;;) {
    if (t == 0) s_tile = atomicAdd(&st->tile_counter, 1);
    __syncthreads();
    const int tile = s_tile;
    if (tile >= ntiles) break;
    const PartTile T = b.tiles[tile];
    const int m = T.pos;
    const int B = b.seg_begin[cur][m], cnt = b.seg_count[cur][m];
    const int pr = b.split_pair[m];
    int row[PART_RPT];
    bool ok[PART_RPT];
#pragma unroll
    for (int i = 0; i < PART_RPT; ++i) {
      const int idx = T.begin + i * PART_THREADS + t;
      ok[i] = idx < T.end;
      row[i] = ok[i] ? (src ? src[idx] : idx) : 0;
      if (YABT_BOUNDS_CHECKED && ok[i] && (row[i] < 0 || row[i] >= p.n)) {
        atomicOr(&st->err, DERR_BOUNDS);
        ok[i] = false;
        row[i] = 0;
      }
    }
    if (pr < 0) {
#pragma unroll
      for (int i = 0; i < PART_RPT; ++i) {
        if (!ok[i]) continue;
        const int idx = T.begin + i * PART_THREADS + t;
        b.fin[idx] = row[i];
      }
      __syncthreads();
      continue;
    }
    const int f = b.split_f[m];
    const unsigned thr = (unsigned)b.split_b[m];
    // the row's bin of the split feature: one byte of the feature-major copy,
    // else a byte of the row's slab in the tiled matrix
    const FeatAddr fa = b.faddr[f];
    const uint8_t* col = io.bins_fm ? io.bins_fm + (size_t)f * p.n : io.bins + fa.off + fa.pos;
    const size_t stride = io.bins_fm ? 1 : (size_t)fa.width;
    bool lf[PART_RPT];
    unsigned bal[PART_RPT];
#pragma unroll
    for (int i = 0; i < PART_RPT; ++i) {
      lf[i] = ok[i] && (unsigned)__ldg(col + (size_t)row[i] * stride) <= thr;
      bal[i] = __ballot_sync(0xffffffffu, lf[i]);
      if (lane == 0) s_wc[i][warp] = __popc(bal[i]);
    }
    __syncthreads();
    // warp 0: tile total, then a warp-wide decoupled look-back over up to 32
    // predecessor tiles of the same node per step
    if (warp == 0) {
      int run = 0;
      if (t == 0) {
        for (int i = 0; i < PART_RPT; ++i)
          for (int w = 0; w < NW; ++w) { s_wpre[i][w] = run; run += s_wc[i][w]; }
      }
      const unsigned Lt = (unsigned)__shfl_sync(0xffffffffu, run, 0);
      unsigned long long* stat = b.tile_status;
      const unsigned ep = epoch & 0x3fffffffu;
      unsigned excl = 0;
      if (T.t_in_node == 0) {
        if (lane == 0) atomicExch(&stat[tile], lb_word(epoch, 2u, Lt));
      } else {
        if (lane == 0) atomicExch(&stat[tile], lb_word(epoch, 1u, Lt));
        int base = tile - 1;                // window [base-31, base], lane j <-> tile base-j
        const int first = tile - T.t_in_node;
        long long spins = 0;
        for (;;) {
          const int j = base - lane;
          unsigned long long w = 0;
          unsigned wf = 2u;                 // tiles before the node's first count as "inclusive 0"
          unsigned wv = 0;
          if (j >= first) {
            w = *(volatile unsigned long long*)&stat[j];
            const bool cur = (unsigned)(w >> 34) == ep;
            wf = cur ? (unsigned)(w >> 32) & 3u : 0u;
            wv = (unsigned)(w & 0xffffffffu);
          }
          const unsigned notready = __ballot_sync(0xffffffffu, wf == 0u);
          const unsigned incl = __ballot_sync(0xffffffffu, wf == 2u);
          // lanes up to the first inclusive tile must all be ready
          const int stop = incl ? __ffs(incl) - 1 : 31;
          const unsigned need = stop >= 31 ? 0xffffffffu : ((1u << (stop + 1)) - 1u);
          if (notready & need) {
            if (++spins > (1LL << 22)) { if (lane == 0) atomicOr(&st->err, DERR_LOOKBACK_TIMEOUT); break; }
            continue;
          }
          unsigned v = (lane <= stop && j >= first) ? wv : 0u;
          for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          excl += v;
          if (incl) break;
          base -= 32;
        }
        if (lane == 0) atomicExch(&stat[tile], lb_word(epoch, 2u, excl + Lt));
      }
      if (lane == 0) {
        s_excl = (int)excl;
        if (T.last) {
          const int Ltot = (int)(excl + Lt);
          b.seg_begin[nxt][2 * pr] = B; b.seg_count[nxt][2 * pr] = Ltot;
          b.seg_begin[nxt][2 * pr + 1] = B + Ltot; b.seg_count[nxt][2 * pr + 1] = cnt - Ltot;
        }
      }
    }
    __syncthreads();
    const int excl = s_excl;
    const int off_in_node = T.begin - B;
    const unsigned lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int i = 0; i < PART_RPT; ++i) {
      if (!ok[i]) continue;
      const int rl = s_wpre[i][warp] + __popc(bal[i] & lt_mask);   // left rank in tile
      int pos;
      if (lf[i]) pos = B + excl + rl;
      else {
        const int rr = off_in_node - excl + (i * PART_THREADS + t - rl);
        pos = B + cnt - 1 - rr;
      }
      if (pos < B || pos >= B + cnt) { atomicOr(&st->err, DERR_SEGMENT_OVERFLOW); continue; }
      dst[pos] = row[i];
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ plan next level
// One block: histogram items for the smaller children (local row counts come
// from the partition), or the leaf ranges of the children when no level follows.
// Item slots of pair q, unit u: [U * pre_q + u * nch_q, + nch_q) where nch_q is
// the pair's chunk count and pre_q its exclusive prefix over pairs.
__global__ void __launch_bounds__(1024)
k_plan(GrowParams p, GrowBufs b, int level_gate) {
  pdl_wait();
  pdl_trigger();
  GrowState* st = b.st;
  if (level_gate == LEVEL_DYN && (level_gate = st->plan_level) < 1) return;
  if (st->plan_level != level_gate) return;
  const int d = level_gate, nxt = (d + 1) & 1;
  const int P = st->P;
  __shared__ int s_chunk, s_total;
  if (!st->active) {
    const int src = nxt == 0 ? SRC_LIST0 : SRC_LIST1;
    for (int q = threadIdx.x; q < 2 * P; q += blockDim.x) {
      const int gid = b.act_gid[nxt][q];
      b.leaf_src[gid] = src;
      b.leaf_begin[gid] = b.seg_begin[nxt][q];
      b.leaf_count[gid] = b.seg_count[nxt][q];
    }
    if (threadIdx.x == 0) { st->plan_level = -1; st->n_items = 0; }
    return;
  }
  // node_tpre[q] <- chunk count of pair q; job_nitems[q] <- its prefix
  if ((threadIdx.x >> 5) == 0) {
    const int lane = threadIdx.x & 31;
    long long R = 0;
    for (int q = lane; q < P; q += 32) R += b.seg_count[nxt][b.pair_sil[q] ? 2 * q : 2 * q + 1];
    for (int o = 16; o; o >>= 1) R += __shfl_xor_sync(0xffffffffu, R, o);
    const int chunk = item_chunk(R, p.U);
    if (lane == 0) {
      st->hist_rows[min(d + 1, 63)] = R;
      st->acc_child_rows += R;
      st->acc_launches += 1;
    }
    for (int q = lane; q < P; q += 32) {
      const int sc = b.seg_count[nxt][b.pair_sil[q] ? 2 * q : 2 * q + 1];
      b.node_tpre[q] = (sc + chunk - 1) / chunk;
    }
    __syncwarp();
    const int tot = warp_excl_scan(b.node_tpre, b.job_nitems, P);
    if (lane == 0) {
      const int slots = tot * p.U;
      const bool ok = slots <= p.max_items;
      if (!ok) atomicOr(&st->err, DERR_ITEM_OVERFLOW);
      s_chunk = chunk; s_total = ok ? slots : 0;
      st->n_items = ok ? slots : 0; st->item_counter = 0; st->plan_level = -1;
    }
  }
  __syncthreads();
  const int chunk = s_chunk;
  if (s_total == 0) return;
  if (P <= FIN_SMEM_NODES) {
    // pair tables staged in shared memory, then one thread per item slot: slot i
    // of pair q, unit u, chunk c is U * pre[q] + u * nch[q] + c
    __shared__ int s_pre[FIN_SMEM_NODES + 1], s_nch[FIN_SMEM_NODES], s_sb[FIN_SMEM_NODES], s_sc[FIN_SMEM_NODES];
    for (int q = threadIdx.x; q < P; q += blockDim.x) {
      const int sp = b.pair_sil[q] ? 2 * q : 2 * q + 1;
      s_pre[q] = b.job_nitems[q];
      s_nch[q] = b.node_tpre[q];
      s_sb[q] = b.seg_begin[nxt][sp];
      s_sc[q] = b.seg_count[nxt][sp];
    }
    if (threadIdx.x == 0) s_pre[P] = s_total / p.U;
    __syncthreads();
    for (int e = threadIdx.x; e < P * p.U; e += blockDim.x) {
      const int q = e / p.U, u = e % p.U;
      b.job_first[e] = p.U * s_pre[q] + u * s_nch[q];
      b.job_nitems[e] = s_nch[q];
    }
    for (int i = threadIdx.x; i < s_total; i += blockDim.x) {
      int lo = 0, hi = P - 1;                 // last pair with U * pre <= i
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.U * s_pre[mid] <= i) lo = mid; else hi = mid - 1;
      }
      const int q = lo, r = i - p.U * s_pre[q], nch = s_nch[q];
      const int u = r / nch, c = r - u * nch;
      HistItem it;
      it.begin = s_sb[q] + c * chunk;
      it.count = min(chunk, s_sc[q] - c * chunk);
      it.unit = u; it.job = q; it.slot = i;
      it.used = 0; it.pad[0] = it.pad[1] = 0;
      b.items[i] = it;
    }
    return;
  }
  // job tables (pair-major, unit-minor)
  for (int e = threadIdx.x; e < P * p.U; e += blockDim.x) {
    const int q = e / p.U, u = e % p.U;
    const int nch = b.node_tpre[q];
    b.job_first[e] = p.U * b.job_nitems[q] + u * nch;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < P * p.U; e += blockDim.x) {
    const int q = e / p.U, u = e % p.U;
    const int sp = b.pair_sil[q] ? 2 * q : 2 * q + 1;
    const int sb = b.seg_begin[nxt][sp], sc = b.seg_count[nxt][sp];
    const int first = b.job_first[e], nch = b.node_tpre[q];
    for (int c = 0; c < nch; ++c) {
      HistItem it;
      it.begin = sb + c * chunk;
      it.count = min(chunk, sc - c * chunk);
      it.unit = u; it.job = q; it.slot = first + c;
      it.used = 0; it.pad[0] = it.pad[1] = 0;
      b.items[first + c] = it;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < P * p.U; e += blockDim.x) b.job_nitems[e] = b.node_tpre[e / p.U];
}

// One block: tree metadata, and the leaves' row intervals sorted by start.
// The leaf row ranges (in `fin` or a final list; they share one offset space
// and are disjoint) tile [0, n), so k_leaf_assign can map every position to
// its leaf with a binary search.
__global__ void __launch_bounds__(1024)
k_finish(GrowParams p, GrowBufs b, int* meta, long long n_root) {
  pdl_wait();
  pdl_trigger();
  GrowState* st = b.st;
  const int nn = st->n_nodes;
  __shared__ int s_nl;
  if (threadIdx.x == 0) {
    meta[0] = nn;
    meta[1] = st->depth_max + 1;
    meta[2] = (int)(st->err | st->xerr);
    meta[3] = st->level;
    if (nn == 1) {   // single-leaf tree: the root owns every row
      b.leaf_src[0] = SRC_IDENTITY; b.leaf_begin[0] = 0; b.leaf_count[0] = (int)n_root;
    }
    s_nl = 0;
  }
  __syncthreads();
  // rank leaves (feature < 0 is not visible here; leaves are nodes with node_bin < 0)
  for (int g = threadIdx.x; g < nn; g += blockDim.x) {
    if (b.node_bin[g] >= 0) continue;
    // order by (begin, non-empty, id): an empty range sorts before the
    // non-empty range that starts at the same position
    const int bg = b.leaf_begin[g], ng = b.leaf_count[g] > 0;
    int rank = 0;
    for (int q = 0; q < nn; ++q) {
      if (b.node_bin[q] >= 0) continue;
      const int bq = b.leaf_begin[q], nq = b.leaf_count[q] > 0;
      if (bq < bg || (bq == bg && (nq < ng || (nq == ng && q < g)))) ++rank;
    }
    b.split_f[rank] = g;            // reuse per-node scratch: sorted leaf gids
    atomicAdd(&s_nl, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) st->n_leaves = s_nl;
}

// Writes leaf_of_row[row] = leaf for every position of the final leaf ranges
// (SRC_IDENTITY positions are root positions: root[i], or i without a root list).
__global__ void k_leaf_assign(GrowParams p, GrowBufs b, int* __restrict__ leaf_of_row, const int* __restrict__ root,
                              long long n_root) {
  pdl_wait();
  GrowState* st = b.st;
  const int nl = st->n_leaves;
  extern __shared__ int sm_leaf[];          // [nl] begins, [nl] gids, [nl] srcs
  int* sb = sm_leaf;
  int* sg = sm_leaf + nl;
  int* ss = sm_leaf + 2 * nl;
  for (int i = threadIdx.x; i < nl; i += blockDim.x) {
    const int g = b.split_f[i];
    sb[i] = b.leaf_begin[g]; sg[i] = g; ss[i] = b.leaf_src[g];
  }
  __syncthreads();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_root;
       i += (long long)gridDim.x * blockDim.x) {
    int lo = 0, hi = nl - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (sb[mid] <= i) lo = mid; else hi = mid - 1;
    }
    const int src = ss[lo];
    int row;
    if (src == SRC_IDENTITY) row = root ? root[i] : (int)i;
    else if (src == SRC_FIN) row = b.fin[i];
    else row = b.rows[src == SRC_LIST0 ? 0 : 1][i];
    if (YABT_BOUNDS_CHECKED && (row < 0 || row >= p.n || sg[lo] < 0 || sg[lo] >= p.maxn)) {
      atomicOr(&st->err, DERR_BOUNDS);
      continue;
    }
    leaf_of_row[row] = sg[lo];
  }
}

// Leaf of every row 0..n-1 of the grown tree, by its split bins: bin <= split
// bin goes left (the same routing as the partition and as Tree.apply on the
// imputed features, yabt/tree.py:82-116, since bin(x) <= b <=> x <= edges[b]).
__global__ void k_apply_all(GrowParams p, GrowBufs b, TreeIO io) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < p.n;
       i += (long long)gridDim.x * blockDim.x) {
    long long node = 0;
    for (int depth = 0; depth <= p.levels_max && io.feature[node] >= 0; ++depth) {
      const long long f = io.feature[node];
      if (YABT_BOUNDS_CHECKED && (f >= p.F || io.left[node] < 0 || io.left[node] >= p.maxn ||
                                  io.right[node] < 0 || io.right[node] >= p.maxn)) {
        atomicOr(&b.st->err, DERR_BOUNDS);
        break;
      }
      const unsigned bin = io.bins_fm[f * p.n + i];
      node = bin <= (unsigned)b.node_bin[node] ? io.left[node] : io.right[node];
    }
    io.leaf_of_row[i] = (int)node;
  }
}

cudaError_t launch_apply_all(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int nsm, cudaStream_t s) {
  const int grid = (int)std::min<long long>((p.n + 255) / 256, 8LL * nsm);
  k_apply_all<<<std::max(grid, 1), 256, 0, s>>>(p, b, io);
  count_launches(1);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ best-first growth
// Restates the heap grower, yabt/tree.py:206-360: candidate leaves ordered by
// (-gain, push order); the best one is split, its rows partitioned stably, the
// smaller child histogrammed and the sibling obtained by subtraction, and both
// children become candidates when depth < max_depth and their gain > 0. Push
// order equals node-id order (a node is pushed right after it is created), so
// ties go to the lower node id. One split per step, with the level-wise
// kernels doing the partition (one node), the item plan and the histogram:
//     k_bf_pick -> k_partition -> k_plan -> k_hist -> k_reduce -> k_bf_scan
// Every live leaf keeps its rows in rows[0] at a disjoint range and its full
// histogram in hist[0] at its slot (the left child inherits the parent's slot,
// the right child takes a new one: at most max_leaves slots). Leaves that are
// never split again may keep their rows in rows[1] (SRC_LIST1).

// Per (child, feature): best bin of one feature of a candidate node, with the
// exact left sums of the winning bin. v: the lane's 8 bins (exclusive of
// nothing: raw bin sums), per channel. Lane 0 writes the record and folds the
// feature into node_key[c].
template <int C>
__device__ __forceinline__ void bf_scan_feature(const GrowParams& p, const GrowBufs& b, const TreeIO& io,
                                                long long (&v)[C][8], int c, int f, float pm, float ginv,
                                                float hinv) {
  const int lane = threadIdx.x & 31;
  const float lam = p.lam, gam = p.gamma, mcw = p.mcw, fmsl = (float)p.msl;
  const bool fok = !(p.use_fmask && io.fmask && !io.fmask[f]);
  long long lt[C];
#pragma unroll
  for (int k = 0; k < C; ++k) {
#pragma unroll
    for (int i = 1; i < 8; ++i) v[k][i] += v[k][i - 1];
    long long x = v[k][7];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    lt[k] = __shfl_sync(0xffffffffu, x, 31);
    const long long excl = x - v[k][7];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[k][i] += excl;
  }
  const float G = __fmul_rn(__ll2float_rn(lt[0]), ginv);
  const float H = (C == 3) ? __fmul_rn(__ll2float_rn(lt[1]), hinv) : __ll2float_rn(lt[C - 1]);
  const float Cn = __ll2float_rn(lt[C - 1]);
  const float t3 = __fdiv_rn(__fmul_rn(G, G), __fadd_rn(H, lam));
  const float boost = p.use_imat ? __fadd_rn(1.f, __fmul_rn(p.ib, pm)) : 1.f;
  float bsel = -INFINITY, bgain = -INFINITY;
  int bbin = 0;
  long long bgl = 0, bhl = 0, bcl = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int bin = lane * 8 + i;
    const float GL = __fmul_rn(__ll2float_rn(v[0][i]), ginv);
    const float CL = __ll2float_rn(v[C - 1][i]);
    const float HL = (C == 3) ? __fmul_rn(__ll2float_rn(v[1][i]), hinv) : CL;
    const float GR = __fsub_rn(G, GL), HR = __fsub_rn(H, HL), CR = __fsub_rn(Cn, CL);
    const float t1 = __fdiv_rn(__fmul_rn(GL, GL), __fadd_rn(HL, lam));
    const float t2 = __fdiv_rn(__fmul_rn(GR, GR), __fadd_rn(HR, lam));
    float gain = __fsub_rn(__fmul_rn(0.5f, __fsub_rn(__fadd_rn(t1, t2), t3)), gam);
    const bool valid = fok && bin != YABT_NB - 1 && CL >= fmsl && CR >= fmsl && HL >= mcw && HR >= mcw;
    if (!valid) gain = -INFINITY;
    const float sel = p.use_imat ? __fmul_rn(gain, boost) : gain;
    if (i == 0 || sel > bsel) {
      bsel = sel; bgain = gain; bbin = bin;
      bgl = v[0][i]; bhl = v[C - 2][i]; bcl = v[C - 1][i];
    }
  }
  // warp argmax: larger sel wins, ties -> lower bin
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float os = __shfl_xor_sync(0xffffffffu, bsel, o);
    const int ob = __shfl_xor_sync(0xffffffffu, bbin, o);
    const float og = __shfl_xor_sync(0xffffffffu, bgain, o);
    const long long ogl = __shfl_xor_sync(0xffffffffu, bgl, o);
    const long long ohl = __shfl_xor_sync(0xffffffffu, bhl, o);
    const long long ocl = __shfl_xor_sync(0xffffffffu, bcl, o);
    if (os > bsel || (os == bsel && ob < bbin)) {
      bsel = os; bbin = ob; bgain = og; bgl = ogl; bhl = ohl; bcl = ocl;
    }
  }
  if (lane == 0) {
    BfCand r;
    r.sel = bsel; r.gain = bgain; r.f = f; r.bin = bbin; r.flag = 0;
    r.gl = bgl; r.cl = bcl; r.hl = (C == 3) ? bhl : bcl;
    r.g = lt[0]; r.c = lt[C - 1]; r.h = (C == 3) ? lt[1] : lt[C - 1];
    b.bf_feat[(size_t)c * p.F + f] = r;
    atomicMax(&b.node_key[c], ((unsigned long long)f2ord(bsel) << 32) | (0xffffffffu - (unsigned)f));
  }
}

// The same in the arithmetic of the reference's C / Numba grower
// (yabt/_cgrow/grow.c:124-199 best_split): float64 sums of the bins (here the
// exact sums, converted), float64 gain in the same operand order without
// contraction, candidate bins b < nbins - 1 with nbins = min(edges + 1, 256),
// first maximum of gain * boost with a strict '>', and bin -1 when the
// feature has no valid split. The node's feature is chosen in k_bf_pick.
template <int C>
__device__ __forceinline__ void bf_scan_feature_f64(const GrowParams& p, const GrowBufs& b, const TreeIO& io,
                                                    long long (&v)[C][8], int c, int f, float pm, double ginv,
                                                    double hinv) {
  const int lane = threadIdx.x & 31;
  const double lam = (double)p.lam, gam = (double)p.gamma, mcw = (double)p.mcw, msl = (double)p.msl;
  const bool fok = !(p.use_fmask && io.fmask && !io.fmask[f]);
  const int nb = min(io.edge_cnt[f] + 1, YABT_NB);
  long long lt[C];
#pragma unroll
  for (int k = 0; k < C; ++k) {
#pragma unroll
    for (int i = 1; i < 8; ++i) v[k][i] += v[k][i - 1];
    long long x = v[k][7];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    lt[k] = __shfl_sync(0xffffffffu, x, 31);
    const long long excl = x - v[k][7];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[k][i] += excl;
  }
  const double G = __dmul_rn((double)lt[0], ginv);
  const double H = (C == 3) ? __dmul_rn((double)lt[1], hinv) : (double)lt[C - 1];
  const double Cn = (double)lt[C - 1];
  const double parent = __ddiv_rn(__dmul_rn(G, G), __dadd_rn(H, lam));
  const double bo = p.use_imat ? (double)__fadd_rn(1.f, __fmul_rn(p.ib, pm)) : 1.0;
  double bsel = -INFINITY, bgain = -INFINITY;
  int bbin = -1;
  long long bgl = 0, bhl = 0, bcl = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int bin = lane * 8 + i;
    const double GL = __dmul_rn((double)v[0][i], ginv);
    const double CL = (double)v[C - 1][i];
    const double HL = (C == 3) ? __dmul_rn((double)v[1][i], hinv) : CL;
    const double GR = __dsub_rn(G, GL), HR = __dsub_rn(H, HL), CR = __dsub_rn(Cn, CL);
    if (!(fok && bin < nb - 1 && CL >= msl && CR >= msl && HL >= mcw && HR >= mcw)) continue;
    const double t1 = __ddiv_rn(__dmul_rn(GL, GL), __dadd_rn(HL, lam));
    const double t2 = __ddiv_rn(__dmul_rn(GR, GR), __dadd_rn(HR, lam));
    const double gain = __dsub_rn(__dmul_rn(0.5, __dsub_rn(__dadd_rn(t1, t2), parent)), gam);
    const double sel = __dmul_rn(gain, bo);
    if (sel > bsel) {
      bsel = sel; bgain = gain; bbin = bin;
      bgl = v[0][i]; bhl = v[C - 2][i]; bcl = v[C - 1][i];
    }
  }
  // warp: the first maximum in bin order (larger sel, ties -> lower bin; no valid bin = -1 last)
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const double os = __shfl_xor_sync(0xffffffffu, bsel, o);
    const int ob = __shfl_xor_sync(0xffffffffu, bbin, o);
    const double og = __shfl_xor_sync(0xffffffffu, bgain, o);
    const long long ogl = __shfl_xor_sync(0xffffffffu, bgl, o);
    const long long ohl = __shfl_xor_sync(0xffffffffu, bhl, o);
    const long long ocl = __shfl_xor_sync(0xffffffffu, bcl, o);
    const bool take = ob >= 0 && (bbin < 0 || os > bsel || (os == bsel && ob < bbin));
    if (take) {
      bsel = os; bbin = ob; bgain = og; bgl = ogl; bhl = ohl; bcl = ocl;
    }
  }
  if (lane == 0) {
    BfCand r;
    r.sel = bsel; r.gain = (float)bgain; r.f = f; r.bin = bbin; r.flag = 0;
    r.gl = bgl; r.cl = bcl; r.hl = (C == 3) ? bhl : bcl;
    r.g = lt[0]; r.c = lt[C - 1]; r.h = (C == 3) ? lt[1] : lt[C - 1];
    b.bf_feat[(size_t)c * p.F + f] = r;
  }
}

template <int C>
__device__ __forceinline__ void bf_scan_any(const GrowParams& p, const GrowBufs& b, const TreeIO& io,
                                            long long (&v)[C][8], int c, int f, float pm, const GrowState* st) {
  if (p.bf_f64) bf_scan_feature_f64<C>(p, b, io, v, c, f, pm, (double)st->ginv, (double)st->hinv);
  else bf_scan_feature<C>(p, b, io, v, c, f, pm, st->ginv, st->hinv);
}

// Scan of the root (root != 0: the level-0 histogram in `small`) or of the two
// children of the node the last k_bf_pick split. Blocks [0, fblocks): one warp
// per feature handles both children (the left child's slot is the parent's,
// so the parent's bins are read before either child is written). Blocks
// beyond: the children's row ranges (copied back from rows[1] to rows[0] when
// the children stay candidates).
template <int C>
__global__ void __launch_bounds__(SCAN_WARPS * 32)
k_bf_scan(GrowParams p, GrowBufs b, TreeIO io, int root) {
  GrowState* st = b.st;
  const int fblocks = (p.F + SCAN_WARPS - 1) / SCAN_WARPS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t FB = (size_t)p.F * YABT_NB;
  const size_t HN = (size_t)C * FB;
  if (root) {
    if (!st->active) return;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      b.leaf_src[0] = SRC_IDENTITY; b.leaf_begin[0] = 0; b.leaf_count[0] = (int)io.n_root;
      b.node_slot[0] = 0;
      st->bf_next_slot = 1; st->bf_split = -2; st->bf_scan = 1;
    }
  } else {
    if (st->bf_split < 0) return;
    if (blockIdx.x >= fblocks) {
      // children row ranges; while they stay candidates their rows go back to rows[0]
      const int nl = st->n_nodes - 2, nr = nl + 1;
      const int B = b.seg_begin[0][0], cnt = b.seg_count[0][0];
      const int keep = st->bf_scan;
      if (blockIdx.x == fblocks && threadIdx.x == 0) {
        const int src = keep ? SRC_LIST0 : SRC_LIST1;
        b.leaf_src[nl] = src; b.leaf_begin[nl] = b.seg_begin[1][0]; b.leaf_count[nl] = b.seg_count[1][0];
        b.leaf_src[nr] = src; b.leaf_begin[nr] = b.seg_begin[1][1]; b.leaf_count[nr] = b.seg_count[1][1];
      }
      if (keep) {
        const int nb = gridDim.x - fblocks;
        for (int i = (blockIdx.x - fblocks) * blockDim.x + threadIdx.x; i < cnt; i += nb * blockDim.x)
          b.rows[0][B + i] = b.rows[1][B + i];
      }
      return;
    }
    if (!st->bf_scan) return;
  }
  const int f = blockIdx.x * SCAN_WARPS + warp;
  if (blockIdx.x >= fblocks || f >= p.F) return;
  const long long* sm = b.small + (size_t)f * YABT_NB + lane * 8;
  const long long* scnt = b.small + (size_t)(C - 1) * FB + (size_t)f * (YABT_NB / 2) + lane * 4;
  long long vs[C][8];
#pragma unroll
  for (int c = 0; c < C - 1; ++c) {
    const longlong2* q = reinterpret_cast<const longlong2*>(sm + c * FB);
#pragma unroll
    for (int i = 0; i < 4; ++i) { const longlong2 t = q[i]; vs[c][2 * i] = t.x; vs[c][2 * i + 1] = t.y; }
  }
  {
    const longlong2* q = reinterpret_cast<const longlong2*>(scnt);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const longlong2 t = q[i];
      vs[C - 1][4 * i + 0] = (long long)((unsigned long long)t.x & 0xffffffffULL);
      vs[C - 1][4 * i + 1] = (long long)((unsigned long long)t.x >> 32);
      vs[C - 1][4 * i + 2] = (long long)((unsigned long long)t.y & 0xffffffffULL);
      vs[C - 1][4 * i + 3] = (long long)((unsigned long long)t.y >> 32);
    }
  }
  if (root) {
    if (p.max_depth > 0) {
      long long* dst = b.hist[0] + (size_t)f * YABT_NB + lane * 8;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        longlong2* q = reinterpret_cast<longlong2*>(dst + c * FB);
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = make_longlong2(vs[c][2 * i], vs[c][2 * i + 1]);
      }
    }
    bf_scan_any<C>(p, b, io, vs, 0, f, b.pathmax[0][f], st);
    return;
  }
  // children of node m: the small one from `small`, the other = parent - small
  const int m = st->bf_split;
  const int nl = st->n_nodes - 2, nr = nl + 1;
  const int ps = b.node_slot[nl], rs = b.node_slot[nr];
  const bool sil = b.pair_sil[0] != 0;
  long long vo[C][8];
  {
    const long long* par = b.hist[0] + (size_t)ps * HN + (size_t)f * YABT_NB + lane * 8;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const longlong2* q = reinterpret_cast<const longlong2*>(par + c * FB);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const longlong2 t = q[i];
        vo[c][2 * i] = t.x - vs[c][2 * i];
        vo[c][2 * i + 1] = t.y - vs[c][2 * i + 1];
      }
    }
  }
  float pm = 0.f;
  if (p.use_imat) {
    pm = fmaxf(b.pathmax[0][(size_t)ps * p.F + f], io.imat[(size_t)io.feature[m] * p.F + f]);
    __syncwarp();
    if (lane == 0) {
      b.pathmax[0][(size_t)ps * p.F + f] = pm;
      b.pathmax[0][(size_t)rs * p.F + f] = pm;
    }
  }
  __syncwarp();
#pragma unroll
  for (int ch = 0; ch < 2; ++ch) {
    long long v[C][8];
    const bool from_small = (ch == 0) == sil;
#pragma unroll
    for (int c = 0; c < C; ++c)
#pragma unroll
      for (int i = 0; i < 8; ++i) v[c][i] = from_small ? vs[c][i] : vo[c][i];
    long long* dst = b.hist[0] + (size_t)(ch == 0 ? ps : rs) * HN + (size_t)f * YABT_NB + lane * 8;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      longlong2* q = reinterpret_cast<longlong2*>(dst + c * FB);
#pragma unroll
      for (int i = 0; i < 4; ++i) q[i] = make_longlong2(v[c][2 * i], v[c][2 * i + 1]);
    }
    bf_scan_any<C>(p, b, io, v, ch, f, pm, st);
  }
}

__device__ __forceinline__ float bf_value(const GrowParams& p, const GrowState* st, long long g, long long h) {
  if (p.bf_f64) {
    // -lr * G / (H + lambda) on the float64 sums, yabt/_cgrow/grow.c:318-323,355-363
    const double G = __dmul_rn((double)g, (double)st->ginv);
    const double H = p.general ? __dmul_rn((double)h, (double)st->hinv) : (double)h;
    return (float)__ddiv_rn(__dmul_rn(-(double)p.lr, G), __dadd_rn(H, (double)p.lam));
  }
  // leaf value -lr * G / (H + lambda) in double on the float32 sums, yabt/tree.py:233-243
  const float G = __fmul_rn(__ll2float_rn(g), st->ginv);
  const float H = p.general ? __fmul_rn(__ll2float_rn(h), st->hinv) : __ll2float_rn(h);
  return (float)(-(double)p.lr * (double)G / ((double)H + (double)p.lam));
}

// float64 mode: the child's feature is the first maximum of sel over features
// with a valid split (yabt/_cgrow/grow.c:189-199); the whole block reduces.
// Returns F when no feature has one.
__device__ int bf_best_feature_f64(const GrowParams& p, const BfCand* __restrict__ rec) {
  __shared__ double s_sel[32];
  __shared__ int s_f[32];
  __shared__ int s_best;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double bs = -INFINITY;
  int bf = p.F;
  for (int f = threadIdx.x; f < p.F; f += blockDim.x) {
    const BfCand& r = rec[f];
    if (r.bin >= 0 && (bf == p.F || r.sel > bs)) { bs = r.sel; bf = f; }
  }
  auto better = [&](double os, int of) { return of < p.F && (bf == p.F || os > bs || (os == bs && of < bf)); };
  for (int o = 16; o; o >>= 1) {
    const double os = __shfl_xor_sync(0xffffffffu, bs, o);
    const int of = __shfl_xor_sync(0xffffffffu, bf, o);
    if (better(os, of)) { bs = os; bf = of; }
  }
  if (lane == 0) { s_sel[warp] = bs; s_f[warp] = bf; }
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    bs = lane < nw ? s_sel[lane] : -INFINITY;
    bf = lane < nw ? s_f[lane] : p.F;
    for (int o = 16; o; o >>= 1) {
      const double os = __shfl_xor_sync(0xffffffffu, bs, o);
      const int of = __shfl_xor_sync(0xffffffffu, bf, o);
      if (better(os, of)) { bs = os; bf = of; }
    }
    if (lane == 0) s_best = bf;
  }
  __syncthreads();
  const int res = s_best;
  __syncthreads();
  return res;
}

// One block. Commits the candidates the last k_bf_scan produced, pops the best
// candidate (largest gain, ties -> lower node id) and sets up its split: the
// tree arrays of the node and its two children, and the partition of its row
// range (one active position, `part_gate` selects the source list).
__global__ void __launch_bounds__(1024)
k_bf_pick(GrowParams p, GrowBufs b, TreeIO io, int part_gate) {
  GrowState* st = b.st;
  if (!st->active) return;
  __shared__ unsigned long long s_key;
  const int split = st->bf_split;
  const int n0 = st->n_nodes;
  // A: commit the scanned nodes (the root, or the two newest nodes)
  const int ncommit = !st->bf_scan ? 0 : split == -2 ? 1 : split >= 0 ? 2 : 0;
  for (int c = 0; c < ncommit; ++c) {
    int f;
    if (p.bf_f64) {
      f = bf_best_feature_f64(p, b.bf_feat + (size_t)c * p.F);
    } else {
      const unsigned long long key = b.node_key[c];
      f = (int)(0xffffffffu - (unsigned)(key & 0xffffffffULL));
    }
    if (threadIdx.x == 0) {
      const int gid = split == -2 ? 0 : n0 - 2 + c;
      BfCand r = b.bf_feat[(size_t)c * p.F + ((unsigned)f < (unsigned)p.F ? f : 0)];
      if ((unsigned)f >= (unsigned)p.F) r.gain = -INFINITY;     // no valid split at all
      r.flag = (b.node_depth[gid] < p.max_depth && r.gain > 0.f) ? 1 : 0;
      b.bf_cand[gid] = r;
      if (split == -2) io.value[0] = bf_value(p, st, r.g, r.h);
    }
  }
  __syncthreads();
  if (threadIdx.x < 2) b.node_key[threadIdx.x] = 0ULL;
  if (threadIdx.x == 0) s_key = 0ULL;
  __syncthreads();
  // B: pop the best candidate
  const int leaves = (n0 + 1) / 2;
  if (leaves < p.max_leaves) {
    for (int g = threadIdx.x; g < n0; g += blockDim.x) {
      const BfCand& r = b.bf_cand[g];
      // ties: the earlier push (lower node id) for the heap grower; the lower
      // active-leaf slot for the C / Numba grower (grow.c:299-306)
      const unsigned tie = p.bf_f64 ? (unsigned)b.node_slot[g] : (unsigned)g;
      if (r.flag) atomicMax(&s_key, ((unsigned long long)f2ord(r.gain) << 32) | (0xffffffffu - tie));
    }
  }
  __syncthreads();
  const unsigned long long key = s_key;
  if (key == 0ULL || n0 + 2 > p.maxn) {
    if (threadIdx.x == 0) {
      if (key != 0ULL) atomicOr(&st->err, DERR_NODE_OVERFLOW);
      st->active = 0; st->bf_split = -1; st->bf_scan = 0;
      st->level = -1; st->part_level = -1; st->plan_level = -1;
    }
    return;
  }
  __shared__ int s_pick;
  if (threadIdx.x == 0) {
    const unsigned tie = 0xffffffffu - (unsigned)(key & 0xffffffffULL);
    int m = (int)tie;
    if (p.bf_f64)            // the slot names the node: the leaf that holds it
      for (int g = 0; g < n0; ++g)
        if (b.bf_cand[g].flag && (unsigned)b.node_slot[g] == tie) { m = g; break; }
    s_pick = m;
  }
  __syncthreads();
  const int m = s_pick;
  const BfCand r = b.bf_cand[m];
  const int B = b.leaf_begin[m], cnt = b.leaf_count[m];
  const int nt = (cnt + PART_TILE - 1) / PART_TILE;
  if (threadIdx.x == 0) {
    const int f = r.f, bin = r.bin, ne = io.edge_cnt[f];
    const int nl = n0, nr = n0 + 1, d = b.node_depth[m] + 1;
    b.bf_cand[m].flag = 0;
    io.feature[m] = f;
    io.threshold[m] = io.edges[io.edge_off[f] + min(bin, ne - 1)];
    io.gate[m] = fmaxf(io.scales[f], 1e-12f);
    io.value[m] = 0.f;
    io.left[m] = nl; io.right[m] = nr;
    b.node_bin[m] = bin;
    const float vL = bf_value(p, st, r.gl, r.hl);
    const float vR = bf_value(p, st, r.g - r.gl, r.h - r.hl);
    for (int k = 0; k < 2; ++k) {
      const int q = n0 + k;
      io.feature[q] = -1; io.threshold[q] = 0.f; io.left[q] = -1; io.right[q] = -1;
      io.value[q] = k == 0 ? vL : vR; io.gate[q] = 1.f;
      b.node_depth[q] = d; b.node_bin[q] = -1;
      b.bf_cand[q].flag = 0;
    }
    b.node_slot[nl] = b.node_slot[m];
    b.node_slot[nr] = st->bf_next_slot;
    st->bf_next_slot = st->bf_next_slot + 1;
    // the partition of one active position (pair 0); smaller child by row count
    b.seg_begin[0][0] = B; b.seg_count[0][0] = cnt;
    // children inherit the region; the partition's last tile fills in the split
    // point (a rank with no rows of the node has no tile)
    b.seg_begin[1][0] = B; b.seg_count[1][0] = 0;
    b.seg_begin[1][1] = B; b.seg_count[1][1] = cnt;
    b.split_pair[0] = 0; b.split_f[0] = f; b.split_b[0] = bin;
    b.pair_pos[0] = 0; b.pair_sil[0] = r.cl <= r.c - r.cl;
    const int leaves_after = leaves + 1;
    const int scan = d < p.max_depth && leaves_after < p.max_leaves;
    st->n_nodes = n0 + 2;
    st->depth_max = max(st->depth_max, d);
    st->bf_split = m; st->bf_scan = scan;
    st->P = 1; st->M = 1;
    st->n_tiles = nt; st->tile_counter = 0;
    st->epoch = st->epoch + 1;
    st->part_level = part_gate;
    st->plan_level = scan ? part_gate : -1;
    st->level = scan ? 1 : -1;           // the histogram kernels run at level 1 (rows[1])
    st->active = leaves_after < p.max_leaves ? 1 : 0;
  }
  for (int e = threadIdx.x; e < nt; e += blockDim.x) {
    PartTile t;
    t.pos = 0; t.begin = B + e * PART_TILE; t.end = min(B + cnt, t.begin + PART_TILE);
    t.last = e == nt - 1; t.t_in_node = e;
    t.pad[0] = t.pad[1] = t.pad[2] = 0;
    b.tiles[e] = t;
  }
}

cudaError_t launch_bf_root_scan(const GrowParams& p, const GrowBufs& b, const TreeIO& io, cudaStream_t s) {
  PhaseScope ph(PH_SCAN, s);
  const int fblocks = (p.F + SCAN_WARPS - 1) / SCAN_WARPS;
  if (!p.general) k_bf_scan<2><<<fblocks, SCAN_WARPS * 32, 0, s>>>(p, b, io, 1);
  else k_bf_scan<3><<<fblocks, SCAN_WARPS * 32, 0, s>>>(p, b, io, 1);
  count_launches(1);
  return cudaGetLastError();
}

// One best-first step, first half: pop the best candidate, partition its rows
// and histogram the smaller child into `small`. Step 1 splits the root, whose
// rows are root positions (partition gate 0); later steps read rows[0] (gate 2).
cudaError_t launch_bf_pick_partition(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int step, int nsm,
                                     cudaStream_t s) {
  const int gate = step == 1 ? 0 : 2;
  {
    PhaseScope ph(PH_FINALIZE, s);
    k_bf_pick<<<1, 1024, 0, s>>>(p, b, io, gate);
  }
  const int pgrid = std::max(1, std::min(p.max_tiles, 4 * nsm));
  {
    PhaseScope ph(PH_PARTITION, s);
    k_partition<<<pgrid, PART_THREADS, 0, s>>>(p, b, io, gate);
  }
  {
    PhaseScope ph(PH_PLAN, s);
    k_plan<<<1, 1024, 0, s>>>(p, b, gate);
  }
  count_launches(3);
  return cudaGetLastError();
}

cudaError_t launch_bf_split(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int step, int nsm,
                            cudaStream_t s) {
  const cudaError_t e = launch_bf_pick_partition(p, b, io, step, nsm, s);
  if (e != cudaSuccess) return e;
  return launch_hist_kernels(p, b, io, 1, 1, nsm, s, nullptr, 0);
}

// max |g| over several gradient arrays into the hessian word too (one
// quantisation scale shared by both histogram channels)
cudaError_t launch_absmax_shared(const float* const* arrays, int count, long long n_root, const int* root,
                                 GrowState* st, int nsm, cudaStream_t s) {
  PhaseScope ph(PH_BEGIN, s);
  cudaError_t e = cudaMemsetAsync(&st->amax_g, 0, 2 * sizeof(unsigned), s);
  if (e != cudaSuccess) return e;
  const int grid = (int)std::min<long long>((n_root + 255) / 256, 8LL * nsm);
  for (int i = 0; i < count; ++i) k_absmax<<<std::max(grid, 1), 256, 0, s>>>(arrays[i], nullptr, n_root, root, st);
  count_launches(count);
  e = cudaMemcpyAsync(&st->amax_h, &st->amax_g, sizeof(unsigned), cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// Second half: the children's histograms, scans and row ranges.
cudaError_t launch_bf_scan(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int nsm, cudaStream_t s) {
  PhaseScope ph(PH_SCAN, s);
  const int fblocks = (p.F + SCAN_WARPS - 1) / SCAN_WARPS;
  const int grid = fblocks + std::max(1, std::min<int>(nsm, (int)((p.n + 2047) / 2048)));
  if (!p.general) k_bf_scan<2><<<grid, SCAN_WARPS * 32, 0, s>>>(p, b, io, 0);
  else k_bf_scan<3><<<grid, SCAN_WARPS * 32, 0, s>>>(p, b, io, 0);
  count_launches(1);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ host side
struct HostStep {
  int S, LIMBS, C;
};

static inline int jobs_bound(int d, int max_pairs) {
  if (d == LEVEL_DYN) return max_pairs;       // any level of a device-side loop
  if (d == 0) return 1;
  long long j = 1LL << min(d - 1, 30);
  return (int)std::min<long long>(j, max_pairs);
}

// ------------------------------------------------------------------ device-side level loop
// Kernels run inside device-side level loops, counted on the device (the host
// cannot know how many levels a loop ran): every pass of a loop's body adds
// its kernels here.
__device__ unsigned long long g_loop_launches;

// Condition of a device-side level loop (a CUDA graph WHILE node, abi.cu):
// another level runs while the tree is active and below its level limit.
// Inside the loop body (body_kernels > 0) it also counts the body's kernels.
__global__ void k_level_loop_cond(const GrowState* __restrict__ st, int levels_max, cudaGraphConditionalHandle h,
                                  int body_kernels) {
  const bool more = st->active && st->level < levels_max;
  cudaGraphSetConditional(h, more ? 1u : 0u);
  if (body_kernels > 0) atomicAdd(&g_loop_launches, (unsigned long long)body_kernels);
}

// The condition kernel of a loop: before the loop (body_kernels 0) or as the
// body's last kernel (body_kernels = the body's kernels, itself included).
cudaError_t launch_level_loop_cond(const GrowParams& p, const GrowBufs& b, cudaGraphConditionalHandle h,
                                   int body_kernels, cudaStream_t s) {
  k_level_loop_cond<<<1, 1, 0, s>>>(b.st, p.levels_max, h, body_kernels);
  return cudaGetLastError();
}

cudaError_t loop_launches_reset(cudaStream_t s) {
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_loop_launches);
  return e != cudaSuccess ? e : cudaMemsetAsync(ptr, 0, sizeof(unsigned long long), s);
}

cudaError_t loop_launches_read(long long* out) {
  unsigned long long v = 0;
  const cudaError_t e = cudaMemcpyFromSymbol(&v, g_loop_launches, sizeof(v));
  *out = (long long)v;
  return e;
}

// Launches of one level. Returns a CUDA error code (0 on success).
cudaError_t launch_level_hist(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int d,
                              int nsm, cudaStream_t s, cudaEvent_t after_hist, int root_counts) {
  return launch_hist_kernels(p, b, io, d, jobs_bound(d, p.max_pairs), nsm, s, after_hist, root_counts);
}

// The split of a level in two halves: the scan (features [f_lo, f_hi)) and
// the choice of the splits with the partition and the next level's plan. A
// feature-sliced sharded fit gathers every rank's best split per node between
// the two (yabt_grow_xgather).
cudaError_t launch_level_scan(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int d,
                              int nsm, cudaStream_t s) {
  (void)nsm;
  const int jobs = jobs_bound(d, p.max_pairs);
  const int fblocks = (p.f_hi - p.f_lo + SCAN_WARPS - 1) / SCAN_WARPS;
  cudaError_t e;
  {
    PhaseScope ph(PH_SCAN, s);
    e = p.general ? launch_pdl(k_scan<3>, dim3(jobs * fblocks), dim3(SCAN_WARPS * 32), 0, s, p, b, io, d)
                  : launch_pdl(k_scan<2>, dim3(jobs * fblocks), dim3(SCAN_WARPS * 32), 0, s, p, b, io, d);
  }
  count_launches(1);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_level_choose(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int d,
                                int nsm, cudaStream_t s) {
  cudaError_t e;
  {
    PhaseScope ph(PH_FINALIZE, s);
    e = launch_pdl(k_finalize, dim3(1), dim3(1024), 0, s, p, b, io, d);
  }
  if (e != cudaSuccess) return e;
  const int pgrid = std::max(1, std::min(p.max_tiles, 4 * nsm));
  {
    PhaseScope ph(PH_PARTITION, s);
    e = launch_pdl(k_partition, dim3(pgrid), dim3(PART_THREADS), 0, s, p, b, io, d);
  }
  if (e != cudaSuccess) return e;
  {
    PhaseScope ph(PH_PLAN, s);
    e = launch_pdl(k_plan, dim3(1), dim3(1024), 0, s, p, b, d);
  }
  count_launches(3);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_level_split(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int d,
                               int nsm, cudaStream_t s) {
  const cudaError_t e = launch_level_scan(p, b, io, d, nsm, s);
  if (e != cudaSuccess) return e;
  return launch_level_choose(p, b, io, d, nsm, s);
}

cudaError_t launch_tree_begin(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int nsm,
                              cudaStream_t s) {
  PhaseScope ph(PH_BEGIN, s);
  cudaError_t e = cudaMemsetAsync(&b.st->amax_g, 0, 2 * sizeof(unsigned), s);
  if (e != cudaSuccess) return e;

  const int grid = (int)std::min<long long>((io.n_root + 255) / 256, 8LL * nsm);
  e = launch_pdl(k_absmax, dim3(std::max(grid, 1)), dim3(256), 0, s, io.g, (const float*)(p.general ? io.h : nullptr),
                 (long long)io.n_root, io.root_rows, b.st);
  count_launches(1);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_tree_init(const GrowParams& p, const GrowBufs& b, const TreeIO& io, cudaStream_t s) {
  PhaseScope ph(PH_BEGIN, s);
  const cudaError_t e = launch_pdl(k_tree_init, dim3(1), dim3(1024), 0, s, p, b, io);
  count_launches(1);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_tree_finish(const GrowParams& p, const GrowBufs& b, const TreeIO& io, int* meta,
                               int* leaf_of_row, int nsm, cudaStream_t s) {
  PhaseScope ph(PH_FINISH, s);
  cudaError_t e = launch_pdl(k_finish, dim3(1), dim3(1024), 0, s, p, b, meta, (long long)io.n_root);
  if (e != cudaSuccess) return e;
  const int grid = (int)std::min<long long>((io.n_root + 511) / 512, 4LL * nsm);
  e = launch_pdl(k_leaf_assign, dim3(std::max(grid, 1)), dim3(512), 3 * (p.max_leaves + 1) * sizeof(int), s, p, b,
                 leaf_of_row, (const int*)io.root_rows, (long long)io.n_root);
  count_launches(2);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace yabt
