// Draft trees inside the device round (greedy): EAGLE-2 top-w expansion, path-probability
// frontier and verify selection, tree verification, acceptance, compaction and the drafter
// update, all from one CUDA graph with one host synchronisation per round.
//
// The reference drafts trees level by level on the host (python/woodcock/spec.py:216-303,
// src/core/spec.cpp:86-187) and verifies them with a tree mask (spec.cpp:189-224). Here the
// tree lives in a device TreeState and every decision is a small kernel between the drafter
// and target passes:
//   begin    node 0 = the newest committed token (or a forced tree's nodes, for tests);
//   expand   per frontier row: the drafter head's softmax and its top-w rows as children, in
//            frontier order, each child's path probability = parent's * q (spec.cpp:117-128);
//   frontier the w nodes of the newest level with the largest path probability (ties: earlier
//            node first) get drafter cache slots, positions n-1+depth and ancestor bit masks
//            (committed entries + drafted ancestors + itself, spec.cpp:158-171);
//   select   all drafted nodes if they fit the budget, else the root plus the `budget` nodes of
//            largest path probability (ties: shallower, then earlier; StaticPolicy.select_verify)
//            in node order, as verify rows with positions n+depth and tree-mask bits;
//   accept   verify_tree_greedy (src/sampling/sampling.cpp:95-106): from the root, the first
//            child in node order whose token is the target's argmax at its parent;
//   compact  target K/V rows n+keep[i] -> n+i in every layer (KVCache::compact,
//            src/cache/kv_cache.cpp:21-31); the taps of the kept rows feed the drafter update.
#pragma once

#include "common.cuh"
#include "misc.cuh"

namespace wc {

constexpr int TR_MAXN = 128;  // tree nodes per round, root included
constexpr int TR_MAXW = 16;   // rows of one drafter pass (frontier width)
constexpr int TR_MAXV = 16;   // verified rows (one target pass)

struct TreeState {
  int n;           // nodes so far (node 0 = root)
  int pending;     // children written by the last expansion, counted into n by the next step
  int level_lo;    // first node of the newest level
  int n_frontier;  // rows of the current drafter pass and head
  int N;           // verify rows
  int n_keep;      // kept verify rows (root + accepted path)
  int n_new;       // committed length after this round (applied once the cache is compacted)
  int forced_on;   // 1: the round verifies the forced tree f_* instead of drafting one
  int f_n;
  int pad[3];
  int token[TR_MAXN], parent[TR_MAXN], depth[TR_MAXN], slot[TR_MAXN];
  double phat[TR_MAXN];
  int prop_tok[TR_MAXN];  // the drafter head's own argmax at a node (test readout), -1 if none
  float prop_z[TR_MAXN];
  int fr_node[TR_MAXW], fr_tok[TR_MAXW], fr_pos[TR_MAXW], fr_fbrow[TR_MAXW];
  unsigned long long fr_mask[TR_MAXW];
  unsigned long long hkeys[TR_MAXW];  // drafter head argmax keys (the expansion reads the logits)
  int vnode[TR_MAXV], vtok[TR_MAXV], vpar[TR_MAXV], vpos[TR_MAXV], keep[TR_MAXV];
  unsigned long long vmask[TR_MAXV];
  unsigned long long vkeys[TR_MAXV];
  int f_tok[TR_MAXN], f_par[TR_MAXN];
};

struct TreeStepParams {
  TreeState* ts;
  RoundState* st;
  int level;        // depth of the nodes this step creates / forwards
  int W;            // width
  int budget;       // verify budget (select)
  int max_rows;     // verify rows the graph was built for (select)
  // expand
  const float* z;   // [rows][Vh] drafter head logits
  int Vh;
  const int* vocab_map;
  int vocab;
  // begin / store_fb
  const float* root_fb;
  float* fb_store;  // [1 + slots][H]: row 0 = the root's feature, row s + 1 = slot s
  int H;
  const float* h;   // drafter pass output rows [rows][H]
  const float* norm_w;
  float eps;
  int post_norm;
  int* out_host_view;
};

__device__ __forceinline__ void tree_commit(TreeState* ts) {
  if (ts->pending) {
    ts->level_lo = ts->n;
    ts->n += ts->pending;
    ts->pending = 0;
  }
}

// node 0 and (forced trees) every node; the root's feature into fb_store row 0
__global__ void tree_begin_kernel(__grid_constant__ const TreeStepParams p) {
  pdl_launch_dependents();
  pdl_wait();
  TreeState* ts = p.ts;
  if (threadIdx.x == 0) {
    ts->n = 1;
    ts->pending = 0;
    ts->level_lo = 0;
    ts->n_frontier = 1;
    ts->fr_node[0] = 0;
    ts->token[0] = p.st->x_n;
    ts->parent[0] = -1;
    ts->depth[0] = 0;
    ts->slot[0] = -1;
    ts->phat[0] = 1.0;
    ts->prop_tok[0] = -1;
    ts->prop_z[0] = 0.f;
    if (ts->forced_on) {
      const int fn = min(ts->f_n, TR_MAXN);
      for (int v = 1; v < fn; ++v) {
        const int pa = ts->f_par[v];
        const bool ok = pa >= 0 && pa < v;
        ts->token[v] = ts->f_tok[v];
        ts->parent[v] = ok ? pa : 0;
        ts->depth[v] = ts->depth[ok ? pa : 0] + 1;
        ts->slot[v] = -1;
        ts->phat[v] = 1.0;
        ts->prop_tok[v] = -1;
        ts->prop_z[v] = 0.f;
        if (!ok) raise_error(&p.st->err, kErrTree);
      }
      ts->n = fn;
    }
    for (int i = 0; i < TR_MAXV; ++i) ts->vkeys[i] = 0ull;
    for (int i = 0; i < TR_MAXW; ++i) ts->hkeys[i] = 0ull;
  }
  for (int i = threadIdx.x; i < p.H; i += blockDim.x) p.fb_store[i] = p.root_fb[i];
}

// One block per frontier row: the head row's max, softmax sum and (greedy drafting) top-W rows
// as children of the frontier node, larger logit first, lower row first on equal logits.
__global__ void __launch_bounds__(256) tree_expand_kernel(__grid_constant__ const TreeStepParams p) {
  pdl_launch_dependents();
  pdl_wait();
  TreeState* ts = p.ts;
  const int r = blockIdx.x;
  if (r >= ts->n_frontier) return;
  __shared__ float s_v[8];
  __shared__ int s_i[8];
  __shared__ float s_sum[8];
  __shared__ int s_sel[TR_MAXW];
  __shared__ float s_selv[TR_MAXW];
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const float* z = p.z + size_t(r) * p.Vh;
  const int v = ts->fr_node[r];
  const bool forced = ts->forced_on != 0;
  const int W = forced ? 1 : min(p.W, p.Vh);
  float zmax = 0.f, zsum = 0.f;
  for (int j = 0; j < W; ++j) {  // j-th largest, excluding rows already taken
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < p.Vh; i += blockDim.x) {
      bool taken = false;
      for (int q = 0; q < j; ++q) taken |= s_sel[q] == i;
      const float x = z[i];
      if (!taken && (x > bv || (x == bv && i < bi))) {
        bv = x;
        bi = i;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      s_v[warp] = bv;
      s_i[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      float b = s_v[0];
      int ix = s_i[0];
      for (int w = 1; w < int(blockDim.x / kWarp); ++w)
        if (s_v[w] > b || (s_v[w] == b && s_i[w] < ix)) {
          b = s_v[w];
          ix = s_i[w];
        }
      s_sel[j] = ix;
      s_selv[j] = b;
    }
    __syncthreads();
    if (j == 0) {  // the softmax denominator around the row's max
      zmax = s_selv[0];
      float a = 0.f;
      for (int i = tid; i < p.Vh; i += blockDim.x) a += expf(z[i] - zmax);
      a = warp_sum(a);
      if (lane == 0) s_sum[warp] = a;
      __syncthreads();
      if (tid == 0) {
        float t = 0.f;
        for (int w = 0; w < int(blockDim.x / kWarp); ++w) t += s_sum[w];
        s_sum[0] = t;
      }
      __syncthreads();
      zsum = s_sum[0];
    }
  }
  if (tid != 0) return;
  const int first = s_sel[0];
  ts->prop_tok[v] = p.vocab_map ? p.vocab_map[first] : first;
  ts->prop_z[v] = s_selv[0];
  if (forced) {
    if (r == 0) ts->pending = 0;
    return;
  }
  const int base = ts->n + r * W;
  for (int j = 0; j < W; ++j) {
    const int c = base + j;
    if (c >= TR_MAXN) {
      raise_error(&p.st->err, kErrTree);
      break;
    }
    const int row = s_sel[j];
    int tok = p.vocab_map ? p.vocab_map[row] : row;
    if (tok < 0 || tok >= p.vocab) {
      raise_error(&p.st->err, kErrTokenRange);
      tok = 0;
    }
    ts->token[c] = tok;
    ts->parent[c] = v;
    ts->depth[c] = p.level;
    ts->slot[c] = -1;
    ts->phat[c] = ts->phat[v] * double(expf(s_selv[j] - zmax) / zsum);
    ts->prop_tok[c] = -1;
    ts->prop_z[c] = 0.f;
  }
  if (r == 0) ts->pending = ts->n_frontier * W;
}

// The nodes of depth `level` that the drafter forwards next: their slots, positions, parent
// features and ancestor masks over the drafted slots (bit s = slot s, counted from the
// committed length).
__global__ void tree_frontier_kernel(__grid_constant__ const TreeStepParams p) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x != 0) return;
  TreeState* ts = p.ts;
  tree_commit(ts);
  int fr[TR_MAXW];
  int m = 0;
  if (ts->forced_on) {  // every node of this depth that has children, in node order
    for (int v = 1; v < ts->n; ++v) {
      if (ts->depth[v] != p.level) continue;
      bool has_child = false;
      for (int c = v + 1; c < ts->n && !has_child; ++c) has_child = ts->parent[c] == v;
      if (!has_child) continue;
      if (m == p.W) {
        raise_error(&p.st->err, kErrTree);
        break;
      }
      fr[m++] = v;
    }
  } else {  // the W nodes of the newest level with the largest path probability, earlier first on ties
    const int lo = ts->level_lo, hi = ts->n;
    for (; m < p.W && m < hi - lo; ++m) {
      int best = -1;
      for (int v = lo; v < hi; ++v) {
        bool taken = false;
        for (int q = 0; q < m; ++q) taken |= fr[q] == v;
        if (!taken && (best < 0 || ts->phat[v] > ts->phat[best])) best = v;
      }
      fr[m] = best;
    }
  }
  const int n_commit = p.st->n;
  for (int i = 0; i < m; ++i) {
    const int v = fr[i];
    const int s = (p.level - 1) * p.W + i;
    ts->slot[v] = s;
    ts->fr_node[i] = v;
    ts->fr_tok[i] = ts->token[v];
    ts->fr_pos[i] = n_commit - 1 + p.level;
    const int pa = ts->parent[v];
    ts->fr_fbrow[i] = pa > 0 ? ts->slot[pa] + 1 : 0;
    unsigned long long mask = 1ull << s;
    for (int u = pa; u > 0; u = ts->parent[u]) mask |= 1ull << ts->slot[u];
    ts->fr_mask[i] = mask;
  }
  ts->n_frontier = m;
}

// The features of the nodes a drafter pass just forwarded: RMSNorm(h) * norm (post-norm
// drafters) or h, into their fb_store rows.
__global__ void __launch_bounds__(256) tree_store_fb_kernel(__grid_constant__ const TreeStepParams p) {
  pdl_launch_dependents();
  pdl_wait();
  TreeState* ts = p.ts;
  const int r = blockIdx.x;
  if (r >= ts->n_frontier) return;
  __shared__ float red[8];
  const float* hr = p.h + size_t(r) * p.H;
  float* dst = p.fb_store + size_t(ts->slot[ts->fr_node[r]] + 1) * p.H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < p.H; i += blockDim.x) ss = fmaf(hr[i], hr[i], ss);
  ss = warp_sum(ss);
  if (threadIdx.x % kWarp == 0) red[threadIdx.x / kWarp] = ss;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < int(blockDim.x / kWarp); ++w) t += red[w];
  const float inv = 1.f / sqrtf(t / float(p.H) + p.eps);
  for (int i = threadIdx.x; i < p.H; i += blockDim.x) dst[i] = p.post_norm ? hr[i] * inv * p.norm_w[i] : hr[i];
}

// The verify tree: all drafted nodes within the budget, else the root plus the `budget` nodes of
// largest path probability (ties: shallower, then earlier), in node order; rows get positions
// n + depth and ancestor bits over the verify rows (self included).
__global__ void tree_select_kernel(__grid_constant__ const TreeStepParams p) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x != 0) return;
  TreeState* ts = p.ts;
  tree_commit(ts);
  const int total = ts->n - 1;
  bool kept[TR_MAXN];
  for (int v = 0; v < TR_MAXN; ++v) kept[v] = v < ts->n;
  if (!ts->forced_on && total > p.budget) {
    for (int v = 1; v < ts->n; ++v) kept[v] = false;
    for (int k = 0; k < p.budget; ++k) {
      int best = -1;
      for (int v = 1; v < ts->n; ++v) {
        if (kept[v]) continue;
        if (best < 0 || ts->phat[v] > ts->phat[best] ||
            (ts->phat[v] == ts->phat[best] && ts->depth[v] < ts->depth[best]))
          best = v;
      }
      kept[best] = true;
    }
  }
  int rowof[TR_MAXN];
  int N = 0;
  for (int v = 0; v < ts->n; ++v) {
    rowof[v] = -1;
    if (!kept[v]) continue;
    if (N == p.max_rows) {
      raise_error(&p.st->err, kErrTree);
      break;
    }
    rowof[v] = N;
    const int pa = ts->parent[v];
    const int pr = pa >= 0 ? rowof[pa] : -1;
    if (pa >= 0 && pr < 0) raise_error(&p.st->err, kErrTree);  // a kept node's parent is kept
    ts->vnode[N] = v;
    ts->vtok[N] = ts->token[v];
    ts->vpar[N] = pr;
    ts->vpos[N] = p.st->n + ts->depth[v];
    ts->vmask[N] = (pr >= 0 ? ts->vmask[pr] : 0ull) | (1ull << N);
    ++N;
  }
  ts->N = N;
}

// verify_tree_greedy (src/sampling/sampling.cpp:95-106) on the target's argmax keys; the
// accepted tokens and the next token into the round state, the kept rows into keep[].
__global__ void tree_accept_kernel(__grid_constant__ const TreeStepParams p) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x != 0) return;
  TreeState* ts = p.ts;
  RoundState* st = p.st;
  const int N = ts->N;
  int am[TR_MAXV];
  for (int i = 0; i < N; ++i) am[i] = int(argmax_key_index(ts->vkeys[i]));
  int v = 0, a = 0;
  ts->keep[0] = 0;
  for (;;) {
    int c = -1;
    for (int u = v + 1; u < N && c < 0; ++u)
      if (ts->vpar[u] == v && ts->vtok[u] == am[v]) c = u;
    if (c < 0 || a >= MAXK) break;
    st->acc[a++] = ts->vtok[c];
    ts->keep[a] = c;
    v = c;
  }
  const int next = am[v];
  st->acc[a] = next;
  st->a = a;
  st->n_out = a + 1;
  st->L_upd = a + 1;
  st->x_n = next;
  ts->n_keep = a + 1;
  ts->n_new = st->n + a + 1;
  for (int i = 0; i < TR_MAXV; ++i) ts->vkeys[i] = 0ull;
  if (p.out_host_view) {
    p.out_host_view[0] = a + 1;
    for (int i = 0; i <= a; ++i) p.out_host_view[1 + i] = st->acc[i];
  }
}

// KVCache::compact for every layer and KV head of a cache: rows n + keep[i] -> n + i. One thread
// owns the same 16-byte piece of every row and moves the rows in increasing i; keep[] increases
// and keep[i] >= i, so a row is read before any step overwrites it.
struct TreeCompactParams {
  const TreeState* ts;
  const RoundState* st;
  void* K;
  void* V;
  long long layer_elems;  // elements per layer: Hk * cap * D
  long long stride_h;     // elements per KV head: cap * D
  int D;
  int esize;              // bytes per element
  int cap;
};

__global__ void tree_compact_kernel(__grid_constant__ const TreeCompactParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int layer = blockIdx.x, hk = blockIdx.y;
  const int nk = p.ts->n_keep, n = p.st->n;
  const int pieces = p.D * p.esize / 16;
  if (n + p.ts->N > p.cap) return;  // the verify raised kErrCapacity already
  for (int which = 0; which < 2; ++which) {
    char* base = static_cast<char*>(which ? p.V : p.K) +
                 (size_t(layer) * p.layer_elems + size_t(hk) * p.stride_h) * p.esize;
    for (int c = threadIdx.x; c < pieces; c += blockDim.x)
      for (int i = 1; i < nk; ++i) {
        const int src = p.ts->keep[i];
        if (src == i) continue;
        const uint4 x = *reinterpret_cast<const uint4*>(base + (size_t(n + src) * p.D * p.esize) + c * 16);
        *reinterpret_cast<uint4*>(base + (size_t(n + i) * p.D * p.esize) + c * 16) = x;
      }
  }
}

// The kept rows' taps [3][i][Ht] for the drafter update; then the committed length advances
// (the compaction before this kernel read the old one).
struct TreeTapsParams {
  TreeState* ts;
  RoundState* st;
  const float* in;   // [3][rows][Ht]
  float* out;        // [3][rows][Ht]
  int rows;
  int Ht;
};

__global__ void tree_taps_kernel(__grid_constant__ const TreeTapsParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int f = blockIdx.x, i = blockIdx.y;
  if (f == 0 && i == 0 && threadIdx.x == 0) p.st->n = p.ts->n_new;
  if (i >= p.ts->n_keep) return;
  const float* src = p.in + (size_t(f) * p.rows + p.ts->keep[i]) * p.Ht;
  float* dst = p.out + (size_t(f) * p.rows + i) * p.Ht;
  for (int k = threadIdx.x; k < p.Ht; k += blockDim.x) dst[k] = src[k];
}

}  // namespace wc
