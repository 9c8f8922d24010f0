// Small kernels of the round and of the ops API: embedding gathers, row ops,
// acceptance (greedy / stochastic), KV append / read / compaction and the device
// bookkeeping that lets a whole round replay from one CUDA graph.
#pragma once

#include "common.cuh"

namespace wc {

constexpr int MAXK = 16;     // longest chain per round
constexpr int MAXKEYS = 2 * MAXK + 2;
constexpr int MAXTREE = 64;  // tree nodes per acceptance call

// Device-resident decoder state (one per decoder). The host reads it only at the
// round's single synchronisation.
struct RoundState {
  int n;        // committed tokens before x_n == target cache size
  int dc_len;   // drafter cache size (real entries)
  int x_n;      // newest committed token (not yet in the target cache)
  int a;        // drafts accepted by the last round
  int n_out;    // tokens emitted by the last round (a + 1)
  int L_upd;    // rows of the drafter update (a + 1)
  int err;      // device error word
  int pad;
  int tokens[MAXK + 1];   // verify input [x_n, d_1..d_K]
  int acc[MAXK + 1];      // accepted tokens d_1..d_a, next
  int forced[MAXK];       // oracle-drafter tokens (-1 = drafter's own)
  unsigned long long keys[MAXKEYS];  // argmax keys: draft steps [0, K), verify rows [K, 2K+1)
  unsigned long long draft_keys[MAXK];  // the last round's draft-step keys, kept when keys reset
  unsigned long long rng[2];         // sampled decoding: Philox seed, counter base of the next round
  float temperature;                 // sampled decoding: T (0 = greedy)
  int top_k;                         // sampled decoding: top-k warping of the target (0 = off)
  float top_p;                       // sampled decoding: top-p warping of the target (1 = off)
  int pad2;
};

// ----------------------------------------------------------------------------- activation packing

// Writes the GEMV input form of L rows (one block per row): fragments of x * w (bf16 models)
// or fp32 rows x * w [16][K] (fp32 models), the row's sum of squares of x into ss[l]
// (a single-part statistic), and optionally an fp32 copy of x. Rows come from fp32
// activations (src + l * ld) or from an embedding table gathered by token id; for the
// verify input the tokens are [x_n, d_1..d_K] resolved from the round state.
struct PackParams {
  const float* src;
  const int* row_map;  // source row of output row l: src + row_map[l] * ld (nullptr = l)
  int ld;
  const void* table;   // [vocab][K] of table_dtype (when src == nullptr)
  int table_dtype;
  const int* tokens;
  RoundState* st;      // tokens from the round state (verify input)
  const int* vocab_map;
  int vocab;
  int K;
  int L;
  const int* L_dev;
  const float* w;      // scale written into the fragments (norm gain) or nullptr
  uint32_t* xf;        // rows in the model's fragment format
  int xf_width;        // fragment width (bf16: K padded to whole slabs)
  int xf_fp32;
  float* ss;           // [16] or nullptr
  float* copy;         // [L][K] fp32 copy of x or nullptr
  int* err;
};

__global__ void pack_rows_kernel(__grid_constant__ const PackParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int l = blockIdx.x;
  const int L = p.L_dev ? *p.L_dev : p.L;
  if (l >= L) return;
  __shared__ int s_tok;
  __shared__ float red[32];
  if (threadIdx.x == 0) {
    int tok = 0;
    if (!p.src) {
      if (p.st) {
        if (l == 0) tok = p.st->x_n;
        else if (p.st->forced[l - 1] >= 0) tok = p.st->forced[l - 1];
        else {
          const uint32_t idx = argmax_key_index(p.st->keys[l - 1]);
          tok = p.vocab_map ? p.vocab_map[idx] : int(idx);
        }
      } else {
        tok = p.tokens[l];
      }
      if (tok < 0 || tok >= p.vocab) {
        raise_error(p.st ? &p.st->err : p.err, kErrTokenRange);
        tok = 0;
      }
      if (p.st) p.st->tokens[l] = tok;
    }
    s_tok = tok;
  }
  __syncthreads();
  float ss = 0.f;
  for (int k = threadIdx.x; k < p.K; k += blockDim.x) {
    float v;
    if (p.src) v = p.src[size_t(p.row_map ? p.row_map[l] : l) * p.ld + k];
    else {
      const size_t o = size_t(s_tok) * p.K + k;
      v = p.table_dtype == 1 ? bf16_bits_to_f32(static_cast<const uint16_t*>(p.table)[o])
                             : static_cast<const float*>(p.table)[o];
    }
    ss = fmaf(v, v, ss);
    if (p.copy) p.copy[size_t(l) * p.K + k] = v;
    const float x = p.w ? v * p.w[k] : v;
    if (p.xf_fp32) reinterpret_cast<float*>(p.xf)[size_t(l) * p.K + k] = x;
    else xf_store(p.xf, p.xf_width, l, k, x);
  }
  if (p.ss) {
    ss = warp_sum(ss);
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float a = 0.f;
      for (int w = 0; w < int(blockDim.x / 32); ++w) a += red[w];
      p.ss[l] = a;
    }
  }
}

// 1/rms of every row of an embedding table (the drafter's auxiliary-stream norm per token)
__global__ void row_inv_kernel(const void* table, int dtype, int rows, int K, float eps, float* out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (warp >= rows) return;
  double ss = 0.0;
  for (int k = lane; k < K; k += 32) {
    const size_t o = size_t(warp) * K + k;
    const float v = dtype == 1 ? bf16_bits_to_f32(static_cast<const uint16_t*>(table)[o]) : static_cast<const float*>(table)[o];
    ss += double(v) * double(v);
  }
  ss = warp_sum_d(ss);
  if (lane == 0) out[warp] = 1.f / sqrtf(float(ss / K) + eps);
}

// ----------------------------------------------------------------------------- ops API row kernels

// y = x * rsqrt(mean(x^2) + eps) * w with a double sum of squares (cpu_ops.cpp:50-59)
__global__ void rmsnorm_rows_kernel(const float* x, float* y, int d, const float* w, float eps) {
  const size_t r = blockIdx.x;
  const float* xr = x + r * d;
  float* yr = y + r * d;
  __shared__ double red[32];
  double ss = 0.0;
  for (int i = threadIdx.x; i < d; i += blockDim.x) ss += double(xr[i]) * double(xr[i]);
  ss = warp_sum_d(ss);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    double v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.0;
    v = warp_sum_d(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = 1.f / sqrtf(float(red[0] / d) + eps);
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x) yr[i] = xr[i] * inv * w[i];
}

// rotate-half RoPE on x[L][heads][D] with a host-built (cos, sin) table [max_pos][D/2]
__global__ void rope_rows_kernel(float* x, int heads, int D, const int* positions, const float2* table, int max_pos,
                                 int* err) {
  const int l = blockIdx.x, half = D / 2;
  int pos = positions[l];
  if (pos < 0 || pos >= max_pos) {
    if (threadIdx.x == 0) raise_error(err, kErrPosition);
    return;
  }
  const float2* row = table + size_t(pos) * half;
  for (int idx = threadIdx.x; idx < heads * half; idx += blockDim.x) {
    const int h = idx / half, i = idx % half;
    float* v = x + (size_t(l) * heads + h) * D;
    const float x1 = v[i], x2 = v[i + half];
    v[i] = x1 * row[i].x - x2 * row[i].y;
    v[i + half] = x2 * row[i].x + x1 * row[i].y;
  }
}

__global__ void silu_mul_kernel(float* g, const float* u, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float v = g[i];
    g[i] = v / (1.f + expf(-v)) * u[i];
  }
}

// one row in place; -inf -> 0; double sum (cpu_ops.cpp:86-96)
__global__ void softmax_row_kernel(float* x, int n) {
  __shared__ float fmax_s[32];
  __shared__ double dsum_s[32];
  const int tid = threadIdx.x, nw = blockDim.x / 32;
  float m = -INFINITY;
  for (int i = tid; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
  m = warp_max(m);
  if (tid % 32 == 0) fmax_s[tid / 32] = m;
  __syncthreads();
  if (tid < 32) {
    float v = tid < nw ? fmax_s[tid] : -INFINITY;
    v = warp_max(v);
    if (tid == 0) fmax_s[0] = v;
  }
  __syncthreads();
  m = fmax_s[0];
  double s = 0.0;
  for (int i = tid; i < n; i += blockDim.x) {
    const float v = x[i];
    const float e = (isinf(v) && v < 0.f) ? 0.f : expf(v - m);
    x[i] = e;
    s += e;
  }
  s = warp_sum_d(s);
  if (tid % 32 == 0) dsum_s[tid / 32] = s;
  __syncthreads();
  if (tid < 32) {
    double v = tid < nw ? dsum_s[tid] : 0.0;
    v = warp_sum_d(v);
    if (tid == 0) dsum_s[0] = v;
  }
  __syncthreads();
  const float inv = float(1.0 / dsum_s[0]);
  for (int i = tid; i < n; i += blockDim.x) x[i] *= inv;
}

__global__ void argmax_rows_kernel(const float* x, int n, int* out) {
  __shared__ unsigned long long best;
  if (threadIdx.x == 0) best = 0ull;
  __syncthreads();
  const float* xr = x + size_t(blockIdx.x) * n;
  unsigned long long k = 0ull;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const unsigned long long c = argmax_key(xr[i], uint32_t(i));
    if (c > k) k = c;
  }
  atomicMax(&best, k);
  __syncthreads();
  if (threadIdx.x == 0) out[blockIdx.x] = int(argmax_key_index(best));
}

__global__ void keys_to_index_kernel(const unsigned long long* keys, int n, const int* vocab_map, int* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const uint32_t idx = argmax_key_index(keys[i]);
    out[i] = vocab_map ? vocab_map[idx] : int(idx);
  }
}

// ----------------------------------------------------------------------------- KV arena

// k, v [L][Hk][D] fp32 -> arena rows [start, start+L) of one layer ([Hk][cap][D])
__global__ void kv_append_kernel(void* K, void* V, int dtype, int Hk, int D, int cap, int start, const float* k,
                                 const float* v, int L) {
  const size_t total = size_t(L) * Hk * D;
  for (size_t idx = blockIdx.x * size_t(blockDim.x) + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
    const int d = int(idx % D), h = int((idx / D) % Hk), l = int(idx / (size_t(D) * Hk));
    const size_t dst = (size_t(h) * cap + start + l) * D + d;
    if (dtype == 1) {
      static_cast<uint16_t*>(K)[dst] = f32_to_bf16_bits(k[idx]);
      static_cast<uint16_t*>(V)[dst] = f32_to_bf16_bits(v[idx]);
    } else {
      static_cast<float*>(K)[dst] = k[idx];
      static_cast<float*>(V)[dst] = v[idx];
    }
  }
}

__global__ void kv_read_kernel(const void* K, const void* V, int dtype, int Hk, int D, int cap, int T, float* k,
                               float* v) {
  const size_t total = size_t(T) * Hk * D;
  for (size_t idx = blockIdx.x * size_t(blockDim.x) + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
    const int d = int(idx % D), h = int((idx / D) % Hk), t = int(idx / (size_t(D) * Hk));
    const size_t src = (size_t(h) * cap + t) * D + d;
    if (dtype == 1) {
      k[idx] = bf16_bits_to_f32(static_cast<const uint16_t*>(K)[src]);
      v[idx] = bf16_bits_to_f32(static_cast<const uint16_t*>(V)[src]);
    } else {
      k[idx] = static_cast<const float*>(K)[src];
      v[idx] = static_cast<const float*>(V)[src];
    }
  }
}

// In-place compaction: rows start+keep[i] -> start+i for every (layer, head, K|V) slab.
// One block per slab stages all kept rows in shared memory before writing, so the
// result equals the reference's increasing-order memmove (kv_cache.cpp:21-31) for any
// keep list (dst <= src aliasing included).
__global__ void kv_compact_kernel(void* K, void* V, int dtype, int D, int cap, int slabs, const int* keep, int n_keep,
                                  int start) {
  extern __shared__ float stage[];  // [n_keep][D]
  const int slab = blockIdx.x;      // layer * Hk + head, K then V
  const bool is_v = slab >= slabs;
  void* base = is_v ? V : K;
  const size_t slab_off = size_t(is_v ? slab - slabs : slab) * cap * D;
  for (int idx = threadIdx.x; idx < n_keep * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    const size_t src = slab_off + size_t(start + keep[i]) * D + d;
    stage[idx] = dtype == 1 ? bf16_bits_to_f32(static_cast<const uint16_t*>(base)[src]) : static_cast<const float*>(base)[src];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < n_keep * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    const size_t dst = slab_off + size_t(start + i) * D + d;
    if (dtype == 1) static_cast<uint16_t*>(base)[dst] = f32_to_bf16_bits(stage[idx]);
    else static_cast<float*>(base)[dst] = stage[idx];
  }
}

// ----------------------------------------------------------------------------- acceptance

// verify_tree_greedy (sampling.cpp:95-106): from the root, follow the first child (in
// node order = draw order) whose token equals the target argmax at the current node.
__global__ void accept_greedy_tree_kernel(const int* am, const int* tokens, const int* parents, int N, int* out_path,
                                          int* out_n, int* out_next, int* err) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  for (int v = 1; v < N; ++v)
    if (parents[v] < 0 || parents[v] >= v) {
      raise_error(err, kErrTree);
      *out_n = 0;
      *out_next = am[0];
      return;
    }
  int v = 0, np = 0;
  while (true) {
    const int want = am[v];
    int nxt = -1;
    for (int c = v + 1; c < N; ++c)
      if (parents[c] == v && tokens[c] == want) {
        nxt = c;
        break;
      }
    if (nxt < 0) {
      *out_n = np;
      *out_next = want;
      return;
    }
    out_path[np++] = nxt;
    v = nxt;
  }
}

// Block-wide fp64 sum over n values (1024 threads).
__device__ double block_sum_d(double v, double* red) {
  v = warp_sum_d(v);
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    double x = lane < int(blockDim.x / 32) ? red[lane] : 0.0;
    x = warp_sum_d(x);
    if (lane == 0) red[32] = x;
  }
  __syncthreads();
  return red[32];
}

// Inverse-CDF draw: first i with cumsum(p)[i] > u * sum(p) (np.searchsorted side="right"),
// clipped to n-1 (sampling.py:190-193). Each thread owns a contiguous chunk; for n up
// to 4096 thread 0 scans alone, so the cumsum is the reference's sequential one.
__device__ int block_sample(const double* p, int n, double u, double* red, int* sel) {
  const int tid = threadIdx.x, nt = blockDim.x;
  if (n <= 4096) {
    if (tid == 0) {
      double tot = 0.0;
      for (int i = 0; i < n; ++i) tot += p[i];
      const double target = u * tot;
      double c = 0.0;
      int r = n - 1;
      for (int i = 0; i < n; ++i) {
        c += p[i];
        if (c > target) {
          r = i;
          break;
        }
      }
      *sel = r;
    }
    __syncthreads();
    const int r = *sel;
    __syncthreads();
    return r;
  }
  const int chunk = (n + nt - 1) / nt;
  const int i0 = min(n, tid * chunk), i1 = min(n, i0 + chunk);
  double s = 0.0;
  for (int i = i0; i < i1; ++i) s += p[i];
  // exclusive prefix over chunk sums (in shared memory, sequential per warp leader)
  __shared__ double chunk_sum[1024];
  chunk_sum[tid] = s;
  __syncthreads();
  if (tid == 0) {
    double c = 0.0;
    for (int t = 0; t < nt; ++t) {
      const double x = chunk_sum[t];
      chunk_sum[t] = c;
      c += x;
    }
    red[33] = c;  // total
    *sel = n - 1;
  }
  __syncthreads();
  const double target = u * red[33];
  double c = chunk_sum[tid];
  for (int i = i0; i < i1; ++i) {
    c += p[i];
    if (c > target) {
      atomicMin(sel, i);
      break;
    }
  }
  __syncthreads();
  const int r = *sel;
  __syncthreads();
  return r;
}

// verify_tree_stochastic (sampling.py:143-177) with Philox uniforms. Single block.
// pw, qw: scratch [V] fp64 each.
__global__ void __launch_bounds__(1024) accept_stochastic_tree_kernel(
    const double* p, const double* q, int V, const int* tokens, const int* parents, int N, uint64_t seed,
    uint64_t offset, double* pw, double* qw, int* out_path, int* out_n, int* out_next, int* out_used, int* err) {
  __shared__ double red[40];
  __shared__ int sel;
  const int tid = threadIdx.x;
  for (int v = 1; v < N; ++v)
    if (parents[v] < 0 || parents[v] >= v || tokens[v] < 0 || tokens[v] >= V) {
      if (tid == 0) {
        raise_error(err, kErrTree);
        *out_n = 0;
        *out_next = 0;
        *out_used = 0;
      }
      return;
    }
  uint64_t ctr = offset;
  int v = 0, np = 0;
  while (true) {
    for (int i = tid; i < V; i += blockDim.x) pw[i] = p[size_t(v) * V + i];
    __syncthreads();
    bool has_kids = false;
    for (int c = v + 1; c < N; ++c) has_kids |= parents[c] == v;
    if (!has_kids) {
      const double u = philox_uniform(seed, ctr++);
      const int r = block_sample(pw, V, u, red, &sel);
      if (tid == 0) {
        *out_n = np;
        *out_next = r;
        *out_used = int(ctr - offset);
      }
      return;
    }
    for (int i = tid; i < V; i += blockDim.x) qw[i] = q[size_t(v) * V + i];
    __syncthreads();
    int accepted = -1;
    for (int c = v + 1; c < N; ++c) {
      if (parents[c] != v) continue;
      const int x = tokens[c];
      const double qx = qw[x];
      if (qx > 0) {
        const double u = philox_uniform(seed, ctr++);
        const double ratio = pw[x] / qx;
        if (u < (ratio < 1.0 ? ratio : 1.0)) {
          accepted = c;
          break;
        }
      }
      // p <- norm(max(p - q, 0)), or p / sum(p) when that mass is <= 1e-12
      double s = 0.0;
      for (int i = tid; i < V; i += blockDim.x) s += fmax(pw[i] - qw[i], 0.0);
      s = block_sum_d(s, red);
      if (s <= 1e-12) {
        double tp = 0.0;
        for (int i = tid; i < V; i += blockDim.x) tp += pw[i];
        tp = block_sum_d(tp, red);
        for (int i = tid; i < V; i += blockDim.x) pw[i] = pw[i] / tp;
      } else {
        for (int i = tid; i < V; i += blockDim.x) pw[i] = fmax(pw[i] - qw[i], 0.0) / s;
      }
      __syncthreads();
      if (tid == 0) qw[x] = 0.0;
      __syncthreads();
      double sq = 0.0;
      for (int i = tid; i < V; i += blockDim.x) sq += qw[i];
      sq = block_sum_d(sq, red);
      if (sq <= 0) break;
      for (int i = tid; i < V; i += blockDim.x) qw[i] /= sq;
      __syncthreads();
    }
    if (accepted < 0) {
      const double u = philox_uniform(seed, ctr++);
      const int r = block_sample(pw, V, u, red, &sel);
      if (tid == 0) {
        *out_n = np;
        *out_next = r;
        *out_used = int(ctr - offset);
      }
      return;
    }
    if (tid == 0) out_path[np] = accepted;
    ++np;
    v = accepted;
    __syncthreads();
  }
}

__global__ void philox_uniforms_kernel(uint64_t seed, uint64_t offset, int n, double* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = philox_uniform(seed, offset + uint64_t(i));
}

// ----------------------------------------------------------------------------- drafter auxiliary table
// GEMM operand rows for the per-token auxiliary term: row i = token r0 + i, columns [0, H) zero
// (the feature half of the layer-0 Q/K/V weight), columns [H, 2H) the bf16 high (lo = 0) or low
// (lo = 1) part of embed[t] * (1/rms of the row) * aux_norm, so two GEMMs add up to the fp32 value.
__global__ void aux_rows_kernel(const uint16_t* embed, const float* row_inv, const float* aux_norm, int r0, int H,
                                int lo, uint16_t* out) {
  const int i = blockIdx.x, t = r0 + i;
  const uint16_t* e = embed + size_t(t) * H;
  uint16_t* o = out + size_t(i) * 2 * H;
  const float inv = row_inv[t];
  for (int k = threadIdx.x; k < H; k += blockDim.x) {
    const float x = bf16_bits_to_f32(e[k]) * inv * aux_norm[k];
    const uint16_t hi = f32_to_bf16_bits(x);
    o[k] = 0;
    o[H + k] = lo ? f32_to_bf16_bits(x - bf16_bits_to_f32(hi)) : hi;
  }
}

// ----------------------------------------------------------------------------- bounded-wait self test
// Waits, with the same bounded helper every pipelined kernel uses, on an mbarrier phase that
// nothing completes: after `iters` tries the wait gives up and the kernel raises kErrTimeout in
// the error word and returns, which the host reads at its next synchronisation.
__global__ void wait_selftest_kernel(int* err, uint32_t iters) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait(&bar, 0, iters)) raise_error(err, kErrTimeout);
}

// ----------------------------------------------------------------------------- round bookkeeping

// Greedy chain acceptance (python/woodcock/spec.py:357-362): longest prefix of drafts
// equal to the target argmax, plus the target token at the first mismatch. Chain
// compaction keeps rows 0..a, i.e. the target cache size becomes n + a + 1 (no data
// moves). Resets every argmax key for the next round.
__global__ void accept_chain_kernel(RoundState* st, int K, const int* vocab_map_unused, int* out_host_view) {
  pdl_launch_dependents();
  pdl_wait();
  if (threadIdx.x != 0) return;
  int am[MAXK + 1];
  for (int i = 0; i <= K; ++i) am[i] = int(argmax_key_index(st->keys[K + i]));
  int a = 0;
  while (a < K && st->tokens[a + 1] == am[a]) ++a;
  const int next = am[a];
  for (int i = 0; i < a; ++i) st->acc[i] = st->tokens[i + 1];
  st->acc[a] = next;
  st->a = a;
  st->n_out = a + 1;
  st->L_upd = a + 1;
  st->n += a + 1;
  st->x_n = next;
  for (int i = 0; i < K; ++i) st->draft_keys[i] = st->keys[i];
  for (int i = 0; i < MAXKEYS; ++i) st->keys[i] = 0ull;
  if (out_host_view) {
    out_host_view[0] = a + 1;
    for (int i = 0; i <= a; ++i) out_host_view[1 + i] = st->acc[i];
  }
  (void)vocab_map_unused;
}

// ----------------------------------------------------------------------------- sampled rounds
// probs_from_logits (sampling.py:39-55) as one threshold per row: with x = z / T, top-k keeps
// x >= (k-th largest x) and top-p then keeps the largest x whose descending cumulative
// softmax mass, counted before each of them, stays below top_p; both are "x >= thr", so the
// warped distribution is p_j = [x_j >= thr] exp(x_j - M) / Z. Rows whose values tie exactly
// at the threshold keep every tied token (the reference breaks such ties by sort position).
struct RowWarp {
  float M;    // max of x
  float thr;  // -inf: no warping
  double Z;   // sum of exp(x - M) over the kept tokens
};

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float order_key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

struct WarpParams {
  const float* z;  // [R][ld]
  int V, ld;
  const float* temperature;
  const int* top_k;
  const float* top_p;
  RowWarp* out;                  // [R]
  unsigned long long* zero_keys; // cleared here (the keys a later draw accumulates into)
  int zero_n;
};

template <class T, class Op>
__device__ __forceinline__ T block_reduce(T v, T* red, Op op) {
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = v;
  __syncthreads();
  T a = red[0];
  for (int w = 1; w < int(blockDim.x / 32); ++w) a = op(a, red[w]);
  return a;
}

// One block per row: max, then the top-k key by a count radix select (4 passes of 8 bits),
// the kept mass, the top-p key by a mass radix select, the final normaliser.
__global__ void __launch_bounds__(1024) warp_rows_kernel(__grid_constant__ const WarpParams p) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ unsigned cnt[256];
  __shared__ double mass[256];
  __shared__ float red_f[32];
  __shared__ double red_d[32];
  __shared__ uint32_t s_prefix;
  __shared__ unsigned long long s_above;
  __shared__ double s_above_m;
  __shared__ int s_found;
  const int row = blockIdx.x, tid = threadIdx.x;
  if (row == 0 && p.zero_keys && tid < p.zero_n) p.zero_keys[tid] = 0ull;
  const float* z = p.z + size_t(row) * p.ld;
  const float T = *p.temperature;
  const int k = p.top_k ? *p.top_k : 0;
  const float tp = p.top_p ? *p.top_p : 1.f;
  float m = -INFINITY;
  for (int j = tid; j < p.V; j += blockDim.x) m = fmaxf(m, z[j] / T);
  const float M = block_reduce(m, red_f, [](float a, float b) { return fmaxf(a, b); });
  uint32_t keep_key = 0u;  // elements with order_key(x) >= keep_key stay
  if (k > 0 && k < p.V) {  // the k-th largest x
    uint32_t prefix = 0u;
    unsigned long long above = 0ull;
    for (int shift = 24; shift >= 0; shift -= 8) {
      const uint32_t hi = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int b = tid; b < 256; b += blockDim.x) cnt[b] = 0u;
      __syncthreads();
      for (int j = tid; j < p.V; j += blockDim.x) {
        const uint32_t key = order_key(z[j] / T);
        if ((key & hi) == (prefix & hi)) atomicAdd(&cnt[(key >> shift) & 255u], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        int b = 255;
        for (; b > 0; --b) {
          if (above + cnt[b] >= (unsigned long long)k) break;
          above += cnt[b];
        }
        s_prefix = prefix | (uint32_t(b) << shift);
        s_above = above;
      }
      __syncthreads();
      prefix = s_prefix;
      above = s_above;
    }
    keep_key = prefix;
  }
  double s1 = 0.0;
  for (int j = tid; j < p.V; j += blockDim.x) {
    const float x = z[j] / T;
    if (order_key(x) >= keep_key) s1 += exp(double(x) - double(M));
  }
  const double S1 = block_reduce(s1, red_d, [](double a, double b) { return a + b; });
  if (tp < 1.f) {  // the largest x at which the descending inclusive mass reaches top_p
    const double target = double(tp) * S1;
    uint32_t prefix = 0u;
    double above_m = 0.0;
    bool found = true;
    for (int shift = 24; shift >= 0 && found; shift -= 8) {
      const uint32_t hi = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int b = tid; b < 256; b += blockDim.x) mass[b] = 0.0;
      __syncthreads();
      for (int j = tid; j < p.V; j += blockDim.x) {
        const float x = z[j] / T;
        const uint32_t key = order_key(x);
        if (key >= keep_key && (key & hi) == (prefix & hi)) atomicAdd(&mass[(key >> shift) & 255u], exp(double(x) - double(M)));
      }
      __syncthreads();
      if (tid == 0) {
        int b = 255;
        bool hit = false;
        for (; b >= 0; --b) {
          if (above_m + mass[b] >= target) {
            hit = true;
            break;
          }
          above_m += mass[b];
        }
        s_found = hit ? 1 : 0;
        s_prefix = prefix | (uint32_t(hit ? b : 0) << shift);
        s_above_m = above_m;
      }
      __syncthreads();
      found = s_found != 0;
      prefix = s_prefix;
      above_m = s_above_m;
    }
    if (found && prefix > keep_key) keep_key = prefix;
  }
  double zs = 0.0;
  for (int j = tid; j < p.V; j += blockDim.x) {
    const float x = z[j] / T;
    if (order_key(x) >= keep_key) zs += exp(double(x) - double(M));
  }
  const double Z = block_reduce(zs, red_d, [](double a, double b) { return a + b; });
  if (tid == 0) p.out[row] = RowWarp{M, keep_key ? order_key_value(keep_key) : -INFINITY, Z};
}

// probs_from_logits (sampling.py:39-55) from the warp thresholds: p_j = [x_j >= thr] exp(x_j - M) / Z
__global__ void warped_probs_kernel(const float* z, int V, const float* temperature, const RowWarp* warp, float* out) {
  const int row = blockIdx.y;
  const RowWarp w = warp[row];
  const float T = *temperature;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < V; j += gridDim.x * blockDim.x) {
    const float x = z[size_t(row) * V + j] / T;
    out[size_t(row) * V + j] = x >= w.thr ? float(exp(double(x) - double(w.M)) / w.Z) : 0.f;
  }
}

// Gumbel-max draws over the kept tokens of warped rows (the warped autoregressive step and
// first token): keys[row] = argmax over x_j >= thr of (x_j + Gumbel), stream `stream` + row.
struct SampleRowsParams {
  const float* z;
  int V, ld;
  const float* temperature;
  const RowWarp* warp;
  const unsigned long long* rng;
  int stream;
  unsigned long long* keys;
};

__global__ void __launch_bounds__(256) sample_rows_kernel(__grid_constant__ const SampleRowsParams p) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ unsigned long long s_best;
  const int row = blockIdx.y;
  const float* z = p.z + size_t(row) * p.ld;
  const float T = *p.temperature, thr = p.warp[row].thr;
  const uint64_t seed = p.rng[0], base = p.rng[1] + uint64_t(p.stream + row) * kRngStreamLen;
  if (threadIdx.x == 0) s_best = 0ull;
  __syncthreads();
  const int chunk = (p.V + gridDim.x - 1) / gridDim.x;
  const int j0 = min(p.V, int(blockIdx.x) * chunk), j1 = min(p.V, j0 + chunk);
  unsigned long long best = 0ull;
  for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
    const float x = z[j] / T;
    if (!(x >= thr)) continue;
    const unsigned long long key = argmax_key(x + philox_gumbel_f(seed, base + uint64_t(j)), uint32_t(j));
    if (key > best) best = key;
  }
  if (best) atomicMax(&s_best, best);
  __syncthreads();
  if (threadIdx.x == 0 && s_best) atomicMax(&p.keys[row], s_best);
}
// Softmax statistics of logit rows at temperature T, in slices: block b of a row's nb blocks
// writes (max of z / T, sum of exp(z / T - max)) over its slice. Rows [0, R1) are z1 (length
// V1, row stride V1), then rows [R1, R1 + R2) are z2 (length V2).
struct StatsParams {
  const float* z1;
  int R1, V1, nb1;
  const float* z2;
  int R2, V2, nb2;
  const float* temperature;  // T on the device
  float2* out;               // [R1 * nb1 + R2 * nb2]
};

__global__ void __launch_bounds__(256) logit_stats_kernel(__grid_constant__ const StatsParams p) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32];
  const int b = blockIdx.x;
  const float* z;
  int V, nb, i;
  if (b < p.R1 * p.nb1) {
    z = p.z1 + size_t(b / p.nb1) * p.V1;
    V = p.V1;
    nb = p.nb1;
    i = b % p.nb1;
  } else {
    const int b2 = b - p.R1 * p.nb1;
    z = p.z2 + size_t(b2 / p.nb2) * p.V2;
    V = p.V2;
    nb = p.nb2;
    i = b2 % p.nb2;
  }
  const int chunk = (V + nb - 1) / nb, j0 = min(V, i * chunk), j1 = min(V, j0 + chunk);
  const float T = *p.temperature;
  float m = -INFINITY;
  for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) m = fmaxf(m, z[j] / T);
  m = warp_max(m);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = m;
  __syncthreads();
  float M = -INFINITY;
  for (int w = 0; w < int(blockDim.x / 32); ++w) M = fmaxf(M, red[w]);
  __syncthreads();
  float e = 0.f;
  if (M != -INFINITY)
    for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) e += expf(z[j] / T - M);
  e = warp_sum(e);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = e;
  __syncthreads();
  if (threadIdx.x == 0) {
    float S = 0.f;
    for (int w = 0; w < int(blockDim.x / 32); ++w) S += red[w];
    p.out[b] = make_float2(M, S);
  }
}

// Stochastic chain acceptance (sampling.py:69-82, the chain case of verify_tree_stochastic,
// sampling.py:143-177, with _residual 182-187) on the round's logits: target rows zt [K+1][V]
// at [x_n, d_1..d_K], draft rows zd [K][Vd] (the drafter head's rows; token j is row
// vocab_inv[j], or j without a restricted head). With p_i = softmax(zt_i / T) and
// q_i = softmax(zd_i / T): draft d_{i+1} is accepted when q_i(x) > 0 and u_i < min(1,
// p_i(x) / q_i(x)); at the first rejection (row a) the next token is drawn from
// norm(max(p_a - q_a, 0)) (from p_a when that mass is <= 1e-12), after K acceptances from p_K.
// The draw is the Gumbel-max over the token ids, sliced across the grid; every block repeats
// the (K-step) decision, and the last block to finish reduces the slices in block order and
// commits the round as accept_chain_kernel does, advancing the random counter base.
struct SampleAcceptParams {
  RoundState* st;
  int K;
  const float* zt;
  int V;
  const float* zd;
  int Vd;
  const int* vocab_inv;  // [V] or nullptr
  const float2* stats;   // logit_stats_kernel: target rows (nbt each, unless warped), then draft rows (nbd each)
  int nbt, nbd;
  const RowWarp* warp;   // warped target rows (top-k / top-p), or nullptr
  double* part;          // [gridDim][3]: residual mass, residual key, p key (bits)
  unsigned* counter;     // zero at launch; left at zero
  int* out_host_view;
};

__device__ __forceinline__ int sample_row_of(const SampleAcceptParams& p, int tok) {
  if (tok < 0 || tok >= p.V) return -1;
  if (p.vocab_inv) return p.vocab_inv[tok];
  return tok < p.Vd ? tok : -1;
}

__global__ void __launch_bounds__(256) accept_sampled_kernel(__grid_constant__ const SampleAcceptParams p) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ double sM[MAXK + 1], sS[MAXK + 1], dM[MAXK], dS[MAXK];
  __shared__ float sThr[MAXK + 1];
  __shared__ int s_a;
  __shared__ double red_d[32];
  __shared__ unsigned long long s_kr, s_kp;
  __shared__ bool s_last;
  RoundState* st = p.st;
  const int K = p.K, tid = threadIdx.x;
  const float T = st->temperature;
  const uint64_t seed = st->rng[0], base = st->rng[1];
  // ---- per-row statistics from the slices, in slice order
  if (tid < 2 * K + 1 && tid <= K && p.warp) {
    sM[tid] = p.warp[tid].M;
    sS[tid] = p.warp[tid].Z;
    sThr[tid] = p.warp[tid].thr;
  } else if (tid < 2 * K + 1) {
    const bool tgt = tid <= K;
    const int r = tgt ? tid : tid - K - 1, nb = tgt ? p.nbt : p.nbd;
    const size_t tslices = p.warp ? 0 : size_t(K + 1) * p.nbt;
    const float2* s = p.stats + (tgt ? size_t(r) * p.nbt : tslices + size_t(r) * p.nbd);
    if (tgt) sThr[r] = -INFINITY;
    double M = -INFINITY;
    for (int b = 0; b < nb; ++b) M = fmax(M, double(s[b].x));
    double S = 0.0;
    for (int b = 0; b < nb; ++b)
      if (s[b].x != -INFINITY) S += double(s[b].y) * exp(double(s[b].x) - M);
    if (tgt) {
      sM[r] = M;
      sS[r] = S;
    } else {
      dM[r] = M;
      dS[r] = S;
    }
  }
  if (tid == 0) {
    s_kr = 0ull;
    s_kp = 0ull;
  }
  __syncthreads();
  // ---- the decisions (identical in every block)
  if (tid == 0) {
    int a = 0;
    for (; a < K; ++a) {
      const int x = st->tokens[a + 1];
      const int row = sample_row_of(p, x);
      const double qx = row >= 0 ? exp(double(p.zd[size_t(a) * p.Vd + row] / T) - dM[a]) / dS[a] : 0.0;
      if (!(qx > 0.0)) break;
      const float xt = p.zt[size_t(a) * p.V + x] / T;
      const double px = xt >= sThr[a] ? exp(double(xt) - sM[a]) / sS[a] : 0.0;
      const double u = philox_uniform(seed, base + uint64_t(kRngAcceptStream) * kRngStreamLen + uint64_t(a));
      const double ratio = px / qx;
      if (!(u < (ratio < 1.0 ? ratio : 1.0))) break;
    }
    s_a = a;
  }
  __syncthreads();
  const int a = s_a;
  // ---- this block's slice of the residual (a < K) or bonus (a == K) draw
  const int chunk = (p.V + gridDim.x - 1) / gridDim.x;
  const int j0 = min(p.V, int(blockIdx.x) * chunk), j1 = min(p.V, j0 + chunk);
  const float* zr = p.zt + size_t(a) * p.V;
  const float* qr = a < K ? p.zd + size_t(a) * p.Vd : nullptr;
  double mass = 0.0;
  unsigned long long kr = 0ull, kp = 0ull;
  for (int j = j0 + tid; j < j1; j += blockDim.x) {
    const float xj = zr[j] / T;
    const double pj = xj >= sThr[a] ? exp(double(xj) - sM[a]) / sS[a] : 0.0;
    double rj = pj;
    if (qr) {
      const int row = sample_row_of(p, j);
      const double qj = row >= 0 ? exp(double(qr[row] / T) - dM[a]) / dS[a] : 0.0;
      rj = fmax(pj - qj, 0.0);
    }
    mass += rj;
    const double g = philox_gumbel_d(seed, base + uint64_t(kRngResidualStream) * kRngStreamLen + uint64_t(j));
    if (rj > 0.0) {
      const unsigned long long k = argmax_key(float(log(rj) + g), uint32_t(j));
      if (k > kr) kr = k;
    }
    if (pj > 0.0) {
      const unsigned long long k = argmax_key(float(log(pj) + g), uint32_t(j));
      if (k > kp) kp = k;
    }
  }
  mass = warp_sum_d(mass);
  if (tid % 32 == 0) red_d[tid / 32] = mass;
  if (kr) atomicMax(&s_kr, kr);
  if (kp) atomicMax(&s_kp, kp);
  __syncthreads();
  if (tid == 0) {
    double m2 = 0.0;
    for (int w = 0; w < int(blockDim.x / 32); ++w) m2 += red_d[w];
    double* pp = p.part + size_t(blockIdx.x) * 3;
    pp[0] = m2;
    pp[1] = __longlong_as_double((long long)s_kr);
    pp[2] = __longlong_as_double((long long)s_kp);
    __threadfence();
    s_last = atomicAdd(p.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last || tid != 0) return;
  // ---- last block: reduce the slices in block order and commit
  __threadfence();
  double m_all = 0.0;
  unsigned long long kr_all = 0ull, kp_all = 0ull;
  for (int b = 0; b < int(gridDim.x); ++b) {
    const double* pp = p.part + size_t(b) * 3;
    m_all += __ldcg(pp);
    const unsigned long long k1 = (unsigned long long)__double_as_longlong(__ldcg(pp + 1));
    const unsigned long long k2 = (unsigned long long)__double_as_longlong(__ldcg(pp + 2));
    if (k1 > kr_all) kr_all = k1;
    if (k2 > kp_all) kp_all = k2;
  }
  const bool use_p = a < K && !(m_all > 1e-12);
  const unsigned long long key = use_p ? kp_all : kr_all;
  int next = key ? int(argmax_key_index(key)) : 0;
  if (!key) raise_error(&st->err, kErrSample);
  for (int i = 0; i < a; ++i) st->acc[i] = st->tokens[i + 1];
  st->acc[a] = next;
  st->a = a;
  st->n_out = a + 1;
  st->L_upd = a + 1;
  st->n += a + 1;
  st->x_n = next;
  for (int i = 0; i < MAXKEYS; ++i) st->keys[i] = 0ull;
  st->rng[1] = base + kRngRoundStride;
  *p.counter = 0u;
  if (p.out_host_view) {
    p.out_host_view[0] = a + 1;
    for (int i = 0; i <= a; ++i) p.out_host_view[1 + i] = st->acc[i];
  }
}

// End of the drafter update (and of the drafter prefill): out = RMSNorm(h[L-1]) with the
// drafter's final norm; root_out (head input of the next round's first draft step) and
// root_fb (feature of its first drafter pass: out with post_norm, else h) as fp32 rows and
// as GEMV input fragments (root_fb times the layer-0 input norm gain, with its sum of
// squares); with advance_dc the drafter cache grows by L.
struct FinishParams {
  RoundState* st;
  const int* L_dev;
  int L_static;
  const float* h;
  int d;
  const float* norm_w;
  float eps;
  int post_norm;
  float* root_out;
  float* root_fb;
  uint32_t* xf_out;   // fragments of root_out (no scale)
  uint32_t* xf_fb;    // fragments of root_fb * in_norm0
  const float* in_norm0;
  float* ss_fb;       // [16]: row 0 = sum of root_fb^2
  int xf_width;       // fragment width (bf16: d padded to whole slabs)
  int xf_fp32;
  int advance_dc;
};

__global__ void finish_update_kernel(__grid_constant__ const FinishParams p) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32];
  __shared__ float s_inv;
  const int L = p.L_dev ? *p.L_dev : p.L_static;
  if (L < 1 || L > p.L_static) {
    if (threadIdx.x == 0) raise_error(&p.st->err, kErrRows);
    return;
  }
  const float* hr = p.h + size_t(L - 1) * p.d;
  float ss = 0.f;
  for (int i = threadIdx.x; i < p.d; i += blockDim.x) ss = fmaf(hr[i], hr[i], ss);
  ss = warp_sum(ss);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f;
    for (int w = 0; w < int(blockDim.x / 32); ++w) a += red[w];
    s_inv = 1.f / sqrtf(a / float(p.d) + p.eps);
  }
  __syncthreads();
  float sf = 0.f;
  for (int i = threadIdx.x; i < p.d; i += blockDim.x) {
    const float o = hr[i] * s_inv * p.norm_w[i];
    const float fb = p.post_norm ? o : hr[i];
    p.root_out[i] = o;
    p.root_fb[i] = fb;
    sf = fmaf(fb, fb, sf);
    if (p.xf_fp32) {
      reinterpret_cast<float*>(p.xf_out)[i] = o;
      reinterpret_cast<float*>(p.xf_fb)[i] = fb * p.in_norm0[i];
    } else {
      xf_store(p.xf_out, p.xf_width, 0, i, o);
      xf_store(p.xf_fb, p.xf_width, 0, i, fb * p.in_norm0[i]);
    }
  }
  sf = warp_sum(sf);
  __syncthreads();
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = sf;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f;
    for (int w = 0; w < int(blockDim.x / 32); ++w) a += red[w];
    p.ss_fb[0] = a;
    if (p.advance_dc) p.st->dc_len += L;
  }
}

}  // namespace wc
