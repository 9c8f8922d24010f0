// Skinny GEMM ("GEMV" over L <= 16 rows) for the decode round: y[L][N] = x[L][K] . W[N][K]^T.
//
// Weights stream from HBM exactly once per launch. The input x is assembled in the
// prologue from up to three segments, each a row source (fp32 activations or an
// embedding-table gather by token id) with an optional RMSNorm; this fuses the
// reference's rmsnorm -> linear pairs (src/core/qwen3.cpp:86-101,
// src/core/drafter.cpp:106-128) and the drafter's feature fusion (drafter.cpp:75-89).
// Epilogues: store, residual add (linear(..., accumulate=true)), SwiGLU
// (silu(gate)*up, cpu_ops.cpp:79-84) and a fused argmax over the output rows.
//
// bf16 weights: tensor-core mma.sync m16n8k16 with the weight as the A operand
// (16 output rows) and the activations as B (8 rows per n-tile). Weights are stored
// pre-tiled in A-fragment order (16x16 tile = 512 contiguous bytes, 16 bytes per lane),
// so every warp load is one fully coalesced 512-byte line. Activations are split
// into bf16 hi + lo terms (two MMAs per tile), which keeps them at fp32-level accuracy.
// fp32 weights: CUDA-core FMA, row-major [N][K].
//
// Latency hiding: each block owns a contiguous slice of row blocks. Before it waits
// on the previous kernel (programmatic dependent launch) it bulk-prefetches the start
// of its weight slice into L2, and keeps a prefetch window running ahead of the
// consumption; the activation prologue uses 16-byte loads that are all in flight at
// once, in two passes (RMSNorm statistics, then the bf16 hi/lo split into shared memory).
#pragma once

#include "common.cuh"

namespace wc {

enum Epilogue : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / kWarp;
constexpr int GEMV_KC = 2048;                    // k per shared-memory chunk
constexpr int GEMV_KTC = GEMV_KC / 16;           // k-tiles per chunk
constexpr int GEMV_TPW = GEMV_KTC / GEMV_WARPS;  // k-tiles per warp per chunk
constexpr int GEMV_RBB = 2;                      // row blocks per reduction batch
constexpr int GEMV_MAXL = 16;                    // rows per launch (2 n-tiles)
constexpr int GEMV_MAXSEG = 3;
constexpr long long GEMV_PREFETCH_WINDOW = 384 * 1024;  // bytes of its slice a block keeps in flight

struct Seg {
  const float* src;     // fp32 rows src + l*ld (when table == nullptr)
  const void* table;    // embedding table [vocab][len], row = resolved token of row l
  int table_dtype;      // 0 fp32, 1 bf16
  int ld;
  int len;
  const float* norm_w;  // RMSNorm gain or nullptr
  float* write_back;    // block 0 stores the (normalised) segment rows here when set
  int ld_wb;
};

// Per-row token ids for embedding segments: forced id (>= 0) > argmax key > plain id.
struct TokenSrc {
  const int* tokens;
  const unsigned long long* keys;
  const int* vocab_map;  // head row -> token id, nullptr = identity
  const int* forced;
  int* tok_out;          // block 0 stores the resolved ids here when set
  int vocab;
};

struct GemvParams {
  const void* w;
  int N;       // valid output rows
  int Np;      // padded rows (multiple of 16 * group for bf16)
  int K;       // valid input columns (a multiple of 4, segments too)
  int Kp;      // padded columns (multiple of 16 for bf16)
  int w_dtype;
  int L;
  const int* L_dev;  // dynamic row count (overrides L when set); rows <= L_max
  int L_max;
  int nseg;
  Seg seg[GEMV_MAXSEG];
  float eps;
  TokenSrc tok;
  int epi;
  float* y;
  int ldy;
  const float* base;  // EPI_ADD: y = base + acc (base may equal y)
  int ldb;
  float* y2;          // optional copy of the stored result (tap capture)
  int ldy2;
  unsigned long long* keys;  // EPI_ARGMAX
  int group;          // row blocks per epilogue unit: 2 for SwiGLU (gate block, up block)
  int* err;
};

__device__ __forceinline__ int gemv_rows(const GemvParams& p) {
  int L = p.L_dev ? *p.L_dev : p.L;
  if (L < 0 || L > p.L_max) {
    raise_error(p.err, kErrRows);
    L = L < 0 ? 0 : p.L_max;
  }
  return L;
}

__device__ __forceinline__ int resolve_token(const TokenSrc& t, int l, int* err) {
  int tok;
  if (t.forced && t.forced[l] >= 0) {
    tok = t.forced[l];
  } else if (t.keys) {
    const uint32_t idx = argmax_key_index(t.keys[l]);
    tok = t.vocab_map ? t.vocab_map[idx] : int(idx);
  } else {
    tok = t.tokens[l];
  }
  if (tok < 0 || tok >= t.vocab) {
    raise_error(err, kErrTokenRange);
    tok = 0;
  }
  return tok;
}

// 4 consecutive values (i multiple of 4) of row l of a segment.
__device__ __forceinline__ float4 seg_load4(const Seg& s, int l, int i, const int* toks) {
  if (s.table) {
    const size_t off = size_t(toks[l]) * size_t(s.len) + size_t(i);
    if (s.table_dtype == 1) {
      const uint2 u = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(s.table) + off);
      return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                         __uint_as_float(u.y & 0xFFFF0000u));
    }
    return *reinterpret_cast<const float4*>(static_cast<const float*>(s.table) + off);
  }
  return *reinterpret_cast<const float4*>(s.src + size_t(l) * size_t(s.ld) + size_t(i));
}

// Resolve tokens, then the per-(row, segment) RMSNorm scale: each thread owns columns
// 4*c4 of every row, all of its loads in flight at once; fixed-order block reduction.
__device__ void gemv_prologue_stats(const GemvParams& p, int L, int* s_tok, float* s_inv, float* s_red) {
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  bool need_tok = false;
  for (int s = 0; s < p.nseg; ++s) need_tok |= p.seg[s].table != nullptr;
  if (tid < L) {
    const int t = need_tok ? resolve_token(p.tok, tid, p.err) : 0;
    s_tok[tid] = t;
    if (need_tok && p.tok.tok_out && blockIdx.x == 0) p.tok.tok_out[tid] = t;
  }
  __syncthreads();
  for (int s = 0; s < p.nseg; ++s) {
    const Seg& sg = p.seg[s];
    if (!sg.norm_w) {
      if (tid < L) s_inv[tid * GEMV_MAXSEG + s] = 1.f;
      continue;
    }
    const int len4 = sg.len / 4;
    for (int l0 = 0; l0 < L; l0 += 4) {  // four rows at a time keeps the live registers small
      float ss[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c4 = tid; c4 < len4; c4 += GEMV_THREADS) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (l0 + u < L) v[u] = seg_load4(sg, l0 + u, c4 * 4, s_tok);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (l0 + u < L) ss[u] += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (l0 + u < L) {
          const float w = warp_sum(ss[u]);
          if (lane == 0) s_red[warp * GEMV_MAXL + l0 + u] = w;
        }
      }
    }
    __syncthreads();
    if (tid < L) {
      float tot = 0.f;
      for (int w = 0; w < GEMV_WARPS; ++w) tot += s_red[w * GEMV_MAXL + tid];
      s_inv[tid * GEMV_MAXSEG + s] = 1.f / sqrtf(tot / float(sg.len) + p.eps);
    }
    __syncthreads();
  }
}

__device__ __forceinline__ bool gemv_has_write_back(const GemvParams& p) {
  for (int s = 0; s < p.nseg; ++s)
    if (p.seg[s].write_back) return true;
  return false;
}

// Epilogue for one output element (row l of the activations, output feature n).
__device__ __forceinline__ void gemv_store(const GemvParams& p, int l, int n, float v) {
  if (p.epi == EPI_ADD) v += p.base[size_t(l) * p.ldb + n];
  p.y[size_t(l) * p.ldy + n] = v;
  if (p.y2) p.y2[size_t(l) * p.ldy2 + n] = v;
}

// Bulk L2 prefetch of bytes [b0, b1) of a block's weight slice, split over its warps.
__device__ __forceinline__ void prefetch_slice(const char* slice, long long b0, long long b1) {
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  if (lane != 0) return;
  constexpr long long piece = 32 * 1024;
  for (long long o = b0 + (long long)warp * piece; o < b1; o += (long long)GEMV_WARPS * piece) {
    const long long n = (b1 - o < piece ? b1 - o : piece) & ~15LL;
    if (n > 0) prefetch_l2_bulk(slice + o, uint32_t(n));
  }
}

// ----------------------------------------------------------------------------- bf16 / mma path

// Builds the B operand of chunk `chunk` in shared memory: [nt][kt_local][lane] x uint4 where,
// for lane (g, t) = (lane / 4, lane % 4), .x = hi(x[g][2t], x[g][2t+1]), .y = hi(x[g][2t+8],
// x[g][2t+9]), .z / .w the lo terms, relative to k-tile kt_local and n-tile nt. Rows >= L are
// left unwritten: they only feed output columns that are never stored.
template <int NT>
__device__ void gemv_build_chunk(const GemvParams& p, int L, int chunk, uint4* xs, const int* s_tok,
                                 const float* s_inv, bool write_back) {
  uint32_t* xw = reinterpret_cast<uint32_t*>(xs);
  const int k0 = chunk * GEMV_KC;
  const int kend = min(p.K, k0 + GEMV_KC);
  // segments overlapping [k0, kend): each 4-column group belongs to exactly one segment
  const int kc4 = (kend - k0) / 4;
  const int total = L * kc4;
  constexpr int U = 4;
  for (int base = threadIdx.x; base < total; base += GEMV_THREADS * U) {
    float4 v[U], w[U];
    int segi[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = base + u * GEMV_THREADS;
      segi[u] = -1;
      if (idx < total) {
        const int n = idx / kc4, k = k0 + (idx % kc4) * 4;
        int off = 0;
        for (int s = 0; s < p.nseg; ++s) {
          const Seg& sg = p.seg[s];
          if (k < off + sg.len) {
            segi[u] = s;
            v[u] = seg_load4(sg, n, k - off, s_tok);
            w[u] = sg.norm_w ? *reinterpret_cast<const float4*>(sg.norm_w + (k - off)) : make_float4(1.f, 1.f, 1.f, 1.f);
            break;
          }
          off += sg.len;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = base + u * GEMV_THREADS;
      if (segi[u] < 0) continue;
      const int n = idx / kc4, k = k0 + (idx % kc4) * 4;
      const float inv = s_inv[n * GEMV_MAXSEG + segi[u]];
      const float x0 = v[u].x * inv * w[u].x, x1 = v[u].y * inv * w[u].y;
      const float x2 = v[u].z * inv * w[u].z, x3 = v[u].w * inv * w[u].w;
      if (write_back) {
        int off = 0;
        for (int s = 0; s < segi[u]; ++s) off += p.seg[s].len;
        const Seg& sg = p.seg[segi[u]];
        if (sg.write_back)
          *reinterpret_cast<float4*>(sg.write_back + size_t(n) * sg.ld_wb + (k - off)) = make_float4(x0, x1, x2, x3);
      }
      uint16_t h0, l0, h1, l1, h2, l2, h3, l3;
      split_bf16(x0, h0, l0);
      split_bf16(x1, h1, l1);
      split_bf16(x2, h2, l2);
      split_bf16(x3, h3, l3);
      const int kl = k - k0, ktl = kl >> 4, kk = kl & 15, t = (kk & 7) >> 1, half = kk >> 3;
      const int lane = (n & 7) * 4 + t, nt = n >> 3;
      const size_t word = ((size_t(nt) * GEMV_KTC + ktl) * kWarp + lane) * 4;
      xw[word + half] = pack2(h0, h1);
      xw[word + 2 + half] = pack2(l0, l1);
      xw[word + 4 + half] = pack2(h2, h3);  // lane + 1 holds columns 2t+2, 2t+3
      xw[word + 6 + half] = pack2(l2, l3);
    }
  }
}

template <int NT>
__global__ void __launch_bounds__(GEMV_THREADS, 2) gemv_bf16_kernel(const GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint4* xs = reinterpret_cast<uint4*>(smem);                                        // NT * KTC * 32 uint4
  float* red = reinterpret_cast<float*>(smem + size_t(NT) * GEMV_KTC * kWarp * 16);  // RBB*NT*W*32*4
  float* s_inv = red + GEMV_RBB * NT * GEMV_WARPS * kWarp * 4;                       // MAXL * MAXSEG
  float* s_red = s_inv + GEMV_MAXL * GEMV_MAXSEG;                                    // WARPS * MAXL
  int* s_tok = reinterpret_cast<int*>(s_red + GEMV_WARPS * GEMV_MAXL);               // MAXL
  unsigned long long* s_key = reinterpret_cast<unsigned long long*>(s_tok + GEMV_MAXL);  // MAXL

  pdl_launch_dependents();
  const int G = p.group;
  const int nunits = p.Np / (16 * G);
  const int u0 = int((long long)blockIdx.x * nunits / gridDim.x);
  const int u1 = int((long long)(blockIdx.x + 1) * nunits / gridDim.x);
  const int KT = p.Kp / 16;
  const long long rb_bytes = (long long)KT * 512;
  const char* slice = static_cast<const char*>(p.w) + (long long)u0 * G * rb_bytes;
  const long long slice_bytes = (long long)(u1 - u0) * G * rb_bytes;
  // weights do not depend on the previous kernel: start streaming them before waiting on it
  prefetch_slice(slice, 0, slice_bytes < GEMV_PREFETCH_WINDOW ? slice_bytes : GEMV_PREFETCH_WINDOW);
  pdl_wait();

  const int L = gemv_rows(p);
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  if (tid < GEMV_MAXL) s_key[tid] = 0ull;
  gemv_prologue_stats(p, L, s_tok, s_inv, s_red);

  const int nchunks = (KT + GEMV_KTC - 1) / GEMV_KTC;
  const bool wb = blockIdx.x == 0 && gemv_has_write_back(p);
  if (nchunks == 1) {
    gemv_build_chunk<NT>(p, L, 0, xs, s_tok, s_inv, wb);
    __syncthreads();
  }
  const uint4* W = static_cast<const uint4*>(p.w);
  const int units_per_batch = GEMV_RBB / G;

  for (int ub = u0; ub < u1; ub += units_per_batch) {
    const int nrb = min(units_per_batch, u1 - ub) * G;  // row blocks in this batch
    const int rb0 = ub * G;
    {  // keep the prefetch window running ahead of consumption
      const long long done = (long long)(rb0 - u0 * G) * rb_bytes;
      const long long a = done + GEMV_PREFETCH_WINDOW, b = a + (long long)nrb * rb_bytes;
      if (ub > u0 && a < slice_bytes) prefetch_slice(slice, a, b < slice_bytes ? b : slice_bytes);
    }
    float acc[GEMV_RBB][NT][4];
#pragma unroll
    for (int j = 0; j < GEMV_RBB; ++j)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][nt][e] = 0.f;

    for (int c = 0; c < nchunks; ++c) {
      if (nchunks > 1) {
        __syncthreads();
        gemv_build_chunk<NT>(p, L, c, xs, s_tok, s_inv, wb && ub == u0);
        __syncthreads();
      }
      const int kt0 = c * GEMV_KTC;
      const int ktn = min(GEMV_KTC, KT - kt0);
#pragma unroll
      for (int j = 0; j < GEMV_RBB; ++j) {
        if (j >= nrb) break;
        const uint4* wt = W + (size_t(rb0 + j) * KT + kt0) * kWarp + lane;
        uint4 a[GEMV_TPW];
#pragma unroll
        for (int i = 0; i < GEMV_TPW; ++i) {
          const int kl = warp + i * GEMV_WARPS;
          if (kl < ktn) a[i] = ldg_stream(wt + size_t(kl) * kWarp);
        }
#pragma unroll
        for (int i = 0; i < GEMV_TPW; ++i) {
          const int kl = warp + i * GEMV_WARPS;
          if (kl < ktn) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint4 b = xs[(size_t(nt) * GEMV_KTC + kl) * kWarp + lane];
              mma_bf16_16816(acc[j][nt], a[i], b.x, b.y);
              mma_bf16_16816(acc[j][nt], a[i], b.z, b.w);
            }
          }
        }
      }
    }
    // cross-warp reduction of the split-K partials
#pragma unroll
    for (int j = 0; j < GEMV_RBB; ++j)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        *reinterpret_cast<float4*>(&red[(((j * NT + nt) * GEMV_WARPS + warp) * kWarp + lane) * 4]) =
            make_float4(acc[j][nt][0], acc[j][nt][1], acc[j][nt][2], acc[j][nt][3]);
    __syncthreads();
    const int jcount = (p.epi == EPI_SWIGLU) ? nrb / 2 : nrb;
    for (int idx = tid; idx < jcount * NT * kWarp * 4; idx += GEMV_THREADS) {
      const int e = idx % 4, ln = (idx / 4) % kWarp, nt = (idx / (4 * kWarp)) % NT, jj = idx / (4 * kWarp * NT);
      const int g = ln / 4, t = ln % 4;
      const int l = nt * 8 + 2 * t + (e & 1);
      const int r16 = g + ((e & 2) ? 8 : 0);
      if (l >= L) continue;
      if (p.epi == EPI_SWIGLU) {
        const int jg = jj * 2, ju = jj * 2 + 1;
        float gs = 0.f, us = 0.f;
#pragma unroll
        for (int w = 0; w < GEMV_WARPS; ++w) {
          gs += red[(((jg * NT + nt) * GEMV_WARPS + w) * kWarp + ln) * 4 + e];
          us += red[(((ju * NT + nt) * GEMV_WARPS + w) * kWarp + ln) * 4 + e];
        }
        const int n = ((rb0 / 2) + jj) * 16 + r16;
        if (n < p.N) p.y[size_t(l) * p.ldy + n] = gs / (1.f + expf(-gs)) * us;
      } else {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < GEMV_WARPS; ++w) s += red[(((jj * NT + nt) * GEMV_WARPS + w) * kWarp + ln) * 4 + e];
        const int n = (rb0 + jj) * 16 + r16;
        if (n < p.N) {
          if (p.epi == EPI_ARGMAX) {
            if (p.y) p.y[size_t(l) * p.ldy + n] = s;
            atomicMax(&s_key[l], argmax_key(s, uint32_t(n)));
          } else {
            gemv_store(p, l, n, s);
          }
        }
      }
    }
    __syncthreads();
  }
  if (p.epi == EPI_ARGMAX && tid < L && s_key[tid] != 0ull) atomicMax(&p.keys[tid], s_key[tid]);
}

template <int NT>
size_t gemv_bf16_smem() {
  return size_t(NT) * GEMV_KTC * kWarp * 16 + size_t(GEMV_RBB) * NT * GEMV_WARPS * kWarp * 4 * 4 +
         GEMV_MAXL * GEMV_MAXSEG * 4 + GEMV_WARPS * GEMV_MAXL * 4 + GEMV_MAXL * 4 + GEMV_MAXL * 8 + 16;
}

// ----------------------------------------------------------------------------- fp32 / FMA path

// x lives in smem as fp32 [L][Kp]; each warp computes whole output rows, lanes split K.
__global__ void __launch_bounds__(GEMV_THREADS) gemv_f32_kernel(const GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* xs = reinterpret_cast<float*>(smem);  // L_max * Kp
  float* s_inv = xs + size_t(p.L_max) * p.Kp;
  float* s_red = s_inv + GEMV_MAXL * GEMV_MAXSEG;
  int* s_tok = reinterpret_cast<int*>(s_red + GEMV_WARPS * GEMV_MAXL);
  unsigned long long* s_key = reinterpret_cast<unsigned long long*>(s_tok + GEMV_MAXL);

  pdl_launch_dependents();
  pdl_wait();
  const int L = gemv_rows(p);
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  if (tid < GEMV_MAXL) s_key[tid] = 0ull;
  gemv_prologue_stats(p, L, s_tok, s_inv, s_red);
  const bool wb = blockIdx.x == 0 && gemv_has_write_back(p);
  const int kq = p.K / 4;
  for (int idx = tid; idx < L * kq; idx += GEMV_THREADS) {
    const int l = idx / kq, k = (idx % kq) * 4;
    int off = 0;
    for (int s = 0; s < p.nseg; ++s) {
      const Seg& sg = p.seg[s];
      if (k < off + sg.len) {
        const float4 v = seg_load4(sg, l, k - off, s_tok);
        const float inv = s_inv[l * GEMV_MAXSEG + s];
        const float4 w = sg.norm_w ? *reinterpret_cast<const float4*>(sg.norm_w + (k - off))
                                   : make_float4(1.f, 1.f, 1.f, 1.f);
        const float4 x = make_float4(v.x * inv * w.x, v.y * inv * w.y, v.z * inv * w.z, v.w * inv * w.w);
        *reinterpret_cast<float4*>(&xs[size_t(l) * p.Kp + k]) = x;
        if (wb && sg.write_back) *reinterpret_cast<float4*>(sg.write_back + size_t(l) * sg.ld_wb + (k - off)) = x;
        break;
      }
      off += sg.len;
    }
  }
  for (int idx = tid; idx < L * (p.Kp - p.K); idx += GEMV_THREADS)
    xs[size_t(idx / (p.Kp - p.K)) * p.Kp + p.K + idx % (p.Kp - p.K)] = 0.f;
  __syncthreads();
  const int rows_per_unit = p.group;  // SwiGLU: gate row n and up row n are rows 2n, 2n+1 (interleaved)
  const int nunits = p.N;             // one unit = one output feature (1 or 2 weight rows)
  const int u0 = int((long long)blockIdx.x * nunits / gridDim.x);
  const int u1 = int((long long)(blockIdx.x + 1) * nunits / gridDim.x);
  const float* W = static_cast<const float*>(p.w);
  unsigned long long best[GEMV_MAXL];
#pragma unroll
  for (int l = 0; l < GEMV_MAXL; ++l) best[l] = 0ull;
  for (int u = u0 + warp; u < u1; u += GEMV_WARPS) {
    float acc[2][GEMV_MAXL];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int l = 0; l < GEMV_MAXL; ++l) acc[r][l] = 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (r >= rows_per_unit) break;
      const float* wr = W + size_t(u * rows_per_unit + r) * p.Kp;
      for (int k = lane * 4; k < p.Kp; k += kWarp * 4) {
        const float4 w4 = ldg_stream_f4(reinterpret_cast<const float4*>(wr + k));
#pragma unroll
        for (int l = 0; l < GEMV_MAXL; ++l) {
          if (l < L) {
            const float4 x4 = *reinterpret_cast<const float4*>(&xs[size_t(l) * p.Kp + k]);
            acc[r][l] = fmaf(w4.x, x4.x, fmaf(w4.y, x4.y, fmaf(w4.z, x4.z, fmaf(w4.w, x4.w, acc[r][l]))));
          }
        }
      }
    }
#pragma unroll
    for (int l = 0; l < GEMV_MAXL; ++l) {
      if (l < L) {
        const float s0 = warp_sum(acc[0][l]);
        const float s1 = rows_per_unit == 2 ? warp_sum(acc[1][l]) : 0.f;
        if (lane == 0) {
          if (p.epi == EPI_SWIGLU) {
            p.y[size_t(l) * p.ldy + u] = s0 / (1.f + expf(-s0)) * s1;
          } else if (p.epi == EPI_ARGMAX) {
            if (p.y) p.y[size_t(l) * p.ldy + u] = s0;
            const unsigned long long k = argmax_key(s0, uint32_t(u));
            if (k > best[l]) best[l] = k;
          } else {
            gemv_store(p, l, u, s0);
          }
        }
      }
    }
  }
  if (p.epi == EPI_ARGMAX) {
    if (lane == 0) {
#pragma unroll
      for (int l = 0; l < GEMV_MAXL; ++l)
        if (l < L && best[l]) atomicMax(&s_key[l], best[l]);
    }
    __syncthreads();
    if (tid < L && s_key[tid] != 0ull) atomicMax(&p.keys[tid], s_key[tid]);
  }
}

inline size_t gemv_f32_smem(int L_max, int Kp) {
  return size_t(L_max) * Kp * 4 + GEMV_MAXL * GEMV_MAXSEG * 4 + GEMV_WARPS * GEMV_MAXL * 4 + GEMV_MAXL * 4 +
         GEMV_MAXL * 8 + 16;
}

}  // namespace wc
