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
#pragma once

#include "common.cuh"

namespace wc {

enum Epilogue : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / kWarp;
constexpr int GEMV_KC = 2048;                  // k per smem chunk
constexpr int GEMV_KTC = GEMV_KC / 16;         // k-tiles per chunk
constexpr int GEMV_TPW = GEMV_KTC / GEMV_WARPS;  // k-tiles per warp per chunk
constexpr int GEMV_RBB = 2;                    // row blocks per reduction batch
constexpr int GEMV_MAXL = 16;                  // rows per launch (2 n-tiles)
constexpr int GEMV_MAXSEG = 3;

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
  int K;       // valid input columns
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
  const void* prefetch_next;   // weights of the next launch: bulk-prefetched into L2
  long long prefetch_bytes;
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

__device__ __forceinline__ float seg_value(const Seg& s, int l, int i, const int* toks) {
  if (s.table) {
    const size_t off = size_t(toks[l]) * size_t(s.len) + size_t(i);
    return s.table_dtype == 1 ? bf16_bits_to_f32(static_cast<const uint16_t*>(s.table)[off])
                              : static_cast<const float*>(s.table)[off];
  }
  return s.src[size_t(l) * size_t(s.ld) + size_t(i)];
}

// Shared prologue: resolve tokens and compute the per-(row, segment) RMSNorm scale.
__device__ void gemv_prologue_stats(const GemvParams& p, int L, int* s_tok, float* s_inv) {
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  if (tid < L) {
    bool need = false;
    for (int s = 0; s < p.nseg; ++s) need |= p.seg[s].table != nullptr;
    const int t = need ? resolve_token(p.tok, tid, p.err) : 0;
    s_tok[tid] = t;
    if (need && p.tok.tok_out && blockIdx.x == 0) p.tok.tok_out[tid] = t;
  }
  __syncthreads();
  for (int item = warp; item < L * p.nseg; item += GEMV_WARPS) {
    const int l = item / p.nseg, s = item % p.nseg;
    const Seg& sg = p.seg[s];
    float inv = 1.f;
    if (sg.norm_w) {
      float ss = 0.f;
      for (int i = lane; i < sg.len; i += kWarp) {
        const float v = seg_value(sg, l, i, s_tok);
        ss = fmaf(v, v, ss);
      }
      ss = warp_sum(ss);
      inv = 1.f / sqrtf(ss / float(sg.len) + p.eps);
    }
    if (lane == 0) s_inv[l * GEMV_MAXSEG + s] = inv;
  }
  __syncthreads();
}

// Value of input column k (global index) of row l after normalisation; 0 in padding.
__device__ __forceinline__ float gemv_input(const GemvParams& p, int l, int k, const int* s_tok,
                                            const float* s_inv) {
  int off = 0;
  for (int s = 0; s < p.nseg; ++s) {
    const Seg& sg = p.seg[s];
    if (k < off + sg.len) {
      const int i = k - off;
      float v = seg_value(sg, l, i, s_tok);
      if (sg.norm_w) v = v * s_inv[l * GEMV_MAXSEG + s] * sg.norm_w[i];
      return v;
    }
    off += sg.len;
  }
  return 0.f;
}

__device__ __forceinline__ void gemv_write_back(const GemvParams& p, int l, int k, float v) {
  int off = 0;
  for (int s = 0; s < p.nseg; ++s) {
    const Seg& sg = p.seg[s];
    if (k < off + sg.len) {
      if (sg.write_back) sg.write_back[size_t(l) * sg.ld_wb + (k - off)] = v;
      return;
    }
    off += sg.len;
  }
}

__device__ __forceinline__ bool gemv_has_write_back(const GemvParams& p) {
  for (int s = 0; s < p.nseg; ++s)
    if (p.seg[s].write_back) return true;
  return false;
}

// Epilogue for one output element (row l of the activations, output feature n).
__device__ __forceinline__ void gemv_store(const GemvParams& p, int l, int n, float v) {
  if (p.epi == EPI_ADD) {
    v += p.base[size_t(l) * p.ldb + n];
  }
  p.y[size_t(l) * p.ldy + n] = v;
  if (p.y2) p.y2[size_t(l) * p.ldy2 + n] = v;
}

__device__ __forceinline__ void gemv_prefetch_next(const GemvParams& p) {
  if (!p.prefetch_next || p.prefetch_bytes <= 0) return;
  // each block prefetches its share, in 64 KB bulk requests issued by one thread per warp
  const long long per_block = ((p.prefetch_bytes + gridDim.x - 1) / gridDim.x + 15) & ~15LL;
  const long long b0 = per_block * blockIdx.x;
  long long b1 = b0 + per_block;
  if (b1 > p.prefetch_bytes) b1 = p.prefetch_bytes;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  if (lane != 0) return;
  const char* base = static_cast<const char*>(p.prefetch_next);
  for (long long o = b0 + (long long)warp * 65536; o < b1; o += (long long)GEMV_WARPS * 65536) {
    long long n = b1 - o;
    if (n > 65536) n = 65536;
    n &= ~15LL;
    if (n > 0) prefetch_l2_bulk(base + o, uint32_t(n));
  }
}

// ----------------------------------------------------------------------------- bf16 / mma path

// smem B-fragment layout of one chunk: [nt][kt_local][lane] x uint4, where for lane (g, t) =
// (lane / 4, lane % 4): .x = hi(x[g][2t], x[g][2t+1]), .y = hi(x[g][2t+8], x[g][2t+9]),
// .z/.w = the lo terms, all relative to k-tile kt_local and n-tile nt.
template <int NT>
__device__ void gemv_build_chunk(const GemvParams& p, int L, int chunk, uint4* xs, const int* s_tok,
                                 const float* s_inv, bool write_back) {
  uint32_t* xw = reinterpret_cast<uint32_t*>(xs);
  const int k0 = chunk * GEMV_KC;
  const int kcount = min(GEMV_KC, p.Kp - k0);
  const int pairs = kcount / 2;
  for (int idx = threadIdx.x; idx < NT * 8 * pairs; idx += GEMV_THREADS) {
    const int n = idx / pairs, pr = idx % pairs;
    const int kl = pr * 2, k = k0 + kl;
    float v0 = 0.f, v1 = 0.f;
    if (n < L) {
      if (k < p.K) v0 = gemv_input(p, n, k, s_tok, s_inv);
      if (k + 1 < p.K) v1 = gemv_input(p, n, k + 1, s_tok, s_inv);
      if (write_back) {
        if (k < p.K) gemv_write_back(p, n, k, v0);
        if (k + 1 < p.K) gemv_write_back(p, n, k + 1, v1);
      }
    }
    uint16_t h0, l0, h1, l1;
    split_bf16(v0, h0, l0);
    split_bf16(v1, h1, l1);
    const int ktl = kl / 16, kk = kl % 16, t = (kk % 8) / 2, half = kk / 8;
    const int g = n % 8, nt = n / 8, lane = g * 4 + t;
    const size_t word = ((size_t(nt) * GEMV_KTC + ktl) * kWarp + lane) * 4;
    xw[word + half] = pack2(h0, h1);
    xw[word + 2 + half] = pack2(l0, l1);
  }
}

template <int NT>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_bf16_kernel(const GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  uint4* xs = reinterpret_cast<uint4*>(smem);                                   // NT * KTC * 32 uint4
  float* red = reinterpret_cast<float*>(smem + size_t(NT) * GEMV_KTC * kWarp * 16);  // RBB*NT*W*32*4
  float* s_inv = red + GEMV_RBB * NT * GEMV_WARPS * kWarp * 4;                 // MAXL * MAXSEG
  int* s_tok = reinterpret_cast<int*>(s_inv + GEMV_MAXL * GEMV_MAXSEG);          // MAXL
  unsigned long long* s_key = reinterpret_cast<unsigned long long*>(s_tok + GEMV_MAXL + 2);  // MAXL (8B aligned)

  gemv_prefetch_next(p);
  const int L = gemv_rows(p);
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  if (tid < GEMV_MAXL) s_key[tid] = 0ull;
  gemv_prologue_stats(p, L, s_tok, s_inv);

  const int G = p.group;
  const int nunits = p.Np / (16 * G);
  const int u0 = int((long long)blockIdx.x * nunits / gridDim.x);
  const int u1 = int((long long)(blockIdx.x + 1) * nunits / gridDim.x);
  const int KT = p.Kp / 16;
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
        if (n < p.N) {
          const float v = gs / (1.f + expf(-gs)) * us;
          p.y[size_t(l) * p.ldy + n] = v;
        }
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
         GEMV_MAXL * GEMV_MAXSEG * 4 + (GEMV_MAXL + 2) * 4 + GEMV_MAXL * 8 + 16;
}

// ----------------------------------------------------------------------------- fp32 / FMA path

// x lives in smem as fp32 [L][Kp]; each warp computes whole output rows, lanes split K.
__global__ void __launch_bounds__(GEMV_THREADS) gemv_f32_kernel(const GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* xs = reinterpret_cast<float*>(smem);                    // L_max * Kp
  float* s_inv = xs + size_t(p.L_max) * p.Kp;
  int* s_tok = reinterpret_cast<int*>(s_inv + GEMV_MAXL * GEMV_MAXSEG);
  unsigned long long* s_key = reinterpret_cast<unsigned long long*>(s_tok + GEMV_MAXL + 2);

  gemv_prefetch_next(p);
  const int L = gemv_rows(p);
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  if (tid < GEMV_MAXL) s_key[tid] = 0ull;
  gemv_prologue_stats(p, L, s_tok, s_inv);
  const bool wb = blockIdx.x == 0 && gemv_has_write_back(p);
  for (int idx = tid; idx < L * p.Kp; idx += GEMV_THREADS) {
    const int l = idx / p.Kp, k = idx % p.Kp;
    float v = 0.f;
    if (k < p.K) {
      v = gemv_input(p, l, k, s_tok, s_inv);
      if (wb) gemv_write_back(p, l, k, v);
    }
    xs[idx] = v;
  }
  __syncthreads();
  const int rows_per_unit = p.group;  // SwiGLU: gate row n and up row n are rows 2n, 2n+1 (interleaved)
  const int nunits = p.N;             // one unit = one output feature (1 or 2 weight rows)
  const int u0 = int((long long)blockIdx.x * nunits / gridDim.x);
  const int u1 = int((long long)(blockIdx.x + 1) * nunits / gridDim.x);
  const float* W = static_cast<const float*>(p.w);
  unsigned long long best[GEMV_MAXL];
  for (int l = 0; l < GEMV_MAXL; ++l) best[l] = 0ull;
  for (int u = u0 + warp; u < u1; u += GEMV_WARPS) {
    float acc[2][GEMV_MAXL];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int l = 0; l < GEMV_MAXL; ++l) acc[r][l] = 0.f;
    for (int r = 0; r < rows_per_unit; ++r) {
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
    if (lane == 0)
      for (int l = 0; l < L; ++l)
        if (best[l]) atomicMax(&s_key[l], best[l]);
    __syncthreads();
    if (tid < L && s_key[tid] != 0ull) atomicMax(&p.keys[tid], s_key[tid]);
  }
}

inline size_t gemv_f32_smem(int L_max, int Kp) {
  return size_t(L_max) * Kp * 4 + GEMV_MAXL * GEMV_MAXSEG * 4 + (GEMV_MAXL + 2) * 4 + GEMV_MAXL * 8 + 16;
}

// ----------------------------------------------------------------------------- weight tiling

// Row-major W[N][K] (fp32 or bf16 source) -> bf16 A-fragment tiles of [Np][Kp]; zero padding.
// With interleave_rows = R > 0 (SwiGLU), row block 2j takes gate rows [16j, 16j+16) and row
// block 2j+1 the up rows [16j, 16j+16), where the source holds gate rows [0, R) then up rows.
__global__ void tile_bf16_kernel(const void* src, int src_dtype, int N, int K, int Np, int Kp, int interleave_rows,
                                 uint16_t* dst) {
  const size_t total = size_t(Np) * Kp;
  for (size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
    const size_t tile = idx / 256;
    const int within = int(idx % 256);
    const int KT = Kp / 16;
    const int rb = int(tile / KT), kt = int(tile % KT);
    const int lane = within / 8, e = within % 8;
    const int g = lane / 4, t = lane % 4;
    const int r = g + ((e & 2) ? 8 : 0);
    const int c = 2 * t + (e & 1) + ((e & 4) ? 8 : 0);
    int row = rb * 16 + r;
    const int col = kt * 16 + c;
    if (interleave_rows > 0) {
      const int pair = rb / 2;
      row = (rb % 2 == 0) ? pair * 16 + r : interleave_rows + pair * 16 + r;
      if (pair * 16 + r >= interleave_rows) row = N;  // padding
    }
    float v = 0.f;
    if (row < N && col < K) {
      const size_t s = size_t(row) * K + col;
      v = src_dtype == 1 ? bf16_bits_to_f32(static_cast<const uint16_t*>(src)[s]) : static_cast<const float*>(src)[s];
    }
    dst[idx] = f32_to_bf16_bits(v);
  }
}

// Row-major fp32 copy with row padding (Kp) and optional gate/up interleave (row 2n = gate n,
// row 2n+1 = up n).
__global__ void copy_f32_rows_kernel(const void* src, int src_dtype, int N, int K, int Kp, int interleave_rows,
                                     float* dst) {
  const size_t total = size_t(N) * Kp;
  for (size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
    const int r = int(idx / Kp), c = int(idx % Kp);
    int row = r;
    if (interleave_rows > 0) row = (r % 2 == 0) ? r / 2 : interleave_rows + r / 2;
    float v = 0.f;
    if (c < K) {
      const size_t s = size_t(row) * K + c;
      v = src_dtype == 1 ? bf16_bits_to_f32(static_cast<const uint16_t*>(src)[s]) : static_cast<const float*>(src)[s];
    }
    dst[idx] = v;
  }
}

}  // namespace wc
