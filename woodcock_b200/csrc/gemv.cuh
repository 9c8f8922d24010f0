// Skinny GEMM ("GEMV" over L <= 16 rows) for the decode round:
//   y[L][N] = sum_s inv_s[l] * (x_s[L][K_s] . W_s[N][K_s]^T).
//
// Inputs arrive already in the GEMV's input form ("fragments", common.cuh): the producing
// kernel wrote them pre-multiplied by this GEMV's RMSNorm gain, together with partial sums
// of squares of its rows. The per-row 1/rms (inv_s) is applied to the accumulators, so a
// normalised input costs no prologue pass. This covers the reference's rmsnorm -> linear
// pairs (src/core/qwen3.cpp:86-101, src/core/drafter.cpp:106-128) and the drafter's per-tap
// RMSNorm + fc fusion (drafter.cpp:75-89). A segment can instead gather embedding rows by
// token id (the drafter's auxiliary stream, drafter.cpp:110-116), scaled by a per-token
// 1/rms table built at load time.
//
// bf16 weights are pre-tiled in mma.m16n8k16 A-fragment order (16x16 tile = 512 contiguous
// bytes). One block per SM: a producer warp streams the block's weights through an 8-stage
// ring of 16 KB shared-memory slabs with 1-D bulk (TMA) copies marked L2 evict-first; the
// first stages are issued before the kernel waits on its predecessor (programmatic
// dependent launch). After the wait the producer bulk-copies the input rows' RMSNorm
// statistics and the activation fragments of the block's K-chunk into shared memory once,
// so the MMA loop reads only shared memory. Eight MMA warps split each slab's k-tiles and
// issue two MMAs per tile and n-tile (activation hi and lo bf16 terms, fp32-level
// accuracy), then release the slot through an mbarrier. At the end of each 16-feature unit
// they hand their per-warp sums to four epilogue warps through two shared-memory buffers
// and continue with the next unit, so the cross-warp reduction and the epilogue's global
// traffic overlap the weight stream.
//
// Four instances: the default (64 KB activation chunk, up to 2048 columns at 8 rows); the
// wide one (80 KB chunk, 7-stage ring: K up to 2560 without splitting) and its 16-row form
// (128 KB chunk, 4-stage ring, one reduction buffer: K up to 2048 at 9-16 rows); and the streamed
// one (ACS: whole K in one block for projections with at most one unit per SM, the
// activation streamed in 16 KB pieces through a 4-deep ring beside the weight slab each
// piece multiplies). Otherwise, when K exceeds the chunk, K is split: the blocks of one row
// range write fp32 partials and the last of them to arrive (one fence and one atomic per
// block) adds them in chunk order and runs the epilogue, so results do not depend on
// arrival order. Epilogues: store, residual add (linear(..., accumulate=true)), SwiGLU
// (silu(gate)*up, cpu_ops.cpp:79-84, gate/up row blocks interleaved) and a fused argmax;
// stored results can also be emitted as fragments for up to two consumers (times their norm
// gains) and as per-unit sums of squares for their 1/rms. Optionally, as its own stream
// ends, each block prefetches its share of the next GEMV's weights into L2.
//
// fp32 weights (row-major [N][Kp]) run the same interface on CUDA cores: fragments are
// then plain fp32 rows [16][len].
#pragma once

#include "common.cuh"

namespace wc {

enum Epilogue : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_ARGMAX = 3 };

constexpr int GEMV_MAXL = 16;  // rows per launch (2 n-tiles)
constexpr int GEMV_MAXSEG = 3;
constexpr int GV_CWARPS = 8;                        // MMA warps
constexpr int GV_CTHREADS = GV_CWARPS * kWarp;      // 256
constexpr int GV_EWARPS = 4;                        // epilogue warps
constexpr int GV_ETHREADS = GV_EWARPS * kWarp;      // 128
constexpr int GV_THREADS = GV_CTHREADS + kWarp + GV_ETHREADS;  // + one producer warp + the epilogue warps
constexpr int GV_SLAB = 32;                         // k-tiles per ring stage: 512 columns
constexpr int GV_COLS = GV_SLAB * 16;
constexpr int GV_STAGE_BYTES = GV_SLAB * 512;       // 16 KB
constexpr int GV_NSTAGE = 8;                        // ring stages at 8 rows (7 at 16 rows)
constexpr int GV_ACT_BYTES = 64 * 1024;             // activation chunk buffer
constexpr int GV_TPW = GV_SLAB / GV_CWARPS;         // k-tiles per warp per slab
constexpr int GV_F32_THREADS = 256;
constexpr int GV_F32_WARPS = GV_F32_THREADS / kWarp;
constexpr int GV_SIDE_BLOCKS = 16;                  // blocks that run a head's side job
constexpr int GV_ACS_DEPTH = GV_ACT_BYTES / GV_STAGE_BYTES;  // streamed activation pieces in flight (4)

__host__ __device__ constexpr int gv_nstage(int NT) { return NT == 1 ? GV_NSTAGE : GV_NSTAGE - 1; }

// Host-computed properties of a launch's inputs (GemvParams::flags).
enum GemvFlags : int { GV_F_TOK = 1, GV_F_SS = 2, GV_F_TABLE = 4 };

// Slabs of K per activation chunk: 4 (2048 columns) for 8 rows, 2 for 16 rows.
__host__ __device__ constexpr int gv_chunk_slabs(int NT) { return GV_ACT_BYTES / (GV_STAGE_BYTES * NT); }
// The wide instance (8 rows): a 5-slab activation chunk (K up to 2560, e.g. Qwen3-4B's hidden
// width) in 80 KB, with a 7-stage weight ring, so those projections need not split K.
constexpr int GV_WIDE_ACT_BYTES = 80 * 1024;
constexpr int GV_WIDE_SLABS = GV_WIDE_ACT_BYTES / GV_STAGE_BYTES;
// The wide instance at 16 rows: a 4-slab chunk (K up to 2048 for both n-tiles) in 128 KB beside a
// 4-stage weight ring, so the 9-16-row verifies (chains of 8 and more, draft trees) do not split
// the hidden-width projections and split the 6144-wide ones in 3 instead of 6. It keeps one
// reduction buffer instead of two to make room for the 4th stage: a unit's partial sums are
// written only after all of its slabs, so the epilogue drains the buffer while the MMA warps
// run the next unit, and the ring depth bounds the weight stream (bytes in flight per SM).
constexpr int GV_WIDE2_ACT_BYTES = 128 * 1024;
constexpr int GV_WIDE2_SLABS = GV_WIDE2_ACT_BYTES / (2 * GV_STAGE_BYTES);

// Fragment width of an input of K columns: bf16 models pad to whole ring slabs.
__host__ __device__ inline int xf_width(bool bf16, int K) { return bf16 ? (K + GV_COLS - 1) / GV_COLS * GV_COLS : K; }

// Per-row token ids for embedding segments: forced id (>= 0) > argmax key > plain id.
struct TokenSrc {
  const int* tokens;
  const unsigned long long* keys;
  const int* vocab_map;  // head row -> token id, nullptr = identity
  const int* forced;
  int* tok_out;          // block 0 stores the resolved ids here when set
  int vocab;
};

// One input segment: consecutive columns of the GEMV input.
struct XSeg {
  const uint32_t* xf;     // fragments (width lenp) or nullptr for an embedding segment
  const float* ss;        // [nparts][16] partial sums of squares of the rows; nullptr = not normalised
  int nparts;
  int len;                // true width (RMSNorm mean, embedding row length)
  int lenp;               // padded width: xf_width(len); the weight layout uses the same padding
  float eps;
  const void* table;      // embedding segment: [vocab][len] rows (bf16 or fp32 as the weights)
  const float* norm_w;    //   times this gain
  const float* row_inv;   //   times row_inv[token] (1/rms of the row), or 1 when nullptr
};

// Fragments of the stored result times w (the consumer's norm gain, or none).
struct XOut {
  uint32_t* xf;
  const float* w;
};

struct GemvParams {
  const void* w;
  int N, Np, Kp, group;  // group: row blocks per epilogue unit (2 for SwiGLU)
  int L;
  const int* L_dev;      // dynamic row count (overrides L when set); rows <= L_max
  int L_max;
  int nseg;
  XSeg seg[GEMV_MAXSEG];
  TokenSrc tok;
  int epi;
  int flags;             // GemvFlags of the segments (set by the launcher)
  // acs = 1 (8 rows, group 1, one unit per block, no embedding segment; launched as the
  // kernel's ACS instance): the whole K in one block, the activation streamed beside the
  // weights in 16 KB pieces through a 4-deep ring in the activation buffer instead of split K
  int acs;
  float* y;              // fp32 result rows (optional except for argmax logits)
  int ldy;
  const float* base;     // EPI_ADD: y = base + acc (base may equal y)
  int ldb;
  int base_tok;          // EPI_ADD: base row of row l = the row of l's token (tok), not l
                         // (the drafter's per-token auxiliary Q/K/V table)
  float* y2;             // optional second copy of the stored result (tap capture)
  int ldy2;
  unsigned long long* keys;  // EPI_ARGMAX: per-row max keys (atomicMax)
  // EPI_ARGMAX with `temperature` set (T on the device, > 0): the key of row l is a draw from
  // softmax(v / T), the argmax of v / T + Gumbel noise (element n of stream rng_stream + l
  // from rng = [seed, counter base] on the device); the stored logits stay v
  const float* temperature;
  const unsigned long long* rng;
  int rng_stream;
  int pad_rng;
  int nout;
  XOut out[2];
  int out_width;         // fragment width of the outputs (xf_width(N))
  float* ss_out;         // bf16: [units][16] sum of y^2 per row over each unit's features;
                         // fp32: [gridDim.x][16] per block
  // bf16 work split: gridDim.x = nkc * gpk; block b owns K-chunk b % nkc (kc_slabs slabs)
  // and the (b / nkc)-th of gpk contiguous unit ranges
  int nkc, kc_slabs, gpk;
  float* partial;        // nkc > 1: [nkc][Np / 16][16 features][16 rows] fp32 partial sums
  int* counters;         // nkc > 1: [gpk] arrivals per unit range (left at zero)
  const void* pf;        // L2 prefetch of upcoming weights (up to two regions), split over the blocks
  size_t pf_bytes;
  const void* pf2;
  size_t pf2_bytes;
  // side job of a drafter head, in blocks < side_blocks:
  //   side_y = side_src * inv(seg 0) * side_w, the next chain step's feature
  const float* side_src;
  int side_len, side_width, side_blocks;
  const float* side_w;
  float* side_y;
  XOut side_out;
  float* side_ss;        // [side_blocks][16]
  int* err;
};

__device__ __forceinline__ int gemv_rows(const int* L_dev, int L0, int L_max, int* err) {
  int L = L_dev ? *L_dev : L0;
  if (L < 0 || L > L_max) {
    raise_error(err, kErrRows);
    L = L < 0 ? 0 : L_max;
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

// Tokens, then s_inv[s * 16 + l] = the 1/rms of row l of segment s (0 for l >= L). The
// partial sums are added in a fixed order: 16 part groups per row, then the groups.
// Runs on 256 threads (named barrier 1); s_part holds 256 floats.
__device__ void gemv_prologue(const GemvParams& p, int L, int* s_tok, float* s_inv, float* s_part) {
  const int tid = threadIdx.x;
  bool need_tok = false;
  for (int s = 0; s < p.nseg; ++s) need_tok |= p.seg[s].xf == nullptr;
  if (tid < L) {
    const int t = need_tok ? resolve_token(p.tok, tid, p.err) : 0;
    s_tok[tid] = t;
    if (need_tok && p.tok.tok_out && blockIdx.x == 0) p.tok.tok_out[tid] = t;
  }
  named_sync(1, 256);
  const int l = tid & 15, g = tid >> 4;
  for (int s = 0; s < p.nseg; ++s) {
    const XSeg& sg = p.seg[s];
    if (sg.xf && sg.ss) {
      float a = 0.f;
      for (int q = g; q < sg.nparts; q += 16) a += sg.ss[q * 16 + l];
      s_part[g * 16 + l] = a;
      named_sync(1, 256);
      if (tid < 16) {
        float t = 0.f;
#pragma unroll
        for (int q = 0; q < 16; ++q) t += s_part[q * 16 + tid];
        s_inv[s * 16 + tid] = tid < L ? 1.f / sqrtf(t / float(sg.len) + sg.eps) : 0.f;
      }
      named_sync(1, 256);
    } else if (tid < 16) {
      s_inv[s * 16 + tid] = tid >= L ? 0.f : (!sg.xf && sg.row_inv) ? sg.row_inv[s_tok[tid]] : 1.f;
    }
  }
  named_sync(1, 256);
}

// B operand of one k-tile of an embedding segment for this lane: {hi(2t), hi(2t+8), lo(2t),
// lo(2t+8)} of row nt*8 + g, i.e. table[tok] * norm_w in fragment form (zero past L or len).
__device__ __forceinline__ uint4 xseg_table_b(const XSeg& s, int kt_in_seg, int nt, int lane, int L, const int* s_tok) {
  const int g = lane >> 2, t = lane & 3, l = nt * 8 + g;
  if (l >= L || kt_in_seg * 16 >= s.len) return make_uint4(0, 0, 0, 0);
  const int c = kt_in_seg * 16 + 2 * t;
  const uint16_t* row = static_cast<const uint16_t*>(s.table) + size_t(s_tok[l]) * s.len;
  const uint32_t e0 = *reinterpret_cast<const uint32_t*>(row + c);
  const uint32_t e1 = *reinterpret_cast<const uint32_t*>(row + c + 8);
  const float2 w0 = *reinterpret_cast<const float2*>(s.norm_w + c);
  const float2 w1 = *reinterpret_cast<const float2*>(s.norm_w + c + 8);
  uint4 b;
  split2_bf16(__uint_as_float(e0 << 16) * w0.x, __uint_as_float(e0 & 0xFFFF0000u) * w0.y, b.x, b.z);
  split2_bf16(__uint_as_float(e1 << 16) * w1.x, __uint_as_float(e1 & 0xFFFF0000u) * w1.y, b.y, b.w);
  return b;
}

// Segment holding global slab `slab` (slabs of 512 padded columns); *first = its first slab.
__device__ __forceinline__ int gemv_seg_of(const GemvParams& p, int slab, int* first) {
  int f = 0;
  for (int s = 0; s < p.nseg; ++s) {
    const int n = p.seg[s].lenp / GV_COLS;
    if (slab < f + n || s + 1 == p.nseg) {
      *first = f;
      return s;
    }
    f += n;
  }
  *first = 0;
  return 0;
}

// The head's side job over this block's slice of the feature (s_inv[l] = seg 0's 1/rms).
// `nthreads` threads take part (named barrier 1); s_red holds (nthreads / 32) * 16 floats.
__device__ void gemv_side_job(const GemvParams& p, int L, const float* s_inv, float* s_red, int nthreads, bool bf16) {
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const int per = (p.side_len + p.side_blocks - 1) / p.side_blocks;
  const int f0 = min(p.side_len, int(blockIdx.x) * per), f1 = min(p.side_len, f0 + per);
  for (int l = 0; l < L; ++l) {
    float a = 0.f;
    for (int f = f0 + tid; f < f1; f += nthreads) {
      const float o = p.side_src[size_t(l) * p.side_len + f] * s_inv[l] * p.side_w[f];
      if (p.side_y) p.side_y[size_t(l) * p.side_len + f] = o;
      if (p.side_out.xf) {
        const float x = p.side_out.w ? o * p.side_out.w[f] : o;
        if (bf16) xf_store(p.side_out.xf, p.side_width, l, f, x);
        else reinterpret_cast<float*>(p.side_out.xf)[size_t(l) * p.side_len + f] = x;
      }
      a = fmaf(o, o, a);
    }
    a = warp_sum(a);
    if (lane == 0) s_red[warp * 16 + l] = a;
  }
  named_sync(1, nthreads);
  if (p.side_ss && tid < 16) {
    float a = 0.f;
    if (tid < L)
      for (int w = 0; w < nthreads / kWarp; ++w) a += s_red[w * 16 + tid];
    p.side_ss[blockIdx.x * 16 + tid] = a;
  }
}

// Epilogue of one output element: feature n of unit u (row r16 of its block), row l; v0 the
// sum (SwiGLU: gate), v1 the up sum. Writes y / y2 / fragments, returns y^2 for the unit's
// sum of squares; argmax goes to the block key.
// the value an EPI_ARGMAX key ranks: the logit, or with a temperature the perturbed logit
__device__ __forceinline__ float gemv_pick_value(const GemvParams& p, int l, int n, float v) {
  if (!p.temperature) return v;
  return v / *p.temperature +
         philox_gumbel_f(p.rng[0], p.rng[1] + uint64_t(p.rng_stream + l) * kRngStreamLen + uint64_t(n));
}

// The global inputs of one element's epilogue: the residual (which may be the output buffer
// itself) and the consumers' norm gains. Callers load them for all of a thread's elements
// before storing any result, so the loads are one round trip instead of one per element.
struct EpiIn {
  float base;
  float w[2];
};

__device__ __forceinline__ EpiIn gemv_epi_load(const GemvParams& p, int n, int l, const int* btok) {
  EpiIn e;
  e.base = p.epi == EPI_ADD ? p.base[size_t(p.base_tok ? btok[l] : l) * p.ldb + n] : 0.f;
  e.w[0] = (p.nout > 0 && p.out[0].w) ? __ldg(p.out[0].w + n) : 1.f;
  e.w[1] = (p.nout > 1 && p.out[1].w) ? __ldg(p.out[1].w + n) : 1.f;
  return e;
}

// EPI_ARGMAX element: stores the logit and returns its ranking key; callers keep the best key
// of each row in registers and fold it into the block's key once (a shared atomic per element
// serialises the 128 epilogue threads on a handful of row addresses).
__device__ __forceinline__ unsigned long long gemv_argmax_item(const GemvParams& p, int n, int l, float v) {
  if (p.y) p.y[size_t(l) * p.ldy + n] = v;
  return argmax_key(gemv_pick_value(p, l, n, v), uint32_t(n));
}

__device__ __forceinline__ float gemv_epilogue_in(const GemvParams& p, int n, int l, float v0, float v1,
                                                  EpiIn e, unsigned long long* s_key) {
  float v = v0;
  if (p.epi == EPI_ARGMAX) {
    if (p.y) p.y[size_t(l) * p.ldy + n] = v;
    atomicMax(&s_key[l], argmax_key(gemv_pick_value(p, l, n, v), uint32_t(n)));
    return 0.f;
  }
  if (p.epi == EPI_SWIGLU) v = v0 / (1.f + expf(-v0)) * v1;
  if (p.epi == EPI_ADD) v += e.base;
  if (p.y) p.y[size_t(l) * p.ldy + n] = v;
  if (p.y2) p.y2[size_t(l) * p.ldy2 + n] = v;
#pragma unroll
  for (int o = 0; o < 2; ++o)
    if (o < p.nout) xf_store(p.out[o].xf, p.out_width, l, n, p.out[o].w ? v * e.w[o] : v);
  return v * v;
}

__device__ __forceinline__ float gemv_epilogue(const GemvParams& p, int n, int l, float v0, float v1,
                                               unsigned long long* s_key) {
  return gemv_epilogue_in(p, n, l, v0, v1, gemv_epi_load(p, n, l, nullptr), s_key);
}

// Tokens (GV_F_TOK) and s_inv[s * 16 + l] = the 1/rms of row l of segment s (0 for l >= L),
// run by the MMA warps (named barrier 1). Every statistics load of every segment is issued
// before the first is used, so the prologue costs one global round trip. The partial sums are
// added in a fixed order: parts g, g + 16, g + 32, ... per row and part group, then the 16
// groups. s_part holds GEMV_MAXSEG x 256 floats.
// Byte offsets (or -1) at which the producer stages each normalised segment's statistics in
// a shared buffer of `cap` bytes: in segment order, while they fit and are 16-byte aligned.
// Producer and MMA warps evaluate the same rule.
__device__ __forceinline__ void gemv_ss_plan(const GemvParams& p, size_t cap, int (&stg)[GEMV_MAXSEG]) {
  size_t off = 0;
#pragma unroll
  for (int s = 0; s < GEMV_MAXSEG; ++s) {
    stg[s] = -1;
    if (s < p.nseg && p.seg[s].xf && p.seg[s].ss) {
      const size_t bytes = size_t(p.seg[s].nparts) * 64;
      if ((reinterpret_cast<uintptr_t>(p.seg[s].ss) & 15) == 0 && off + bytes <= cap) {
        stg[s] = int(off);
        off += bytes;
      }
    }
  }
}

__device__ void gemv_prologue_fast(const GemvParams& p, int L, int* s_tok, float* s_inv, float* s_part,
                                   const unsigned char* stage, const int (&stg)[GEMV_MAXSEG], uint64_t* ss_bar) {
  const int tid = threadIdx.x;
  if (p.flags & GV_F_TOK) {
    if (tid < L) {
      const int t = resolve_token(p.tok, tid, p.err);
      s_tok[tid] = t;
      if (p.tok.tok_out && blockIdx.x == 0) p.tok.tok_out[tid] = t;
    }
    named_sync(1, GV_CTHREADS);
  }
  if (p.flags & GV_F_SS) {
    const int l = tid & 15, g = tid >> 4;
    float v[GEMV_MAXSEG][8];
    bool staged = false;
#pragma unroll
    for (int s = 0; s < GEMV_MAXSEG; ++s) {  // global statistics first: their loads are in flight below
      const XSeg& sg = p.seg[s];
      const bool on = s < p.nseg && sg.xf && sg.ss && stg[s] < 0;
      staged |= stg[s] >= 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int q = g + 16 * i;
        v[s][i] = (on && q < sg.nparts) ? __ldcg(sg.ss + q * 16 + l) : 0.f;
      }
    }
    if (staged && !mbar_wait(ss_bar, 0)) raise_error(p.err, kErrTimeout);
#pragma unroll
    for (int s = 0; s < GEMV_MAXSEG; ++s) {
      const XSeg& sg = p.seg[s];
      float a = 0.f;
      if (stg[s] >= 0) {
        const float* st = reinterpret_cast<const float*>(stage + stg[s]);
        for (int q = g; q < sg.nparts; q += 16) a += st[q * 16 + l];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) a += v[s][i];
        if (s < p.nseg && sg.xf && sg.ss)
          for (int q = g + 128; q < sg.nparts; q += 16) a += __ldcg(sg.ss + q * 16 + l);
      }
      s_part[s * 256 + g * 16 + l] = a;
    }
    named_sync(1, GV_CTHREADS);
  }
  if (tid < GEMV_MAXSEG * 16) {
    const int s = tid >> 4, l = tid & 15;
    float inv = 0.f;
    if (s < p.nseg && l < L) {
      const XSeg& sg = p.seg[s];
      if (sg.xf && sg.ss) {
        float t = 0.f;
#pragma unroll
        for (int q = 0; q < 16; ++q) t += s_part[s * 256 + q * 16 + l];
        inv = 1.f / sqrtf(t / float(sg.len) + sg.eps);
      } else {
        inv = (!sg.xf && sg.row_inv) ? sg.row_inv[s_tok[l]] : 1.f;
      }
    }
    s_inv[tid] = inv;
  }
  named_sync(1, GV_CTHREADS);
}

// Shared-memory carve-up of the bf16 kernel (byte offsets, every region 16-byte aligned).
template <int NT, bool WIDE = false>
struct GvLayout {
  static constexpr int NS = WIDE ? (NT == 1 ? gv_nstage(NT) - 1 : 4) : gv_nstage(NT);
  static constexpr int NRB = WIDE && NT == 2 ? 1 : 2;  // reduction buffers
  static constexpr int ACT_BYTES = WIDE ? (NT == 1 ? GV_WIDE_ACT_BYTES : GV_WIDE2_ACT_BYTES) : GV_ACT_BYTES;
  static constexpr int CHS = ACT_BYTES / (GV_STAGE_BYTES * NT);            // slabs per activation chunk
  static constexpr size_t ring = 0;                                        // NS x 16 KB weight slabs
  static constexpr size_t act = ring + size_t(NS) * GV_STAGE_BYTES;        // [NT][CHS][32 kt][32 lanes] uint4
  static constexpr size_t bars = act + ACT_BYTES;  // full[NS] empty[NS] act red_full[2] red_empty[2] ss act_full[4] act_empty[4]
  static constexpr size_t nbars = 2 * NS + 6 + 2 * GV_ACS_DEPTH;
  static constexpr size_t red = bars + (nbars * 8 + 15) / 16 * 16;         // [NRB buffers][2 row blocks][NT][W][32][4] floats
  static constexpr size_t red_buf = size_t(2) * NT * GV_CWARPS * kWarp * 4;  // floats per buffer
  static constexpr size_t red_bytes = NRB * red_buf * 4;
  static constexpr size_t inv = red + red_bytes;                           // [3][16] floats
  static constexpr size_t part = inv + GEMV_MAXSEG * 16 * 4;               // [3][256] floats
  static constexpr size_t sq = part + GEMV_MAXSEG * 256 * 4;               // [2][16 features][16 rows] floats
  static constexpr size_t tok = sq + 2 * 256 * 4;                          // [16] ints
  static constexpr size_t btok = tok + 16 * 4;                             // [16] ints (epilogue's tokens)
  static constexpr size_t flag = btok + 16 * 4;                            // [4] ints
  static constexpr size_t key = flag + 16;                                 // [16] u64
  static constexpr size_t total = key + 16 * 8;
  static_assert(red_buf * 4 >= 8 * 256 * 4 || NT == 2, "split-K staging needs 8 KB of the reduction buffers");
};

// Warp roles: 0-7 MMA (named barrier 1), 8 the bulk-copy producer, 9-12 epilogue (named
// barrier 2). The MMA warps hand each unit's per-warp sums to the epilogue warps through
// shared-memory buffers (NRB of them; mbarriers red_full / red_empty) and go straight on to the next
// unit's slabs, so the cross-warp reduction, the epilogue's global traffic and the split-K
// hand-off overlap the weight stream instead of stalling it.
template <int NT, bool ACS = false, bool WIDE = false>
__global__ void __launch_bounds__(GV_THREADS, 1) gemv_bf16_kernel(__grid_constant__ const GemvParams pk) {
  static_assert(!(ACS && WIDE) && (!ACS || NT == 1), "kernel instances: ACS is 8-row, ACS and WIDE exclusive");
  using Lay = GvLayout<NT, WIDE>;
  constexpr int NS = Lay::NS;
  constexpr int CHS = Lay::CHS;
  extern __shared__ __align__(128) unsigned char gv_smem[];
  unsigned char* ring = gv_smem + Lay::ring;
  unsigned char* act = gv_smem + Lay::act;
  uint64_t* full = reinterpret_cast<uint64_t*>(gv_smem + Lay::bars);
  uint64_t* empty = full + NS;
  uint64_t* act_bar = empty + NS;
  uint64_t* red_full = act_bar + 1;
  uint64_t* red_empty = red_full + 2;
  uint64_t* ss_bar = red_empty + 2;
  uint64_t* act_full = ss_bar + 1;                 // [GV_ACS_DEPTH] (acs)
  uint64_t* act_empty = act_full + GV_ACS_DEPTH;   // [GV_ACS_DEPTH]
  float* red = reinterpret_cast<float*>(gv_smem + Lay::red);
  float* s_inv = reinterpret_cast<float*>(gv_smem + Lay::inv);
  float* s_part = reinterpret_cast<float*>(gv_smem + Lay::part);
  float* s_sq = reinterpret_cast<float*>(gv_smem + Lay::sq);
  int* s_tok = reinterpret_cast<int*>(gv_smem + Lay::tok);
  int* s_btok = reinterpret_cast<int*>(gv_smem + Lay::btok);
  int* s_flag = reinterpret_cast<int*>(gv_smem + Lay::flag);
  unsigned long long* s_key = reinterpret_cast<unsigned long long*>(gv_smem + Lay::key);
  const uint4* act4 = reinterpret_cast<const uint4*>(act);
  // parameters are read in place (a copy to shared memory cost ~0.4 us per launch: the
  // threads' distinct words serialise in the constant cache)
  const GemvParams& p = pk;

  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const int G = p.group;
  const int nunits = p.Np / (16 * G);
  const int KT = p.Kp >> 4;
  const int nslab = KT / GV_SLAB;
  // 32-bit work split (gi < grid <= a few hundred, nunits < 2^14): no 64-bit divisions
  const unsigned nkc = unsigned(p.nkc), gpk = unsigned(p.gpk);
  const int kc = int(blockIdx.x % nkc), gi = int(blockIdx.x / nkc);
  const int u0 = int(unsigned(gi) * unsigned(nunits) / gpk), u1 = int(unsigned(gi + 1) * unsigned(nunits) / gpk);
  const int s0 = kc * p.kc_slabs, s1 = min(nslab, s0 + p.kc_slabs), ns = s1 - s0;
  const int total = (u1 - u0) * G * ns;  // ring stages: unit, row block of the unit, slab
  if (tid == GV_CWARPS * kWarp) {  // the producer lane: every barrier a bulk copy completes, one fence
    for (int s = 0; s < NS; ++s) mbar_init(full + s, 1);
    mbar_init(act_bar, 1);
    mbar_init(ss_bar, 1);
    for (int b = 0; b < GV_ACS_DEPTH; ++b) mbar_init(act_full + b, 1);
    mbar_fence_init();
  } else if (tid < NS) {  // arrivals from threads only: ordered by the barrier below
    mbar_init(empty + tid, GV_CWARPS);
  } else if (tid >= 32 && tid < 32 + GV_ACS_DEPTH) {
    mbar_init(act_empty + (tid - 32), GV_CWARPS);
  } else if (tid >= 64 && tid < 66) {
    mbar_init(red_full + (tid - 64), GV_CTHREADS);
  } else if (tid >= 96 && tid < 98) {
    mbar_init(red_empty + (tid - 96), GV_ETHREADS);
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == GV_CWARPS) {  // ---- producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      const char* w = static_cast<const char*>(p.w);
      auto issue = [&](int q) {
        const int st = q % NS, rbl = q / ns, si = q % ns;
        const size_t rb = size_t(u0) * G + rbl;
        mbar_arrive_expect_tx(full + st, GV_STAGE_BYTES);
        bulk_g2s_hint(ring + st * GV_STAGE_BYTES, w + (rb * KT + size_t(s0 + si) * GV_SLAB) * 512, GV_STAGE_BYTES,
                      full + st, pol);
      };
      int issued = 0;
      // weights do not depend on the previous kernel: fill the ring before waiting on it
      for (; issued < min(total, NS); ++issued) issue(issued);
      pdl_wait();
      // statistics of the normalised segments, into the reduction buffers (unused until the
      // first unit is handed over), ahead of the larger activation copy
      int stg[GEMV_MAXSEG];
      gemv_ss_plan(p, Lay::red_bytes, stg);
      uint32_t ss_bytes = 0;
#pragma unroll
      for (int s = 0; s < GEMV_MAXSEG; ++s)
        if (stg[s] >= 0) ss_bytes += uint32_t(p.seg[s].nparts) * 64;
      if (ss_bytes) {
        mbar_arrive_expect_tx(ss_bar, ss_bytes);
#pragma unroll
        for (int s = 0; s < GEMV_MAXSEG; ++s)
          if (stg[s] >= 0)
            bulk_g2s(reinterpret_cast<unsigned char*>(red) + stg[s], p.seg[s].ss, uint32_t(p.seg[s].nparts) * 64, ss_bar);
      }
      // the activation fragments of this K-chunk (embedding segments are built by the MMA warps)
      bool ok = true;
      int as = 0, af = 0;  // acs: segment of the next activation piece and its first slab
      auto issue_act = [&](int j) {  // acs: activation piece j (slab s0 + j) into ring slot j % depth
        const int sl = s0 + j;
        while (as + 1 < p.nseg && sl >= af + p.seg[as].lenp / GV_COLS) af += p.seg[as++].lenp / GV_COLS;
        const XSeg& sg = p.seg[as];
        uint64_t* bar = act_full + j % GV_ACS_DEPTH;
        mbar_arrive_expect_tx(bar, GV_STAGE_BYTES);
        bulk_g2s(act + (j % GV_ACS_DEPTH) * GV_STAGE_BYTES,
                 reinterpret_cast<const char*>(sg.xf) + size_t(sl - af) * GV_SLAB * 512, GV_STAGE_BYTES, bar);
      };
      if (ACS) {
        // pieces j and weight slabs j are consumed together; slot j % depth frees after step
        // j - depth and weight slot j % NS after step j - NS: issue in the order they free
        int aiss = 0;
        for (; aiss < min(ns, GV_ACS_DEPTH); ++aiss) issue_act(aiss);
        for (int k = 0; ok && (issued < total || aiss < ns); ++k) {
          if (issued < total && issued == k + NS) {
            const int st = issued % NS;
            if (!mbar_wait(empty + st, ((issued / NS) - 1) & 1, 1u << 26)) {
              raise_error(p.err, kErrTimeout);
              ok = false;
              break;
            }
            issue(issued++);
          }
          if (aiss < ns && aiss == k + GV_ACS_DEPTH) {
            const int sa = aiss % GV_ACS_DEPTH;
            if (!mbar_wait(act_empty + sa, ((aiss / GV_ACS_DEPTH) - 1) & 1, 1u << 26)) {
              raise_error(p.err, kErrTimeout);
              ok = false;
              break;
            }
            issue_act(aiss++);
          }
        }
        // the block's shared memory must outlive every activation copy issued into it
        for (int j = max(0, aiss - GV_ACS_DEPTH); j < aiss; ++j)
          if (!mbar_wait(act_full + j % GV_ACS_DEPTH, (j / GV_ACS_DEPTH) & 1)) raise_error(p.err, kErrTimeout);
      } else {
        uint32_t act_bytes = 0;
        {
          int s = 0, f = 0;
          for (int sl = s0; sl < s1; ++sl) {
            while (s + 1 < p.nseg && sl >= f + p.seg[s].lenp / GV_COLS) f += p.seg[s++].lenp / GV_COLS;
            if (p.seg[s].xf) act_bytes += NT * GV_STAGE_BYTES;
          }
        }
        mbar_arrive_expect_tx(act_bar, act_bytes);
        {
          int s = 0, f = 0;
          for (int sl = s0; sl < s1; ++sl) {
            while (s + 1 < p.nseg && sl >= f + p.seg[s].lenp / GV_COLS) f += p.seg[s++].lenp / GV_COLS;
            const XSeg& sg = p.seg[s];
            if (!sg.xf) continue;
            for (int nt = 0; nt < NT; ++nt)
              bulk_g2s(act + (nt * CHS + (sl - s0)) * GV_STAGE_BYTES,
                       reinterpret_cast<const char*>(sg.xf) + (size_t(nt) * (sg.lenp >> 4) + size_t(sl - f) * GV_SLAB) * 512,
                       GV_STAGE_BYTES, act_bar);
          }
        }
        for (; issued < total; ++issued) {
          const int st = issued % NS;
          if (!mbar_wait(empty + st, ((issued / NS) - 1) & 1, 1u << 26)) {
            raise_error(p.err, kErrTimeout);
            ok = false;
            break;
          }
          issue(issued);
        }
      }
      // the HBM stream of this block is issued: fetch our share of the next GEMV's weights
      for (int rgn = 0; rgn < 2 && ok; ++rgn) {
        const char* pfp = static_cast<const char*>(rgn ? p.pf2 : p.pf);
        const size_t pfb = rgn ? p.pf2_bytes : p.pf_bytes;
        if (!pfp || pfb < 16) continue;
        const size_t per = ((pfb / gridDim.x) + 15) & ~size_t(15);
        const size_t b0 = per * blockIdx.x, b1 = min(pfb & ~size_t(15), b0 + per);
        for (size_t o = b0; o < b1; o += (1u << 20)) prefetch_l2_bulk(pfp + o, uint32_t(min(size_t(1u << 20), b1 - o)));
      }
      // the block's shared memory must outlive every copy issued into it, also when the
      // consumers gave up on a wait: wait (bounded) for the last copy of each slot
      for (int q = max(0, issued - NS); q < issued; ++q)
        if (!mbar_wait(full + q % NS, (q / NS) & 1)) raise_error(p.err, kErrTimeout);
      if (!ACS && !mbar_wait(act_bar, 0)) raise_error(p.err, kErrTimeout);
      if (ss_bytes && !mbar_wait(ss_bar, 0)) raise_error(p.err, kErrTimeout);
    }
    return;
  }

  if (warp > GV_CWARPS) {  // ---- epilogue warps
    const int et = tid - (GV_CWARPS + 1) * kWarp;
    pdl_wait();
    const int L = gemv_rows(p.L_dev, p.L, p.L_max, nullptr);
    if (et < 16) {
      s_key[et] = 0ull;
      s_btok[et] = (p.base_tok && et < L) ? resolve_token(p.tok, et, nullptr) : 0;
    }
    named_sync(2, GV_ETHREADS);
    bool ok = true;
    unsigned long long kbest[NT];  // EPI_ARGMAX: best key of this thread's row(s) (fixed per k)
    int krow[NT];
#pragma unroll
    for (int k = 0; k < NT; ++k) {
      const int idx = et + k * GV_ETHREADS;
      kbest[k] = 0ull;
      krow[k] = (idx / (4 * kWarp)) * 8 + 2 * (((idx / 4) % kWarp) % 4) + ((idx % 4) & 1);
    }
    for (int u = u0, j = 0; u < u1; ++u, ++j) {
      const int b = j & 1;
      // this thread's elements of the unit; their epilogue inputs load while the MMAs run
      int ln_[NT], e_[NT], nt_[NT], l_[NT], r16_[NT];
      bool live[NT];
      EpiIn ein[NT];
#pragma unroll
      for (int k = 0; k < NT; ++k) {
        const int idx = et + k * GV_ETHREADS;
        e_[k] = idx % 4;
        ln_[k] = (idx / 4) % kWarp;
        nt_[k] = idx / (4 * kWarp);
        l_[k] = nt_[k] * 8 + 2 * (ln_[k] % 4) + (e_[k] & 1);
        r16_[k] = ln_[k] / 4 + ((e_[k] & 2) ? 8 : 0);
        live[k] = p.nkc == 1 && l_[k] < L && u * 16 + r16_[k] < p.N;
        if (live[k]) ein[k] = gemv_epi_load(p, u * 16 + r16_[k], l_[k], s_btok);
      }
      const int rbi = j % Lay::NRB;
      if (ok && !mbar_wait(red_full + rbi, (j / Lay::NRB) & 1)) {
        raise_error(p.err, kErrTimeout);
        ok = false;
      }
      const float* rb = red + rbi * Lay::red_buf;
      float* sq = s_sq + b * 256;
      float v[NT][2];
#pragma unroll
      for (int k = 0; k < NT; ++k) {
        v[k][0] = v[k][1] = 0.f;
#pragma unroll
        for (int r = 0; r < 2; ++r)
          if (r < G)
#pragma unroll
            for (int w = 0; w < GV_CWARPS; ++w)
              v[k][r] += rb[(((r * NT + nt_[k]) * GV_CWARPS + w) * kWarp + ln_[k]) * 4 + e_[k]];
      }
      mbar_arrive(red_empty + rbi);  // this thread's reads of the buffer are done
#pragma unroll
      for (int k = 0; k < NT; ++k) {
        if (p.nkc > 1) {  // this chunk's share, reduced below by the last block of the range
#pragma unroll
          for (int r = 0; r < 2; ++r)
            if (r < G)
              p.partial[((size_t(kc) * (p.Np >> 4) + size_t(u) * G + r) * 16 + r16_[k]) * 16 + l_[k]] = v[k][r];
        } else if (p.epi == EPI_ARGMAX) {
          if (live[k]) {
            const unsigned long long key = gemv_argmax_item(p, u * 16 + r16_[k], l_[k], v[k][0]);
            kbest[k] = key > kbest[k] ? key : kbest[k];
          }
        } else {
          sq[r16_[k] * 16 + l_[k]] =
              live[k] ? gemv_epilogue_in(p, u * 16 + r16_[k], l_[k], v[k][0], v[k][1], ein[k], s_key) : 0.f;
        }
      }
      if (p.nkc == 1 && p.ss_out) {  // fixed-order sum over the unit's 16 features
        named_sync(2, GV_ETHREADS);
        if (et < 16) {
          float a = 0.f;
          if (et < L)
            for (int f = 0; f < 16; ++f) a += sq[f * 16 + et];
          p.ss_out[size_t(u) * 16 + et] = a;
        }
      }
    }
#pragma unroll
    for (int k = 0; k < NT; ++k)
      if (kbest[k]) atomicMax(&s_key[krow[k]], kbest[k]);
    if (p.nkc > 1) {
      // ---- split K: the last block of this unit range adds the chunks in order
      __threadfence();
      named_sync(2, GV_ETHREADS);
      if (et == 0) s_flag[0] = atomicAdd(&p.counters[gi], 1) == p.nkc - 1;
      named_sync(2, GV_ETHREADS);
      if (s_flag[0]) {
        __threadfence();
        if (p.epi == EPI_ARGMAX) {
          // heads: many units per range and no epilogue inputs; 16 units at a time, every
          // partial load of a group in flight together, the best key per row in registers
          constexpr int FU = 16, PER = FU * 256 / GV_ETHREADS;
          unsigned long long fbest[NT * 8];
#pragma unroll
          for (int r = 0; r < NT * 8; ++r) fbest[r] = 0ull;
          for (int ub = u0; ub < u1; ub += FU) {
            const int nu = min(FU, u1 - ub), per = 16 * L, items = nu * per;
            float v0[PER];
#pragma unroll
            for (int i = 0; i < PER; ++i) v0[i] = 0.f;
            for (int c = 0; c < p.nkc; ++c) {
#pragma unroll
              for (int i = 0; i < PER; ++i) {
                const int it = et + i * GV_ETHREADS;
                if (it < items) {
                  const int uu = it / per, r16 = (it % per) / L, l = it % L;
                  v0[i] += __ldcg(&p.partial[((size_t(c) * (p.Np >> 4) + size_t(ub + uu)) * 16 + r16) * 16 + l]);
                }
              }
            }
#pragma unroll
            for (int i = 0; i < PER; ++i) {
              const int it = et + i * GV_ETHREADS;
              if (it < items) {
                const int uu = it / per, r16 = (it % per) / L, l = it % L;
                const int n = (ub + uu) * 16 + r16;
                if (n < p.N) {
                  const unsigned long long key = gemv_argmax_item(p, n, l, v0[i]);
#pragma unroll
                  for (int r = 0; r < NT * 8; ++r)
                    if (r == l && key > fbest[r]) fbest[r] = key;
                }
              }
            }
          }
#pragma unroll
          for (int r = 0; r < NT * 8; ++r)
            if (fbest[r]) atomicMax(&s_key[r], fbest[r]);
        } else {
          // up to 4 units at a time: every global input of the group before any store
          constexpr int FU = 4, PER = FU * 256 / GV_ETHREADS;
          float* s_sq8 = red;  // [FU][16 features][16 rows]; every unit of this block has been reduced
          for (int ub = u0; ub < u1; ub += FU) {
            const int nu = min(FU, u1 - ub), per = 16 * L, items = nu * per;
            float v0[PER], v1[PER];
            EpiIn ein[PER];
#pragma unroll
            for (int i = 0; i < PER; ++i) {
              v0[i] = v1[i] = 0.f;
              const int it = et + i * GV_ETHREADS;
              if (it < items) {
                const int uu = it / per, r16 = (it % per) / L, l = it % L;
                const int n = (ub + uu) * 16 + r16;
                if (n < p.N) ein[i] = gemv_epi_load(p, n, l, s_btok);
              }
            }
            for (int c = 0; c < p.nkc; ++c) {
#pragma unroll
              for (int i = 0; i < PER; ++i) {
                const int it = et + i * GV_ETHREADS;
                if (it < items) {
                  const int uu = it / per, r16 = (it % per) / L, l = it % L;
                  const float* src = &p.partial[((size_t(c) * (p.Np >> 4) + size_t(ub + uu) * G) * 16 + r16) * 16 + l];
                  v0[i] += __ldcg(src);
                  if (G == 2) v1[i] += __ldcg(src + 256);
                }
              }
            }
#pragma unroll
            for (int i = 0; i < PER; ++i) {
              const int it = et + i * GV_ETHREADS;
              if (it < items) {
                const int uu = it / per, r16 = (it % per) / L, l = it % L;
                const int n = (ub + uu) * 16 + r16;
                s_sq8[(uu * 16 + r16) * 16 + l] = n < p.N ? gemv_epilogue_in(p, n, l, v0[i], v1[i], ein[i], s_key) : 0.f;
              }
            }
            named_sync(2, GV_ETHREADS);
            if (p.ss_out && et < nu * 16) {  // fixed-order sum over each unit's 16 features
              const int uu = et / 16, l = et % 16;
              float a = 0.f;
              if (l < L)
                for (int f = 0; f < 16; ++f) a += s_sq8[(uu * 16 + f) * 16 + l];
              p.ss_out[size_t(ub + uu) * 16 + l] = a;
            }
            named_sync(2, GV_ETHREADS);
          }
        }
        if (et == 0) p.counters[gi] = 0;  // ready for the next launch
      }
    }
    named_sync(2, GV_ETHREADS);
    if (p.epi == EPI_ARGMAX && et < L && s_key[et] != 0ull) atomicMax(&p.keys[et], s_key[et]);
    return;
  }

  // ---- MMA warps
  pdl_wait();
  const int L = gemv_rows(p.L_dev, p.L, p.L_max, p.err);
  {
    int stg[GEMV_MAXSEG];
    gemv_ss_plan(p, Lay::red_bytes, stg);
    gemv_prologue_fast(p, L, s_tok, s_inv, s_part, reinterpret_cast<const unsigned char*>(red), stg, ss_bar);
  }
  if (p.flags & GV_F_TABLE) {  // embedding segments of this chunk: built from the table straight into the buffer
    bool table = false;
    int s = 0, f = 0;
    for (int sl = s0; sl < s1; ++sl) {
      while (s + 1 < p.nseg && sl >= f + p.seg[s].lenp / GV_COLS) f += p.seg[s++].lenp / GV_COLS;
      const XSeg& sg = p.seg[s];
      if (sg.xf) continue;
      table = true;
      for (int idx = tid; idx < NT * GV_SLAB * kWarp; idx += GV_CTHREADS) {
        const int nt = idx / (GV_SLAB * kWarp), kt = (idx / kWarp) % GV_SLAB, ln = idx % kWarp;
        reinterpret_cast<uint4*>(act)[((nt * CHS + (sl - s0)) * GV_SLAB + kt) * kWarp + ln] =
            xseg_table_b(sg, (sl - f) * GV_SLAB + kt, nt, ln, L, s_tok);
      }
    }
    if (table) named_sync(1, GV_CTHREADS);
  }
  bool ok = true;
  if (!ACS && !mbar_wait(act_bar, 0)) {
    raise_error(p.err, kErrTimeout);
    ok = false;
  }
  int seg_first0;
  const int seg0 = gemv_seg_of(p, s0, &seg_first0);
  const int seg_end0 = seg_first0 + p.seg[seg0].lenp / GV_COLS;
  int q = 0;
  for (int u = u0, j = 0; u < u1; ++u, ++j) {
    float tot[2][NT][4];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) tot[r][nt][e] = 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (r >= G) break;
      // independent accumulators per k-tile and hi / lo term: the MMAs of a slab do not wait
      // on one another (a single accumulator chains them at the MMA latency)
      constexpr int NA = 2 * GV_TPW;
      float acc[NT][NA][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < NA; ++c)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[nt][c][e] = 0.f;
      int seg = seg0, seg_end = seg_end0;
      for (int si = 0; si < ns; ++si, ++q) {
        const int st = q % NS;
        if (ok && !mbar_wait(full + st, (q / NS) & 1)) {
          raise_error(p.err, kErrTimeout);
          ok = false;
        }
        if (ACS && ok && !mbar_wait(act_full + si % GV_ACS_DEPTH, (si / GV_ACS_DEPTH) & 1)) {
          raise_error(p.err, kErrTimeout);
          ok = false;
        }
        // acs: this slab's activation piece sits in ring slot si % depth (8 rows: NT == 1)
        const int abase = ACS ? (si % GV_ACS_DEPTH) * GV_SLAB : si * GV_SLAB;
        if (ok) {
          const uint4* A = reinterpret_cast<const uint4*>(ring + st * GV_STAGE_BYTES);
#pragma unroll
          for (int i = 0; i < GV_TPW; ++i) {
            const int kl = warp + i * GV_CWARPS;
            const uint4 a = A[kl * kWarp + lane];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint4 b = act4[(nt * CHS * GV_SLAB + abase + kl) * kWarp + lane];
              mma_bf16_16816(acc[nt][2 * i], a, b.x, b.y);
              mma_bf16_16816(acc[nt][2 * i + 1], a, b.z, b.w);
            }
          }
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(empty + st);
          if (ACS) mbar_arrive(act_empty + si % GV_ACS_DEPTH);
        }
        const int gs = s0 + si;
        if (gs + 1 == seg_end || si + 1 == ns) {  // fold with the segment's 1/rms per activation row
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int l = nt * 8 + 2 * (lane & 3) + (e & 1);
              float a = 0.f;
#pragma unroll
              for (int c = 0; c < NA; ++c) {
                a += acc[nt][c][e];
                acc[nt][c][e] = 0.f;
              }
              tot[r][nt][e] += a * s_inv[seg * 16 + l];
            }
          if (gs + 1 == seg_end && seg + 1 < p.nseg) {
            ++seg;
            seg_end += p.seg[seg].lenp / GV_COLS;
          }
        }
      }
    }
    // ---- hand the unit's per-warp sums to the epilogue warps
    const int rbi = j % Lay::NRB;
    if (j >= Lay::NRB && ok && !mbar_wait(red_empty + rbi, ((j / Lay::NRB) - 1) & 1)) {
      raise_error(p.err, kErrTimeout);
      ok = false;
    }
    float* rb = red + rbi * Lay::red_buf;
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        if (r < G)
          *reinterpret_cast<float4*>(&rb[(((r * NT + nt) * GV_CWARPS + warp) * kWarp + lane) * 4]) =
              make_float4(tot[r][nt][0], tot[r][nt][1], tot[r][nt][2], tot[r][nt][3]);
    mbar_arrive(red_full + rbi);
  }
  if (p.side_src && int(blockIdx.x) < p.side_blocks) gemv_side_job(p, L, s_inv, s_part, GV_CTHREADS, true);
}

template <int NT, bool WIDE = false>
constexpr size_t gemv_bf16_smem() {
  return GvLayout<NT, WIDE>::total + 128;
}
static_assert(gemv_bf16_smem<1>() <= kSmemOptinBytes && gemv_bf16_smem<2>() <= kSmemOptinBytes &&
                  gemv_bf16_smem<1, true>() <= kSmemOptinBytes && gemv_bf16_smem<2, true>() <= kSmemOptinBytes,
              "a GEMV layout exceeds the per-block shared memory");

// ----------------------------------------------------------------------------- fp32 models
// Inputs are staged in shared memory with their 1/rms applied, then one warp per output
// feature (or gate/up pair) runs CUDA-core FMA over the fp32 row; same epilogues.
__global__ void __launch_bounds__(GV_F32_THREADS) gemv_f32_kernel(__grid_constant__ const GemvParams p) {
  extern __shared__ __align__(16) unsigned char gf_smem[];
  float* xs = reinterpret_cast<float*>(gf_smem);  // [L_max][Kp]
  float* s_inv = xs + size_t(p.L_max) * p.Kp;   // [3][16]
  float* s_part = s_inv + GEMV_MAXSEG * 16;     // [256]
  float* s_ss = s_part + 256;                   // [16]
  int* s_tok = reinterpret_cast<int*>(s_ss + 16);
  unsigned long long* s_key = reinterpret_cast<unsigned long long*>(s_tok + 16);

  pdl_launch_dependents();
  pdl_wait();
  const int L = gemv_rows(p.L_dev, p.L, p.L_max, p.err);
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  if (tid < 16) {
    s_key[tid] = 0ull;
    s_ss[tid] = 0.f;
  }
  gemv_prologue(p, L, s_tok, s_inv, s_part);
  for (int idx = tid; idx < L * p.Kp; idx += GV_F32_THREADS) {
    const int l = idx / p.Kp, k = idx % p.Kp;
    float v = 0.f;
    int off = 0;
    for (int s = 0; s < p.nseg; ++s) {
      const XSeg& sg = p.seg[s];
      if (k < off + sg.len) {
        const int i = k - off;
        v = sg.xf ? reinterpret_cast<const float*>(sg.xf)[size_t(l) * sg.len + i]
                  : static_cast<const float*>(sg.table)[size_t(s_tok[l]) * sg.len + i] * sg.norm_w[i];
        v *= s_inv[s * 16 + l];
        break;
      }
      off += sg.len;
    }
    xs[idx] = v;
  }
  __syncthreads();
  const int G = p.group;
  const int nunits = p.N;
  const int u0 = int((long long)blockIdx.x * nunits / gridDim.x);
  const int u1 = int((long long)(blockIdx.x + 1) * nunits / gridDim.x);
  const float* W = static_cast<const float*>(p.w);
  unsigned long long best[GEMV_MAXL];
  float ssl[GEMV_MAXL];
#pragma unroll
  for (int l = 0; l < GEMV_MAXL; ++l) {
    best[l] = 0ull;
    ssl[l] = 0.f;
  }
  for (int u = u0 + warp; u < u1; u += GV_F32_WARPS) {
    float acc[2][GEMV_MAXL];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int l = 0; l < GEMV_MAXL; ++l) acc[r][l] = 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      if (r >= G) break;
      const float* wr = W + size_t(u * G + r) * p.Kp;
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
        const float s1 = G == 2 ? warp_sum(acc[1][l]) : 0.f;
        if (lane == 0) {
          if (p.epi == EPI_ARGMAX) {
            if (p.y) p.y[size_t(l) * p.ldy + u] = s0;
            const unsigned long long k = argmax_key(gemv_pick_value(p, l, u, s0), uint32_t(u));
            if (k > best[l]) best[l] = k;
          } else {
            float v = (p.epi == EPI_SWIGLU) ? s0 / (1.f + expf(-s0)) * s1 : s0;
            if (p.epi == EPI_ADD) v += p.base[size_t(l) * p.ldb + u];
            if (p.y) p.y[size_t(l) * p.ldy + u] = v;
            if (p.y2) p.y2[size_t(l) * p.ldy2 + u] = v;
            for (int o = 0; o < p.nout; ++o)
              reinterpret_cast<float*>(p.out[o].xf)[size_t(l) * p.N + u] = p.out[o].w ? v * p.out[o].w[u] : v;
            ssl[l] = fmaf(v, v, ssl[l]);
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
  if (p.ss_out) {  // fixed order: lane 0 of each warp holds its features' partials
    if (lane == 0) {
#pragma unroll
      for (int l = 0; l < GEMV_MAXL; ++l) s_part[warp * 16 + l] = ssl[l];
    }
    __syncthreads();
    if (tid < 16) {
      float a = 0.f;
      if (tid < L)
        for (int w = 0; w < GV_F32_WARPS; ++w) a += s_part[w * 16 + tid];
      p.ss_out[blockIdx.x * 16 + tid] = a;
    }
  }
  if (p.side_src && int(blockIdx.x) < p.side_blocks) {
    __syncthreads();
    gemv_side_job(p, L, s_inv, s_part, GV_F32_THREADS, false);
  }
}

inline size_t gemv_f32_smem(int L_max, int Kp) {
  return size_t(L_max) * Kp * 4 + GEMV_MAXSEG * 16 * 4 + 256 * 4 + 16 * 4 + 16 * 4 + 16 * 8 + 64;
}

}  // namespace wc
