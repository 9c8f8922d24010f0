// Persistent layer-stack kernel for the target's verify pass (and the autoregressive step).
//
// The multi-kernel round pays, per dependent step, a kernel's start-up after its dependency
// wait, its tail and the launch gap; at batch 1 those add up to more than the weight stream
// itself. Here one CTA per SM runs the whole layer stack as a list of jobs (GEMV, attention,
// split-K finalize) separated by grid-wide barriers; the launch is cooperative, so every CTA
// is resident and the barriers cannot wait for a CTA that never starts. Every barrier wait is
// bounded and raises kErrTimeout when it expires.
//
// Weights never wait for data: a producer warp walks the same job list and streams each
// GEMV job's weight slabs for this CTA through a 4-stage shared-memory ring (bulk copies,
// L2 evict-first), blocked only by free slots, so HBM keeps streaming through barriers and
// attention. Consumers, after each barrier, fence the async proxy, bulk-copy the job's
// activation fragments into shared memory, fold the per-row 1/rms and run the MMA loop and
// epilogue of gemv.cuh. Attention runs on S CTAs per KV head (prefix slices, 8 warps of
// 16-position tiles; rule-based visibility as attention.cuh) and combines the S partial
// softmax states through global memory: the last CTA of a head to arrive merges them in a
// fixed order and emits the O projection's input fragments. A GEMV whose K exceeds the
// activation buffer writes split-K partials; a finalize job after the next barrier adds them
// in chunk order and runs the epilogue.
#pragma once

#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"

namespace wc {

enum JobType : int { JOB_GEMV = 0, JOB_ATTN = 1, JOB_FIN = 2 };

constexpr int SK_CWARPS = 8;
constexpr int SK_CTHREADS = SK_CWARPS * kWarp;
constexpr int SK_THREADS = SK_CTHREADS + kWarp;
constexpr int SK_NSTAGE = 8;
constexpr int SK_ACT_BYTES = 64 * 1024;  // 4 slabs of 8-row fragments
constexpr int SK_RED_BYTES = 2 * GV_CWARPS * kWarp * 4 * 4;
constexpr int SK_SSP_PARTS = 256;        // partial sums of squares staged with the activations
constexpr int SK_SSP_BYTES = SK_SSP_PARTS * 16 * 4;
constexpr int SK_D = 128;                // head dim of the attention job
constexpr int SK_LD = SK_D + 8;
constexpr int SK_MAXR = 16;              // query rows per KV head (one m-tile)
constexpr int SK_MAXL = 8;               // new rows
constexpr int SK_BLK = 16;
constexpr int SK_MAXS = 16;              // CTAs per KV head
constexpr int SK_TILE_BYTES = 2 * SK_BLK * SK_LD * 2;  // K + V tile
constexpr int SK_NTILE = 4;                            // prefix tile buffers (warps 0..3)
// union region U: a GEMV job's activations | reduction | staged statistics, or an attention
// job's q / tail / raw rows / RoPE rows, its prefix tiles and, after the tiles, the warp outputs
constexpr int SK_ATT_BASE = 2 * SK_MAXR * SK_LD * 2 + SK_TILE_BYTES + (SK_MAXR + 2 * SK_MAXL) * SK_D * 4 +
                            SK_MAXL * (SK_D / 2) * 8 + 2 * SK_D * 4 + SK_MAXL * 4;
constexpr int SK_TILES_OFF = 40 * 1024;                           // prefix tiles start
constexpr int SK_ATT_OW = SK_CWARPS * SK_MAXR * SK_D * 4;         // warp outputs (after the tiles)
constexpr int SK_U_BYTES = SK_ACT_BYTES + SK_RED_BYTES + SK_SSP_BYTES;
static_assert(SK_ATT_BASE <= SK_TILES_OFF, "attention buffers overlap the prefix tiles");
static_assert(SK_TILES_OFF + SK_NTILE * SK_TILE_BYTES <= SK_U_BYTES, "prefix tiles exceed the union region");
static_assert(SK_ATT_OW <= SK_U_BYTES, "warp outputs exceed the union region");

struct AttnJob {
  AttnParams a;
  float* part;    // [Hk][S][MAXR][D + 2]: acc, m, l per row
  int* counters;  // [Hk] arrivals (left at zero)
  int S;          // CTAs per KV head
  int pad;
};

struct __align__(16) Job {
  int type;
  int pad[3];
  GemvParams g;  // JOB_GEMV; JOB_FIN reads g.partial / g.nkc and runs g's epilogue
  AttnJob at;
};
static_assert(sizeof(Job) % 16 == 0, "jobs are bulk-copied");

struct StackParams {
  const Job* jobs;
  int njobs;
  unsigned* bar;  // grid barrier counter, zero at launch
  int* err;
};

// grid barrier: arrive after this CTA's writes of the job, then wait for all CTAs
__device__ __forceinline__ void sk_arrive(unsigned* bar) {
  __threadfence();
  atomicAdd(bar, 1u);
}
__device__ __forceinline__ bool sk_wait(const unsigned* bar, unsigned target) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(bar) : "memory");
    if (v >= target) return true;
    if (i > 32) __nanosleep(64);
  }
  return false;
}

// this CTA's share of a bf16 GEMV job: K-chunk kc, unit range [u0, u1), slabs [s0, s1)
struct SkShare {
  int kc, gi, u0, u1, s0, s1, ns, total;
};
__device__ __forceinline__ SkShare sk_share(const GemvParams& p) {
  SkShare s;
  const int G = p.group, nunits = p.Np / (16 * G), nslab = (p.Kp >> 4) / GV_SLAB;
  s.kc = int(blockIdx.x) % p.nkc;
  s.gi = int(blockIdx.x) / p.nkc;
  if (s.gi >= p.gpk) {
    s.u0 = s.u1 = 0;
  } else {
    s.u0 = int((long long)s.gi * nunits / p.gpk);
    s.u1 = int((long long)(s.gi + 1) * nunits / p.gpk);
  }
  s.s0 = s.kc * p.kc_slabs;
  s.s1 = min(nslab, s.s0 + p.kc_slabs);
  s.ns = s.s1 - s.s0;
  s.total = (s.u1 - s.u0) * G * s.ns;
  return s;
}

// ---------------------------------------------------------------------------- attention job
// This CTA's part of the attention of KV head hk (rank of S): prefix slice + (last rank)
// the new rows; partial state to global, the last CTA of the head merges and emits.
__device__ void sk_attention(const AttnJob& J, unsigned char* U, float* mw, float* lw, float* cw, int* s_flag) {
  const AttnParams& p = J.a;
  constexpr int D = SK_D, LD = SK_LD, NDT = D / 8, d4 = D / 4, EPL = D / kWarp;
  const int S = J.S;
  const int hk = int(blockIdx.x) / S, rank = int(blockIdx.x) % S;
  if (hk >= p.Hk) return;
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp, g = lane >> 2, t = lane & 3;
  const int rep = p.H / p.Hk, Lm = p.L_max;
  uint16_t* qh = reinterpret_cast<uint16_t*>(U);
  uint16_t* ql = qh + SK_MAXR * LD;
  uint16_t* tail = ql + SK_MAXR * LD;                                     // [K,V][BLK][LD]
  float* raw = reinterpret_cast<float*>(tail + 2 * SK_BLK * LD);          // [MAXR + 2 MAXL][D]
  float2* rp = reinterpret_cast<float2*>(raw + (SK_MAXR + 2 * SK_MAXL) * D);  // [MAXL][D/2]
  float* wq = reinterpret_cast<float*>(rp + SK_MAXL * (D / 2));
  float* wk = wq + D;
  int* spos = reinterpret_cast<int*>(wk + D);
  unsigned char* tiles = U + SK_TILES_OFF;
  float* ow = reinterpret_cast<float*>(U);  // [WARPS][MAXR][D] after the tiles are done
  const uint16_t* Kg = static_cast<const uint16_t*>(p.Kc) + hk * p.stride_h;
  const uint16_t* Vg = static_cast<const uint16_t*>(p.Vc) + hk * p.stride_h;

  // ---- one round trip: lengths, raw rows, norm gains, RoPE rows (positions n + l), prefix tiles
  int L = p.L_dev ? *p.L_dev : p.L;
  const int n = (p.n_dev ? *p.n_dev : 0) + p.n_add;
  if (L < 0 || L > Lm) {
    if (tid == 0) raise_error(p.err, kErrRows);
    L = L < 0 ? 0 : Lm;
  }
  const int R = L * rep;
  const int nc = max(0, min(n, p.cap));  // prefix rows that exist in the cache
  const int chunk = ((nc + S - 1) / S + SK_BLK - 1) / SK_BLK * SK_BLK;
  const int q0 = min(nc, rank * chunk), q1 = min(nc, q0 + chunk);
  const int ntiles = (q1 - q0 + SK_BLK - 1) / SK_BLK;
  {  // prefix tiles: warp w < NTILE takes tile w
    const int tl = warp;
    uint16_t* kb = reinterpret_cast<uint16_t*>(tiles + size_t(warp % SK_NTILE) * SK_TILE_BYTES);
    uint16_t* vb = kb + SK_BLK * LD;
    if (warp < SK_NTILE && tl < ntiles) {
      const int pos0 = q0 + tl * SK_BLK;
      constexpr int cpr = D / 8;
      for (int c = lane; c < SK_BLK * cpr; c += kWarp) {
        const int row = c / cpr, col = (c % cpr) * 8, pos = pos0 + row;
        const bool ok = pos < q1;
        const long long off = ok ? (long long)pos * p.stride_p + col : 0;
        cp_async16(kb + row * LD + col, Kg + off, ok ? 16 : 0);
        cp_async16(vb + row * LD + col, Vg + off, ok ? 16 : 0);
      }
    }
    cp_async_commit();
  }
  constexpr int RAWV = (SK_MAXR + 2 * SK_MAXL) * d4 / SK_CTHREADS;
  const int nraw_max = Lm * rep + 2 * Lm;
  float4 rv[RAWV];
#pragma unroll
  for (int i = 0; i < RAWV; ++i) {
    const int idx = tid + i * SK_CTHREADS;
    if (idx < nraw_max * d4) {
      const int row = idx / d4, c = (idx % d4) * 4;
      int head, l;
      if (row < Lm * rep) {
        l = row / rep;
        head = hk * rep + row % rep;
      } else {
        const int j = row - Lm * rep;
        l = j % Lm;
        head = p.H + (j < Lm ? 0 : p.Hk) + hk;
      }
      rv[i] = *reinterpret_cast<const float4*>(p.qkv + size_t(l) * p.ld_qkv + size_t(head) * D + c);
    }
  }
  constexpr int ROPEV = SK_MAXL * (D / 2) / SK_CTHREADS;
  float2 rr[ROPEV];
#pragma unroll
  for (int i = 0; i < ROPEV; ++i) {
    const int idx = tid + i * SK_CTHREADS;
    const int pos = p.positions ? 0 : n + idx / (D / 2);
    if (!p.positions && idx < Lm * (D / 2) && pos < p.max_pos) rr[i] = p.rope[size_t(pos) * (D / 2) + idx % (D / 2)];
  }
  const float wqv = tid < D ? (p.q_norm ? p.q_norm[tid] : 1.f) : 0.f;
  const float wkv = tid < D ? (p.k_norm ? p.k_norm[tid] : 1.f) : 0.f;
  if (tid < D) {
    wq[tid] = wqv;
    wk[tid] = wkv;
  }
#pragma unroll
  for (int i = 0; i < RAWV; ++i) {
    const int idx = tid + i * SK_CTHREADS;
    if (idx < nraw_max * d4) *reinterpret_cast<float4*>(&raw[(idx / d4) * D + (idx % d4) * 4]) = rv[i];
  }
  if (!p.positions) {
#pragma unroll
    for (int i = 0; i < ROPEV; ++i) {
      const int idx = tid + i * SK_CTHREADS;
      if (idx < Lm * (D / 2)) rp[idx] = rr[i];
    }
  }
  if (tid < Lm) {
    const int pos = p.positions ? p.positions[tid] : n + tid;
    const bool bad = pos < 0 || pos >= p.max_pos;
    if (bad && tid < L) raise_error(p.err, kErrPosition);
    spos[tid] = bad ? 0 : pos;
  }
  const bool owns_tail = rank == S - 1;
  if (owns_tail)  // the tail tile holds the new rows only (zero elsewhere)
    for (int c = tid; c < SK_BLK * (D / 8); c += SK_CTHREADS) {
      *reinterpret_cast<uint4*>(tail + (c / (D / 8)) * LD + (c % (D / 8)) * 8) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(tail + SK_BLK * LD + (c / (D / 8)) * LD + (c % (D / 8)) * 8) = make_uint4(0, 0, 0, 0);
    }
  named_sync(1, SK_CTHREADS);
  if (p.positions) {  // explicit positions: the RoPE rows need them first
    for (int idx = tid; idx < L * (D / 2); idx += SK_CTHREADS)
      rp[idx] = p.rope[size_t(spos[idx / (D / 2)]) * (D / 2) + idx % (D / 2)];
  }
  for (int idx = tid; idx < (16 - R > 0 ? 16 - R : 0) * LD; idx += SK_CTHREADS) {
    qh[R * LD + idx] = 0;
    ql[R * LD + idx] = 0;
  }
  named_sync(1, SK_CTHREADS);

  // ---- q / k RMSNorm + RoPE; q -> bf16 hi / lo, new k / v -> bf16 tail tile and cache
  const bool cache_ok = n + L <= p.cap;
  if (!cache_ok && tid == 0 && rank == 0) raise_error(p.err, kErrCapacity);
  for (int it = warp; it < R + 2 * L; it += SK_CWARPS) {
    const bool is_q = it < R;
    const int j = it - R;
    const bool is_k = !is_q && j < L;
    const int l = is_q ? it / rep : j % L;
    const int rrow = is_q ? it : Lm * rep + (is_k ? 0 : Lm) + l;
    float v[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) v[e] = raw[rrow * D + lane * EPL + e];
    if ((is_q && p.q_norm) || (is_k && p.k_norm)) {
      const float* w = is_q ? wq : wk;
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) ss = fmaf(v[e], v[e], ss);
      ss = warp_sum(ss);
      const float inv = 1.f / sqrtf(ss / float(D) + p.eps);
#pragma unroll
      for (int e = 0; e < EPL; ++e) v[e] = v[e] * inv * w[lane * EPL + e];
    }
    if (is_q || is_k) {  // rotate-half: dims d and d + D/2 sit in lanes lane and lane ^ 16
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
        const int d = lane * EPL + e;
        const float2 cs = rp[l * (D / 2) + d % (D / 2)];
        v[e] = (d < D / 2) ? (v[e] * cs.x - partner * cs.y) : (v[e] * cs.x + partner * cs.y);
      }
    }
    if (is_q) {
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        uint16_t h, lo;
        split_bf16(v[e], h, lo);
        qh[it * LD + lane * EPL + e] = h;
        ql[it * LD + lane * EPL + e] = lo;
      }
    } else {
      uint16_t bv[EPL];
#pragma unroll
      for (int e = 0; e < EPL; ++e) bv[e] = f32_to_bf16_bits(v[e]);
      if (owns_tail) {
        uint16_t* dst = tail + (is_k ? 0 : SK_BLK * LD) + l * LD;
#pragma unroll
        for (int e = 0; e < EPL; ++e) dst[lane * EPL + e] = bv[e];
      }
      if (rank == 0 && p.write_cache && cache_ok) {
        uint16_t* dst = static_cast<uint16_t*>(is_k ? p.Kc : p.Vc) + hk * p.stride_h + (long long)(n + l) * p.stride_p;
#pragma unroll
        for (int e = 0; e < EPL; ++e) dst[lane * EPL + e] = bv[e];
      }
    }
  }
  cp_async_wait<0>();
  named_sync(1, SK_CTHREADS);

  // ---- tiles
  float o[NDT][4];
  float mrow[2], lrow[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mrow[h] = -INFINITY;
    lrow[h] = 0.f;
  }
#pragma unroll
  for (int dt = 0; dt < NDT; ++dt)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[dt][e] = 0.f;
  auto tile = [&](const uint16_t* kb, const uint16_t* vb, int pos_base, int end) {
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t bk[4], ah[4], al[4];
      ldsm_x4(bk, kb + ((lane & 7) + 8 * (lane >> 4)) * LD + ks * 16 + 8 * ((lane >> 3) & 1));
      const int qoff = (lane & 15) * LD + ks * 16 + 8 * (lane >> 4);
      ldsm_x4(ah, qh + qoff);
      ldsm_x4(al, ql + qoff);
      mma_bf16_16816r(s[0], ah, bk[0], bk[1]);
      mma_bf16_16816r(s[0], al, bk[0], bk[1]);
      mma_bf16_16816r(s[1], ah, bk[2], bk[3]);
      mma_bf16_16816r(s[1], al, bk[2], bk[3]);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = g + 8 * h;
      const int l = (r < R ? r : 0) / rep;
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int pos = pos_base + nt * 8 + 2 * t + c;
          bool vis = r < R && pos < end;
          if (vis) {
            if (pos < n) {
              vis = p.window <= 0 || pos >= n + l - p.window + 1;
            } else {
              const int jj = pos - n;
              vis = p.newmask ? ((p.newmask[l] >> jj) & 1ull) != 0 : jj <= l;
              if (vis && p.window > 0) vis = pos >= n + l - p.window + 1;
            }
          }
          const float sv = vis ? p.scale * s[nt][2 * h + c] : -INFINITY;
          s[nt][2 * h + c] = sv;
          mx = fmaxf(mx, sv);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(mrow[h], mx);
      const float alpha = (mn == -INFINITY || mrow[h] == -INFINITY) ? (mn == -INFINITY ? 1.f : 0.f) : expf(mrow[h] - mn);
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const float sv = s[nt][2 * h + c];
          const float e = (sv == -INFINITY) ? 0.f : expf(sv - mn);
          s[nt][2 * h + c] = e;
          sum += e;
        }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      lrow[h] = lrow[h] * alpha + sum;
      mrow[h] = mn;
#pragma unroll
      for (int dt = 0; dt < NDT; ++dt) {
        o[dt][2 * h] *= alpha;
        o[dt][2 * h + 1] *= alpha;
      }
    }
    uint32_t ph[4], plo[4];
    split2_bf16(s[0][0], s[0][1], ph[0], plo[0]);
    split2_bf16(s[0][2], s[0][3], ph[1], plo[1]);
    split2_bf16(s[1][0], s[1][1], ph[2], plo[2]);
    split2_bf16(s[1][2], s[1][3], ph[3], plo[3]);
#pragma unroll
    for (int dp = 0; dp < D / 16; ++dp) {
      uint32_t bv[4];
      ldsm_x4_trans(bv, vb + (lane & 15) * LD + dp * 16 + 8 * (lane >> 4));
      mma_bf16_16816r(o[2 * dp], ph, bv[0], bv[1]);
      mma_bf16_16816r(o[2 * dp], plo, bv[0], bv[1]);
      mma_bf16_16816r(o[2 * dp + 1], ph, bv[2], bv[3]);
      mma_bf16_16816r(o[2 * dp + 1], plo, bv[2], bv[3]);
    }
  };
  if (warp < SK_NTILE && warp < ntiles) {
    const uint16_t* kb = reinterpret_cast<const uint16_t*>(tiles + size_t(warp) * SK_TILE_BYTES);
    tile(kb, kb + SK_BLK * LD, q0 + warp * SK_BLK, q1);
  }
  for (int tl = warp + SK_NTILE; warp < SK_NTILE && tl < ntiles; tl += SK_NTILE) {  // longer prefixes: reload
    uint16_t* kb = reinterpret_cast<uint16_t*>(tiles + size_t(warp) * SK_TILE_BYTES);
    uint16_t* vb = kb + SK_BLK * LD;
    __syncwarp();
    const int pos0 = q0 + tl * SK_BLK;
    constexpr int cpr = D / 8;
    for (int c = lane; c < SK_BLK * cpr; c += kWarp) {
      const int row = c / cpr, col = (c % cpr) * 8, pos = pos0 + row;
      const bool ok = pos < q1;
      const long long off = ok ? (long long)pos * p.stride_p + col : 0;
      cp_async16(kb + row * LD + col, Kg + off, ok ? 16 : 0);
      cp_async16(vb + row * LD + col, Vg + off, ok ? 16 : 0);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();
    tile(kb, vb, pos0, q1);
  }
  if (owns_tail && warp == SK_CWARPS - 1) tile(tail, tail + SK_BLK * LD, n, n + L);
  named_sync(1, SK_CTHREADS);  // tiles done: ow may overwrite them

  // ---- merge the warps, write this CTA's partial state
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = g + 8 * h;
    if (r < R) {
#pragma unroll
      for (int dt = 0; dt < NDT; ++dt)
        *reinterpret_cast<float2*>(&ow[(warp * SK_MAXR + r) * D + dt * 8 + 2 * t]) = make_float2(o[dt][2 * h], o[dt][2 * h + 1]);
      if (t == 0) {
        mw[warp * SK_MAXR + r] = mrow[h];
        lw[warp * SK_MAXR + r] = lrow[h];
      }
    }
  }
  named_sync(1, SK_CTHREADS);
  float* mypart = J.part + (size_t(hk) * S + rank) * SK_MAXR * (D + 2);
  if (warp * kWarp < R * SK_CWARPS) {  // per-row warp weights
    const bool act = tid < R * SK_CWARPS;
    const int r = act ? tid / SK_CWARPS : 0, w = tid % SK_CWARPS;
    const float mv = act ? mw[w * SK_MAXR + r] : -INFINITY;
    float M = mv;
#pragma unroll
    for (int o2 = 1; o2 < SK_CWARPS; o2 <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
    const float wt = (mv == -INFINITY) ? 0.f : expf(mv - M);
    float lt = act ? wt * lw[w * SK_MAXR + r] : 0.f;
#pragma unroll
    for (int o2 = 1; o2 < SK_CWARPS; o2 <<= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o2);
    __syncwarp();
    if (act) {
      mw[w * SK_MAXR + r] = wt;
      if (w == 0) {
        mypart[r * (D + 2) + D] = M;
        mypart[r * (D + 2) + D + 1] = lt;
      }
    }
  }
  named_sync(1, SK_CTHREADS);
  for (int idx = tid; idx < R * D; idx += SK_CTHREADS) {
    const int r = idx / D, d = idx % D;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < SK_CWARPS; ++w) acc = fmaf(mw[w * SK_MAXR + r], ow[(w * SK_MAXR + r) * D + d], acc);
    mypart[r * (D + 2) + d] = acc;
  }
  // ---- the last CTA of the head merges the S partial states in rank order
  __threadfence();
  named_sync(1, SK_CTHREADS);
  if (tid == 0) s_flag[0] = atomicAdd(&J.counters[hk], 1) == S - 1;
  named_sync(1, SK_CTHREADS);
  if (!s_flag[0]) return;
  __threadfence();
  const float* hp = J.part + size_t(hk) * S * SK_MAXR * (D + 2);
  float* sm_m = reinterpret_cast<float*>(U);  // [MAXR][MAXS] (U is free: this CTA's tiles are done)
  float* sm_l = sm_m + SK_MAXR * SK_MAXS;
  for (int idx = tid; idx < R * SK_MAXS; idx += SK_CTHREADS) {  // every (row, CTA) state at once
    const int r = idx / SK_MAXS, q = idx % SK_MAXS;
    sm_m[idx] = q < S ? __ldcg(&hp[(q * SK_MAXR + r) * (D + 2) + D]) : -INFINITY;
    sm_l[idx] = q < S ? __ldcg(&hp[(q * SK_MAXR + r) * (D + 2) + D + 1]) : 0.f;
  }
  named_sync(1, SK_CTHREADS);
  if (tid < R) {  // per-row weights of the CTAs, in rank order
    float M = -INFINITY;
    for (int q = 0; q < S; ++q) M = fmaxf(M, sm_m[tid * SK_MAXS + q]);
    float lt = 0.f;
    for (int q = 0; q < S; ++q) {
      const float mq = sm_m[tid * SK_MAXS + q];
      if (mq != -INFINITY) lt += expf(mq - M) * sm_l[tid * SK_MAXS + q];
    }
    for (int q = 0; q < SK_MAXS; ++q) {
      const float mq = sm_m[tid * SK_MAXS + q];
      cw[tid * SK_MAXS + q] = (q >= S || mq == -INFINITY) ? 0.f : expf(mq - M) / lt;
    }
  }
  named_sync(1, SK_CTHREADS);
  for (int idx = tid; idx < R * D; idx += SK_CTHREADS) {
    const int r = idx / D, d = idx % D;
    float v[SK_MAXS];
#pragma unroll
    for (int q = 0; q < SK_MAXS; ++q) v[q] = q < S ? __ldcg(&hp[(q * SK_MAXR + r) * (D + 2) + d]) : 0.f;
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < SK_MAXS; ++q) acc = fmaf(cw[r * SK_MAXS + q], v[q], acc);
    attn_emit(p, r / rep, (hk * rep + r % rep) * D + d, acc);
  }
  if (tid == 0) J.counters[hk] = 0;
}

// ---------------------------------------------------------------------------- standalone attention
// The attention job as its own launch for the per-kernel round: S blocks per KV head and no
// thread-block cluster (a cluster of large blocks waits for enough free SMs in one GPC);
// the last block of a head merges the S partial states from global memory. Each block
// covers at most SK_NTILE x 16 prefix rows, so the cache capacity must be <= S x 64.
__global__ void __launch_bounds__(SK_CTHREADS) attention_flat_kernel(__grid_constant__ const AttnJob J) {
  extern __shared__ __align__(128) unsigned char af_smem[];
  unsigned char* U = af_smem;
  float* mw = reinterpret_cast<float*>(U + SK_U_BYTES);  // [W][MAXR]
  float* lw = mw + SK_CWARPS * SK_MAXR;                   // [W][MAXR]
  float* cw = lw + SK_CWARPS * SK_MAXR;                   // [MAXR][MAXS]
  int* s_flag = reinterpret_cast<int*>(cw + SK_MAXR * SK_MAXS);
  pdl_launch_dependents();
  pdl_wait();
  sk_attention(J, U, mw, lw, cw, s_flag);
}

constexpr size_t attention_flat_smem() {
  return size_t(SK_U_BYTES) + 2 * SK_CWARPS * SK_MAXR * 4 + SK_MAXR * SK_MAXS * 4 + 16;
}

// ---------------------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(SK_THREADS, 1) stack_kernel(__grid_constant__ const StackParams sp) {
  extern __shared__ __align__(128) unsigned char sk_smem[];
  unsigned char* ring = sk_smem;                                                 // NSTAGE x 16 KB
  unsigned char* U = ring + SK_NSTAGE * GV_STAGE_BYTES;                          // union region
  unsigned char* act = U;                                                        // GEMV fragments
  float* red = reinterpret_cast<float*>(U + SK_ACT_BYTES);                       // [2][W][32][4]
  float* ssp = reinterpret_cast<float*>(U + SK_ACT_BYTES + SK_RED_BYTES);        // [parts][16]
  Job* s_job = reinterpret_cast<Job*>(U + SK_U_BYTES);                           // [2] job parameters
  uint64_t* full = reinterpret_cast<uint64_t*>(s_job + 2);                       // [NSTAGE]
  uint64_t* empty = full + SK_NSTAGE;                                            // [NSTAGE]
  uint64_t* act_bar = empty + SK_NSTAGE;                                         // [1]
  uint64_t* job_bar = act_bar + 1;                                               // [2]
  float* s_inv = reinterpret_cast<float*>(job_bar + 2);                          // [3][16]
  float* s_part = s_inv + GEMV_MAXSEG * 16;                                      // [256]
  float* s_sq = s_part + 256;                                                    // [16][16]
  float* mw = s_sq + 256;                                                        // [W][MAXR]
  float* lw = mw + SK_CWARPS * SK_MAXR;                                          // [W][MAXR]
  int* s_tok = reinterpret_cast<int*>(lw + SK_CWARPS * SK_MAXR);                 // [16]
  int* s_flag = s_tok + 16;                                                      // [4]
  unsigned long long* s_key = reinterpret_cast<unsigned long long*>(s_flag + 4);  // [16]

  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  if (tid == 0) {
    for (int s = 0; s < SK_NSTAGE; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, SK_CWARPS);
    }
    mbar_init(act_bar, 1);
    mbar_init(job_bar, 1);
    mbar_init(job_bar + 1, 1);
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == SK_CWARPS) {  // ---- producer: every GEMV job's weight slabs, in job order
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      int q = 0;  // ring stage counter across jobs
      bool ok = true;
      for (int j = 0; j < sp.njobs && ok; ++j) {
        const Job& J = sp.jobs[j];
        if (J.type != JOB_GEMV) continue;
        const GemvParams& p = J.g;
        const SkShare sh = sk_share(p);
        const char* w = static_cast<const char*>(p.w);
        const int KT = p.Kp >> 4;
        for (int i = 0; i < sh.total; ++i, ++q) {
          const int st = q % SK_NSTAGE;
          if (q >= SK_NSTAGE && !mbar_wait(empty + st, ((q / SK_NSTAGE) - 1) & 1, 1u << 26)) {
            raise_error(sp.err, kErrTimeout);
            ok = false;
            break;
          }
          const int rbl = i / sh.ns, si = i % sh.ns;
          const size_t rb = size_t(sh.u0) * p.group + rbl;
          mbar_arrive_expect_tx(full + st, GV_STAGE_BYTES);
          bulk_g2s_hint(ring + st * GV_STAGE_BYTES, w + (rb * KT + size_t(sh.s0 + si) * GV_SLAB) * 512,
                        GV_STAGE_BYTES, full + st, pol);
        }
        // this CTA's share of the next GEMV job into L2 now: it streams while the consumers
        // still work through this job, the barriers and any attention in between
        for (int j2 = j + 1; j2 < sp.njobs && ok; ++j2) {
          if (sp.jobs[j2].type != JOB_GEMV) continue;
          const GemvParams& p2 = sp.jobs[j2].g;
          const SkShare s2 = sk_share(p2);
          const char* w2 = static_cast<const char*>(p2.w);
          const int KT2 = p2.Kp >> 4;
          for (int rbl = 0; rbl < (s2.u1 - s2.u0) * p2.group; ++rbl) {
            const size_t rb = size_t(s2.u0) * p2.group + rbl;
            prefetch_l2_bulk(w2 + (rb * KT2 + size_t(s2.s0) * GV_SLAB) * 512, uint32_t(s2.ns) * GV_STAGE_BYTES);
          }
          break;
        }
      }
      for (int qq = max(0, q - SK_NSTAGE); qq < q; ++qq)
        if (!mbar_wait(full + qq % SK_NSTAGE, (qq / SK_NSTAGE) & 1)) raise_error(sp.err, kErrTimeout);
    }
    return;
  }

  // ---- consumers
  int q = 0;          // ring stage counter, in the producer's order
  bool ok = true;
  if (tid == 0 && sp.njobs > 0) {  // job parameters travel one job ahead into shared memory
    mbar_arrive_expect_tx(job_bar, sizeof(Job));
    bulk_g2s(s_job, sp.jobs, sizeof(Job), job_bar);
  }
  for (int j = 0; j < sp.njobs; ++j) {
    if (tid == 0 && j + 1 < sp.njobs) {  // slot (j + 1) & 1 last held job j - 1, finished by all threads
      mbar_arrive_expect_tx(job_bar + ((j + 1) & 1), sizeof(Job));
      bulk_g2s(s_job + ((j + 1) & 1), sp.jobs + j + 1, sizeof(Job), job_bar + ((j + 1) & 1));
    }
    if (!mbar_wait(job_bar + (j & 1), (j >> 1) & 1)) {
      raise_error(sp.err, kErrTimeout);
      ok = false;
    }
    const Job& J = s_job[j & 1];
    const int type = J.type;
    // wait for every CTA to finish job j - 1
    if (j > 0) {
      if (tid == 0 && !sk_wait(sp.bar, unsigned(j) * gridDim.x)) raise_error(sp.err, kErrTimeout);
      named_sync(1, SK_CTHREADS);
    }
    if (type == JOB_GEMV) {
      const GemvParams& p = J.g;
      const SkShare sh = sk_share(p);
      const int G = p.group;
      const int L = gemv_rows(p.L_dev, p.L, p.L_max, p.err);
      if (tid < 16) s_key[tid] = 0ull;
      int parts = 0;
      bool tbl = false;  // embedding segments need the token prologue
      for (int sg = 0; sg < p.nseg; ++sg) {
        if (p.seg[sg].xf && p.seg[sg].ss) parts += p.seg[sg].nparts;
        tbl |= p.seg[sg].xf == nullptr;
      }
      const bool staged = sh.total > 0 && parts <= SK_SSP_PARTS && !tbl;
      // This chunk's activation fragments and the inputs' partial sums of squares, written by
      // other CTAs before the barrier: cp.async (generic proxy) by every consumer thread, so no
      // proxy fence is needed after the barrier's acquire.
      if (sh.total > 0) {
        for (int sl = sh.s0; sl < sh.s1; ++sl) {
          int f0;
          const XSeg& sg = p.seg[gemv_seg_of(p, sl, &f0)];
          if (!sg.xf) continue;
          const char* src = reinterpret_cast<const char*>(sg.xf) + size_t(sl - f0) * GV_SLAB * 512;
          unsigned char* dst = act + (sl - sh.s0) * GV_STAGE_BYTES;
          for (int c = tid; c < GV_STAGE_BYTES / 16; c += SK_CTHREADS) cp_async16(dst + c * 16, src + c * 16, 16);
        }
        if (staged) {
          int off = 0;
          for (int sg = 0; sg < p.nseg; ++sg)
            if (p.seg[sg].xf && p.seg[sg].ss) {
              const float* src = p.seg[sg].ss;
              for (int c = tid; c < p.seg[sg].nparts * 4; c += SK_CTHREADS)
                cp_async16(ssp + off * 16 + c * 4, src + c * 4, 16);
              off += p.seg[sg].nparts;
            }
        }
      }
      cp_async_commit();
      if (!staged) gemv_prologue(p, L, s_tok, s_inv, s_part);
      bool table = false;
      for (int sl = sh.s0; sl < sh.s1; ++sl) {
        int f0;
        const XSeg& sg = p.seg[gemv_seg_of(p, sl, &f0)];
        if (sg.xf) continue;
        table = true;
        for (int idx = tid; idx < GV_SLAB * kWarp; idx += SK_CTHREADS) {
          const int kt = idx / kWarp, ln = idx % kWarp;
          reinterpret_cast<uint4*>(act)[((sl - sh.s0) * GV_SLAB + kt) * kWarp + ln] =
              xseg_table_b(sg, (sl - f0) * GV_SLAB + kt, 0, ln, L, s_tok);
        }
      }
      if (table) named_sync(1, SK_CTHREADS);
      cp_async_wait<0>();
      named_sync(1, SK_CTHREADS);
      if (staged) {  // 1/rms per (segment, row) from the staged partial sums, fixed order
        const int l = tid & 15, g = tid >> 4;
        int off = 0;
        for (int sg = 0; sg < p.nseg; ++sg) {
          const XSeg& xs = p.seg[sg];
          if (xs.xf && xs.ss) {
            float a = 0.f;
            for (int q2 = g; q2 < xs.nparts; q2 += 16) a += ssp[(off + q2) * 16 + l];
            s_part[g * 16 + l] = a;
            named_sync(1, SK_CTHREADS);
            if (tid < 16) {
              float t2 = 0.f;
#pragma unroll
              for (int q2 = 0; q2 < 16; ++q2) t2 += s_part[q2 * 16 + tid];
              s_inv[sg * 16 + tid] = tid < L ? 1.f / sqrtf(t2 / float(xs.len) + xs.eps) : 0.f;
            }
            named_sync(1, SK_CTHREADS);
            off += xs.nparts;
          } else if (tid < 16) {
            s_inv[sg * 16 + tid] = tid < L ? 1.f : 0.f;
          }
        }
        named_sync(1, SK_CTHREADS);
      }
      const uint4* act4 = reinterpret_cast<const uint4*>(act);
      int seg_first0 = 0;
      const int seg0 = sh.ns > 0 ? gemv_seg_of(p, sh.s0, &seg_first0) : 0;
      const int seg_end0 = seg_first0 + p.seg[seg0].lenp / GV_COLS;
      for (int u = sh.u0; u < sh.u1; ++u) {
        float tot[2][4];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int e = 0; e < 4; ++e) tot[r][e] = 0.f;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          if (r >= G) break;
          constexpr int NA = 2 * GV_TPW;  // independent accumulators (see gemv.cuh)
          float acc[NA][4];
#pragma unroll
          for (int c = 0; c < NA; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[c][e] = 0.f;
          int seg = seg0, seg_end = seg_end0;
          for (int si = 0; si < sh.ns; ++si, ++q) {
            const int st = q % SK_NSTAGE;
            if (ok && !mbar_wait(full + st, (q / SK_NSTAGE) & 1)) {
              raise_error(p.err, kErrTimeout);
              ok = false;
            }
            if (ok) {
              const uint4* A = reinterpret_cast<const uint4*>(ring + st * GV_STAGE_BYTES);
#pragma unroll
              for (int i = 0; i < GV_TPW; ++i) {
                const int kl = warp + i * SK_CWARPS;
                const uint4 a = A[kl * kWarp + lane];
                const uint4 b = act4[(si * GV_SLAB + kl) * kWarp + lane];
                mma_bf16_16816(acc[2 * i], a, b.x, b.y);
                mma_bf16_16816(acc[2 * i + 1], a, b.z, b.w);
              }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + st);
            const int gs = sh.s0 + si;
            if (gs + 1 == seg_end || si + 1 == sh.ns) {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int l = 2 * (lane & 3) + (e & 1);
                float a = 0.f;
#pragma unroll
                for (int c = 0; c < NA; ++c) {
                  a += acc[c][e];
                  acc[c][e] = 0.f;
                }
                tot[r][e] += a * s_inv[seg * 16 + l];
              }
              if (gs + 1 == seg_end && seg + 1 < p.nseg) {
                ++seg;
                seg_end += p.seg[seg].lenp / GV_COLS;
              }
            }
          }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r)
          if (r < G)
            *reinterpret_cast<float4*>(&red[((r * SK_CWARPS + warp) * kWarp + lane) * 4]) =
                make_float4(tot[r][0], tot[r][1], tot[r][2], tot[r][3]);
        named_sync(1, SK_CTHREADS);
        if (tid < kWarp * 4) {
          const int e = tid % 4, ln = tid / 4;
          const int l = 2 * (ln % 4) + (e & 1), r16 = ln / 4 + ((e & 2) ? 8 : 0);
          float v[2] = {0.f, 0.f};
#pragma unroll
          for (int r = 0; r < 2; ++r)
            if (r < G)
#pragma unroll
              for (int w = 0; w < SK_CWARPS; ++w) v[r] += red[((r * SK_CWARPS + w) * kWarp + ln) * 4 + e];
          if (p.nkc > 1) {
#pragma unroll
            for (int r = 0; r < 2; ++r)
              if (r < G) p.partial[((size_t(sh.kc) * (p.Np >> 4) + size_t(u) * G + r) * 16 + r16) * 16 + l] = v[r];
          } else {
            float sq = 0.f;
            if (l < L && u * 16 + r16 < p.N) sq = gemv_epilogue(p, u * 16 + r16, l, v[0], v[1], s_key);
            s_sq[r16 * 16 + l] = sq;
          }
        }
        named_sync(1, SK_CTHREADS);
        if (p.nkc == 1 && p.ss_out && tid < 16) {
          float a = 0.f;
          if (tid < L)
            for (int f = 0; f < 16; ++f) a += s_sq[f * 16 + tid];
          p.ss_out[size_t(u) * 16 + tid] = a;
        }
      }
      named_sync(1, SK_CTHREADS);
      if (p.epi == EPI_ARGMAX && tid < L && s_key[tid] != 0ull) atomicMax(&p.keys[tid], s_key[tid]);
    } else if (type == JOB_ATTN) {
      sk_attention(J.at, U, mw, lw, s_part, s_flag);  // s_part: [MAXR][MAXS] merge weights
    } else {  // JOB_FIN: add the split-K chunks of units blockIdx.x, + gridDim.x, ... in order
      const GemvParams& p = J.g;
      const int G = p.group, nunits = p.Np / (16 * G);
      const int L = gemv_rows(p.L_dev, p.L, p.L_max, p.err);
      for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
        if (tid < 16 * L) {
          const int r16 = tid / L, l = tid % L;
          float v[2] = {0.f, 0.f};
#pragma unroll
          for (int r = 0; r < 2; ++r)
            if (r < G)
              for (int c = 0; c < p.nkc; ++c)
                v[r] += __ldcg(&p.partial[((size_t(c) * (p.Np >> 4) + size_t(u) * G + r) * 16 + r16) * 16 + l]);
          const int n = u * 16 + r16;
          s_sq[r16 * 16 + l] = n < p.N ? gemv_epilogue(p, n, l, v[0], v[1], s_key) : 0.f;
        }
        named_sync(1, SK_CTHREADS);
        if (p.ss_out && tid < 16) {
          float a = 0.f;
          if (tid < L)
            for (int f = 0; f < 16; ++f) a += s_sq[f * 16 + tid];
          p.ss_out[size_t(u) * 16 + tid] = a;
        }
        named_sync(1, SK_CTHREADS);
      }
    }
    // this CTA is done with job j
    named_sync(1, SK_CTHREADS);
    if (tid == 0) sk_arrive(sp.bar);
  }
}

constexpr size_t stack_smem() {
  return size_t(SK_NSTAGE) * GV_STAGE_BYTES + SK_U_BYTES + 2 * sizeof(Job) + (2 * SK_NSTAGE + 4) * 8 +
         GEMV_MAXSEG * 16 * 4 +
         256 * 4 + 256 * 4 + 2 * SK_CWARPS * SK_MAXR * 4 + 16 * 4 + 4 * 4 + 16 * 8 + 128;
}

}  // namespace wc
