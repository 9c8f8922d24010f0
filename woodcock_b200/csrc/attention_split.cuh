// Decode / verify attention over a bf16 KV cache, split along the sequence, for the rounds'
// few new rows (L <= 16, up to 32 query rows per KV head). Same contract as attention_kernel
// (attention.cuh) for rule-based visibility (causal new rows, optional tree bits in newmask,
// optional window); the reference computation is ops::attention (src/backends/cpu_ops.cpp)
// after the per-head q/k RMSNorm and RoPE of qwen3.cpp:86-101 / drafter.cpp:106-128.
//
// With mask_from_prefix the newmask bits count from the committed length (*n_dev) and cover the
// rows appended earlier in the round too (drafted tree levels).
//
// Grid (S + 1, Hk), 16 warps (8 when a block holds two m-tiles of query rows), no clusters. Blocks 0..S-1 of KV head hk each own a slice of
// the committed prefix [0, npre); block S owns the tail [npre, n + L): rows appended earlier in
// the same round, then the new rows, which it normalises, rotates, rounds to bf16 and appends
// to the cache. When the caller marks the prefix stable (its rows were written by completed
// work, as in the decoder's round graphs), each block fetches its prefix tiles and the RoPE
// rows before the programmatic-dependent wait, so that traffic overlaps the QKV projection.
// After the wait every block loads its head's q rows (one round trip), normalises and rotates
// them into bf16 hi / lo tiles, runs S = Q K^T, online softmax and O += P V on m16n8k16 MMAs
// (16 tiles of 16 positions per block and pass), merges its warps pairwise in shared memory and stores
// its partial state (unnormalised o, running max m, sum l per query row) to global scratch.
// The last block of the head to arrive (one fence and one atomic per block) combines the S + 1
// partial states in block order, so the result does not depend on arrival order, and writes
// the O projection's input fragments. There are no spin waits.
#pragma once

#include "attention.cuh"
#include "common.cuh"

namespace wc {

constexpr int AS_BLK = 16;                    // positions per tile
constexpr int AS_CHUNK = 16 * AS_BLK;         // positions in shared memory at once (16 tiles)
constexpr int AS_MAXR = 32;                   // query rows per KV head
constexpr int AS_MAXL = 16;                   // new rows per launch
constexpr int AS_MAXS = 64;                   // prefix blocks per KV head
constexpr int AS_MAXHK = 64;                  // KV heads (arrival counters)

struct AttnSplitParams {
  AttnParams a;
  float* part_o;   // [Hk][S + 1][AS_MAXR][D]: unnormalised o per query row
  float* part_ml;  // [Hk][S + 1][AS_MAXR][2]: running max m and sum l per query row
  int* counters;  // [Hk] arrivals, zero between launches
  int S;          // prefix blocks per KV head
  int pad;
};

template <int D, int NW>
struct AsLayout {
  static constexpr int LD = D + 8;  // padded bf16 row stride: conflict-free ldmatrix rows
  static constexpr size_t kv_bytes = size_t(2) * AS_CHUNK * LD * 2;              // K | V tiles
  static constexpr size_t raw_bytes = size_t(AS_MAXR + 2 * AS_MAXL) * D * 4;     // raw q | k | v rows
  static constexpr size_t mg_bytes = size_t(NW / 2) * AS_MAXR * D * 4;           // pairwise warp merge (after the tiles)
  static constexpr size_t region_a = kv_bytes + raw_bytes > mg_bytes ? kv_bytes + raw_bytes : mg_bytes;
  static constexpr size_t q_bytes = size_t(AS_MAXR) * LD * 2;                    // per hi / lo
  static constexpr size_t cw_bytes = size_t(AS_MAXR) * (AS_MAXS + 1) * 4;        // merge weights
  static constexpr size_t region_q = 2 * q_bytes > cw_bytes ? 2 * q_bytes : cw_bytes;
  static constexpr size_t rope_off = region_a + region_q;                        // [MAXL][D/2] float2
  static constexpr size_t w_off = rope_off + size_t(AS_MAXL) * RopeSmem<D>::kRow * 8;      // q_norm, k_norm
  static constexpr size_t ml_off = w_off + 2 * D * 4;                            // [NW/2][MAXR] m, l
  static constexpr size_t pos_off = ml_off + size_t(NW) * AS_MAXR * 4;           // [MAXL] ints
  static constexpr size_t mlall_off = pos_off + AS_MAXL * 4;                     // [MAXS + 1][MAXR][2]
  static constexpr size_t flag_off = mlall_off + size_t(AS_MAXS + 1) * AS_MAXR * 2 * 4;
  static constexpr size_t total = flag_off + 16;
};

template <int D, int NW>
constexpr size_t attention_split_smem() {
  return AsLayout<D, NW>::total;
}

template <int D, int MT, int NW>
__global__ void __launch_bounds__(NW * 32) attention_split_kernel(__grid_constant__ const AttnSplitParams sp) {
  static_assert(16 % NW == 0 || NW == 16, "16 tiles per chunk over NW warps");
  constexpr int AS_THREADS = NW * kWarp;
  constexpr int AS_WARPS = NW;
  constexpr int AS_TPW = 16 / NW;  // tiles per warp and chunk
  using Lay = AsLayout<D, NW>;
  constexpr int LD = Lay::LD;
  constexpr int NDT = D / 8;
  constexpr int d4 = D / 4;
  const AttnParams& p = sp.a;
  extern __shared__ __align__(16) unsigned char as_smem[];
  uint16_t* kbuf = reinterpret_cast<uint16_t*>(as_smem);                       // [CHUNK][LD]
  uint16_t* vbuf = kbuf + AS_CHUNK * LD;                                         // [CHUNK][LD]
  float* raw = reinterpret_cast<float*>(as_smem + Lay::kv_bytes);                // [MAXR + 2 MAXL][D]
  float* mg = reinterpret_cast<float*>(as_smem);                                 // [NW/2][MAXR][D]
  uint16_t* qh = reinterpret_cast<uint16_t*>(as_smem + Lay::region_a);           // [MAXR][LD]
  uint16_t* ql = qh + AS_MAXR * LD;
  float* cw = reinterpret_cast<float*>(as_smem + Lay::region_a);                 // [MAXR][S + 1]
  float2* rp = reinterpret_cast<float2*>(as_smem + Lay::rope_off);               // [MAXL][D/2]
  float* wq = reinterpret_cast<float*>(as_smem + Lay::w_off);
  float* wk = wq + D;
  float* mw = reinterpret_cast<float*>(as_smem + Lay::ml_off);                   // [NW/2][MAXR]
  float* lw = mw + (AS_WARPS / 2) * AS_MAXR;
  int* spos = reinterpret_cast<int*>(as_smem + Lay::pos_off);
  int* s_flag = reinterpret_cast<int*>(as_smem + Lay::flag_off);

  const int S = sp.S, split = blockIdx.x, hk = blockIdx.y;
  const bool is_tail = split == S;
  const int rep = p.H / p.Hk;
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const int g = lane >> 2, t = lane & 3;
  const int Lm = p.L_max;
  const uint16_t* Kg = static_cast<const uint16_t*>(p.Kc) + hk * p.stride_h;
  const uint16_t* Vg = static_cast<const uint16_t*>(p.Vc) + hk * p.stride_h;

  for (int i = tid; i < D; i += AS_THREADS) {  // norm gains: independent of the previous kernel
    wq[i] = p.q_norm ? p.q_norm[i] : 1.f;
    wk[i] = p.k_norm ? p.k_norm[i] : 1.f;
  }
  // this block's slice [q0, q1) of the prefix [0, npre): 16-position granules spread over S blocks
  int q0 = 0, q1 = 0;
  auto set_slice = [&](int npre) {
    if (is_tail) return;
    const int granules = (npre + AS_BLK - 1) / AS_BLK;
    const int g0 = int((long long)split * granules / S), g1 = int((long long)(split + 1) * granules / S);
    q0 = min(npre, g0 * AS_BLK);
    q1 = min(npre, g1 * AS_BLK);
  };
  // positions [c0, c0 + CHUNK) of the slice into the tile buffers, up to the end of the last
  // tile in use; rows past q1 inside that tile are zero (their P is 0, and 0 * V must stay 0)
  auto load_chunk = [&](int c0) {
    constexpr int cpr = D / 8;  // 16-byte pieces per row
    const int rows = min(AS_CHUNK, (q1 - c0 + AS_BLK - 1) / AS_BLK * AS_BLK);
    for (int c = tid; c < rows * cpr; c += AS_THREADS) {
      const int row = c / cpr, col = (c % cpr) * 8, pos = c0 + row;
      const bool ok = pos < q1;
      const long long off = ok ? (long long)pos * p.stride_p + col : 0;
      cp_async16(kbuf + row * LD + col, Kg + off, ok ? 16 : 0);
      cp_async16(vbuf + row * LD + col, Vg + off, ok ? 16 : 0);
    }
    cp_async_commit();
  };
  constexpr int ROPEV = (AS_MAXL * (D / 2) + AS_THREADS - 1) / AS_THREADS;
  auto load_rope = [&](const int* pos_of_row) {  // rp[l] = table row of position pos_of_row(l)
    float2 rr[ROPEV];
#pragma unroll
    for (int i = 0; i < ROPEV; ++i) {
      const int idx = tid + i * AS_THREADS, l = idx / (D / 2);
      rr[i] = make_float2(1.f, 0.f);
      if (l < Lm) {
        const int pos = pos_of_row[l];
        if (pos >= 0 && pos < p.max_pos) rr[i] = p.rope[size_t(pos) * (D / 2) + idx % (D / 2)];
      }
    }
#pragma unroll
    for (int i = 0; i < ROPEV; ++i) {
      const int idx = tid + i * AS_THREADS;
      if (idx < Lm * (D / 2)) rp[RopeSmem<D>::at(idx / (D / 2), idx % (D / 2))] = rr[i];
    }
  };

  int npre = -1;
  bool rope_ready = false;
  if (p.stable_prefix && p.n_dev) {
    npre = *p.n_dev;
    if (npre < 0 || npre > p.cap) npre = 0;  // reported below through n
    set_slice(npre);
    if (q1 > q0) load_chunk(q0);
    if (!p.positions) {  // positions npre + n_add + l are known before the wait
      if (tid < Lm) spos[tid] = npre + p.n_add + tid;
      __syncthreads();
      load_rope(spos);
      rope_ready = true;
    }
  }

  pdl_launch_dependents();
  pdl_wait();

  // ---- lengths; raw q rows of this KV head (and, in the tail block, the new k / v rows)
  int L = p.L_dev ? *p.L_dev : p.L;
  const int nd = p.n_dev ? *p.n_dev : 0;
  const int n = nd + p.n_add;
  const int mlo = p.mask_from_prefix ? nd : n;  // first position whose visibility the bits decide
  if (L < 0 || L > Lm) {
    if (tid == 0 && split == 0 && hk == 0) raise_error(p.err, kErrRows);
    L = L < 0 ? 0 : Lm;
  }
  const int R = L * rep;
  if (R > AS_MAXR || Lm > AS_MAXL || (!p.stable_prefix && n > p.cap)) {  // uniform over the grid
    if (tid == 0 && split == 0 && hk == 0) raise_error(p.err, kErrRows);
    cp_async_wait<0>();
    return;
  }
  if (npre < 0) {  // prefix not marked stable: everything before n is prefix
    npre = n;
    set_slice(npre);
    if (q1 > q0) load_chunk(q0);
  }
  const int nraw = is_tail ? Lm * rep + 2 * Lm : Lm * rep;
  {
    constexpr int RAWV = (AS_MAXR + 2 * AS_MAXL) * d4 / AS_THREADS;
    float4 rv[RAWV];
#pragma unroll
    for (int i = 0; i < RAWV; ++i) {
      const int idx = tid + i * AS_THREADS;
      if (idx < nraw * d4) {
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
    int mypos = 0;
    if (tid < Lm && p.positions) mypos = p.positions[tid];
#pragma unroll
    for (int i = 0; i < RAWV; ++i) {
      const int idx = tid + i * AS_THREADS;
      if (idx < nraw * d4) *reinterpret_cast<float4*>(&raw[(idx / d4) * D + (idx % d4) * 4]) = rv[i];
    }
    __syncthreads();  // every spos read of the early RoPE fetch is done
    if (tid < Lm) {
      int pos = p.positions ? mypos : n + tid;
      if (pos < 0 || pos >= p.max_pos) {
        if (tid < L && split == 0) raise_error(p.err, kErrPosition);
        pos = 0;
      }
      spos[tid] = pos;
    }
  }
  const int tl = n + L - npre;  // tail positions [npre, n + L)
  if (tl > 2 * AS_BLK || npre > n) {  // uniform over the grid
    if (tid == 0 && split == 0 && hk == 0) raise_error(p.err, kErrRows);
    cp_async_wait<0>();
    return;
  }
  const bool cache_ok = n + L <= p.cap;
  if (is_tail) {  // the tail tiles: rows appended earlier in this round from the cache, zero elsewhere
    constexpr int cpr = D / 8;
    for (int c = tid; c < 2 * AS_BLK * cpr; c += AS_THREADS) {
      const int ti = c / cpr, col = (c % cpr) * 8, pos = npre + ti;
      if (pos < n && pos < p.cap) {
        cp_async16(kbuf + ti * LD + col, Kg + (long long)pos * p.stride_p + col, 16);
        cp_async16(vbuf + ti * LD + col, Vg + (long long)pos * p.stride_p + col, 16);
      } else {
        *reinterpret_cast<uint4*>(kbuf + ti * LD + col) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(vbuf + ti * LD + col) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
    if (!cache_ok && tid == 0) raise_error(p.err, kErrCapacity);
  }
  __syncthreads();
  if (!rope_ready || n != npre + p.n_add) load_rope(spos);
  for (int idx = tid; idx < (MT * 16 - R) * LD; idx += AS_THREADS) {  // padding query rows
    qh[R * LD + idx] = 0;
    ql[R * LD + idx] = 0;
  }
  __syncthreads();

  // ---- per-head RMSNorm + RoPE, eight lanes per row (lane j of the eight holds elements
  // [j * EPQ, (j + 1) * EPQ); the rotate-half partner of element d < D/2 sits in lane j ^ 4):
  // q -> bf16 hi / lo tiles; in the tail block new k / v -> bf16, tail tile and cache
  constexpr int EPQ = D / 8;
  const int nrows = R + (is_tail ? 2 * L : 0);
  const int sub = lane & 7;
  for (int base = 0; base < nrows; base += AS_THREADS / 8) {  // uniform across the block
    const int it = base + warp * 4 + (lane >> 3);
    const bool valid = it < nrows;
    const bool is_q = it < R;
    const int j = it - R;
    const bool is_k = !is_q && j < L;
    const int l = valid ? (is_q ? it / rep : j % L) : 0;
    const int rrow = is_q ? (l * rep + it % rep) : Lm * rep + (is_k ? 0 : Lm) + l;
    float v[EPQ];
#pragma unroll
    for (int e = 0; e < EPQ; e += 4) {
      const float4 x4 = valid ? *reinterpret_cast<const float4*>(&raw[rrow * D + sub * EPQ + e])
                              : make_float4(0.f, 0.f, 0.f, 0.f);
      v[e] = x4.x;
      v[e + 1] = x4.y;
      v[e + 2] = x4.z;
      v[e + 3] = x4.w;
    }
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < EPQ; ++e) ss = fmaf(v[e], v[e], ss);
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss += __shfl_xor_sync(0xffffffffu, ss, 4);
    if (valid && ((is_q && p.q_norm) || (is_k && p.k_norm))) {
      const float* w = is_q ? wq : wk;
      const float inv = rsqrtf(ss / float(D) + p.eps);
#pragma unroll
      for (int e = 0; e < EPQ; ++e) v[e] = v[e] * inv * w[sub * EPQ + e];
    }
    const bool rot = valid && (is_q || is_k);
#pragma unroll
    for (int e = 0; e < EPQ; ++e) {  // rotate-half
      const float partner = __shfl_xor_sync(0xffffffffu, v[e], 4);
      const int d = sub * EPQ + e;
      if (rot) {
        const float2 cs = rp[RopeSmem<D>::at(l, d % (D / 2))];
        v[e] = (d < D / 2) ? (v[e] * cs.x - partner * cs.y) : (v[e] * cs.x + partner * cs.y);
      }
    }
    if (!valid) continue;
    if (is_q) {
#pragma unroll
      for (int e = 0; e < EPQ; ++e) {
        uint16_t h, lo;
        split_bf16(v[e], h, lo);
        qh[it * LD + sub * EPQ + e] = h;
        ql[it * LD + sub * EPQ + e] = lo;
      }
    } else {
      uint16_t bv[EPQ];
#pragma unroll
      for (int e = 0; e < EPQ; ++e) bv[e] = f32_to_bf16_bits(v[e]);
      const int ti = n + l - npre;
      uint16_t* dst = (is_k ? kbuf : vbuf) + ti * LD;
#pragma unroll
      for (int e = 0; e < EPQ; ++e) dst[sub * EPQ + e] = bv[e];
      if (p.write_cache && cache_ok) {
        uint16_t* cd = static_cast<uint16_t*>(is_k ? p.Kc : p.Vc) + hk * p.stride_h + (long long)(n + l) * p.stride_p;
#pragma unroll
        for (int e = 0; e < EPQ; ++e) cd[sub * EPQ + e] = bv[e];
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- tiles
  float o[MT][NDT][4];
  float mrow[MT][2], lrow[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mrow[mt][h] = -INFINITY;
      lrow[mt][h] = 0.f;
    }
#pragma unroll
    for (int dt = 0; dt < NDT; ++dt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mt][dt][e] = 0.f;
  }
  // one 16-position tile at kb / vb: positions pos_base.., visible below `end`
  auto tile = [&](const uint16_t* kb, const uint16_t* vb, int pos_base, int end) {
    float s[MT][2][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[mt][nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t bk[4];
      ldsm_x4(bk, kb + ((lane & 7) + 8 * (lane >> 4)) * LD + ks * 16 + 8 * ((lane >> 3) & 1));
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t ah[4], al[4];
        const int qoff = (mt * 16 + (lane & 15)) * LD + ks * 16 + 8 * (lane >> 4);
        ldsm_x4(ah, qh + qoff);
        ldsm_x4(al, ql + qoff);
        mma_bf16_16816r(s[mt][0], ah, bk[0], bk[1]);
        mma_bf16_16816r(s[mt][0], al, bk[0], bk[1]);
        mma_bf16_16816r(s[mt][1], ah, bk[2], bk[3]);
        mma_bf16_16816r(s[mt][1], al, bk[2], bk[3]);
      }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = mt * 16 + g + 8 * h;
        const int l = (r < R ? r : 0) / rep;
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int pos = pos_base + nt * 8 + 2 * t + c;
            bool vis = r < R && pos < end;
            if (vis) {
              if (pos < mlo) {
                vis = p.window <= 0 || pos >= n + l - p.window + 1;
              } else {
                const int jj = pos - mlo;
                vis = p.newmask ? ((p.newmask[l] >> jj) & 1ull) != 0 : jj <= l;
                if (vis && p.window > 0) vis = pos >= n + l - p.window + 1;
              }
            }
            const float sv = vis ? (p.scale * kLog2e) * s[mt][nt][2 * h + c] : -INFINITY;  // log2 units
            s[mt][nt][2 * h + c] = sv;
            mx = fmaxf(mx, sv);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(mrow[mt][h], mx);
        const float alpha = (mn == -INFINITY || mrow[mt][h] == -INFINITY) ? (mn == -INFINITY ? 1.f : 0.f)
                                                                          : ex2_approx(mrow[mt][h] - mn);
        float sum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const float sv = s[mt][nt][2 * h + c];
            const float e = (sv == -INFINITY) ? 0.f : ex2_approx(sv - mn);
            s[mt][nt][2 * h + c] = e;
            sum += e;
          }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        lrow[mt][h] = lrow[mt][h] * alpha + sum;
        mrow[mt][h] = mn;
#pragma unroll
        for (int dt = 0; dt < NDT; ++dt) {
          o[mt][dt][2 * h] *= alpha;
          o[mt][dt][2 * h + 1] *= alpha;
        }
      }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {  // O += P V: the score C-fragments are the A fragments of P (hi + lo)
      uint32_t ph[4], plo[4];
      split2_bf16(s[mt][0][0], s[mt][0][1], ph[0], plo[0]);
      split2_bf16(s[mt][0][2], s[mt][0][3], ph[1], plo[1]);
      split2_bf16(s[mt][1][0], s[mt][1][1], ph[2], plo[2]);
      split2_bf16(s[mt][1][2], s[mt][1][3], ph[3], plo[3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t bv[4];
        ldsm_x4_trans(bv, vb + (lane & 15) * LD + dp * 16 + 8 * (lane >> 4));
        mma_bf16_16816r(o[mt][2 * dp], ph, bv[0], bv[1]);
        mma_bf16_16816r(o[mt][2 * dp], plo, bv[0], bv[1]);
        mma_bf16_16816r(o[mt][2 * dp + 1], ph, bv[2], bv[3]);
        mma_bf16_16816r(o[mt][2 * dp + 1], plo, bv[2], bv[3]);
      }
    }
  };
  bool worked = false;
  if (is_tail) {
    if (warp < (tl + AS_BLK - 1) / AS_BLK) {
      tile(kbuf + warp * AS_BLK * LD, vbuf + warp * AS_BLK * LD, npre + warp * AS_BLK, n + L);
      worked = true;
    }
  } else {
    for (int c0 = q0; c0 < q1; c0 += AS_CHUNK) {
      if (c0 > q0) {  // longer slices: the next chunk (one more round trip)
        __syncthreads();
        load_chunk(c0);
        cp_async_wait<0>();
        __syncthreads();
      }
#pragma unroll
      for (int i = 0; i < AS_TPW; ++i) {
        const int tl_idx = warp + AS_WARPS * i, pb = c0 + tl_idx * AS_BLK;
        if (pb < q1) {
          tile(kbuf + tl_idx * AS_BLK * LD, vbuf + tl_idx * AS_BLK * LD, pb, q1);
          worked = true;
        }
      }
    }
  }
  __syncthreads();  // the tile buffers are free: they hold the pairwise warp merge from here

  // ---- the block's partial state: warps merge pairwise in a fixed order (w += w + half), so
  // warp 0 ends with the block's (m, l, o) in registers
  if (!worked) {  // an idle warp contributes nothing
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mrow[mt][h] = -INFINITY;
        lrow[mt][h] = 0.f;
      }
  }
#pragma unroll
  for (int half = AS_WARPS / 2; half >= 1; half >>= 1) {
    if (warp >= half && warp < 2 * half) {  // the upper half writes its state
      const int slot = warp - half;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = mt * 16 + g + 8 * h;
#pragma unroll
          for (int dt = 0; dt < NDT; ++dt)
            *reinterpret_cast<float2*>(&mg[(slot * AS_MAXR + r) * D + dt * 8 + 2 * t]) =
                make_float2(o[mt][dt][2 * h], o[mt][dt][2 * h + 1]);
          if (t == 0) {
            mw[slot * AS_MAXR + r] = mrow[mt][h];
            lw[slot * AS_MAXR + r] = lrow[mt][h];
          }
        }
    }
    __syncthreads();
    if (warp < half) {  // the lower half folds its partner in
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = mt * 16 + g + 8 * h;
          const float m2 = mw[warp * AS_MAXR + r], l2 = lw[warp * AS_MAXR + r];
          const float M = fmaxf(mrow[mt][h], m2);
          const float a1 = mrow[mt][h] == -INFINITY ? 0.f : ex2_approx(mrow[mt][h] - M);
          const float a2 = m2 == -INFINITY ? 0.f : ex2_approx(m2 - M);
          lrow[mt][h] = a1 * lrow[mt][h] + a2 * l2;
          mrow[mt][h] = M;
#pragma unroll
          for (int dt = 0; dt < NDT; ++dt) {
            const float2 v = *reinterpret_cast<const float2*>(&mg[(warp * AS_MAXR + r) * D + dt * 8 + 2 * t]);
            o[mt][dt][2 * h] = a1 * o[mt][dt][2 * h] + a2 * v.x;
            o[mt][dt][2 * h + 1] = a1 * o[mt][dt][2 * h + 1] + a2 * v.y;
          }
        }
    }
    __syncthreads();
  }
  if (warp == 0) {  // the block's partial state, straight from warp 0's registers
    float* po = sp.part_o + (size_t(hk) * (S + 1) + split) * AS_MAXR * D;
    float* ml = sp.part_ml + (size_t(hk) * (S + 1) + split) * AS_MAXR * 2;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = mt * 16 + g + 8 * h;
        if (r >= R) continue;
#pragma unroll
        for (int dt = 0; dt < NDT; ++dt)
          *reinterpret_cast<float2*>(&po[size_t(r) * D + dt * 8 + 2 * t]) =
              make_float2(o[mt][dt][2 * h], o[mt][dt][2 * h + 1]);
        if (t == 0) *reinterpret_cast<float2*>(&ml[r * 2]) = make_float2(mrow[mt][h], lrow[mt][h]);
      }
  }
  // ---- arrival; the last block of this KV head combines the S + 1 partial states in order
  __syncthreads();  // every partial store of this block has been issued
  if (tid == 0) {
    __threadfence();
    s_flag[0] = atomicAdd(&sp.counters[hk], 1) == S;
  }
  __syncthreads();
  if (!s_flag[0]) return;
  __threadfence();
  const float* hml = sp.part_ml + size_t(hk) * (S + 1) * AS_MAXR * 2;
  const float* ho = sp.part_o + size_t(hk) * (S + 1) * AS_MAXR * D;
  float* sml = reinterpret_cast<float*>(as_smem + Lay::mlall_off);  // [S + 1][MAXR][2]
  for (int c = tid; c < (S + 1) * AS_MAXR * 2 / 4; c += AS_THREADS)
    *reinterpret_cast<float4*>(sml + 4 * c) = __ldcg(reinterpret_cast<const float4*>(hml) + c);
  __syncthreads();
  for (int r = warp; r < R; r += AS_WARPS) {  // per-row split weights exp(m_s - M) / sum_s exp(m_s - M) l_s
    float M = -INFINITY;
    for (int s2 = lane; s2 <= S; s2 += kWarp) M = fmaxf(M, sml[(s2 * AS_MAXR + r) * 2]);
    for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
    float lt = 0.f;
    for (int s2 = lane; s2 <= S; s2 += kWarp) {
      const float mv = sml[(s2 * AS_MAXR + r) * 2];
      const float wv = mv == -INFINITY ? 0.f : ex2_approx(mv - M);
      cw[r * (AS_MAXS + 1) + s2] = wv;
      lt = fmaf(wv, sml[(s2 * AS_MAXR + r) * 2 + 1], lt);
    }
    for (int o2 = 16; o2 > 0; o2 >>= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o2);
    __syncwarp();
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    for (int s2 = lane; s2 <= S; s2 += kWarp) cw[r * (AS_MAXS + 1) + s2] *= inv;
  }
  __syncthreads();
  for (int it = tid; it < R * (D / 4); it += AS_THREADS) {
    const int r = it / (D / 4), c = (it % (D / 4)) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 <= S; s0 += 8) {  // eight splits' loads in flight at a time
      float4 v[8];
      float wv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int s2 = s0 + u;
        wv[u] = s2 <= S ? cw[r * (AS_MAXS + 1) + s2] : 0.f;
        v[u] = wv[u] != 0.f ? __ldcg(reinterpret_cast<const float4*>(ho + (size_t(s2) * AS_MAXR + r) * D + c))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        acc.x = fmaf(wv[u], v[u].x, acc.x);
        acc.y = fmaf(wv[u], v[u].y, acc.y);
        acc.z = fmaf(wv[u], v[u].z, acc.z);
        acc.w = fmaf(wv[u], v[u].w, acc.w);
      }
    }
    const int l = r / rep, h = hk * rep + r % rep;
    attn_emit(p, l, h * D + c, acc.x);
    attn_emit(p, l, h * D + c + 1, acc.y);
    attn_emit(p, l, h * D + c + 2, acc.z);
    attn_emit(p, l, h * D + c + 3, acc.w);
  }
  if (tid == 0) sp.counters[hk] = 0;  // ready for the next launch
}

}  // namespace wc
