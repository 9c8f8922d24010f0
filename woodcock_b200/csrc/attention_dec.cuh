// Decode / verify attention for bf16 KV caches, built around as few dependent global round
// trips as possible (at batch 1 each one costs about a microsecond while the weight stream
// keeps HBM busy).
//
// Same contract as attention_kernel (attention.cuh) for rule-based visibility (causal new
// rows, optional tree bits in newmask, optional window). One cluster of 8 CTAs per KV head;
// each CTA owns a slice of the committed prefix [0, npre) and every warp of it one or two
// 16-position tiles. When the caller marks the prefix as stable (its length and rows were
// written by work that has completed before this kernel starts, as in the decoder's round
// graphs), the prefix tiles and its length are fetched before the kernel waits on its
// predecessor, so they overlap the QKV projection. After the wait: one round trip for the
// raw q / k / v rows and the lengths, one for the RoPE rows; the new K/V rows are normalised,
// rotated, rounded to bf16 and placed straight into a shared-memory tail tile (positions
// [npre, n + L): rows appended earlier in the same round, then the new rows) owned by the
// last CTA, and CTA 0 appends them to the cache. S = Q K^T and O += P V run on m16n8k16
// MMAs with Q and P split into bf16 hi + lo terms; warps merge in shared memory, CTAs through
// distributed shared memory, and the result is emitted as the O projection's input fragments.
// With one m-tile (at most 16 query rows per KV head) every CTA pushes the column slices of its
// merged partial state into the CTA that owns those columns, so one cluster barrier suffices
// and each CTA merges and emits from its own shared memory (no final barrier); two m-tiles
// merge by reading the peers' partial states between two barriers.
#pragma once

#include <cooperative_groups.h>

#include "attention.cuh"
#include "common.cuh"

namespace wc {

constexpr int AD_THREADS = 256;
constexpr int AD_WARPS = AD_THREADS / kWarp;
constexpr int AD_MAXR = 32;   // query rows per KV head (two 16-row m-tiles)
constexpr int AD_MAXL = 16;   // new rows per launch
constexpr int AD_BLK = 16;    // positions per tile
constexpr int AD_TPW = 2;     // prefix tiles per warp in flight
constexpr int AD_CLUSTER = 8;

template <int D>
struct AdLayout {
  static constexpr int LD = D + 8;  // padded bf16 row stride: conflict-free ldmatrix rows
  static constexpr size_t q_bytes = size_t(AD_MAXR) * LD * 2;                          // per hi / lo
  static constexpr size_t tile_bytes = size_t(2) * AD_BLK * LD * 2;                     // K + V
  static constexpr size_t kv_bytes = size_t(AD_WARPS) * AD_TPW * tile_bytes;
  static constexpr size_t ow_bytes = size_t(AD_WARPS) * AD_MAXR * D * 4;               // warp outputs
  static constexpr size_t region_a = kv_bytes > ow_bytes ? kv_bytes : ow_bytes;
  static constexpr size_t tail_bytes = 2 * tile_bytes;
  static constexpr size_t raw_bytes = size_t(AD_MAXR + 2 * AD_MAXL) * D * 4;
  static constexpr size_t pacc_bytes = size_t(AD_MAXR) * D * 4;
  static constexpr size_t region_b = raw_bytes > pacc_bytes ? raw_bytes : pacc_bytes;
  static constexpr size_t base_total = 2 * q_bytes + region_a + tail_bytes + region_b + 2 * D * 4 +
                                       size_t(AD_MAXL) * RopeSmem<D>::kRow * 8 + AD_MAXL * 4 + 2 * AD_WARPS * AD_MAXR * 4 +
                                       2 * AD_MAXR * 4 + 64;
  // one-m-tile merge: partial column slices pushed by every CTA of the cluster
  static constexpr size_t rx_off = (base_total + 15) / 16 * 16;
  static constexpr size_t rx_bytes = size_t(AD_CLUSTER) * 16 * (D / AD_CLUSTER) * 4 + size_t(AD_CLUSTER) * 16 * 2 * 4;
  static constexpr size_t total = rx_off + rx_bytes;
};

template <int D>
constexpr size_t attention_dec_smem() {
  return AdLayout<D>::total;
}
static_assert(attention_dec_smem<128>() <= kSmemOptinBytes && attention_dec_smem<64>() <= kSmemOptinBytes,
              "the decode attention layout exceeds the per-block shared memory");

template <int D, int MT>
__global__ void __launch_bounds__(AD_THREADS, 1) attention_dec_kernel(__grid_constant__ const AttnParams p) {
  using Lay = AdLayout<D>;
  constexpr int LD = Lay::LD;
  constexpr int NDT = D / 8;  // 8-wide output tiles
  constexpr int d4 = D / 4;
  extern __shared__ __align__(16) unsigned char ad_smem[];
  unsigned char* sm = ad_smem;
  uint16_t* qh = reinterpret_cast<uint16_t*>(sm);                          // [MAXR][LD]
  uint16_t* ql = qh + AD_MAXR * LD;                                        // [MAXR][LD]
  unsigned char* reg_a = sm + 2 * Lay::q_bytes;                            // prefix tiles | warp outputs
  uint16_t* tail = reinterpret_cast<uint16_t*>(reg_a + Lay::region_a);     // [2 tiles][K,V][BLK][LD]
  unsigned char* reg_b = reinterpret_cast<unsigned char*>(tail) + Lay::tail_bytes;  // raw rows | partials
  float* raw = reinterpret_cast<float*>(reg_b);                            // [MAXR + 2 MAXL][D]
  float* pacc = reinterpret_cast<float*>(reg_b);                           // [MAXR][D]
  float* wq = reinterpret_cast<float*>(reg_b + Lay::region_b);             // [D]
  float* wk = wq + D;                                                      // [D]
  float2* rp = reinterpret_cast<float2*>(wk + D);                          // [MAXL][padded D/2]
  int* spos = reinterpret_cast<int*>(rp + AD_MAXL * RopeSmem<D>::kRow);   // [MAXL]
  float* mw = reinterpret_cast<float*>(spos + AD_MAXL);                    // [WARPS][MAXR]
  float* lw = mw + AD_WARPS * AD_MAXR;                                     // [WARPS][MAXR]
  float* pm = lw + AD_WARPS * AD_MAXR;                                     // [MAXR]
  float* pl = pm + AD_MAXR;                                                // [MAXR]
  float* ow = reinterpret_cast<float*>(reg_a);                             // [WARPS][MAXR][D]

  cg::cluster_group cluster = cg::this_cluster();
  // scalar parameters used in the dependent phases, read before the dependency wait and held in
  // registers (a parameter-space read there costs a constant-cache miss on the critical path)
  float pv_eps = p.eps, pv_scale = p.scale * kLog2e;  // scores in log2 units
  int pv_window = p.window;
  const float* pv_qn = p.q_norm;
  const float* pv_kn = p.k_norm;
  const unsigned long long* pv_nm = p.newmask;
  asm volatile("" : "+f"(pv_eps), "+f"(pv_scale), "+r"(pv_window), "+l"(pv_qn), "+l"(pv_kn), "+l"(pv_nm));
  const int S = int(cluster.num_blocks());
  const int rank = int(cluster.block_rank());
  const int hk = blockIdx.y;
  const int rep = p.H / p.Hk;
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const int g = lane >> 2, t = lane & 3;
  const int Lm = p.L_max;
  const uint16_t* Kg = static_cast<const uint16_t*>(p.Kc) + hk * p.stride_h;
  const uint16_t* Vg = static_cast<const uint16_t*>(p.Vc) + hk * p.stride_h;

  // committed prefix length (stable: written by completed work) and the norm gains, together
  const int npre_stable = (p.stable_prefix && p.n_dev) ? *p.n_dev : 0;
  for (int i = tid; i < D; i += AD_THREADS) {  // weights: independent of the previous kernel
    wq[i] = pv_qn ? pv_qn[i] : 1.f;
    wk[i] = pv_kn ? pv_kn[i] : 1.f;
  }
  // this CTA's slice of the committed prefix [0, npre), in 16-position tiles
  int q0 = 0, q1 = 0, ntiles = 0;
  auto set_prefix = [&](int npre) {
    const int chunk = ((npre + S - 1) / S + AD_BLK - 1) / AD_BLK * AD_BLK;
    q0 = min(npre, rank * chunk);
    q1 = min(npre, q0 + chunk);
    ntiles = (q1 - q0 + AD_BLK - 1) / AD_BLK;
  };
  // batch b: this warp's tiles warp + WARPS * (b * TPW + i), i < TPW, into its own buffers
  auto load_batch = [&](int b) {
#pragma unroll
    for (int i = 0; i < AD_TPW; ++i) {
      const int tile = warp + AD_WARPS * (b * AD_TPW + i);
      uint16_t* kb = reinterpret_cast<uint16_t*>(reg_a + (size_t(warp) * AD_TPW + i) * Lay::tile_bytes);
      uint16_t* vb = kb + AD_BLK * LD;
      if (tile >= ntiles) continue;
      const int pos0 = q0 + tile * AD_BLK;
      constexpr int cpr = D / 8;  // 16-byte chunks per row
#pragma unroll
      for (int c = lane; c < AD_BLK * cpr; c += kWarp) {
        const int row = c / cpr, col = (c % cpr) * 8, pos = pos0 + row;
        const bool ok = pos < q1;
        const long long off = ok ? (long long)pos * p.stride_p + col : 0;
        cp_async16(kb + row * LD + col, Kg + off, ok ? 16 : 0);
        cp_async16(vb + row * LD + col, Vg + off, ok ? 16 : 0);
      }
    }
    cp_async_commit();
  };
  int npre = -1;
  bool rope_ready = false;
  constexpr int ROPEV = AD_MAXL * (D / 2) / AD_THREADS;
  if (p.stable_prefix) {
    npre = npre_stable;
    if (npre < 0 || npre > p.cap) npre = 0;  // reported below through n
    set_prefix(npre);
    load_batch(0);
    if (!p.positions) {  // positions npre + n_add + l are known: fetch the RoPE rows now
      const int n0 = npre + p.n_add;
      float2 rr[ROPEV > 0 ? ROPEV : 1];
#pragma unroll
      for (int i = 0; i < ROPEV; ++i) {
        const int idx = tid + i * AD_THREADS, pos = n0 + idx / (D / 2);
        if (idx < Lm * (D / 2) && pos >= 0 && pos < p.max_pos) rr[i] = p.rope[size_t(pos) * (D / 2) + idx % (D / 2)];
      }
#pragma unroll
      for (int i = 0; i < ROPEV; ++i) {
        const int idx = tid + i * AD_THREADS;
        if (idx < Lm * (D / 2)) rp[RopeSmem<D>::at(idx / (D / 2), idx % (D / 2))] = rr[i];
      }
      rope_ready = true;
    }
  }

  pdl_launch_dependents();
  pdl_wait();

  // ---- round trip 1: lengths, raw q / k / v rows (all L_max rows), positions
  int L = p.L_dev ? *p.L_dev : p.L;
  const int nd = p.n_dev ? *p.n_dev : 0;
  constexpr int RAWV = (AD_MAXR + 2 * AD_MAXL) * d4 / AD_THREADS;
  const int nraw_max = Lm * rep + 2 * Lm;
  float4 rv[RAWV];
#pragma unroll
  for (int i = 0; i < RAWV; ++i) {
    const int idx = tid + i * AD_THREADS;
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
  int mypos = 0;
  if (tid < Lm && p.positions) mypos = p.positions[tid];
  const int n = nd + p.n_add;
  if (L < 0 || L > Lm) {
    if (tid == 0) raise_error(p.err, kErrRows);
    L = L < 0 ? 0 : Lm;
  }
  const int R = L * rep;
  if (R > AD_MAXR || Lm > AD_MAXL) {
    if (tid == 0) raise_error(p.err, kErrRows);
    cp_async_wait<0>();
    return;  // uniform across the cluster
  }
  if (npre < 0) {  // prefix not marked stable: everything before n is prefix, loaded now
    npre = n;
    set_prefix(npre);
    load_batch(0);
  }
  const bool owns_tail = rank == S - 1;
  const int tl = n + L - npre;  // tail positions [npre, n + L)
  if (tl > 2 * AD_BLK || npre > n) {
    if (tid == 0) raise_error(p.err, kErrRows);
    cp_async_wait<0>();
    return;
  }
  // raw rows to shared memory (row-major as loaded)
#pragma unroll
  for (int i = 0; i < RAWV; ++i) {
    const int idx = tid + i * AD_THREADS;
    if (idx < nraw_max * d4) *reinterpret_cast<float4*>(&raw[(idx / d4) * D + (idx % d4) * 4]) = rv[i];
  }
  if (tid < Lm) {
    int pos = p.positions ? mypos : n + tid;
    if (pos < 0 || pos >= p.max_pos) {
      if (tid < L) raise_error(p.err, kErrPosition);
      pos = 0;
    }
    spos[tid] = pos;
  }
  // tail tiles: earlier rows of this round from the cache, zero elsewhere (new rows land below)
  if (owns_tail) {
    constexpr int cpr = D / 8;
    for (int c = tid; c < 2 * AD_BLK * cpr; c += AD_THREADS) {
      const int ti = c / cpr, col = (c % cpr) * 8, pos = npre + ti;
      uint16_t* kb = tail + (ti / AD_BLK) * 2 * AD_BLK * LD;
      uint16_t* vb = kb + AD_BLK * LD;
      const int row = ti % AD_BLK;
      if (pos < n && pos < p.cap) {
        cp_async16(kb + row * LD + col, Kg + (long long)pos * p.stride_p + col, 16);
        cp_async16(vb + row * LD + col, Vg + (long long)pos * p.stride_p + col, 16);
      } else {  // new rows are written below, after two barriers; the rest stays zero
        *reinterpret_cast<uint4*>(kb + row * LD + col) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(vb + row * LD + col) = make_uint4(0, 0, 0, 0);
      }
    }
  }
  cp_async_commit();
  __syncthreads();

  // ---- round trip 2: RoPE rows (unless fetched before the wait)
  if (!rope_ready || n != npre + p.n_add) {
    float2 rr[ROPEV > 0 ? ROPEV : 1];
#pragma unroll
    for (int i = 0; i < ROPEV; ++i) {
      const int idx = tid + i * AD_THREADS;
      if (idx < L * (D / 2)) rr[i] = p.rope[size_t(spos[idx / (D / 2)]) * (D / 2) + idx % (D / 2)];
    }
#pragma unroll
    for (int i = 0; i < ROPEV; ++i) {
      const int idx = tid + i * AD_THREADS;
      if (idx < L * (D / 2)) rp[RopeSmem<D>::at(idx / (D / 2), idx % (D / 2))] = rr[i];
    }
  }
  // zero the padding query rows (they only feed output rows that are never stored)
  for (int idx = tid; idx < (MT * 16 - R > 0 ? MT * 16 - R : 0) * LD; idx += AD_THREADS) {
    qh[R * LD + idx] = 0;
    ql[R * LD + idx] = 0;
  }
  __syncthreads();

  // ---- per-head RMSNorm + RoPE, eight lanes per row (lane j of the eight holds elements
  // [j * EPQ, (j + 1) * EPQ); the rotate-half partner of element d < D/2 sits in lane j ^ 4):
  // q -> bf16 hi / lo tiles; new k / v -> bf16, tail tile + cache. Every row of a block is in
  // flight in one pass; only the blocks that store k / v (the tail owner, rank 0 for the
  // cache) process those rows.
  const bool cache_ok = n + L <= p.cap;
  if (!cache_ok && tid == 0) raise_error(p.err, kErrCapacity);
  constexpr int EPQ = D / 8;
  const bool need_kv = owns_tail || (rank == 0 && p.write_cache && cache_ok);
  const int nrows = R + (need_kv ? 2 * L : 0);
  const int sub = lane & 7;
  for (int base = 0; base < nrows; base += AD_THREADS / 8) {  // uniform across the block
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
    if (valid && ((is_q && pv_qn) || (is_k && pv_kn))) {
      const float* w = is_q ? wq : wk;
      const float inv = rsqrtf(ss / float(D) + pv_eps);
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
      if (owns_tail) {
        const int ti = n + l - npre;
        uint16_t* dst = tail + (ti / AD_BLK) * 2 * AD_BLK * LD + (is_k ? 0 : AD_BLK * LD) + (ti % AD_BLK) * LD;
#pragma unroll
        for (int e = 0; e < EPQ; ++e) dst[sub * EPQ + e] = bv[e];
      }
      if (rank == 0 && p.write_cache && cache_ok) {
        uint16_t* dst = static_cast<uint16_t*>(is_k ? p.Kc : p.Vc) + hk * p.stride_h + (long long)(n + l) * p.stride_p;
#pragma unroll
        for (int e = 0; e < EPQ; ++e) dst[sub * EPQ + e] = bv[e];
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- tiles: each warp its prefix tiles, the last CTA's last warps the tail tiles
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
  // one 16-position tile: positions pos_base.., visible below `end`
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
    // masked online softmax; each row's 16 scores live in one lane quad
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
              if (pos < n) {
                vis = pv_window <= 0 || pos >= n + l - pv_window + 1;
              } else {
                const int jj = pos - n;
                vis = pv_nm ? ((pv_nm[l] >> jj) & 1ull) != 0 : jj <= l;
                if (vis && pv_window > 0) vis = pos >= n + l - pv_window + 1;
              }
            }
            const float sv = vis ? pv_scale * s[mt][nt][2 * h + c] : -INFINITY;
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
    // O += P V: the score C-fragments are the A fragments of P (hi + lo)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
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
  bool worked = false;  // this warp ran at least one tile (idle warps skip the merge traffic)
  const int nbatch = (ntiles + AD_WARPS * AD_TPW - 1) / (AD_WARPS * AD_TPW);
  for (int b = 0; b < nbatch; ++b) {
    if (b > 0) {  // longer prefixes: refill this warp's buffers (one more round trip per batch)
      __syncwarp();
      load_batch(b);
      cp_async_wait<0>();
      __syncwarp();
    }
#pragma unroll
    for (int i = 0; i < AD_TPW; ++i) {
      const int tl_idx = warp + AD_WARPS * (b * AD_TPW + i);
      if (tl_idx >= ntiles) continue;
      const uint16_t* kb = reinterpret_cast<const uint16_t*>(reg_a + (size_t(warp) * AD_TPW + i) * Lay::tile_bytes);
      tile(kb, kb + AD_BLK * LD, q0 + tl_idx * AD_BLK, q1);
      worked = true;
    }
  }
  if (owns_tail) {
    const int ntail = (tl + AD_BLK - 1) / AD_BLK;
    const int j = AD_WARPS - 1 - warp;  // warps 7 and 6
    if (j < ntail) {
      const uint16_t* kb = tail + j * 2 * AD_BLK * LD;
      tile(kb, kb + AD_BLK * LD, npre + j * AD_BLK, n + L);
      worked = true;
    }
  }
  __syncthreads();  // every warp is done with its tiles: region A now holds warp outputs

  // ---- merge the warps' states in shared memory
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + g + 8 * h;
      if (r < R) {
        if (worked) {
#pragma unroll
          for (int dt = 0; dt < NDT; ++dt) {
            *reinterpret_cast<float2*>(&ow[(warp * AD_MAXR + r) * D + dt * 8 + 2 * t]) =
                make_float2(o[mt][dt][2 * h], o[mt][dt][2 * h + 1]);
          }
        }
        if (t == 0) {
          mw[warp * AD_MAXR + r] = mrow[mt][h];
          lw[warp * AD_MAXR + r] = lrow[mt][h];
        }
      }
    }
  }
  __syncthreads();
  // per-row weights once (row r, warp w): thread r * 8 + w
  if (warp * kWarp < R * AD_WARPS) {  // whole warps take part in the shuffles
    const bool act = tid < R * AD_WARPS;
    const int r = act ? tid / AD_WARPS : 0, w = tid % AD_WARPS;
    const float mv = act ? mw[w * AD_MAXR + r] : -INFINITY;
    float M = mv;
#pragma unroll
    for (int o2 = 1; o2 < AD_WARPS; o2 <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
    const float wt = (mv == -INFINITY) ? 0.f : ex2_approx(mv - M);
    float lt = act ? wt * lw[w * AD_MAXR + r] : 0.f;
#pragma unroll
    for (int o2 = 1; o2 < AD_WARPS; o2 <<= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o2);
    __syncwarp();
    if (act) {
      mw[w * AD_MAXR + r] = wt;  // the warp's weight for row r
      if (w == 0) {
        pm[r] = M;
        pl[r] = lt;
      }
    }
  }
  __syncthreads();
  for (int idx = tid; idx < R * D; idx += AD_THREADS) {
    const int r = idx / D, d = idx % D;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < AD_WARPS; ++w) {
      const float wt = mw[w * AD_MAXR + r];
      if (wt != 0.f) acc = fmaf(wt, ow[(w * AD_MAXR + r) * D + d], acc);  // idle warps have weight 0
    }
    pacc[r * D + d] = acc;
  }
  if constexpr (MT == 1) {
    constexpr int CW = D / AD_CLUSTER;  // output columns this CTA merges and emits
    float* rx = reinterpret_cast<float*>(ad_smem + Lay::rx_off);  // [source CTA][16 rows][CW]
    float* rml = rx + AD_CLUSTER * 16 * CW;                         // [source CTA][16 rows][m, l]
    __syncthreads();  // pacc complete
    for (int idx = tid; idx < R * D; idx += AD_THREADS) {
      const int r = idx / D, d = idx % D;
      cluster.map_shared_rank(rx, d / CW)[(rank * 16 + r) * CW + d % CW] = pacc[r * D + d];
    }
    if (tid < R * AD_CLUSTER) {
      const int r = tid / AD_CLUSTER, j = tid % AD_CLUSTER;
      float* dst = cluster.map_shared_rank(rml, j) + (rank * 16 + r) * 2;
      dst[0] = pm[r];
      dst[1] = pl[r];
    }
    cluster.sync();  // every CTA's slices have landed; only local shared memory is read below
    float* cw = lw;  // [MAXR][CLUSTER] weights / l
    if (warp * kWarp < R * AD_CLUSTER) {  // whole warps take part in the shuffles
      const bool act = tid < R * AD_CLUSTER;
      const int r = act ? tid / AD_CLUSTER : 0, s2 = tid % AD_CLUSTER;
      const float mv = act ? rml[(s2 * 16 + r) * 2] : -INFINITY;
      const float lv = act ? rml[(s2 * 16 + r) * 2 + 1] : 0.f;
      float M = mv;
#pragma unroll
      for (int o2 = 1; o2 < AD_CLUSTER; o2 <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
      const float wt = (mv == -INFINITY) ? 0.f : ex2_approx(mv - M);
      float lt = wt * lv;
#pragma unroll
      for (int o2 = 1; o2 < AD_CLUSTER; o2 <<= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o2);
      if (act) cw[r * AD_CLUSTER + s2] = wt / lt;
    }
    __syncthreads();
    for (int idx = tid; idx < R * CW; idx += AD_THREADS) {
      const int r = idx / CW, c = idx % CW;
      float acc = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < AD_CLUSTER; ++s2) acc = fmaf(cw[r * AD_CLUSTER + s2], rx[(s2 * 16 + r) * CW + c], acc);
      const int l = r / rep, h = hk * rep + r % rep;
      attn_emit(p, l, h * D + rank * CW + c, acc);
    }
    return;  // no peer reads this CTA's shared memory after the barrier
  }
  cluster.sync();
  // ---- merge the cluster's CTAs through distributed shared memory. This CTA emits elements
  // [e0, e1) of the R x D output; per-row CTA weights first (thread = row * 8 + CTA).
  const int per = (R * D + S - 1) / S, e0 = min(R * D, rank * per), e1 = min(R * D, e0 + per);
  const int r0 = e0 / D, r1 = e1 > e0 ? (e1 - 1) / D + 1 : r0;
  float* cw = lw;  // [MAXR][CLUSTER] weights / l (the warp sums are no longer needed)
  if (warp * kWarp < (r1 - r0) * AD_CLUSTER) {  // whole warps take part in the shuffles
    const bool act = tid < (r1 - r0) * AD_CLUSTER;
    const int r = r0 + (act ? tid / AD_CLUSTER : 0), s2 = tid % AD_CLUSTER;
    const float mv = (act && s2 < S) ? cluster.map_shared_rank(pm, s2)[r] : -INFINITY;
    const float lv = (act && s2 < S) ? cluster.map_shared_rank(pl, s2)[r] : 0.f;
    float M = mv;
#pragma unroll
    for (int o2 = 1; o2 < AD_CLUSTER; o2 <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
    const float wt = (mv == -INFINITY) ? 0.f : ex2_approx(mv - M);
    float lt = wt * lv;
#pragma unroll
    for (int o2 = 1; o2 < AD_CLUSTER; o2 <<= 1) lt += __shfl_xor_sync(0xffffffffu, lt, o2);
    if (act) cw[r * AD_CLUSTER + s2] = wt / lt;
  }
  __syncthreads();
  for (int idx = e0 + tid; idx < e1; idx += AD_THREADS) {
    const int r = idx / D, d = idx % D;
    float acc = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < AD_CLUSTER; ++s2)
      if (s2 < S) acc = fmaf(cw[r * AD_CLUSTER + s2], cluster.map_shared_rank(pacc, s2)[r * D + d], acc);
    const int l = r / rep, h = hk * rep + r % rep;
    attn_emit(p, l, h * D + d, acc);
  }
  cluster.sync();
}

}  // namespace wc
