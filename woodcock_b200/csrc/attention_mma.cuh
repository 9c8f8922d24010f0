// Tensor-core decode / verify attention for bf16 KV caches (FlashDecoding on mma.sync).
//
// Same contract as attention_kernel (attention.cuh): one thread-block cluster per KV
// head, blocks split the positions, partial softmax states combine through
// distributed shared memory. Inside a block every warp is an independent split:
// it streams 16-position K/V blocks into its own double-buffered shared tiles with
// cp.async, computes S = Q K^T and O += P V with m16n8k16 MMAs (Q and P split into
// bf16 hi + lo terms, so products keep fp32-level accuracy against the bf16 cache),
// and keeps its own online-softmax state; the four warps are merged in shared
// memory, then the cluster's blocks over DSMEM. New K/V rows are normalised, rotated
// and appended by every block of the cluster (identical values), so each block can
// read the whole range [0, n + L) from the cache.
#pragma once

#include <cooperative_groups.h>

#include "attention.cuh"
#include "common.cuh"

namespace wc {

constexpr int AM_THREADS = 128;
constexpr int AM_WARPS = AM_THREADS / kWarp;
constexpr int AM_MAXR = 32;  // query rows per KV head: two 16-row m-tiles
constexpr int AM_BLK = 16;   // positions per warp iteration
constexpr int AM_CLUSTER = 8;

template <int D>
struct AmLayout {
  static constexpr int LD = D + 8;  // padded bf16 row stride: conflict-free ldmatrix rows
  static constexpr size_t q_bytes = size_t(AM_MAXR) * LD * 2;
  static constexpr size_t kv_bytes = size_t(AM_WARPS) * 2 * 2 * AM_BLK * LD * 2;
  static constexpr size_t ow_bytes = size_t(AM_WARPS) * AM_MAXR * D * 4;
  static constexpr size_t region = kv_bytes > ow_bytes ? kv_bytes : ow_bytes;
};

template <int D>
inline size_t attention_mma_smem(int L_max) {
  using Lay = AmLayout<D>;
  const size_t raw = size_t(AM_MAXR + 2 * L_max) * D * 4;
  const size_t region = Lay::region > raw ? Lay::region : raw;
  return 2 * Lay::q_bytes + region + 2 * D * 4 + size_t(L_max) * (D / 2) * 8 + size_t(L_max) * 4 + 16 +
         2 * AM_WARPS * AM_MAXR * 4 + size_t(AM_MAXR) * D * 4 + 2 * AM_MAXR * 4 + 64;
}

template <int D>
__global__ void __launch_bounds__(AM_THREADS) attention_mma_kernel(__grid_constant__ const AttnParams p) {
  using Lay = AmLayout<D>;
  constexpr int LD = Lay::LD;
  constexpr int NDT = D / 8;  // 8-wide output tiles
  extern __shared__ __align__(16) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int S = int(cluster.num_blocks());
  const int rank = int(cluster.block_rank());
  const int hk = blockIdx.y;
  const int rep = p.H / p.Hk;
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const int g = lane >> 2, t = lane & 3;
  const int Lm = p.L_max;

  const size_t raw_bytes = size_t(AM_MAXR + 2 * Lm) * D * 4;
  const size_t region = Lay::region > raw_bytes ? Lay::region : raw_bytes;
  uint16_t* qh = reinterpret_cast<uint16_t*>(smem);                    // [MAXR][LD]
  uint16_t* ql = qh + AM_MAXR * LD;                                    // [MAXR][LD]
  unsigned char* reg = smem + 2 * Lay::q_bytes;                        // kv tiles | staging | warp outputs
  float* raw = reinterpret_cast<float*>(reg);                          // [MAXR + 2 Lm][D]
  uint16_t* kvb = reinterpret_cast<uint16_t*>(reg);                    // [WARPS][2][2][BLK][LD]
  float* ow = reinterpret_cast<float*>(reg);                           // [WARPS][MAXR][D]
  float* wq = reinterpret_cast<float*>(reg + region);                  // [D]
  float* wk = wq + D;                                                  // [D]
  float2* rp = reinterpret_cast<float2*>(wk + D);                      // [Lm][D/2]
  int* spos = reinterpret_cast<int*>(rp + Lm * (D / 2));               // [Lm]
  float* mw = reinterpret_cast<float*>(spos + ((Lm + 3) & ~3));        // [WARPS][MAXR]
  float* lw = mw + AM_WARPS * AM_MAXR;                                 // [WARPS][MAXR]
  float* pacc = lw + AM_WARPS * AM_MAXR;                               // [MAXR][D]
  float* pm = pacc + AM_MAXR * D;                                      // [MAXR]
  float* pl = pm + AM_MAXR;                                            // [MAXR]

  pdl_launch_dependents();
  pdl_wait();
  int L = p.L_dev ? *p.L_dev : p.L;
  const int n = (p.n_dev ? *p.n_dev : 0) + p.n_add;
  if (L < 0 || L > p.L_max) {
    raise_error(p.err, kErrRows);
    L = L < 0 ? 0 : p.L_max;
  }
  const int R = L * rep;
  const int T = n + L;
  if (R > AM_MAXR) {
    raise_error(p.err, kErrRows);
    return;  // uniform across the cluster
  }

  // ---- stage raw q / k / v rows, norm gains, positions and RoPE rows
  constexpr int d4 = D / 4;
  const int nraw = R + 2 * L;
  for (int idx = tid; idx < nraw * d4; idx += AM_THREADS) {
    const int row = idx / d4, c = (idx % d4) * 4;
    int head, l;
    if (row < R) {
      l = row / rep;
      head = hk * rep + row % rep;
    } else {
      const int j = row - R;
      l = j % L;
      head = p.H + (j < L ? 0 : p.Hk) + hk;
    }
    *reinterpret_cast<float4*>(&raw[row * D + c]) =
        *reinterpret_cast<const float4*>(p.qkv + size_t(l) * p.ld_qkv + size_t(head) * D + c);
  }
  for (int i = tid; i < D; i += AM_THREADS) {
    wq[i] = p.q_norm ? p.q_norm[i] : 1.f;
    wk[i] = p.k_norm ? p.k_norm[i] : 1.f;
  }
  for (int l = tid; l < L; l += AM_THREADS) {
    int pos = p.positions ? p.positions[l] : n + l;
    if (pos < 0 || pos >= p.max_pos) {
      raise_error(p.err, kErrPosition);
      pos = 0;
    }
    spos[l] = pos;
  }
  __syncthreads();
  for (int idx = tid; idx < L * (D / 2); idx += AM_THREADS)
    rp[idx] = p.rope[size_t(spos[idx / (D / 2)]) * (D / 2) + idx % (D / 2)];
  // zero the padding query rows (they only feed output rows that are never stored)
  for (int idx = tid; idx < (2 * 16 - R > 0 ? 2 * 16 - R : 0) * LD; idx += AM_THREADS) {
    qh[R * LD + idx] = 0;
    ql[R * LD + idx] = 0;
  }
  __syncthreads();

  // ---- per-head RMSNorm + RoPE; q -> bf16 hi/lo tiles, k/v -> the cache (every block)
  constexpr int EPL = D / kWarp;
  for (int it = warp; it < nraw; it += AM_WARPS) {
    float v[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) v[e] = raw[it * D + lane * EPL + e];
    const bool is_q = it < R;
    const int j = it - R;
    const bool is_k = !is_q && j < L;
    const int l = is_q ? it / rep : j % L;
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
    } else if (p.write_cache) {
      const int cidx = n + l;
      if (cidx < p.cap) {
        uint16_t* dst = static_cast<uint16_t*>(is_k ? p.Kc : p.Vc) + hk * p.stride_h + (long long)cidx * p.stride_p;
#pragma unroll
        for (int e = 0; e < EPL; ++e) dst[lane * EPL + e] = f32_to_bf16_bits(v[e]);
      } else if (lane == 0) {
        raise_error(p.err, kErrCapacity);
      }
    }
  }
  __threadfence_block();
  __syncthreads();

  // ---- this block's positions, 16 at a time per warp
  const int chunk = (T + S - 1) / S;
  const int p0 = min(T, rank * chunk), p1 = min(T, p0 + chunk);
  const int nblk = (p1 - p0 + AM_BLK - 1) / AM_BLK;
  const int MT = (R + 15) / 16;
  float o[2][NDT][4];
  float mrow[2][2], lrow[2][2];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
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
  uint16_t* mykv = kvb + size_t(warp) * 2 * 2 * AM_BLK * LD;
  const uint16_t* Kg = static_cast<const uint16_t*>(p.Kc) + hk * p.stride_h;
  const uint16_t* Vg = static_cast<const uint16_t*>(p.Vc) + hk * p.stride_h;
  auto load_block = [&](int b, int stage) {
    uint16_t* kb = mykv + size_t(stage) * 2 * AM_BLK * LD;
    uint16_t* vb = kb + AM_BLK * LD;
    const int pos0 = p0 + b * AM_BLK;
    constexpr int cpr = D / 8;  // 16-byte chunks per row
#pragma unroll
    for (int c = lane; c < AM_BLK * cpr; c += kWarp) {
      const int row = c / cpr, col = (c % cpr) * 8, pos = pos0 + row;
      const bool ok = pos < p1 && pos < p.cap;
      const long long off = ok ? (long long)pos * p.stride_p + col : 0;
      cp_async16(kb + row * LD + col, Kg + off, ok ? 16 : 0);
      cp_async16(vb + row * LD + col, Vg + off, ok ? 16 : 0);
    }
    cp_async_commit();
  };
  if (warp < nblk) load_block(warp, 0);
  else cp_async_commit();
  int stage = 0;
  for (int b = warp; b < nblk; b += AM_WARPS) {
    if (b + AM_WARPS < nblk) load_block(b + AM_WARPS, stage ^ 1);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    const uint16_t* kb = mykv + size_t(stage) * 2 * AM_BLK * LD;
    const uint16_t* vb = kb + AM_BLK * LD;
    float s[2][2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[mt][nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t bk[4];
      ldsm_x4(bk, kb + ((lane & 7) + 8 * (lane >> 4)) * LD + ks * 16 + 8 * ((lane >> 3) & 1));
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        if (mt < MT) {
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
    }
    // masked online softmax; each row's 16 scores live in one lane quad
    const int pos_base = p0 + b * AM_BLK;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      if (mt >= MT) continue;
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
            bool vis = r < R && pos < p1;
            if (vis) {
              if (pos < n) {
                vis = p.window <= 0 || pos >= n + l - p.window + 1;
              } else {
                const int jj = pos - n;
                vis = p.newmask ? ((p.newmask[l] >> jj) & 1ull) != 0 : jj <= l;
                if (vis && p.window > 0) vis = pos >= n + l - p.window + 1;
              }
            }
            const float sv = vis ? p.scale * s[mt][nt][2 * h + c] : -INFINITY;
            s[mt][nt][2 * h + c] = sv;
            mx = fmaxf(mx, sv);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float mn = fmaxf(mrow[mt][h], mx);
        const float alpha = (mn == -INFINITY || mrow[mt][h] == -INFINITY) ? (mn == -INFINITY ? 1.f : 0.f)
                                                                          : expf(mrow[mt][h] - mn);
        float sum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const float sv = s[mt][nt][2 * h + c];
            const float e = (sv == -INFINITY) ? 0.f : expf(sv - mn);
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
    for (int mt = 0; mt < 2; ++mt) {
      if (mt >= MT) continue;
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
    __syncwarp();
    stage ^= 1;
  }
  cp_async_wait<0>();
  __syncthreads();  // every warp is done with its K/V tiles: the region now holds warp outputs

  // ---- merge the four warps' states in shared memory
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = mt * 16 + g + 8 * h;
      if (mt < MT && r < R) {
#pragma unroll
        for (int dt = 0; dt < NDT; ++dt) {
          ow[(warp * AM_MAXR + r) * D + dt * 8 + 2 * t] = o[mt][dt][2 * h];
          ow[(warp * AM_MAXR + r) * D + dt * 8 + 2 * t + 1] = o[mt][dt][2 * h + 1];
        }
        if (t == 0) {
          mw[warp * AM_MAXR + r] = mrow[mt][h];
          lw[warp * AM_MAXR + r] = lrow[mt][h];
        }
      }
    }
  }
  __syncthreads();
  for (int idx = tid; idx < R * D; idx += AM_THREADS) {
    const int r = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < AM_WARPS; ++w) M = fmaxf(M, mw[w * AM_MAXR + r]);
    float acc = 0.f, lt = 0.f;
#pragma unroll
    for (int w = 0; w < AM_WARPS; ++w) {
      const float mv = mw[w * AM_MAXR + r];
      const float wt = (mv == -INFINITY) ? 0.f : expf(mv - M);
      acc += wt * ow[(w * AM_MAXR + r) * D + d];
      lt += wt * lw[w * AM_MAXR + r];
    }
    pacc[r * D + d] = acc;
    if (d == 0) {
      pm[r] = M;
      pl[r] = lt;
    }
  }
  cluster.sync();
  // ---- merge the cluster's blocks through distributed shared memory
  for (int r = rank; r < R; r += S) {
    float ms[AM_CLUSTER], M = -INFINITY;
#pragma unroll
    for (int s2 = 0; s2 < AM_CLUSTER; ++s2) {
      ms[s2] = s2 < S ? cluster.map_shared_rank(pm, s2)[r] : -INFINITY;
      M = fmaxf(M, ms[s2]);
    }
    float lt = 0.f, acc = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < AM_CLUSTER; ++s2) {
      if (s2 >= S) continue;
      const float wt = (ms[s2] == -INFINITY) ? 0.f : expf(ms[s2] - M);
      lt += wt * cluster.map_shared_rank(pl, s2)[r];
      if (tid < D) acc += wt * cluster.map_shared_rank(pacc, s2)[r * D + tid];
    }
    if (tid < D) {
      const int l = r / rep, h = hk * rep + r % rep;
      attn_emit(p, l, h * D + tid, acc / lt);
    }
  }
  cluster.sync();
}

}  // namespace wc
