// Decode / verify attention for the round (GQA, L new rows over a KV cache).
//
// One thread-block cluster per KV head; the cluster's blocks split the context
// positions (split-KV) and combine their partial softmax states through
// distributed shared memory, so there is no second launch and no cross-block
// spin-wait. Each block first finishes the new rows of its head: per-head q/k
// RMSNorm (q_norm/k_norm), rotate-half RoPE from a host-built cos/sin table and,
// in block 0, the KV-cache append (the reference's rmsnorm -> rope -> append ->
// attention sequence, src/core/qwen3.cpp:90-96; python/woodcock/target.py:142-153).
//
// Visibility of cache position p for new row l (prefix n = cache size before the rows):
//   p <  n : lo_l <= p, with lo_l = max(0, n + l - window + 1) under a sliding window, else 0;
//   p >= n : bit (p - n) of newmask[l] (nullptr = causal: p - n <= l).
// With mask_from_prefix, n above is the committed length *n_dev instead, so the bits also
// cover rows appended earlier in the same round (drafted tree levels: a drafted node sees the
// committed entries, its drafted ancestors and itself, src/core/spec.cpp:158-171).
// This covers the causal chain, tree masks (prefix + ancestors + self,
// src/sampling/sampling.cpp:85-93) and the drafter window (src/core/qwen3.cpp:44-53).
// A full uint8 mask [L][T] (ops::attention, include/woodcock/ops.h:20) is also accepted.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace wc {

namespace cg = cooperative_groups;

constexpr int ATT_THREADS = 128;
constexpr int ATT_WARPS = ATT_THREADS / kWarp;
constexpr int ATT_TP = 32;        // positions per tile (one per lane)
constexpr int ATT_MAXR = 64;      // query rows (L * heads per KV head) per launch
constexpr int ATT_RPW = ATT_MAXR / ATT_WARPS;
constexpr int ATT_MAXD = 128;
constexpr int ATT_EPL = ATT_MAXD / kWarp;

struct AttnParams {
  // new rows: raw projections qkv [L][(H + 2Hk) * D] (q heads, k heads, v heads)
  const float* qkv;
  int ld_qkv;
  const float* q_norm;
  const float* k_norm;
  float eps;
  const float2* rope;  // [max_pos][D/2] (cos, sin)
  int max_pos;
  const int* positions;  // [L] RoPE positions, nullptr = n + l
  // alternatively ready queries q [L][H][D] (ops API): no new rows, no norm/rope
  const float* q_ready;
  const int* n_dev;      // prefix length = *n_dev + n_add (n_dev may be nullptr)
  int n_add;
  int L;
  const int* L_dev;
  int L_max;
  // cache: element (head h, position p, dim d) at base + h * stride_h + p * stride_p + d
  void* Kc;
  void* Vc;
  int kv_dtype;
  long long stride_h, stride_p;
  int cap;
  int H, Hk, D;
  const unsigned long long* newmask;
  int window;
  const uint8_t* mask_full;  // [L][mask_ld] explicit mask, overrides the rule above
  int mask_ld;
  int T_full;                // ops API (q_ready): T (then n = T and L new rows = 0)
  float scale;
  float* out;
  int ld_out;  // out row stride (floats); head h of row l at out + l*ld_out + h*D
  uint32_t* xf_out;  // optional: the output as input fragments of the o-projection
  int xf_width;      // their (padded) width, >= H*D
  int xf_fp32;       // fp32 models: xf_out holds plain fp32 rows [16][H*D]
  int write_cache;
  int mask_from_prefix;  // newmask bits count from *n_dev (the committed length), not from n
  int stable_prefix;  // n_dev and the cache rows below it were written by completed work
                      // (not by a kernel that may still run): they may be read before the
                      // dependency wait
  int* err;
};

// Shared-memory RoPE table of the new rows, [row][D/2] (cos, sin) pairs stored in groups of 16
// pairs padded to 18: the norm loop's lanes read 16 consecutive pairs of one group per row, and
// with unpadded power-of-two strides every group and row fell into the same banks.
template <int D>
struct RopeSmem {
  static constexpr int kGroups = D / 32;       // 16-pair groups per row
  static constexpr int kRow = kGroups * 18;    // pairs per padded row
  __device__ __forceinline__ static int at(int l, int pair) { return l * kRow + (pair >> 4) * 18 + (pair & 15); }
};

__device__ __forceinline__ void attn_emit(const AttnParams& p, int l, int col, float v) {
  if (p.out) p.out[size_t(l) * p.ld_out + col] = v;
  if (p.xf_out) {
    if (p.xf_fp32) reinterpret_cast<float*>(p.xf_out)[size_t(l) * p.H * p.D + col] = v;
    else xf_store(p.xf_out, p.xf_width, l, col, v);
  }
}

__device__ __forceinline__ float kv_load(const void* base, int dtype, long long off) {
  return dtype == 1 ? bf16_bits_to_f32(static_cast<const uint16_t*>(base)[off]) : static_cast<const float*>(base)[off];
}
__device__ __forceinline__ float kv_round(float v, int dtype) {
  return dtype == 1 ? bf16_bits_to_f32(f32_to_bf16_bits(v)) : v;
}
__device__ __forceinline__ void kv_store(void* base, int dtype, long long off, float v) {
  if (dtype == 1) static_cast<uint16_t*>(base)[off] = f32_to_bf16_bits(v);
  else static_cast<float*>(base)[off] = v;
}

__global__ void __launch_bounds__(ATT_THREADS) attention_kernel(__grid_constant__ const AttnParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int S = int(cluster.num_blocks());
  const int rank = int(cluster.block_rank());
  const int hk = blockIdx.y;
  const int D = p.D, epl = D / kWarp, rep = p.H / p.Hk;
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;
  const int Lm = p.L_max;

  float* qs = reinterpret_cast<float*>(smem);                 // [MAXR][MAXD] queries (normed, roped)
  float* kn = qs + ATT_MAXR * ATT_MAXD;                        // [Lm][MAXD] new K rows
  float* vn = kn + Lm * ATT_MAXD;                              // [Lm][MAXD] new V rows
  float* raw = vn + Lm * ATT_MAXD;                             // [MAXR + 2 Lm][MAXD] staged inputs
  float* wq = raw + (ATT_MAXR + 2 * Lm) * ATT_MAXD;            // [MAXD]
  float* wk = wq + ATT_MAXD;                                   // [MAXD]
  float2* rp = reinterpret_cast<float2*>(wk + ATT_MAXD);       // [Lm][MAXD/2]
  float* kt = reinterpret_cast<float*>(rp + Lm * (ATT_MAXD / 2));  // [TP][MAXD+1]
  float* vt = kt + ATT_TP * (ATT_MAXD + 1);                    // [TP][MAXD]
  float* sc = vt + ATT_TP * ATT_MAXD;                          // [MAXR][TP]
  float* pacc = sc + ATT_MAXR * ATT_TP;                        // [MAXR][MAXD]
  float* pm = pacc + ATT_MAXR * ATT_MAXD;                      // [MAXR]
  float* pl = pm + ATT_MAXR;                                   // [MAXR]
  int* spos = reinterpret_cast<int*>(pl + ATT_MAXR);           // [Lm]

  pdl_launch_dependents();
  pdl_wait();
  int L, n, mlo;
  if (p.q_ready) {
    L = p.L;
    n = p.T_full;
    mlo = n;
  } else {
    L = p.L_dev ? *p.L_dev : p.L;
    n = (p.n_dev ? *p.n_dev : 0) + p.n_add;
    mlo = p.mask_from_prefix ? (p.n_dev ? *p.n_dev : 0) : n;
    if (L < 0 || L > p.L_max) {
      raise_error(p.err, kErrRows);
      L = L < 0 ? 0 : p.L_max;
    }
  }
  const int R = L * rep;
  const int newL = p.q_ready ? 0 : L;
  const int T = n + newL;
  if (R > ATT_MAXR) {
    raise_error(p.err, kErrRows);
    return;  // uniform across the cluster: every block takes this branch
  }

  // ---- stage raw q (rep heads) / k / v rows, norm gains and RoPE rows with 16-byte loads
  const int d4 = D / 4;
  const int nraw = R + 2 * newL;
  for (int idx = tid; idx < nraw * d4; idx += ATT_THREADS) {
    const int row = idx / d4, c = (idx % d4) * 4;
    const float* src;
    if (row < R) {
      const int l = row / rep, h = hk * rep + row % rep;
      src = p.q_ready ? p.q_ready + (size_t(l) * p.H + h) * D : p.qkv + size_t(l) * p.ld_qkv + size_t(h) * D;
    } else {
      const int j = row - R, l = j % newL;
      const int head = p.H + (j < newL ? 0 : p.Hk) + hk;
      src = p.qkv + size_t(l) * p.ld_qkv + size_t(head) * D;
    }
    *reinterpret_cast<float4*>(&raw[row * ATT_MAXD + c]) = *reinterpret_cast<const float4*>(src + c);
  }
  if (!p.q_ready) {
    for (int i = tid; i < D; i += ATT_THREADS) {
      wq[i] = p.q_norm ? p.q_norm[i] : 1.f;
      wk[i] = p.k_norm ? p.k_norm[i] : 1.f;
    }
    for (int l = tid; l < L; l += ATT_THREADS) {
      int pos = p.positions ? p.positions[l] : n + l;
      if (pos < 0 || pos >= p.max_pos) {
        raise_error(p.err, kErrPosition);
        pos = 0;
      }
      spos[l] = pos;
    }
    __syncthreads();
    const int half = D / 2;
    for (int idx = tid; idx < L * half; idx += ATT_THREADS)
      rp[(idx / half) * (ATT_MAXD / 2) + idx % half] = p.rope[size_t(spos[idx / half]) * half + idx % half];
  }
  __syncthreads();

  // ---- per-head RMSNorm + RoPE from shared memory; block 0 of the cluster appends K/V
  const int items = p.q_ready ? R : R + 2 * newL;
  for (int it = warp; it < items; it += ATT_WARPS) {
    float v[ATT_EPL];
#pragma unroll
    for (int e = 0; e < ATT_EPL; ++e) v[e] = e < epl ? raw[it * ATT_MAXD + lane * epl + e] : 0.f;
    if (p.q_ready) {
#pragma unroll
      for (int e = 0; e < ATT_EPL; ++e)
        if (e < epl) qs[it * ATT_MAXD + lane * epl + e] = v[e];
      continue;
    }
    const bool is_q = it < R;
    const int j = it - R;
    const bool is_k = !is_q && j < newL;
    const int l = is_q ? it / rep : j % newL;
    const bool do_norm = is_q ? p.q_norm != nullptr : (is_k && p.k_norm != nullptr);
    if (do_norm) {
      const float* w = is_q ? wq : wk;
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < ATT_EPL; ++e)
        if (e < epl) ss = fmaf(v[e], v[e], ss);
      ss = warp_sum(ss);
      const float inv = 1.f / sqrtf(ss / float(D) + p.eps);
#pragma unroll
      for (int e = 0; e < ATT_EPL; ++e)
        if (e < epl) v[e] = v[e] * inv * w[lane * epl + e];
    }
    if (is_q || is_k) {  // rotate-half RoPE: dims d and d + D/2 pair up across lanes lane ^ 16
      const int half = D / 2;
#pragma unroll
      for (int e = 0; e < ATT_EPL; ++e) {
        if (e < epl) {
          const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
          const int d = lane * epl + e;
          const float2 cs = rp[l * (ATT_MAXD / 2) + d % half];
          v[e] = (d < half) ? (v[e] * cs.x - partner * cs.y) : (v[e] * cs.x + partner * cs.y);
        }
      }
    }
    if (is_q) {
#pragma unroll
      for (int e = 0; e < ATT_EPL; ++e)
        if (e < epl) qs[it * ATT_MAXD + lane * epl + e] = v[e];
    } else {
      float* dst = is_k ? kn : vn;
      const int cidx = n + l;
#pragma unroll
      for (int e = 0; e < ATT_EPL; ++e) {
        if (e >= epl) continue;
        const float r = kv_round(v[e], p.kv_dtype);
        dst[l * ATT_MAXD + lane * epl + e] = r;
        if (p.write_cache && rank == 0) {
          if (cidx < p.cap) {
            kv_store(is_k ? p.Kc : p.Vc, p.kv_dtype, hk * p.stride_h + cidx * p.stride_p + lane * epl + e, r);
          } else if (lane == 0 && e == 0) {
            raise_error(p.err, kErrCapacity);
          }
        }
      }
    }
  }
  __syncthreads();

  // ---- split-KV over [0, T): this block's range, online softmax over tiles of TP positions
  const int chunk = (T + S - 1) / S;
  const int p0 = min(T, rank * chunk), p1 = min(T, p0 + chunk);
  float m[ATT_RPW], ls[ATT_RPW], acc[ATT_RPW][ATT_EPL];
#pragma unroll
  for (int i = 0; i < ATT_RPW; ++i) {
    m[i] = -INFINITY;
    ls[i] = 0.f;
#pragma unroll
    for (int e = 0; e < ATT_EPL; ++e) acc[i][e] = 0.f;
  }
  const int ev = p.kv_dtype == 1 ? 8 : 4;  // elements per 16-byte vector
  const int vpp = D / ev;                   // vectors per position
  for (int t0 = p0; t0 < p1; t0 += ATT_TP) {
    constexpr int MAXV = ATT_TP * ATT_MAXD / 4 / ATT_THREADS;  // 8 vectors per thread at most
    uint4 kv4[MAXV], vv4[MAXV];
    const int nvec = ATT_TP * vpp;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int idx = tid + j * ATT_THREADS;
      kv4[j] = make_uint4(0, 0, 0, 0);
      vv4[j] = make_uint4(0, 0, 0, 0);
      if (idx < nvec) {
        const int pp = idx / vpp, pos = t0 + pp;
        if (pos < p1 && pos < n && pos < p.cap) {
          const long long off = hk * p.stride_h + (long long)pos * p.stride_p + (idx % vpp) * ev;
          const size_t bo = size_t(off) * (p.kv_dtype == 1 ? 2 : 4);
          kv4[j] = *reinterpret_cast<const uint4*>(static_cast<const char*>(p.Kc) + bo);
          vv4[j] = *reinterpret_cast<const uint4*>(static_cast<const char*>(p.Vc) + bo);
        } else if (pos < p1 && pos < n && (idx % vpp) == 0) {
          raise_error(p.err, kErrCapacity);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int idx = tid + j * ATT_THREADS;
      if (idx >= nvec) continue;
      const int pp = idx / vpp, pos = t0 + pp, d0 = (idx % vpp) * ev;
      float* kr = kt + pp * (ATT_MAXD + 1) + d0;
      float* vr = vt + pp * ATT_MAXD + d0;
      if (pos >= n && pos < p1) {  // new rows come from shared memory
        for (int e = 0; e < ev; ++e) {
          kr[e] = kn[(pos - n) * ATT_MAXD + d0 + e];
          vr[e] = vn[(pos - n) * ATT_MAXD + d0 + e];
        }
      } else if (ev == 8) {
        const uint32_t kw[4] = {kv4[j].x, kv4[j].y, kv4[j].z, kv4[j].w};
        const uint32_t vw[4] = {vv4[j].x, vv4[j].y, vv4[j].z, vv4[j].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          kr[2 * q] = __uint_as_float(kw[q] << 16);
          kr[2 * q + 1] = __uint_as_float(kw[q] & 0xFFFF0000u);
          vr[2 * q] = __uint_as_float(vw[q] << 16);
          vr[2 * q + 1] = __uint_as_float(vw[q] & 0xFFFF0000u);
        }
      } else {
        kr[0] = __uint_as_float(kv4[j].x);
        kr[1] = __uint_as_float(kv4[j].y);
        kr[2] = __uint_as_float(kv4[j].z);
        kr[3] = __uint_as_float(kv4[j].w);
        *reinterpret_cast<float4*>(vr) = make_float4(__uint_as_float(vv4[j].x), __uint_as_float(vv4[j].y),
                                                     __uint_as_float(vv4[j].z), __uint_as_float(vv4[j].w));
      }
    }
    __syncthreads();
    // scores: lane = position, all of this warp's rows at once
    float s[ATT_RPW];
#pragma unroll
    for (int i = 0; i < ATT_RPW; ++i) s[i] = 0.f;
    const float* krow = kt + lane * (ATT_MAXD + 1);
    for (int d = 0; d < D; ++d) {
      const float kd = krow[d];
#pragma unroll
      for (int i = 0; i < ATT_RPW; ++i) {
        const int r = warp + i * ATT_WARPS;
        if (r < R) s[i] = fmaf(qs[r * ATT_MAXD + d], kd, s[i]);
      }
    }
    const int pos = t0 + lane;
#pragma unroll
    for (int i = 0; i < ATT_RPW; ++i) {
      const int r = warp + i * ATT_WARPS;
      if (r >= R) continue;
      const int l = r / rep;
      bool vis = pos < p1;
      if (vis) {
        if (p.mask_full) {
          vis = p.mask_full[size_t(l) * p.mask_ld + pos] != 0;
        } else if (pos < mlo) {
          vis = p.window <= 0 || pos >= n + l - p.window + 1;
        } else {
          const int j = pos - mlo;
          vis = p.newmask ? ((p.newmask[l] >> j) & 1ull) != 0 : j <= l;
          if (vis && p.window > 0) vis = pos >= n + l - p.window + 1;
        }
      }
      const float sv = vis ? p.scale * s[i] : -INFINITY;
      const float mt = warp_max(sv);
      const float mn = fmaxf(m[i], mt);
      float e = 0.f, alpha = 1.f;
      if (mn != -INFINITY) {
        e = vis ? expf(sv - mn) : 0.f;
        alpha = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mn);
      }
      ls[i] = ls[i] * alpha + warp_sum(e);
      m[i] = mn;
      sc[r * ATT_TP + lane] = e;
#pragma unroll
      for (int ee = 0; ee < ATT_EPL; ++ee) acc[i][ee] *= alpha;
    }
    __syncwarp();
    // P . V: lane owns dims lane*epl .. +epl, all of this warp's rows at once
    for (int pp = 0; pp < ATT_TP; ++pp) {
      float vvv[ATT_EPL];
      if (epl == 4) {
        const float4 v4 = *reinterpret_cast<const float4*>(&vt[pp * ATT_MAXD + lane * 4]);
        vvv[0] = v4.x;
        vvv[1] = v4.y;
        vvv[2] = v4.z;
        vvv[3] = v4.w;
      } else {
#pragma unroll
        for (int ee = 0; ee < ATT_EPL; ++ee) vvv[ee] = ee < epl ? vt[pp * ATT_MAXD + lane * epl + ee] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < ATT_RPW; ++i) {
        const int r = warp + i * ATT_WARPS;
        if (r < R) {
          const float w = sc[r * ATT_TP + pp];
#pragma unroll
          for (int ee = 0; ee < ATT_EPL; ++ee) acc[i][ee] = fmaf(w, vvv[ee], acc[i][ee]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < ATT_RPW; ++i) {
    const int r = warp + i * ATT_WARPS;
    if (r < R) {
#pragma unroll
      for (int e = 0; e < ATT_EPL; ++e)
        if (e < epl) pacc[r * ATT_MAXD + lane * epl + e] = acc[i][e];
      if (lane == 0) {
        pm[r] = m[i];
        pl[r] = ls[i];
      }
    }
  }
  cluster.sync();
  // ---- combine the S partial states of each row through distributed shared memory
  for (int r = rank; r < R; r += S) {
    float M = -INFINITY;
    for (int s2 = 0; s2 < S; ++s2) M = fmaxf(M, cluster.map_shared_rank(pm, s2)[r]);
    float lt = 0.f, o = 0.f;
    for (int s2 = 0; s2 < S; ++s2) {
      const float ms = cluster.map_shared_rank(pm, s2)[r];
      const float w = (ms == -INFINITY) ? 0.f : expf(ms - M);
      lt += w * cluster.map_shared_rank(pl, s2)[r];
      if (tid < D) o += w * cluster.map_shared_rank(pacc, s2)[r * ATT_MAXD + tid];
    }
    if (tid < D) {
      const int l = r / rep, h = hk * rep + r % rep;
      attn_emit(p, l, h * D + tid, o / lt);
    }
  }
  cluster.sync();
}

inline size_t attention_smem(int L_max) {
  return sizeof(float) * (size_t(ATT_MAXR) * ATT_MAXD + 2 * size_t(L_max) * ATT_MAXD +
                          (size_t(ATT_MAXR) + 2 * L_max) * ATT_MAXD + 2 * ATT_MAXD + size_t(L_max) * ATT_MAXD +
                          ATT_TP * (ATT_MAXD + 1) + ATT_TP * ATT_MAXD + ATT_MAXR * ATT_TP + ATT_MAXR * ATT_MAXD +
                          2 * ATT_MAXR) +
         sizeof(int) * size_t(L_max) + 16;
}

}  // namespace wc
