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
  int write_cache;
  int* err;
};

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

// RMSNorm over one head (lane holds EPL dims d = lane*EPL + e) then rotate-half RoPE.
__device__ __forceinline__ void norm_rope_head(float (&v)[ATT_EPL], int epl, int D, const float* w, float eps,
                                               const float2* rope_row, bool do_norm, bool do_rope) {
  const int lane = threadIdx.x % kWarp;
  if (do_norm) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < ATT_EPL; ++e)
      if (e < epl) ss = fmaf(v[e], v[e], ss);
    ss = warp_sum(ss);
    const float inv = 1.f / sqrtf(ss / float(D) + eps);
#pragma unroll
    for (int e = 0; e < ATT_EPL; ++e)
      if (e < epl) v[e] = v[e] * inv * w[lane * epl + e];
  }
  if (do_rope) {
    const int half = D / 2;
#pragma unroll
    for (int e = 0; e < ATT_EPL; ++e) {
      if (e < epl) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
        const int d = lane * epl + e;
        const float2 cs = rope_row[d % half];
        v[e] = (d < half) ? (v[e] * cs.x - partner * cs.y) : (v[e] * cs.x + partner * cs.y);
      }
    }
  }
}

__global__ void __launch_bounds__(ATT_THREADS) attention_kernel(const AttnParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int S = int(cluster.num_blocks());
  const int rank = int(cluster.block_rank());
  const int hk = blockIdx.y;
  const int D = p.D, epl = D / kWarp, rep = p.H / p.Hk;
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp;

  int L, n;
  if (p.q_ready) {
    L = p.L;
    n = p.T_full;
  } else {
    L = p.L_dev ? *p.L_dev : p.L;
    n = (p.n_dev ? *p.n_dev : 0) + p.n_add;
    if (L < 0 || L > p.L_max) {
      raise_error(p.err, kErrRows);
      L = L < 0 ? 0 : p.L_max;
    }
  }
  const int R = L * rep;
  const int Lm = p.L_max;
  const int newL = p.q_ready ? 0 : L;
  const int T = n + newL;

  float* qs = reinterpret_cast<float*>(smem);              // [MAXR][D]
  float* kn = qs + ATT_MAXR * ATT_MAXD;                     // [Lm][D]
  float* vn = kn + Lm * ATT_MAXD;                           // [Lm][D]
  float* kt = vn + Lm * ATT_MAXD;                           // [TP][D+1]
  float* vt = kt + ATT_TP * (ATT_MAXD + 1);                 // [TP][D]
  float* sc = vt + ATT_TP * ATT_MAXD;                       // [MAXR][TP]
  float* pacc = sc + ATT_MAXR * ATT_TP;                     // [MAXR][D]
  float* pm = pacc + ATT_MAXR * ATT_MAXD;                   // [MAXR]
  float* pl = pm + ATT_MAXR;                                // [MAXR]
  int* spos = reinterpret_cast<int*>(pl + ATT_MAXR);        // [Lm]

  if (R > ATT_MAXR) {
    raise_error(p.err, kErrRows);
    return;  // uniform across the cluster: every block takes this branch
  }
  for (int l = tid; l < L; l += ATT_THREADS) {
    int pos = p.q_ready ? 0 : (p.positions ? p.positions[l] : n + l);
    if (pos < 0 || pos >= p.max_pos) {
      if (!p.q_ready) raise_error(p.err, kErrPosition);
      pos = 0;
    }
    spos[l] = pos;
  }
  __syncthreads();

  // ---- new rows of this head: q (rep heads), k, v
  const int items = p.q_ready ? R : R + 2 * newL;
  for (int it = warp; it < items; it += ATT_WARPS) {
    float v[ATT_EPL];
    if (it < R) {
      const int l = it / rep, rr = it % rep, h = hk * rep + rr;
      if (p.q_ready) {
#pragma unroll
        for (int e = 0; e < ATT_EPL; ++e) v[e] = e < epl ? p.q_ready[(size_t(l) * p.H + h) * D + lane * epl + e] : 0.f;
      } else {
        const float* src = p.qkv + size_t(l) * p.ld_qkv + size_t(h) * D;
#pragma unroll
        for (int e = 0; e < ATT_EPL; ++e) v[e] = e < epl ? src[lane * epl + e] : 0.f;
        norm_rope_head(v, epl, D, p.q_norm, p.eps, p.rope + size_t(spos[l]) * (D / 2), p.q_norm != nullptr, true);
      }
#pragma unroll
      for (int e = 0; e < ATT_EPL; ++e)
        if (e < epl) qs[it * ATT_MAXD + lane * epl + e] = v[e];
    } else {
      const int j = it - R, l = j % newL;
      const bool is_k = j < newL;
      const float* src = p.qkv + size_t(l) * p.ld_qkv + size_t(p.H + (is_k ? 0 : p.Hk) + hk) * D;
#pragma unroll
      for (int e = 0; e < ATT_EPL; ++e) v[e] = e < epl ? src[lane * epl + e] : 0.f;
      norm_rope_head(v, epl, D, p.k_norm, p.eps, p.rope + size_t(spos[l]) * (D / 2), is_k && p.k_norm != nullptr,
                     is_k);
      float* dst = is_k ? kn : vn;
#pragma unroll
      for (int e = 0; e < ATT_EPL; ++e) {
        if (e >= epl) continue;
        const float r = kv_round(v[e], p.kv_dtype);
        dst[l * ATT_MAXD + lane * epl + e] = r;
        if (p.write_cache && rank == 0) {
          const int cidx = n + l;
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

  // ---- split-KV over [0, T): this block's range
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
  for (int t0 = p0; t0 < p1; t0 += ATT_TP) {
    for (int idx = tid; idx < ATT_TP * D; idx += ATT_THREADS) {
      const int pp = idx / D, d = idx % D, pos = t0 + pp;
      float kv = 0.f, vv = 0.f;
      if (pos < p1) {
        if (pos < n) {
          const long long off = hk * p.stride_h + (long long)pos * p.stride_p + d;
          kv = kv_load(p.Kc, p.kv_dtype, off);
          vv = kv_load(p.Vc, p.kv_dtype, off);
        } else {
          kv = kn[(pos - n) * ATT_MAXD + d];
          vv = vn[(pos - n) * ATT_MAXD + d];
        }
      }
      kt[pp * (ATT_MAXD + 1) + d] = kv;
      vt[pp * ATT_MAXD + d] = vv;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < ATT_RPW; ++i) {
      const int r = warp + i * ATT_WARPS;
      if (r < R) {
        const int l = r / rep;
        const int pos = t0 + lane;
        bool vis = pos < p1;
        if (vis) {
          if (p.mask_full) {
            vis = p.mask_full[size_t(l) * p.mask_ld + pos] != 0;
          } else if (pos < n) {
            vis = p.window <= 0 || pos >= n + l - p.window + 1;
          } else {
            const int j = pos - n;
            vis = p.newmask ? ((p.newmask[l] >> j) & 1ull) != 0 : j <= l;
            if (vis && p.window > 0) vis = pos >= n + l - p.window + 1;
          }
        }
        float s = 0.f;
        const float* qr = qs + r * ATT_MAXD;
        const float* kr = kt + lane * (ATT_MAXD + 1);
        for (int d = 0; d < D; ++d) s = fmaf(qr[d], kr[d], s);
        s = vis ? p.scale * s : -INFINITY;
        const float mt = warp_max(s);
        const float mn = fmaxf(m[i], mt);
        float e = 0.f, alpha = 1.f;
        if (mn != -INFINITY) {
          e = vis ? expf(s - mn) : 0.f;
          alpha = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mn);
        }
        ls[i] = ls[i] * alpha + warp_sum(e);
        m[i] = mn;
        sc[r * ATT_TP + lane] = e;
        __syncwarp();
#pragma unroll
        for (int ee = 0; ee < ATT_EPL; ++ee) acc[i][ee] *= alpha;
        if (epl == 4) {
          for (int pp = 0; pp < ATT_TP; ++pp) {
            const float w = sc[r * ATT_TP + pp];
            const float4 v4 = *reinterpret_cast<const float4*>(&vt[pp * ATT_MAXD + lane * 4]);
            acc[i][0] = fmaf(w, v4.x, acc[i][0]);
            acc[i][1] = fmaf(w, v4.y, acc[i][1]);
            acc[i][2] = fmaf(w, v4.z, acc[i][2]);
            acc[i][3] = fmaf(w, v4.w, acc[i][3]);
          }
        } else {
          for (int pp = 0; pp < ATT_TP; ++pp) {
            const float w = sc[r * ATT_TP + pp];
#pragma unroll
            for (int ee = 0; ee < ATT_EPL; ++ee)
              if (ee < epl) acc[i][ee] = fmaf(w, vt[pp * ATT_MAXD + lane * epl + ee], acc[i][ee]);
          }
        }
        __syncwarp();
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
    for (int s = 0; s < S; ++s) M = fmaxf(M, cluster.map_shared_rank(pm, s)[r]);
    float lt = 0.f, o = 0.f;
    for (int s = 0; s < S; ++s) {
      const float ms = cluster.map_shared_rank(pm, s)[r];
      const float w = (ms == -INFINITY) ? 0.f : expf(ms - M);
      lt += w * cluster.map_shared_rank(pl, s)[r];
      if (tid < D) o += w * cluster.map_shared_rank(pacc, s)[r * ATT_MAXD + tid];
    }
    if (tid < D) {
      const int l = r / rep, h = hk * rep + r % rep;
      p.out[size_t(l) * p.ld_out + size_t(h) * D + tid] = o / lt;
    }
  }
  cluster.sync();
}

inline size_t attention_smem(int L_max) {
  return sizeof(float) * (size_t(ATT_MAXR) * ATT_MAXD + 2 * size_t(L_max) * ATT_MAXD + ATT_TP * (ATT_MAXD + 1) +
                          ATT_TP * ATT_MAXD + ATT_MAXR * ATT_TP + ATT_MAXR * ATT_MAXD + 2 * ATT_MAXR) +
         sizeof(int) * size_t(L_max) + 16;
}

}  // namespace wc
