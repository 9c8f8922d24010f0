// Batched tree verification: B independent requests, each verifying a draft token tree of
// `nodes` nodes against its own KV arena. Rows are request-major (row m = r * nodes + i),
// so at B * nodes ~ 2048 rows the projections are compute-bound GEMMs and run on the 5th-gen
// tensor cores: TMA tiles (128B swizzle) into a shared-memory ring, one thread issues
// tcgen05.mma into a TMEM accumulator, four warps read it back with tcgen05.ld for the
// epilogue. Attention is HBM-bound (each request's 4096-row prefix is read once per layer)
// and runs on mma.sync, one block per (request, KV head) with all of its query rows.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace wc {

// ---------------------------------------------------------------------------- tcgen05 GEMM
// C[M][N] = A[M][K] . B[N][K]^T, A and B bf16 row-major (K contiguous), fp32 accumulate.
constexpr int TC_BM = 128;
constexpr int TC_BK = 64;  // one 128-byte swizzle row of bf16
constexpr int TC_STAGES = 4;
constexpr int TC_THREADS = 192;  // warp 0 TMA, warp 1 MMA + TMEM owner, warps 2-5 epilogue

enum TcEpilogue : int {
  TC_STORE = 0,   // c = acc (fp32)
  TC_ADD = 1,     // c = acc + r (fp32; r may alias c)
  TC_SWIGLU = 2,  // tile columns [0, BN/2) gate, [BN/2, BN) up: cb[m][n0/2 + j] = bf16(silu(g_j) * u_j)
  TC_ARGMAX = 3,  // keys[m] = max over columns of (acc, column)
  TC_BF16 = 4,    // cb = bf16(acc)
};

struct GemmTc {
  int M, N, K;
  int epi;
  float* c;
  int ldc;
  const float* r;
  int ldr;
  uint16_t* cb;
  int ldcb;
  unsigned long long* keys;
  int* err;
};

template <int BN>
constexpr size_t gemm_tc_smem() {
  return 1024 + size_t(TC_STAGES) * (TC_BM + BN) * TC_BK * 2 + 256;
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the 128-byte
// swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), leading
// byte offset unused (1), descriptor version 1, layout type 2 (SWIZZLE_128B). The start
// address of the k-th 16-element slice of a row is the tile base + 32 k bytes.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both K-major, M x BN.
template <int BN>
__host__ __device__ constexpr uint32_t umma_idesc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) | (uint32_t(TC_BM >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrives on `bar` once every tcgen05.mma this thread issued before has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_addr(bar))
               : "memory");
}
// 16 consecutive fp32 columns of this thread's TMEM lane (32x32b shape, x16)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                   const __grid_constant__ GemmTc p) {
  static_assert(BN == 128 || BN == 256, "tile width (TMEM columns are allocated in powers of two)");
  constexpr int SA = TC_BM * TC_BK * 2, SB = BN * TC_BK * 2, SS = SA + SB;
  extern __shared__ unsigned char tc_raw[];
  unsigned char* sm = tc_raw + ((1024u - (smem_addr(tc_raw) & 1023u)) & 1023u);  // 1024-aligned for the swizzle
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + TC_STAGES * SS);
  uint64_t* empty = full + TC_STAGES;
  uint64_t* accb = empty + TC_STAGES;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accb + 1);
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int m0 = blockIdx.x * TC_BM, n0 = blockIdx.y * BN;
  const int KB = (p.K + TC_BK - 1) / TC_BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(accb, 1);
    mbar_fence_init();
  }
  if (warp == 1) {  // TMEM: BN fp32 columns x 128 lanes hold the tile's accumulator
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(tslot)),
                 "r"(uint32_t(BN))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_launch_dependents();
  pdl_wait();  // A (and a residual the epilogue reads) come from the previous kernel

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer
      int kb = 0;
      for (; kb < KB; ++kb) {
        const int s = kb % TC_STAGES;
        if (kb >= TC_STAGES && !mbar_wait(empty + s, ((kb / TC_STAGES) - 1) & 1)) {
          raise_error(p.err, kErrTimeout);
          break;
        }
        mbar_arrive_expect_tx(full + s, SS);
        tma_load_2d(sm + s * SS, &ta, kb * TC_BK, m0, full + s);
        tma_load_2d(sm + s * SS + SA, &tb, kb * TC_BK, n0, full + s);
      }
      // shared memory must outlive the copies: wait (bounded) for the last issued stages
      for (int q = max(0, kb - TC_STAGES); q < kb; ++q)
        if (!mbar_wait(full + q % TC_STAGES, (q / TC_STAGES) & 1)) raise_error(p.err, kErrTimeout);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      constexpr uint32_t idesc = umma_idesc_bf16<BN>();
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % TC_STAGES;
        if (!mbar_wait(full + s, (kb / TC_STAGES) & 1)) {
          raise_error(p.err, kErrTimeout);
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_addr(sm + s * SS), b0 = smem_addr(sm + s * SS + SA);
#pragma unroll
        for (int k = 0; k < TC_BK / 16; ++k)
          umma_bf16(tmem, umma_desc_sw128(a0 + 32 * k), umma_desc_sw128(b0 + 32 * k), idesc, (kb | k) != 0);
        umma_commit(empty + s);  // the stage is free once these MMAs have read it
      }
      umma_commit(accb);  // the accumulator is complete once every MMA above has finished
    }
  } else {  // ---- epilogue: warp w reads TMEM lanes [32 (w % 4), 32 (w % 4) + 32)
    const int q = warp & 3;
    const int row = m0 + q * 32 + lane;
    if (!mbar_wait(accb, 0)) raise_error(p.err, kErrTimeout);
    tc_fence_after();
    const uint32_t tl = tmem + (uint32_t(q * 32) << 16);
    const bool rv = row < p.M;
    if (p.epi == TC_SWIGLU) {
      constexpr int H2 = BN / 2;
#pragma unroll 1
      for (int c0 = 0; c0 < H2; c0 += 16) {
        float g[16], u[16];
        tmem_ld16(tl + c0, g);
        tmem_ld16(tl + H2 + c0, u);
        const int f0 = n0 / 2 + c0;
        if (rv && f0 < p.N / 2) {
          uint32_t o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float a = g[2 * i] / (1.f + expf(-g[2 * i])) * u[2 * i];
            const float b = g[2 * i + 1] / (1.f + expf(-g[2 * i + 1])) * u[2 * i + 1];
            o[i] = pack2(f32_to_bf16_bits(a), f32_to_bf16_bits(b));
          }
          uint4* dst = reinterpret_cast<uint4*>(p.cb + size_t(row) * p.ldcb + f0);
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        }
      }
    } else if (p.epi == TC_ARGMAX) {
      unsigned long long best = 0ull;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        tmem_ld16(tl + c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int col = n0 + c0 + i;
          if (col < p.N) {
            const unsigned long long k = argmax_key(v[i], uint32_t(col));
            if (k > best) best = k;
          }
        }
      }
      if (rv && best) atomicMax(&p.keys[row], best);
    } else {
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        tmem_ld16(tl + c0, v);
        if (!rv) continue;
        const int col0 = n0 + c0;
        if (p.epi == TC_BF16) {
          if (col0 + 16 <= p.N) {
            uint32_t o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = pack2(f32_to_bf16_bits(v[2 * i]), f32_to_bf16_bits(v[2 * i + 1]));
            uint4* dst = reinterpret_cast<uint4*>(p.cb + size_t(row) * p.ldcb + col0);
            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
          } else {
            for (int i = 0; i < 16 && col0 + i < p.N; ++i) p.cb[size_t(row) * p.ldcb + col0 + i] = f32_to_bf16_bits(v[i]);
          }
          continue;
        }
        float* dst = p.c + size_t(row) * p.ldc + col0;
        const float* rs = p.epi == TC_ADD ? p.r + size_t(row) * p.ldr + col0 : nullptr;
        if (col0 + 16 <= p.N) {
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            float4 o = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            if (rs) {
              const float4 a = *reinterpret_cast<const float4*>(rs + i);
              o.x += a.x;
              o.y += a.y;
              o.z += a.z;
              o.w += a.w;
            }
            *reinterpret_cast<float4*>(dst + i) = o;
          }
        } else {
          for (int i = 0; i < 16 && col0 + i < p.N; ++i) dst[i] = v[i] + (rs ? rs[i] : 0.f);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(uint32_t(BN))
                 : "memory");
  }
}

// ---------------------------------------------------------------------------- persistent GEMM
// One block per SM loops over the tiles (m fastest, so the blocks that run together share
// weight tiles in L2). Two TMEM accumulators (2 x BN columns): while the four epilogue warps
// drain tile i from one, the MMA thread fills the other with tile i + 1, and the TMA producer
// runs ahead through the shared-memory ring across tile boundaries.
template <int BN>
__device__ __forceinline__ void tc_epilogue_tile(const GemmTc& p, uint32_t tl, int row, int n0) {
  const bool rv = row < p.M;
  if (p.epi == TC_SWIGLU) {
    constexpr int H2 = BN / 2;
#pragma unroll 1
    for (int c0 = 0; c0 < H2; c0 += 16) {
      float g[16], u[16];
      tmem_ld16(tl + c0, g);
      tmem_ld16(tl + H2 + c0, u);
      const int f0 = n0 / 2 + c0;
      if (rv && f0 < p.N / 2) {
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float a = g[2 * i] / (1.f + expf(-g[2 * i])) * u[2 * i];
          const float b = g[2 * i + 1] / (1.f + expf(-g[2 * i + 1])) * u[2 * i + 1];
          o[i] = pack2(f32_to_bf16_bits(a), f32_to_bf16_bits(b));
        }
        uint4* dst = reinterpret_cast<uint4*>(p.cb + size_t(row) * p.ldcb + f0);
        dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
      }
    }
  } else if (p.epi == TC_ARGMAX) {
    unsigned long long best = 0ull;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(tl + c0, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int col = n0 + c0 + i;
        if (col < p.N) {
          const unsigned long long k = argmax_key(v[i], uint32_t(col));
          if (k > best) best = k;
        }
      }
    }
    if (rv && best) atomicMax(&p.keys[row], best);
  } else {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(tl + c0, v);
      if (!rv) continue;
      const int col0 = n0 + c0;
      if (p.epi == TC_BF16) {
        if (col0 + 16 <= p.N) {
          uint32_t o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = pack2(f32_to_bf16_bits(v[2 * i]), f32_to_bf16_bits(v[2 * i + 1]));
          uint4* dst = reinterpret_cast<uint4*>(p.cb + size_t(row) * p.ldcb + col0);
          dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
          dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        } else {
          for (int i = 0; i < 16; ++i)
            if (col0 + i < p.N) p.cb[size_t(row) * p.ldcb + col0 + i] = f32_to_bf16_bits(v[i]);
        }
        continue;
      }
      float* dst = p.c + size_t(row) * p.ldc + col0;
      const float* rs = p.epi == TC_ADD ? p.r + size_t(row) * p.ldr + col0 : nullptr;
      if (col0 + 16 <= p.N) {
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          float4 o = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
          if (rs) {
            const float4 a = *reinterpret_cast<const float4*>(rs + i);
            o.x += a.x;
            o.y += a.y;
            o.z += a.z;
            o.w += a.w;
          }
          *reinterpret_cast<float4*>(dst + i) = o;
        }
      } else {
        for (int i = 0; i < 16; ++i)
          if (col0 + i < p.N) dst[i] = v[i] + (rs ? rs[i] : 0.f);
      }
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    gemm_tcp_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                    const __grid_constant__ GemmTc p) {
  static_assert(BN == 128 || BN == 256, "tile width");
  constexpr int SA = TC_BM * TC_BK * 2, SB = BN * TC_BK * 2, SS = SA + SB;
  extern __shared__ unsigned char tcp_raw[];
  unsigned char* sm = tcp_raw + ((1024u - (smem_addr(tcp_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + TC_STAGES * SS);
  uint64_t* empty = full + TC_STAGES;
  uint64_t* acc_full = empty + TC_STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int KB = (p.K + TC_BK - 1) / TC_BK;
  const int mt = (p.M + TC_BM - 1) / TC_BM, ntiles = mt * ((p.N + BN - 1) / BN);
  const int my_tiles = int(blockIdx.x) < ntiles ? (ntiles - 1 - int(blockIdx.x)) / int(gridDim.x) + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 4);  // one arrival per epilogue warp
    }
    mbar_fence_init();
  }
  if (warp == 1) {  // two accumulators of BN fp32 columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(tslot)),
                 "r"(uint32_t(2 * BN))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer, across tiles
      int q = 0;
      bool ok = true;
      for (int i = 0; i < my_tiles && ok; ++i) {
        const int t = int(blockIdx.x) + i * int(gridDim.x);
        const int m0 = (t % mt) * TC_BM, n0 = (t / mt) * BN;
        for (int kb = 0; kb < KB; ++kb, ++q) {
          const int s = q % TC_STAGES;
          if (q >= TC_STAGES && !mbar_wait(empty + s, ((q / TC_STAGES) - 1) & 1)) {
            raise_error(p.err, kErrTimeout);
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full + s, SS);
          tma_load_2d(sm + s * SS, &ta, kb * TC_BK, m0, full + s);
          tma_load_2d(sm + s * SS + SA, &tb, kb * TC_BK, n0, full + s);
        }
      }
      for (int qq = max(0, q - TC_STAGES); qq < q; ++qq)
        if (!mbar_wait(full + qq % TC_STAGES, (qq / TC_STAGES) & 1)) raise_error(p.err, kErrTimeout);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      constexpr uint32_t idesc = umma_idesc_bf16<BN>();
      int q = 0;
      bool ok = true;
      for (int i = 0; i < my_tiles; ++i) {
        const int b = i & 1;
        if (ok && i >= 2 && !mbar_wait(acc_empty + b, ((i / 2) - 1) & 1)) {
          raise_error(p.err, kErrTimeout);
          ok = false;
        }
        tc_fence_after();
        const uint32_t acc = tmem + uint32_t(b * BN);
        for (int kb = 0; kb < KB && ok; ++kb, ++q) {
          const int s = q % TC_STAGES;
          if (!mbar_wait(full + s, (q / TC_STAGES) & 1)) {
            raise_error(p.err, kErrTimeout);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_addr(sm + s * SS), b0 = smem_addr(sm + s * SS + SA);
#pragma unroll
          for (int k = 0; k < TC_BK / 16; ++k)
            umma_bf16(acc, umma_desc_sw128(a0 + 32 * k), umma_desc_sw128(b0 + 32 * k), idesc, (kb | k) != 0);
          umma_commit(empty + s);
        }
        umma_commit(acc_full + b);  // arrives once this tile's MMAs (all issued above) are done
      }
    }
  } else {  // ---- epilogue warps: TMEM lanes [32 (w % 4), +32)
    const int qd = warp & 3;
    for (int i = 0; i < my_tiles; ++i) {
      const int b = i & 1;
      const int t = int(blockIdx.x) + i * int(gridDim.x);
      const int m0 = (t % mt) * TC_BM, n0 = (t / mt) * BN;
      const int row = m0 + qd * 32 + lane;
      const uint32_t tl = tmem + uint32_t(b * BN) + (uint32_t(qd * 32) << 16);
      // residual epilogue on 128-wide tiles: this row's residual is loaded while the MMAs run
      // (one round trip instead of one per 16 columns); the branch is warp-uniform because the
      // TMEM loads below are warp-collective
      const bool pre = BN == 128 && p.epi == TC_ADD && n0 + BN <= p.N;
      float4 rres[BN == 128 ? BN / 4 : 1];
      if (pre && row < p.M) {
        const float4* rs = reinterpret_cast<const float4*>(p.r + size_t(row) * p.ldr + n0);
#pragma unroll
        for (int q = 0; q < (BN == 128 ? BN / 4 : 1); ++q) rres[q] = rs[q];
      }
      if (!mbar_wait(acc_full + b, (i / 2) & 1)) raise_error(p.err, kErrTimeout);
      tc_fence_after();
      if (pre) {
#pragma unroll
        for (int c0 = 0; c0 < (BN == 128 ? BN : 0); c0 += 16) {
          float v[16];
          tmem_ld16(tl + c0, v);
          if (row < p.M) {
            float* dst = p.c + size_t(row) * p.ldc + n0 + c0;
#pragma unroll
            for (int k = 0; k < 16; k += 4) {
              const float4 a = rres[(c0 + k) / 4];
              *reinterpret_cast<float4*>(dst + k) = make_float4(v[k] + a.x, v[k + 1] + a.y, v[k + 2] + a.z, v[k + 3] + a.w);
            }
          }
        }
      } else {
        tc_epilogue_tile<BN>(p, tl, row, n0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty + b);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(uint32_t(2 * BN))
                 : "memory");
  }
}

// ---------------------------------------------------------------------------- row kernels
// RMSNorm of fp32 rows into bf16 GEMM operands: out[m] = bf16(x[m] / rms(x[m]) * w); rows
// of the embedding table when `tokens` is set (x = the gathered row, also copied into h).
struct RowNormParams {
  const float* x;
  const int* tokens;
  const void* table;  // [vocab][H] bf16
  int vocab;
  float* h_copy;      // with tokens: the gathered fp32 row
  int H;
  const float* w;
  float eps;
  uint16_t* out;
  int ld_out;         // row stride of out (0 = H); lets several normalised blocks share one row
  int M;
  int* err;
};

__global__ void __launch_bounds__(256) row_norm_bf16_kernel(__grid_constant__ const RowNormParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  if (m >= p.M) return;
  __shared__ float red[32];
  __shared__ float s_inv;
  const float* x = p.x ? p.x + size_t(m) * p.H : nullptr;
  const uint16_t* trow = nullptr;
  if (p.tokens) {
    int tok = p.tokens[m];
    if (tok < 0 || tok >= p.vocab) {
      if (threadIdx.x == 0) raise_error(p.err, kErrTokenRange);
      tok = 0;
    }
    trow = static_cast<const uint16_t*>(p.table) + size_t(tok) * p.H;
  }
  float ss = 0.f;
  for (int k = threadIdx.x; k < p.H; k += blockDim.x) {
    const float v = trow ? bf16_bits_to_f32(trow[k]) : x[k];
    if (trow && p.h_copy) p.h_copy[size_t(m) * p.H + k] = v;
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f;
    for (int w = 0; w < int(blockDim.x / 32); ++w) a += red[w];
    s_inv = 1.f / sqrtf(a / float(p.H) + p.eps);
  }
  __syncthreads();
  const float inv = s_inv;
  for (int k = threadIdx.x; k < p.H; k += blockDim.x) {
    const float v = trow ? bf16_bits_to_f32(trow[k]) : x[k];
    p.out[size_t(m) * (p.ld_out ? p.ld_out : p.H) + k] = f32_to_bf16_bits(v * inv * (p.w ? p.w[k] : 1.f));
  }
}

// Per verify row (request r, node i): q / k RMSNorm per head (q_norm, k_norm), rotate-half
// RoPE at position lens[r] + depth_i, q -> bf16 [M][Hq * D] (the attention's queries), k and
// v -> bf16 rows at slot lens[r] + i of the request's cache (the tree is appended as nodes,
// compaction later keeps the accepted path).
struct QkvPostParams {
  const float* qkv;  // [M][(Hq + 2 Hk) D]
  int nodes, Hq, Hk, D;
  const int* lens;   // [B] committed rows per request
  const int* depth;  // [M]
  const float* q_norm;
  const float* k_norm;
  float eps;
  const float2* rope;
  int max_pos;
  uint16_t* q;       // [M][Hq D]
  uint16_t* K;       // this layer's arena [B][Hk][cap][D]
  uint16_t* V;
  int cap;
  int* err;
};

__global__ void __launch_bounds__(128) qkv_post_kernel(__grid_constant__ const QkvPostParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x, r = m / p.nodes, i = m % p.nodes;
  const int D = p.D, half = D / 2, nh = p.Hq + 2 * p.Hk;
  const int pos = p.lens[r] + p.depth[m], slot = p.lens[r] + i;
  if (pos < 0 || pos >= p.max_pos || slot >= p.cap) {
    if (threadIdx.x == 0) raise_error(p.err, pos >= p.max_pos ? kErrPosition : kErrCapacity);
    return;
  }
  const float2* rope = p.rope + size_t(pos) * half;
  const float* row = p.qkv + size_t(m) * nh * D;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp, nw = blockDim.x / kWarp;
  for (int h = warp; h < nh; h += nw) {  // one warp per head
    const float* x = row + size_t(h) * D;
    const bool isq = h < p.Hq, isk = !isq && h < p.Hq + p.Hk;
    float ss = 0.f;
    for (int d = lane; d < D; d += kWarp) ss = fmaf(x[d], x[d], ss);
    ss = warp_sum(ss);
    const float inv = (isq || isk) ? 1.f / sqrtf(ss / float(D) + p.eps) : 1.f;
    const float* w = isq ? p.q_norm : (isk ? p.k_norm : nullptr);
    uint16_t* dst;
    if (isq) dst = p.q + (size_t(m) * p.Hq + h) * D;
    else {
      const int hk = isk ? h - p.Hq : h - p.Hq - p.Hk;
      dst = (isk ? p.K : p.V) + ((size_t(r) * p.Hk + hk) * p.cap + slot) * D;
    }
    for (int d = lane; d < half; d += kWarp) {
      float a = x[d], b = x[d + half];
      if (isq || isk) {
        a *= inv * (w ? w[d] : 1.f);
        b *= inv * (w ? w[d + half] : 1.f);
        const float2 cs = rope[d];
        const float a2 = a * cs.x - b * cs.y, b2 = b * cs.x + a * cs.y;
        a = a2;
        b = b2;
      }
      dst[d] = f32_to_bf16_bits(a);
      dst[d + half] = f32_to_bf16_bits(b);
    }
  }
}

// ---------------------------------------------------------------------------- tree attention
// One block per (request, KV head): all nodes x rep query rows (row = node * rep + j) against
// the request's prefix [0, lens[r]) (visible to every node) and its tree slots lens[r] + t
// (visible when t is an ancestor of the node or the node itself; sampling.py:118-128). Keys
// stream in 64-row tiles (cp.async, double-buffered); S = Q K^T and O += P V on m16n8k16 with
// bf16 Q and P, fp32 scores and online softmax; each warp owns 16 query rows.
constexpr int TA_THREADS = 128;
constexpr int TA_WARPS = TA_THREADS / kWarp;
constexpr int TA_MAXR = 16 * TA_WARPS;  // 64 query rows
constexpr int TA_KT = 64;               // keys per tile
constexpr int TA_MAXN = 64;             // tree nodes
constexpr int TA_NBUF = 3;              // K/V tile ring: two tiles in flight ahead of the one in use

struct TreeAttnParams {
  const uint16_t* q;  // [M][Hq D]
  const uint16_t* K;  // layer arena [B][Hk][cap][D]
  const uint16_t* V;
  int cap;
  const int* lens;     // [B]
  const int* parents;  // [B][nodes]
  int nodes, Hq, Hk;
  float scale;
  uint16_t* out;  // [M][Hq D]
  int nsplit;     // key-range slices per (request, KV head); > 1: partial states, then tree_attn_merge
  int causal;     // chain (prompt) mode: node i sees new rows 0..i; blockIdx.z = tile of TA_MAXR / rep nodes
  float* part_o;  // [B][Hk][nsplit][MAXR][D] unnormalised outputs
  float* part_ml; // [B][Hk][nsplit][MAXR][2] (running max in log2 units, sum)
  int* err;
};

// Queries are staged once in the last tile buffer (moved into registers before that
// buffer's first fill): a block holds 105 KB of shared memory, two per SM.
template <int D>
constexpr size_t tree_attn_smem() {
  return size_t(TA_NBUF) * 2 * size_t(TA_KT) * (D + 8) * 2 + TA_MAXN * 8 + 64;
}

template <int D>
__global__ void __launch_bounds__(TA_THREADS, 2) tree_attention_kernel(__grid_constant__ const TreeAttnParams p) {
  constexpr int LD = D + 8, NK = D / 16, ND = D / 8;
  static_assert(TA_MAXR <= TA_KT, "queries are staged in a tile buffer");
  extern __shared__ __align__(16) unsigned char ta_smem[];
  uint16_t* kv = reinterpret_cast<uint16_t*>(ta_smem);    // [NBUF buffers][K, V][KT][LD]
  uint16_t* qs = kv + size_t(TA_NBUF - 1) * 2 * TA_KT * LD;  // [MAXR][LD] = the last buffer's K tile
  unsigned long long* anc = reinterpret_cast<unsigned long long*>(kv + size_t(TA_NBUF) * 2 * TA_KT * LD);
  const int r = blockIdx.x, hk = blockIdx.y;
  const int sp_i = p.causal ? 0 : blockIdx.z;
  const int tid = threadIdx.x, warp = tid / kWarp, lane = tid % kWarp, g = lane >> 2, t = lane & 3;
  const int rep = p.Hq / p.Hk;
  // causal mode: this block's nodes [i0, i0 + nb); tree mode: all nodes
  const int ntile = TA_MAXR / rep;
  const int i0 = p.causal ? int(blockIdx.z) * ntile : 0;
  const int nb = p.causal ? min(ntile, p.nodes - i0) : p.nodes;
  const int R = nb * rep;
  pdl_launch_dependents();
  pdl_wait();
  const int n = p.lens[r];
  const int total = n + (p.causal ? i0 + nb : p.nodes);  // causal: later rows are invisible to every node here
  const uint16_t* Kr = p.K + (size_t(r) * p.Hk + hk) * p.cap * D;  // one contiguous [cap][D] stream
  const uint16_t* Vr = p.V + (size_t(r) * p.Hk + hk) * p.cap * D;
  constexpr size_t sp = D;  // position stride
  // ancestor sets of the tree nodes (node 0 is the root)
  if (tid == 0 && !p.causal) {
    bool bad = false;
    for (int i = 0; i < p.nodes; ++i) {
      const int par = p.parents[size_t(r) * p.nodes + i];
      if (i == 0 ? par >= 0 : (par < 0 || par >= i)) bad = true;
      anc[i] = (1ull << i) | ((i > 0 && par >= 0 && par < i) ? anc[par] : 0ull);
    }
    if (bad) raise_error(p.err, kErrTree);
  }
  // queries: row rho = node * rep + j  <-  q[(r * nodes + node)][(hk * rep + j) * D]
  for (int c = tid; c < TA_MAXR * (D / 8); c += TA_THREADS) {
    const int rho = c / (D / 8), col = (c % (D / 8)) * 8;
    const bool ok = rho < R;
    const uint16_t* src =
        p.q + (size_t(r * p.nodes + i0 + (ok ? rho / rep : 0)) * p.Hq + hk * rep + (ok ? rho % rep : 0)) * D + col;
    cp_async16(qs + rho * LD + col, src, ok ? 16 : 0);
  }
  auto load_tile = [&](int tile, int buf) {
    uint16_t* kb = kv + size_t(buf) * 2 * TA_KT * LD;
    uint16_t* vb = kb + TA_KT * LD;
    const int p0 = tile * TA_KT;
    for (int c = tid; c < TA_KT * (D / 8); c += TA_THREADS) {
      const int row = c / (D / 8), col = (c % (D / 8)) * 8, pos = p0 + row;
      const bool ok = pos < total;
      const size_t off = ok ? size_t(pos) * sp + col : 0;
      cp_async16(kb + row * LD + col, Kr + off, ok ? 16 : 0);
      cp_async16(vb + row * LD + col, Vr + off, ok ? 16 : 0);
    }
  };
  const int ntiles_all = (total + TA_KT - 1) / TA_KT;
  const int per = (ntiles_all + p.nsplit - 1) / p.nsplit;
  const int tile0 = min(ntiles_all, sp_i * per), ntiles = min(ntiles_all, tile0 + per) - tile0;
  load_tile(tile0, 0);
  cp_async_commit();  // group: queries + tile 0
  if (ntiles > 1) load_tile(tile0 + 1, 1);
  cp_async_commit();  // group: tile 1
  cp_async_wait<1>();
  __syncthreads();  // queries, tile 0 and anc visible

  const bool active = warp * 16 < R;
  const int r0 = warp * 16;
  unsigned long long anc_g = 0ull, anc_g8 = 0ull;  // this thread's two rows' ancestor sets
  const int node_g = i0 + (r0 + g) / rep, node_g8 = i0 + (r0 + g + 8) / rep;  // causal: last visible new row
  if (active && !p.causal) {
    const int ra = r0 + g, rb = r0 + g + 8;
    if (ra < R) anc_g = anc[ra / rep];
    if (rb < R) anc_g8 = anc[rb / rep];
  }
  uint32_t qa[NK][4];
  if (active) {
#pragma unroll
    for (int kk = 0; kk < NK; ++kk) ldsm_x4(qa[kk], qs + (r0 + (lane % 16)) * LD + kk * 16 + (lane / 16) * 8);
  }
  __syncthreads();  // the last buffer is free for its first tile
  float o[ND][4];
#pragma unroll
  for (int j = 0; j < ND; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const float sl2 = p.scale * 1.4426950408889634f;  // scores in log2 units

  for (int tile = 0; tile < ntiles; ++tile) {
    const int buf = tile % TA_NBUF;
    if (tile + 2 < ntiles) load_tile(tile0 + tile + 2, (tile + 2) % TA_NBUF);
    cp_async_commit();
    cp_async_wait<2>();  // this tile's group is complete; the next two may be in flight
    __syncthreads();
    if (active) {
      const uint16_t* kb = kv + size_t(buf) * 2 * TA_KT * LD;
      const uint16_t* vb = kb + TA_KT * LD;
      // ---- S = Q K^T over 64 keys: 8 n-tiles of 8 keys
      float s[TA_KT / 8][4];
#pragma unroll
      for (int j = 0; j < TA_KT / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[j][e] = 0.f;
#pragma unroll
      for (int j = 0; j < TA_KT / 8; ++j) {
#pragma unroll
        for (int kk = 0; kk < NK; kk += 2) {
          uint32_t b[4];  // keys 8j.., dims 16kk + {0, 8, 16, 24}
          ldsm_x4(b, kb + (j * 8 + (lane % 8)) * LD + kk * 16 + (lane / 8) * 8);
          mma_bf16_16816r(s[j], qa[kk], b[0], b[1]);
          mma_bf16_16816r(s[j], qa[kk + 1], b[2], b[3]);
        }
      }
      // ---- visibility, scale, online softmax
      const int p0 = (tile0 + tile) * TA_KT;
      const bool full_prefix = p0 + TA_KT <= n + (p.causal ? i0 + 1 : 0);
      float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int j = 0; j < TA_KT / 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = s[j][e] * sl2;
          if (!full_prefix) {
            const int pos = p0 + j * 8 + 2 * t + (e & 1);
            bool vis;
            if (p.causal) {
              vis = pos <= n + ((e & 2) ? node_g8 : node_g) && pos < total;
            } else {
              const unsigned long long a = (e & 2) ? anc_g8 : anc_g;
              vis = pos < n || (pos < total && ((a >> (pos - n)) & 1ull));
            }
            if (!vis) v = -INFINITY;
          }
          s[j][e] = v;
          tmax[e >> 1] = fmaxf(tmax[e >> 1], v);
        }
      float alpha[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 1));
        tmax[h] = fmaxf(tmax[h], __shfl_xor_sync(0xffffffffu, tmax[h], 2));
        const float mn = fmaxf(mrow[h], tmax[h]);
        alpha[h] = (mn == -INFINITY) ? 1.f : ex2_approx(mrow[h] - mn);
        mrow[h] = mn;
      }
      float lt[2] = {0.f, 0.f};
      uint32_t pa[TA_KT / 16][4];
      // a row with no visible key so far keeps m = -inf: subtract 0 instead (2^-inf = 0)
      const float mg[2] = {mrow[0] == -INFINITY ? 0.f : mrow[0], mrow[1] == -INFINITY ? 0.f : mrow[1]};
#pragma unroll
      for (int j = 0; j < TA_KT / 8; ++j) {
        float e4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          e4[e] = ex2_approx(s[j][e] - mg[e >> 1]);
          lt[e >> 1] += e4[e];
        }
        const int kk = j / 2, hi = j & 1;
        pa[kk][hi * 2 + 0] = pack2(f32_to_bf16_bits(e4[0]), f32_to_bf16_bits(e4[1]));
        pa[kk][hi * 2 + 1] = pack2(f32_to_bf16_bits(e4[2]), f32_to_bf16_bits(e4[3]));
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        lt[h] += __shfl_xor_sync(0xffffffffu, lt[h], 1);
        lt[h] += __shfl_xor_sync(0xffffffffu, lt[h], 2);
        lrow[h] = lrow[h] * alpha[h] + lt[h];
      }
      if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {  // a running maximum moved
#pragma unroll
        for (int dj = 0; dj < ND; ++dj) {
          o[dj][0] *= alpha[0];
          o[dj][1] *= alpha[0];
          o[dj][2] *= alpha[1];
          o[dj][3] *= alpha[1];
        }
      }
      // ---- O += P V: 4 k-steps of 16 keys, 16 n-tiles of 8 dims
#pragma unroll
      for (int kk = 0; kk < TA_KT / 16; ++kk) {
        // A fragment of P: (rows g / g+8, keys 16kk + 2t..) then (keys 16kk + 8 + 2t..)
        const uint32_t a[4] = {pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3]};
#pragma unroll
        for (int dj = 0; dj < ND; dj += 2) {
          uint32_t b[4];  // keys 16kk + (0..7 | 8..15), dims 8dj + (0 | 8)
          ldsm_x4_trans(b, vb + (kk * 16 + (lane % 8) + ((lane / 8) % 2) * 8) * LD + dj * 8 + (lane / 16) * 8);
          mma_bf16_16816r(o[dj], a, b[0], b[1]);
          mma_bf16_16816r(o[dj + 1], a, b[2], b[3]);
        }
      }
    }
    __syncthreads();  // the buffer is refilled next iteration
  }
  cp_async_wait<0>();
  if (!active) return;
  if (p.nsplit > 1) {  // ---- this slice's partial state
    const size_t base = ((size_t(r) * p.Hk + hk) * p.nsplit + sp_i) * TA_MAXR;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int rho = r0 + g + 8 * h;
      if (rho >= R) continue;
      float* po = p.part_o + (base + rho) * D;
#pragma unroll
      for (int dj = 0; dj < ND; ++dj)
        *reinterpret_cast<float2*>(po + dj * 8 + 2 * t) = make_float2(o[dj][2 * h], o[dj][2 * h + 1]);
      if (t == 0) *reinterpret_cast<float2*>(p.part_ml + (base + rho) * 2) = make_float2(mrow[h], lrow[h]);
    }
    return;
  }
  // ---- normalise and store rows g / g+8 of this warp
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int rho = r0 + g + 8 * h;
    if (rho >= R) continue;
    const float inv = lrow[h] > 0.f ? 1.f / lrow[h] : 0.f;
    uint16_t* dst = p.out + (size_t(r * p.nodes + i0 + rho / rep) * p.Hq + hk * rep + rho % rep) * D;
#pragma unroll
    for (int dj = 0; dj < ND; ++dj) {
      const uint32_t v = pack2(f32_to_bf16_bits(o[dj][2 * h] * inv), f32_to_bf16_bits(o[dj][2 * h + 1] * inv));
      *reinterpret_cast<uint32_t*>(dst + dj * 8 + 2 * t) = v;
    }
  }
}

// Merges the slices' partial states of each (request, KV head) in slice order.
template <int D>
__global__ void __launch_bounds__(128) tree_attn_merge_kernel(__grid_constant__ const TreeAttnParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x, hk = blockIdx.y;
  const int rep = p.Hq / p.Hk, R = p.nodes * rep, S = p.nsplit;
  const size_t base = (size_t(r) * p.Hk + hk) * S * TA_MAXR;
  for (int idx = threadIdx.x; idx < R * (D / 2); idx += blockDim.x) {
    const int rho = idx / (D / 2), d = (idx % (D / 2)) * 2;
    float M = -INFINITY;
    for (int s = 0; s < S; ++s) M = fmaxf(M, p.part_ml[(base + size_t(s) * TA_MAXR + rho) * 2]);
    float L = 0.f, o0 = 0.f, o1 = 0.f;
    for (int s = 0; s < S; ++s) {
      const size_t row = base + size_t(s) * TA_MAXR + rho;
      const float2 ml = *reinterpret_cast<const float2*>(p.part_ml + row * 2);
      const float w = ml.x == -INFINITY ? 0.f : ex2_approx(ml.x - M);
      const float2 ov = *reinterpret_cast<const float2*>(p.part_o + row * D + d);
      L += w * ml.y;
      o0 += w * ov.x;
      o1 += w * ov.y;
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    uint16_t* dst = p.out + (size_t(r * p.nodes + rho / rep) * p.Hq + hk * rep + rho % rep) * D + d;
    *reinterpret_cast<uint32_t*>(dst) = pack2(f32_to_bf16_bits(o0 * inv), f32_to_bf16_bits(o1 * inv));
  }
}

// ---------------------------------------------------------------------------- compaction
// KVCache::compact (src/cache/kv_cache.cpp:21-31) for every request and layer: rows
// lens[r] + keep[r][i] -> lens[r] + i, then lens[r] += n_keep[r]. keep must be strictly
// increasing with keep[0] = 0 (checked; kErrTree otherwise), hence keep[i] >= i. Rows are moved
// in increasing i, and one thread moves the same 16-byte chunk c of every row. Row m is written
// only at step m and read only at steps i <= m (keep[i] = m), the read at i = m being skipped, so
// each chunk is read as a source before that thread overwrites it as a destination.
struct BatchCompactParams {
  uint16_t* K;  // [layers][B][Hk][cap][D]
  uint16_t* V;
  int layers, B, cap, Hk, D;
  int* lens;
  const int* keep;  // [B][maxkeep]
  const int* n_keep;
  int maxkeep;
  int* err;
};

__global__ void batch_compact_kernel(__grid_constant__ const BatchCompactParams p) {
  const int r = blockIdx.x, layer = blockIdx.y;
  const int n = p.lens[r], nk = p.n_keep[r];
  const int* keep = p.keep + size_t(r) * p.maxkeep;
  if (nk < 1 || nk > p.maxkeep || keep[0] != 0) {
    if (threadIdx.x == 0) raise_error(p.err, kErrTree);
    return;
  }
  for (int i = 1; i < nk; ++i)
    if (keep[i] <= keep[i - 1] || n + keep[i] >= p.cap) {
      if (threadIdx.x == 0) raise_error(p.err, kErrTree);
      return;
    }
  const int chunks = p.D / 8;  // 16-byte pieces of one head's row
  for (int hk = 0; hk < p.Hk; ++hk) {
    const size_t base = ((size_t(layer) * p.B + r) * p.Hk + hk) * p.cap;
    for (int i = 1; i < nk; ++i) {  // keep[0] = 0 stays in place
      if (keep[i] == i) continue;
      const uint4* sk = reinterpret_cast<const uint4*>(p.K + (base + n + keep[i]) * p.D);
      const uint4* sv = reinterpret_cast<const uint4*>(p.V + (base + n + keep[i]) * p.D);
      uint4* dk = reinterpret_cast<uint4*>(p.K + (base + n + i) * p.D);
      uint4* dv = reinterpret_cast<uint4*>(p.V + (base + n + i) * p.D);
      for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
        dk[c] = sk[c];
        dv[c] = sv[c];
      }
    }
  }
}

__global__ void batch_commit_lens_kernel(int* lens, const int* n_keep, int B) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < B) lens[r] += n_keep[r];
}

// Row-major GEMM copy of a bf16 A-fragment-tiled weight (16 x 16 tiles, KT tiles per row
// block). Output row R: plain (group 1) feature R; SwiGLU (group 2) tile-interleaved:
// within each 2 * half rows, the first `half` are gate rows, the next `half` up rows.
__global__ void detile_rows_kernel(const uint16_t* src, int KT, int group, int half, int Nrows, int K,
                                   uint16_t* dst) {
  const size_t total = size_t(Nrows) * K;
  for (size_t idx = blockIdx.x * size_t(blockDim.x) + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
    const int R = int(idx / K), k = int(idx % K);
    int f, which = 0;
    if (group == 2) {
      const int tile = R / (2 * half), w = R % (2 * half);
      which = w / half;
      f = tile * half + w % half;
    } else {
      f = R;
    }
    const int rb = (f / 16) * group + which, rr = f % 16, c = k % 16;
    const int lane = (rr % 8) * 4 + (c % 8) / 2;
    const int e = (c & 1) | ((rr >= 8) ? 2 : 0) | ((c >= 8) ? 4 : 0);
    dst[idx] = src[(size_t(rb) * KT + k / 16) * 256 + lane * 8 + e];
  }
}

}  // namespace wc
