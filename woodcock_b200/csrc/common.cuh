// Shared device helpers for the woodcock_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wc {

constexpr int kWarp = 32;
// Dynamic shared memory one block may opt into on sm_100 (227 KB); the kernels' layouts are
// checked against it at compile time.
constexpr size_t kSmemOptinBytes = 232448;

// Device error word bits (raised with atomicOr, read by the host at the round's sync).
enum DeviceError : int {
  kErrTokenRange = 1,     // a token id outside [0, vocab)
  kErrCapacity = 2,       // a KV write beyond the arena capacity
  kErrRows = 4,           // a dynamic row count outside the sizes the launch was built for
  kErrPosition = 8,       // a RoPE position beyond the precomputed table
  kErrTree = 16,          // malformed tree (parent >= child)
  kErrTimeout = 32,       // a bounded wait (mbarrier / pipeline) expired
  kErrSample = 64,        // a sampled draw found no token with positive probability
};

__device__ __forceinline__ void raise_error(int* err, int bit) {
  if (err) atomicOr(err, bit);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Two-term bf16 split: v ~= hi + lo with |v - hi - lo| <= 2^-16 |v|. Tensor-core
// products of bf16 weights with (hi, lo) keep fp32-level accuracy on the activations.
__device__ __forceinline__ void split_bf16(float v, uint16_t& hi, uint16_t& lo) {
  hi = f32_to_bf16_bits(v);
  lo = f32_to_bf16_bits(v - bf16_bits_to_f32(hi));
}

// 2^x with the PTX ex2.approx.ftz.f32 instruction (relative error about 2^-22 per the PTX ISA;
// subnormal results flush to zero, 2^-inf = +0). The attention kernels keep scores and running
// maxima in log2 units (e^x = 2^(x log2 e)) and use it for the softmax weights, which they round
// to bf16 or use to weigh fp32 partial states.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t pack2(uint16_t lo_half, uint16_t hi_half) {
  return uint32_t(lo_half) | (uint32_t(hi_half) << 16);
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// Streaming 16-byte load: weights are read once per pass, keep L1 clean.
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float4 ldg_stream_f4(const float4* p) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];\n"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

// Bulk prefetch of [p, p+bytes) into L2 (bytes multiple of 16, p 16-byte aligned).
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

// Programmatic dependent launch: the next kernel in the stream may start once every block
// of this one has called launch_dependents; it must call wait before reading anything this
// kernel writes. Both are no-ops for kernels launched without the PDL attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// Orderable argmax key: larger value first, then the smaller index (first maximum,
// like std::max_element / np.argmax). atomicMax over keys is order-independent.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | static_cast<unsigned long long>(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long k) {
  return 0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull);
}
__device__ __forceinline__ float argmax_key_value(unsigned long long k) {
  uint32_t u = static_cast<uint32_t>(k >> 32);
  u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
  return __uint_as_float(u);
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11), counter (lo, hi, 0, 0), key = seed.
__device__ __forceinline__ uint4 philox4x32_10(uint64_t counter, uint64_t seed) {
  uint32_t c0 = uint32_t(counter), c1 = uint32_t(counter >> 32), c2 = 0, c3 = 0;
  uint32_t k0 = uint32_t(seed), k1 = uint32_t(seed >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
    const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return make_uint4(c0, c1, c2, c3);
}

// fp64 uniform in [0, 1) from element `index` of the stream: 53 bits of words 0 and 1.
__device__ __forceinline__ double philox_uniform(uint64_t seed, uint64_t index) {
  const uint4 r = philox4x32_10(index, seed);
  return (double(r.x >> 5) * 67108864.0 + double(r.y >> 6)) * (1.0 / 9007199254740992.0);
}

// Gumbel(0, 1) noise from element `index` of the stream, -log(-log(u)) with u on the open
// interval (0, 1): argmax_j (z_j / T + g_j) is a draw from softmax(z / T) (the Gumbel-max
// identity; Gumbel 1954, as used for sampling by Maddison, Tarlow & Minka 2014). u takes 53
// bits of words 0 and 1, so the noise is resolved near its upper tail (u -> 1), where the
// argmax over 10^4-10^5 candidates lands: a 24-bit u would quantise -log(u) to multiples
// of 2^-24 there (noise values ~13 apart by ~2.5%) and cap the noise at ~16.6.
__device__ __forceinline__ double philox_u53_open(uint64_t seed, uint64_t index) {
  const uint4 r = philox4x32_10(index, seed);
  return (double(r.x >> 5) * 67108864.0 + double(r.y >> 6) + 0.5) * (1.0 / 9007199254740992.0);
}
// fp64 noise for the residual / bonus draw:
__device__ __forceinline__ double philox_gumbel_d(uint64_t seed, uint64_t index) {
  return -log(-log(philox_u53_open(seed, index)));
}
// the same noise rounded to fp32, for the fused head epilogues and the first-token draw:
__device__ __forceinline__ float philox_gumbel_f(uint64_t seed, uint64_t index) {
  return float(philox_gumbel_d(seed, index));
}

// Random-number layout of sampled decoding. The device keeps (seed, counter base); a
// round (or an autoregressive step, or the prefill's first token) owns kRngStreams
// streams of kRngStreamLen elements from its base, then advances the base by
// kRngRoundStride. Streams 0..15: draft step i / head row l (element = vocabulary row);
// kRngAcceptStream: the acceptance uniform of draft i (element i); kRngResidualStream:
// the Gumbel noise of the residual or bonus draw (element = token id).
constexpr uint64_t kRngStreamLen = 1ull << 21;
constexpr int kRngStreams = 32;
constexpr uint64_t kRngRoundStride = kRngStreamLen * kRngStreams;
constexpr int kRngAcceptStream = 16;
constexpr int kRngResidualStream = 17;

}  // namespace wc

namespace wc {

// ldmatrix: four 8x8 b16 matrices; thread i gives the address of row (i % 8) of matrix i / 8.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* smem_row) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* smem_row) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D with A given as four registers.
__device__ __forceinline__ void mma_bf16_16816r(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 16-byte global -> shared async copy; src_bytes < 16 zero-fills the rest (0 = all zeros).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// bf16 hi/lo halves of two floats packed as (x0 in the low half, x1 in the high half)
__device__ __forceinline__ void split2_bf16(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  uint16_t h0, l0, h1, l1;
  split_bf16(x0, h0, l0);
  split_bf16(x1, h1, l1);
  hi = pack2(h0, h1);
  lo = pack2(l0, l1);
}

}  // namespace wc

namespace wc {

// ---- mbarrier + 1-D bulk (TMA) copies, CTA-local
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(bar)) : "memory");
}
// Bounded wait for the phase with the given parity; false when the bound expired.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t max_iters = 1u << 22) {
  const uint32_t a = smem_addr(bar);
  for (uint32_t i = 0; i < max_iters; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if (i > 64) __nanosleep(32);
  }
  return false;
}
// global -> shared bulk copy completing on `bar` (addresses 16-byte aligned, bytes % 16 == 0)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}
// L2 policy for data read once (streamed weights): evicted before other lines.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}
// bulk_g2s with an L2 cache policy
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;\n" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
      : "memory");
}
// named barrier among `count` threads (warps 0 .. count/32-1)
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// ---- activation fragments: the B-operand layout of the bf16 GEMV, shared by producers and
// consumers. Element (row l < 16, column k) of an input of width K lives in 32-bit word
//   ((nt * (K / 16) + k / 16) * 32 + lane) * 4 + q,   nt = l / 8, lane = (l % 8) * 4 + t,
//   t = (k % 8) / 2, q = (k % 16) / 8 (+2 for the lo term), half-word k % 2,
// i.e. exactly what mma.m16n8k16 expects for B = x^T with hi / lo bf16 terms.
constexpr int XF_NT = 2;  // rows 0..15

__device__ __forceinline__ size_t xf_word(int K, int l, int k, bool lo) {
  const int nt = l >> 3, g = l & 7, kt = k >> 4, kk = k & 15, t = (kk & 7) >> 1, q = kk >> 3;
  return ((size_t(nt) * (K >> 4) + kt) * 32 + g * 4 + t) * 4 + q + (lo ? 2 : 0);
}
// write one element (hi and lo halves)
__device__ __forceinline__ void xf_store(uint32_t* xf, int K, int l, int k, float v) {
  uint16_t h, lo;
  split_bf16(v, h, lo);
  uint16_t* w16 = reinterpret_cast<uint16_t*>(xf);
  w16[xf_word(K, l, k, false) * 2 + (k & 1)] = h;
  w16[xf_word(K, l, k, true) * 2 + (k & 1)] = lo;
}

}  // namespace wc
