// woodcock_b200 runtime: the C ABI of include/woodcock_b200.h.
//
// Host orchestration of the B200 decode round. Weights live on the device in their
// streaming layouts (bf16 A-fragment tiles or fp32 rows); fused projections are
// built at load: Q|K|V stacked, gate/up interleaved by 16-row blocks (SwiGLU
// epilogue), the drafter's main and auxiliary Q/K/V side by side along K. A
// decoder round (draft chain -> verify -> accept -> compact -> drafter update) is
// captured once per chain length as a CUDA graph and replayed with one host
// synchronisation per round; all round state lives in device memory.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "../../include/woodcock_b200.h"
#include "attention.cuh"
#include "attention_dec.cuh"
#include "attention_split.cuh"
#include "attention_mma.cuh"
#include "batch.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "host_io.h"
#include "misc.cuh"
#include "tree.cuh"

using namespace wc;
namespace fs = std::filesystem;

// ============================================================================ errors

namespace {

struct WcError {
  wc_status st;
  std::string msg;
};

[[noreturn]] void fail(wc_status st, const std::string& msg) { throw WcError{st, msg}; }

#define CUDA_TRY(x)                                                                                  \
  do {                                                                                               \
    cudaError_t e_ = (x);                                                                            \
    if (e_ != cudaSuccess) fail(e_ == cudaErrorMemoryAllocation ? WC_ERR_OOM : WC_ERR_CUDA,          \
                                std::string(#x) + ": " + cudaGetErrorString(e_));                    \
  } while (0)

double now_s() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

}  // namespace

// ============================================================================ context

struct RopeTable {
  float2* ptr = nullptr;
  int max_pos = 0;
};

// CUDA-event marks around kernels of a profiled round (a separate graph from the timed one).
enum ProfKind { PK_QKV, PK_ATTN, PK_O, PK_GU, PK_DOWN, PK_HEAD, PK_DRAFT_HEAD, PK_DRAFT_LAYER, PK_COUNT };
constexpr int PK_SLOTS = 16;  // entries of the profile arrays in the C ABI

struct Profiler {
  std::vector<cudaEvent_t> pool;
  size_t next = 0;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> marks;
  cudaEvent_t open[PK_COUNT] = {};
  cudaEvent_t take() {
    if (next == pool.size()) {
      cudaEvent_t e;
      cudaEventCreate(&e);
      pool.push_back(e);
    }
    return pool[next++];
  }
  ~Profiler() {
    for (auto e : pool) cudaEventDestroy(e);
  }
};

struct wc_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int num_sms = 148;
  std::string err;
  int* d_err = nullptr;  // device error word of the ops API
  uint64_t launches = 0;
  bool capturing = false;
  uint64_t capture_launches = 0;
  std::map<std::pair<int, uint32_t>, RopeTable> rope;
  double* pw = nullptr;
  double* qw = nullptr;
  int pw_n = 0;
  int occ_gemv[3] = {1, 1, 1};  // [0] fp32, [1] bf16 NT=1, [2] bf16 NT=2
  size_t max_smem = 0;
  Profiler* prof = nullptr;  // set while a profiled round is being captured
  bool pdl = true;           // programmatic dependent launch between round kernels
  int attn_mode = 4;         // bf16 caches: 4 the cluster kernel (attention_dec.cuh), 2 the
                             // split-sequence kernel (attention_split.cuh; always used for drafted
                             // tree levels), 1 split-KV mma kernel, 0 CUDA cores
  float* as_part_o = nullptr;   // attention_split partial states: [16 KV heads][AS_MAXS + 1][AS_MAXR][128]
  float* as_part_ml = nullptr;  //   and their (m, l): [16][AS_MAXS + 1][AS_MAXR][2]
  int* as_counters = nullptr;   //   per-KV-head arrivals (zero between launches)
  int attn_split_pos = 256;     // capacity positions per prefix block (WC_ATTN_SPLIT_POS)
  int gemv_blocks_per_sm = 1;
  bool gemv_wide = true;                 // 80 KB activation chunks for K up to 2560 (WC_GEMV_WIDE=0: split K)
  bool gemv_acs = true;                  // whole-K blocks with streamed activation pieces (WC_GEMV_ACS=0: split K)
  bool gemv_prefetch = false;            // L2 prefetch of the next GEMV's weights (WC_GEMV_PREFETCH=1;
                                         // measured 1.6% slower on the C3 round: it competes with the
                                         // dependent loads of the kernels in between)
  size_t gemv_prefetch_cap = 64u << 20;  // bytes prefetched at most
  float* gv_partial = nullptr;           // split-K partial sums
  size_t gv_partial_n = 0;               // floats
  int* gv_counters = nullptr;            // split-K arrival counters (zero between launches)
  int gv_counters_n = 0;
  void* pw_scratch = nullptr;            // wc_probs_from_logits: parameters + row thresholds
  int pw_rows = 0;
  uint32_t* lin_xf = nullptr;  // input fragments of the ops-API linear
  int lin_xf_k = 0;
  bool lin_xf_bf16 = false;
};

namespace {

template <class F>
wc_status guard(wc_ctx* ctx, F&& f) {
  try {
    f();
    return WC_OK;
  } catch (const WcError& e) {
    if (ctx) ctx->err = e.msg;
    return e.st;
  } catch (const std::bad_alloc&) {
    if (ctx) ctx->err = "host allocation failed";
    return WC_ERR_OOM;
  } catch (const std::exception& e) {
    if (ctx) ctx->err = e.what();
    return WC_ERR_IO;
  }
}

void prof_begin(wc_ctx* ctx, int kind) {
  if (!ctx->prof) return;
  cudaEvent_t e = ctx->prof->take();
  // external event nodes: a plain record inside stream capture is only a dependency marker
  if (ctx->capturing) cudaEventRecordWithFlags(e, ctx->stream, cudaEventRecordExternal);
  else cudaEventRecord(e, ctx->stream);
  ctx->prof->open[kind] = e;
}

void prof_end(wc_ctx* ctx, int kind) {
  if (!ctx->prof || !ctx->prof->open[kind]) return;
  cudaEvent_t e = ctx->prof->take();
  if (ctx->capturing) cudaEventRecordWithFlags(e, ctx->stream, cudaEventRecordExternal);
  else cudaEventRecord(e, ctx->stream);
  ctx->prof->marks.push_back({kind, {ctx->prof->open[kind], e}});
  ctx->prof->open[kind] = nullptr;
}

void count_launch(wc_ctx* ctx) {
  if (ctx->capturing) ++ctx->capture_launches;
  else ++ctx->launches;
}

void check_launch(wc_ctx* ctx, const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) fail(WC_ERR_CUDA, std::string("launch of ") + what + " failed: " + cudaGetErrorString(e));
  count_launch(ctx);
}

// Launch with optional programmatic dependent launch (the kernel must pdl_wait() before it
// reads anything the previous kernel writes) and an optional cluster along x.
template <typename... KArgs, typename... Args>
void launch_ex(wc_ctx* ctx, const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, bool pdl,
               int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl && ctx->pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster_x > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster_x;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) fail(WC_ERR_CUDA, std::string("launch of ") + what + ": " + cudaGetErrorString(e));
  count_launch(ctx);
}

void* dalloc(size_t bytes) {
  if (bytes == 0) bytes = 16;
  void* p = nullptr;
  const cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(WC_ERR_OOM, "cudaMalloc(" + std::to_string(bytes) + ") failed: " + cudaGetErrorString(e));
  }
  return p;
}

void dfree(void* p) {
  if (p) cudaFree(p);
}

// Host-built rotate-half RoPE table [max_pos][D/2] of (cos, sin) computed with the
// same float expressions as the reference (src/backends/cpu_ops.cpp:64-68).
RopeTable& rope_table(wc_ctx* ctx, int D, float base, int need_pos) {
  uint32_t bits;
  std::memcpy(&bits, &base, 4);
  auto& t = ctx->rope[{D, bits}];
  if (t.max_pos >= need_pos) return t;
  if (ctx->capturing) fail(WC_ERR_INVALID, "RoPE table growth during capture");
  const int max_pos = std::max(need_pos, 32768);
  const int half = D / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = std::pow(base, -2.f * i / D);
  std::vector<float2> host(size_t(max_pos) * half);
  for (int p = 0; p < max_pos; ++p)
    for (int i = 0; i < half; ++i) {
      const float a = float(p) * inv[i];
      host[size_t(p) * half + i] = make_float2(std::cos(a), std::sin(a));
    }
  if (t.ptr) {
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    dfree(t.ptr);
  }
  t.ptr = static_cast<float2*>(dalloc(host.size() * sizeof(float2)));
  CUDA_TRY(cudaMemcpy(t.ptr, host.data(), host.size() * sizeof(float2), cudaMemcpyHostToDevice));
  t.max_pos = max_pos;
  return t;
}

int dtype_size(int dt) { return dt == WC_BF16 ? 2 : 4; }

int src_dtype_code(const std::string& s) {
  if (s == "F32") return 0;
  if (s == "BF16") return 1;
  if (s == "F16") return 2;
  return -1;
}

}  // namespace

// ============================================================================ staged tensors / weights

namespace {

// A tensor uploaded to the device in its source dtype, waiting to be laid out.
struct Staged {
  void* ptr = nullptr;
  int dtype = 0;  // 0 f32, 1 bf16 (f16 is converted to f32 on upload)
  std::vector<int64_t> shape;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

__global__ void f16_to_f32_kernel(const uint16_t* src, float* dst, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    dst[i] = __half2float(__ushort_as_half(src[i]));
}

__global__ void convert_kernel(const void* src, int src_dtype, void* dst, int dst_dtype, size_t n) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    const float v = src_dtype == 1 ? bf16_bits_to_f32(static_cast<const uint16_t*>(src)[i])
                                   : static_cast<const float*>(src)[i];
    if (dst_dtype == 1) static_cast<uint16_t*>(dst)[i] = f32_to_bf16_bits(v);
    else static_cast<float*>(dst)[i] = v;
  }
}

// Tiles a row-major part [N][K] into tile grid positions (rb * rb_stride + rbo, kt + kto)
// of a bf16 A-fragment-tiled matrix with dst_KT k-tiles per row block.
__global__ void tile_part_kernel(const void* src, int src_dtype, int N, int K, uint16_t* dst, int dst_KT,
                                 int rb_stride, int rbo, int kto) {
  const int NB = (N + 15) / 16, KB = (K + 15) / 16;
  const size_t total = size_t(NB) * KB * 256;
  for (size_t idx = blockIdx.x * size_t(blockDim.x) + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
    const size_t tile = idx / 256;
    const int within = int(idx % 256);
    const int rbp = int(tile / KB), ktp = int(tile % KB);
    const int lane = within / 8, e = within % 8, g = lane / 4, t = lane % 4;
    const int r = g + ((e & 2) ? 8 : 0);
    const int c = 2 * t + (e & 1) + ((e & 4) ? 8 : 0);
    const int row = rbp * 16 + r, col = ktp * 16 + c;
    float v = 0.f;
    if (row < N && col < K) {
      const size_t s = size_t(row) * K + col;
      v = src_dtype == 1 ? bf16_bits_to_f32(static_cast<const uint16_t*>(src)[s]) : static_cast<const float*>(src)[s];
    }
    const size_t dtile = size_t(rbp * rb_stride + rbo) * dst_KT + (ktp + kto);
    dst[dtile * 256 + within] = f32_to_bf16_bits(v);
  }
}

// Row-major fp32 part copy: dst[(r * row_stride + row_off) * ld + col_off + c] = src[r][c].
__global__ void copy_part_f32_kernel(const void* src, int src_dtype, int N, int K, float* dst, int ld, int row_stride,
                                     int row_off, int col_off) {
  const size_t total = size_t(N) * K;
  for (size_t idx = blockIdx.x * size_t(blockDim.x) + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
    const int r = int(idx / K), c = int(idx % K);
    const float v = src_dtype == 1 ? bf16_bits_to_f32(static_cast<const uint16_t*>(src)[idx])
                                   : static_cast<const float*>(src)[idx];
    dst[size_t(r * row_stride + row_off) * ld + col_off + c] = v;
  }
}

// Restricted head: new row i = old row ids[i], for the tiled bf16 layout.
__global__ void gather_tiled_rows_kernel(const uint16_t* src, int KT, const int* ids, int n, uint16_t* dst) {
  const int NB = (n + 15) / 16;
  const size_t total = size_t(NB) * KT * 256;
  for (size_t idx = blockIdx.x * size_t(blockDim.x) + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
    const size_t tile = idx / 256;
    const int within = int(idx % 256);
    const int rb = int(tile / KT), kt = int(tile % KT);
    const int lane = within / 8, e = within % 8, g = lane / 4, t = lane % 4;
    const int r = g + ((e & 2) ? 8 : 0);
    const int c = 2 * t + (e & 1) + ((e & 4) ? 8 : 0);
    const int row = rb * 16 + r;
    uint16_t v = 0;
    if (row < n) {
      const int sr = ids[row];
      const int sg = sr % 8, shalf = (sr % 16) / 8;
      const int sc_t = (c % 8) / 2, sc_half = c / 8;
      const int slane = sg * 4 + sc_t;
      const int se = (c % 2) + shalf * 2 + sc_half * 4;
      const size_t stile = size_t(sr / 16) * KT + kt;
      v = src[stile * 256 + slane * 8 + se];
    }
    dst[idx] = v;
  }
}

__global__ void gather_rows_f32_kernel(const float* src, int ld, const int* ids, int n, float* dst) {
  const size_t total = size_t(n) * ld;
  for (size_t idx = blockIdx.x * size_t(blockDim.x) + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x)
    dst[idx] = src[size_t(ids[idx / ld]) * ld + idx % ld];
}

int grid_for(size_t n) { return int(std::min<size_t>((n + 255) / 256, 148 * 16)); }

// One projection in its streaming layout. N = output features; for SwiGLU (group 2)
// the stored matrix holds 2 * N rows (gate and up interleaved by 16-row blocks, or
// rows 2n / 2n+1 in the fp32 layout). The input is one to three segments side by side;
// in the bf16 layout each segment starts on a whole ring slab (512 columns) and its
// padding columns are zero.
struct Lin {
  void* w = nullptr;
  int N = 0, Np = 0, K = 0, Kp = 0, dtype = 0, group = 1;
  int nseg = 1;
  int seg_len[GEMV_MAXSEG] = {0, 0, 0};
  int seg_off[GEMV_MAXSEG] = {0, 0, 0};
  size_t bytes = 0;
  bool owned = true;
};

Lin make_lin(int dtype, int N, std::initializer_list<int> segs, int group) {
  Lin l;
  l.dtype = dtype;
  l.N = N;
  l.group = group;
  const bool bf16 = dtype == WC_BF16;
  int off = 0;
  l.nseg = 0;
  for (int s : segs) {
    if (l.nseg == GEMV_MAXSEG) fail(WC_ERR_INVALID, "too many input segments");
    l.seg_len[l.nseg] = s;
    l.seg_off[l.nseg] = off;
    off += xf_width(bf16, s);
    l.K += s;
    ++l.nseg;
  }
  if (bf16) {
    l.Np = ((N + 15) / 16) * 16 * group;
    l.Kp = off;
    l.bytes = size_t(l.Np) * l.Kp * 2;
  } else {
    l.Np = N * group;
    l.Kp = ((off + 3) / 4) * 4;
    l.bytes = size_t(l.Np) * l.Kp * 4;
  }
  l.w = dalloc(l.bytes);
  CUDA_TRY(cudaMemset(l.w, 0, l.bytes));
  return l;
}

void free_lin(Lin& l) {
  if (l.owned) dfree(l.w);
  l.w = nullptr;
}

// Places a row-major part [rows][cols] at output row row_off of input segment `seg`;
// `which` selects gate (0) / up (1) for a SwiGLU projection.
void lin_put(wc_ctx* ctx, Lin& l, const Staged& s, int rows, int cols, int row_off, int seg, int which) {
  if (seg < 0 || seg >= l.nseg || cols != l.seg_len[seg]) fail(WC_ERR_INVALID, "projection part does not fit");
  const int col_off = l.seg_off[seg];
  if (l.dtype == WC_BF16) {
    if (row_off % 16) fail(WC_ERR_UNSUPPORTED, "projection parts must start on 16-row boundaries");
    const int KT = l.Kp / 16;
    tile_part_kernel<<<grid_for(size_t(rows) * cols), 256, 0, ctx->stream>>>(
        s.ptr, s.dtype, rows, cols, static_cast<uint16_t*>(l.w), KT, l.group, (row_off / 16) * l.group + which,
        col_off / 16);
  } else {
    copy_part_f32_kernel<<<grid_for(size_t(rows) * cols), 256, 0, ctx->stream>>>(
        s.ptr, s.dtype, rows, cols, static_cast<float*>(l.w), l.Kp, l.group, row_off * l.group + which, col_off);
  }
  check_launch(ctx, "weight layout");
}

}  // namespace

struct wc_weight {
  wc_ctx* ctx;
  Lin lin;
};

// ============================================================================ GEMV / attention launchers

namespace {

// A GEMV input held as fragments (common.cuh) with the partial sums of squares of its
// rows ([nparts][16], nullptr when the consumer does not normalise it).
struct XIn {
  const uint32_t* xf = nullptr;
  const float* ss = nullptr;
  int nparts = 0;
};

int max_parts(const wc_ctx*) { return 4096; }

uint32_t* xf_alloc(bool bf16, int K) {
  const size_t bytes = size_t(GEMV_MAXL) * xf_width(bf16, K) * 4;
  auto* p = static_cast<uint32_t*>(dalloc(bytes));
  CUDA_TRY(cudaMemset(p, 0, bytes));  // padding columns and unused rows stay finite
  return p;
}

float* ss_alloc(const wc_ctx* ctx) {
  const size_t bytes = sizeof(float) * max_parts(ctx) * 16;
  auto* p = static_cast<float*>(dalloc(bytes));
  CUDA_TRY(cudaMemset(p, 0, bytes));
  return p;
}

GemvParams gemv_params() {
  GemvParams p;
  std::memset(&p, 0, sizeof(p));
  p.group = 1;
  return p;
}

// A sampled head (sampled decoding): the argmax key of row l becomes a draw from
// softmax(z / T), T read from the device, Gumbel noise from stream `stream` + l.
struct Pick {
  const float* temperature = nullptr;
  const unsigned long long* rng = nullptr;  // [seed, counter base] on the device
  int stream = 0;
};

void apply_pick(GemvParams& p, const Pick* pk) {
  if (!pk || !pk->temperature) return;
  p.temperature = pk->temperature;
  p.rng = pk->rng;
  p.rng_stream = pk->stream;
}

XSeg xs_frag(const XIn& x, int len, bool bf16, float eps = 0.f) {
  XSeg s;
  std::memset(&s, 0, sizeof(s));
  s.xf = x.xf;
  s.ss = x.ss;
  s.nparts = x.nparts;
  s.len = len;
  s.lenp = xf_width(bf16, len);
  s.eps = eps;
  return s;
}

XSeg xs_embed(const void* table, int len, bool bf16, const float* norm_w, const float* row_inv) {
  XSeg s;
  std::memset(&s, 0, sizeof(s));
  s.table = table;
  s.len = len;
  s.lenp = xf_width(bf16, len);
  s.norm_w = norm_w;
  s.row_inv = row_inv;
  return s;
}

// Work split of a bf16 GEMV launch: K-chunks that fit the activation buffer, and blocks
// per chunk so that one block runs per SM.
struct GemvPlan {
  int grid = 1, nkc = 1, kc_slabs = 1, gpk = 1;
  bool wide = false;  // the 80 KB activation-chunk instance
};

GemvPlan gemv_plan(const wc_ctx* ctx, const Lin& W, int L_max) {
  GemvPlan g;
  if (W.dtype != WC_BF16) {
    g.grid = std::max(1, std::min((W.N + GV_F32_WARPS - 1) / GV_F32_WARPS, ctx->num_sms * 2));
    return g;
  }
  const int NT = L_max <= 8 ? 1 : 2;
  const bool wide2 = NT == 2 && ctx->gemv_wide;  // 16 rows: the 128 KB chunk (K to 2048 unsplit)
  const int chs = wide2 ? GV_WIDE2_SLABS : gv_chunk_slabs(NT);
  const int nslab = W.Kp / GV_COLS;
  const int nunits = W.Np / (16 * W.group);
  g.nkc = (nslab + chs - 1) / chs;
  g.wide = wide2;
  if (NT == 1 && g.nkc > 1 && nslab <= GV_WIDE_SLABS && ctx->gemv_wide) {  // K up to 2560: no split
    g.nkc = 1;
    g.wide = true;
  }
  g.kc_slabs = (nslab + g.nkc - 1) / g.nkc;
  const int target = ctx->num_sms * std::min(ctx->gemv_blocks_per_sm, ctx->occ_gemv[NT]);
  g.gpk = std::max(1, std::min(nunits, target / g.nkc));
  g.grid = g.nkc * g.gpk;
  return g;
}

// Blocks of a GEMV launch (the part count of an fp32 GEMV's ss_out and of side jobs).
int gemv_grid(const wc_ctx* ctx, const Lin& W, int L_max) { return gemv_plan(ctx, W, L_max).grid; }

// Part count of a GEMV's ss_out: one per epilogue unit (bf16) or per block (fp32).
int gemv_parts(const wc_ctx* ctx, const Lin& W, int L_max) {
  return W.dtype == WC_BF16 ? W.Np / (16 * W.group) : gemv_grid(ctx, W, L_max);
}

// Part count of a head's side-job sums of squares.
int side_parts(const wc_ctx* ctx, const Lin& W, int L_max) { return std::min(GV_SIDE_BLOCKS, gemv_grid(ctx, W, L_max)); }

// Bytes of `next` to prefetch into L2 while the current GEMV ends (0 = off).
void gemv_prefetch(const wc_ctx* ctx, GemvParams& p, const Lin* next, const Lin* next2 = nullptr) {
  if (!ctx->gemv_prefetch) return;
  if (next && next->dtype == WC_BF16) {
    p.pf = next->w;
    p.pf_bytes = std::min(next->bytes, ctx->gemv_prefetch_cap);
  }
  if (next2 && next2->dtype == WC_BF16) {
    p.pf2 = next2->w;
    p.pf2_bytes = std::min(next2->bytes, ctx->gemv_prefetch_cap);
  }
}

void launch_gemv(wc_ctx* ctx, const Lin& W, GemvParams p) {
  const bool bf16 = W.dtype == WC_BF16;
  p.w = W.w;
  p.N = W.N;
  p.Np = W.Np;
  p.Kp = W.Kp;
  p.group = W.group;
  if (!p.err) p.err = ctx->d_err;
  if (p.nseg != W.nseg) fail(WC_ERR_INVALID, "GEMV input segments do not match the weight");
  for (int s = 0; s < p.nseg; ++s) {
    const XSeg& sg = p.seg[s];
    if (sg.len != W.seg_len[s] || sg.lenp != xf_width(bf16, sg.len))
      fail(WC_ERR_INVALID, "GEMV input width " + std::to_string(sg.len) + " != " + std::to_string(W.seg_len[s]));
    if (sg.xf && sg.ss && (sg.nparts < 1 || sg.nparts > max_parts(ctx)))
      fail(WC_ERR_INVALID, "GEMV input statistics have a bad part count");
    if (!sg.xf && (!sg.table || !sg.norm_w || (bf16 && sg.len % 16)))
      fail(WC_ERR_INVALID, "embedding segments need a table, a gain and a width that is a multiple of 16");
  }
  p.flags = 0;
  for (int s = 0; s < p.nseg; ++s) {
    if (!p.seg[s].xf) p.flags |= GV_F_TOK | GV_F_TABLE;
    if (p.seg[s].xf && p.seg[s].ss) p.flags |= GV_F_SS;
  }
  if (p.L_max < 1 || p.L_max > GEMV_MAXL) fail(WC_ERR_INVALID, "GEMV rows outside 1..16");
  if (p.nout > 2 || ((p.nout > 0 || p.ss_out) && p.epi == EPI_ARGMAX)) fail(WC_ERR_INVALID, "bad GEMV outputs");
  p.out_width = xf_width(bf16, W.N);
  GemvPlan g = gemv_plan(ctx, W, p.L_max);
  // a projection that would split K but has at most one unit per SM runs whole-K blocks,
  // streaming the activation beside the weights (no partials, no last-block hand-off)
  p.acs = 0;
  if (bf16 && ctx->gemv_acs && g.nkc > 1 && p.L_max <= 8 && W.group == 1 && !(p.flags & GV_F_TABLE) &&
      W.Np / 16 <= ctx->num_sms) {
    p.acs = 1;
    g.nkc = 1;
    g.kc_slabs = W.Kp / GV_COLS;
    g.gpk = W.Np / 16;
    g.grid = g.gpk;
  }
  if (p.ss_out && gemv_parts(ctx, W, p.L_max) > max_parts(ctx))
    fail(WC_ERR_INVALID, "GEMV output statistics above the buffer size");
  if (p.side_src) {
    p.side_width = xf_width(bf16, p.side_len);
    p.side_blocks = std::min(GV_SIDE_BLOCKS, g.grid);
  }
  if (bf16) {
    p.nkc = g.nkc;
    p.kc_slabs = g.kc_slabs;
    p.gpk = g.gpk;
    const bool nt2 = p.L_max > 8;
    if (!p.acs && g.kc_slabs > (g.wide ? (nt2 ? GV_WIDE2_SLABS : GV_WIDE_SLABS) : gv_chunk_slabs(nt2 ? 2 : 1)))
      fail(WC_ERR_INVALID, "GEMV chunk above the buffer");
    if (g.nkc > 1) {
      if (size_t(g.nkc) * (W.Np / 16) * 256 > ctx->gv_partial_n || g.gpk > ctx->gv_counters_n)
        fail(WC_ERR_UNSUPPORTED, "GEMV split-K scratch too small for this projection");
      p.partial = ctx->gv_partial;
      p.counters = ctx->gv_counters;
    }
    if (p.acs)
      launch_ex(ctx, "gemv", gemv_bf16_kernel<1, true>, dim3(g.grid), dim3(GV_THREADS), gemv_bf16_smem<1>(), true, 1,
                p);
    else if (g.wide && nt2)
      launch_ex(ctx, "gemv", gemv_bf16_kernel<2, false, true>, dim3(g.grid), dim3(GV_THREADS),
                gemv_bf16_smem<2, true>(), true, 1, p);
    else if (g.wide)
      launch_ex(ctx, "gemv", gemv_bf16_kernel<1, false, true>, dim3(g.grid), dim3(GV_THREADS),
                gemv_bf16_smem<1, true>(), true, 1, p);
    else if (p.L_max <= 8)
      launch_ex(ctx, "gemv", gemv_bf16_kernel<1>, dim3(g.grid), dim3(GV_THREADS), gemv_bf16_smem<1>(), true, 1, p);
    else
      launch_ex(ctx, "gemv", gemv_bf16_kernel<2>, dim3(g.grid), dim3(GV_THREADS), gemv_bf16_smem<2>(), true, 1, p);
  } else {
    const size_t smem = gemv_f32_smem(p.L_max, W.Kp);
    if (smem > ctx->max_smem) fail(WC_ERR_UNSUPPORTED, "fp32 projection too wide for shared memory");
    launch_ex(ctx, "gemv", gemv_f32_kernel, dim3(g.grid), dim3(GV_F32_THREADS), smem, true, 1, p);
  }
}

PackParams pack_params() {
  PackParams p;
  std::memset(&p, 0, sizeof(p));
  return p;
}

// Rows -> GEMV input fragments (+ sums of squares, + fp32 copy); one block per row.
void launch_pack(wc_ctx* ctx, PackParams p, bool bf16, int L_max) {
  if (!p.err) p.err = ctx->d_err;
  p.xf_width = xf_width(bf16, p.K);
  p.xf_fp32 = bf16 ? 0 : 1;
  launch_ex(ctx, "pack", pack_rows_kernel, dim3(L_max), dim3(256), 0, true, 1, p);
}

constexpr int ATT_CLUSTER = 8;

void launch_attention(wc_ctx* ctx, AttnParams p) {
  if (!p.err) p.err = ctx->d_err;
  if (p.D > ATT_MAXD || p.D % 32) fail(WC_ERR_UNSUPPORTED, "head_dim must be a multiple of 32 up to 128");
  if (p.H % p.Hk) fail(WC_ERR_INVALID, "heads must be a multiple of kv_heads");
  const int rep = p.H / p.Hk;
  if (p.L_max * rep > ATT_MAXR) fail(WC_ERR_UNSUPPORTED, "too many query rows per KV head in one launch");
  const uintptr_t al = reinterpret_cast<uintptr_t>(p.Kc) | reinterpret_cast<uintptr_t>(p.Vc) |
                       reinterpret_cast<uintptr_t>(p.q_ready ? p.q_ready : p.qkv);
  if (al % 16 || (p.stride_p * (p.kv_dtype == 1 ? 2 : 4)) % 16 || (p.stride_h * (p.kv_dtype == 1 ? 2 : 4)) % 16 ||
      (!p.q_ready && p.ld_qkv % 4))
    fail(WC_ERR_INVALID, "attention inputs must be 16-byte aligned with 16-byte row strides");
  if (p.xf_out) p.xf_width = xf_width(!p.xf_fp32, p.H * p.D);
  // tensor-core paths: bf16 cache, rule-based visibility, new rows appended by the kernel
  const bool tc_ok = !p.q_ready && !p.mask_full && p.kv_dtype == WC_BF16 && p.write_cache &&
                     (p.D == 128 || p.D == 64) && p.L_max * rep <= AM_MAXR && p.stride_p == p.D;
  // drafted tree levels (mask bits from the committed length) take the split kernel in every mode
  const bool split_ok = tc_ok && p.L_max <= AS_MAXL && p.L_max * rep <= AS_MAXR && p.Hk <= 16;
  if (p.mask_from_prefix && tc_ok && !split_ok) fail(WC_ERR_UNSUPPORTED, "tree level too wide for the decode attention");
  if (split_ok && (ctx->attn_mode == 2 || p.mask_from_prefix)) {
    AttnSplitParams sp;
    std::memset(&sp, 0, sizeof(sp));
    sp.a = p;
    sp.part_o = ctx->as_part_o;
    sp.part_ml = ctx->as_part_ml;
    sp.counters = ctx->as_counters;
    // prefix blocks per KV head: the capacity in slices of attn_split_pos positions (a block holds
    // 256 at once), fixed when the round graph is captured
    sp.S = std::max(1, std::min(AS_MAXS, (p.cap + ctx->attn_split_pos - 1) / ctx->attn_split_pos));
    const bool mt2 = p.L_max * rep > 16;
    const dim3 grid(sp.S + 1, p.Hk);
    if (p.D == 128) {
      if (mt2)
        launch_ex(ctx, "attention_split", attention_split_kernel<128, 2, 8>, grid, dim3(8 * kWarp),
                  attention_split_smem<128, 8>(), true, 1, sp);
      else
        launch_ex(ctx, "attention_split", attention_split_kernel<128, 1, 16>, grid, dim3(16 * kWarp),
                  attention_split_smem<128, 16>(), true, 1, sp);
    } else {
      if (mt2)
        launch_ex(ctx, "attention_split", attention_split_kernel<64, 2, 8>, grid, dim3(8 * kWarp),
                  attention_split_smem<64, 8>(), true, 1, sp);
      else
        launch_ex(ctx, "attention_split", attention_split_kernel<64, 1, 16>, grid, dim3(16 * kWarp),
                  attention_split_smem<64, 16>(), true, 1, sp);
    }
    return;
  }
  if (tc_ok && ctx->attn_mode == 4 && p.L_max <= AD_MAXL && p.L_max * rep <= AD_MAXR) {
    const bool mt2 = p.L_max * rep > 16;
    if (p.D == 128) {
      if (mt2)
        launch_ex(ctx, "attention_dec", attention_dec_kernel<128, 2>, dim3(AD_CLUSTER, p.Hk, 1), dim3(AD_THREADS),
                  attention_dec_smem<128>(), true, AD_CLUSTER, p);
      else
        launch_ex(ctx, "attention_dec", attention_dec_kernel<128, 1>, dim3(AD_CLUSTER, p.Hk, 1), dim3(AD_THREADS),
                  attention_dec_smem<128>(), true, AD_CLUSTER, p);
    } else {
      if (mt2)
        launch_ex(ctx, "attention_dec", attention_dec_kernel<64, 2>, dim3(AD_CLUSTER, p.Hk, 1), dim3(AD_THREADS),
                  attention_dec_smem<64>(), true, AD_CLUSTER, p);
      else
        launch_ex(ctx, "attention_dec", attention_dec_kernel<64, 1>, dim3(AD_CLUSTER, p.Hk, 1), dim3(AD_THREADS),
                  attention_dec_smem<64>(), true, AD_CLUSTER, p);
    }
    return;
  }
  if (tc_ok && ctx->attn_mode >= 1) {
    if (p.D == 128)
      launch_ex(ctx, "attention_mma", attention_mma_kernel<128>, dim3(AM_CLUSTER, p.Hk, 1), dim3(AM_THREADS),
                attention_mma_smem<128>(p.L_max), true, AM_CLUSTER, p);
    else
      launch_ex(ctx, "attention_mma", attention_mma_kernel<64>, dim3(AM_CLUSTER, p.Hk, 1), dim3(AM_THREADS),
                attention_mma_smem<64>(p.L_max), true, AM_CLUSTER, p);
    return;
  }
  launch_ex(ctx, "attention", attention_kernel, dim3(ATT_CLUSTER, p.Hk, 1), dim3(ATT_THREADS),
            attention_smem(p.L_max), true, ATT_CLUSTER, p);
}

AttnParams attn_params() {
  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  return p;
}

}  // namespace

// ============================================================================ C ABI: context

extern "C" wc_status wc_ctx_create(int device, void* stream, wc_ctx** out) {
  if (!out) return WC_ERR_INVALID;
  auto* ctx = new wc_ctx();
  const wc_status st = guard(ctx, [&] {
    CUDA_TRY(cudaSetDevice(device));
    ctx->device = device;
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) fail(WC_ERR_UNSUPPORTED, "woodcock_b200 needs an sm_100 (Blackwell) GPU");
    ctx->num_sms = prop.multiProcessorCount;
    ctx->max_smem = prop.sharedMemPerBlockOptin;
    if (stream) {
      ctx->stream = static_cast<cudaStream_t>(stream);
    } else {
      CUDA_TRY(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking));
      ctx->own_stream = true;
    }
    if (const char* e = std::getenv("WC_PDL")) ctx->pdl = std::atoi(e) != 0;
    if (const char* e = std::getenv("WC_GEMV_BLOCKS_PER_SM")) ctx->gemv_blocks_per_sm = std::max(1, std::atoi(e));
    if (const char* e = std::getenv("WC_ATTN")) ctx->attn_mode = std::atoi(e);
    if (const char* e = std::getenv("WC_ATTN_SPLIT_POS")) ctx->attn_split_pos = std::max(16, std::atoi(e));
    if (const char* e = std::getenv("WC_GEMV_PREFETCH")) ctx->gemv_prefetch = std::atoi(e) != 0;
    if (const char* e = std::getenv("WC_GEMV_ACS")) ctx->gemv_acs = std::atoi(e) != 0;
    if (const char* e = std::getenv("WC_GEMV_WIDE")) ctx->gemv_wide = std::atoi(e) != 0;
    if (const char* e = std::getenv("WC_GEMV_PREFETCH_MB")) ctx->gemv_prefetch_cap = size_t(std::max(0, std::atoi(e))) << 20;
    ctx->d_err = static_cast<int*>(dalloc(sizeof(int)));
    CUDA_TRY(cudaMemset(ctx->d_err, 0, sizeof(int)));
    ctx->gv_partial_n = size_t(8) << 20;  // 32 MB of split-K partials
    ctx->gv_partial = static_cast<float*>(dalloc(sizeof(float) * ctx->gv_partial_n));
    ctx->as_part_o = static_cast<float*>(dalloc(sizeof(float) * 16 * (AS_MAXS + 1) * AS_MAXR * 128));
    ctx->as_part_ml = static_cast<float*>(dalloc(sizeof(float) * 16 * (AS_MAXS + 1) * AS_MAXR * 2));
    ctx->as_counters = static_cast<int*>(dalloc(sizeof(int) * AS_MAXHK));
    CUDA_TRY(cudaMemset(ctx->as_counters, 0, sizeof(int) * AS_MAXHK));
    ctx->gv_counters_n = 8192;
    ctx->gv_counters = static_cast<int*>(dalloc(sizeof(int) * ctx->gv_counters_n));
    CUDA_TRY(cudaMemset(ctx->gv_counters, 0, sizeof(int) * ctx->gv_counters_n));
    const int smax = int(ctx->max_smem);
    CUDA_TRY(cudaFuncSetAttribute(gemv_bf16_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(gemv_bf16_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(gemv_bf16_kernel<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(gemv_bf16_kernel<1, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  smax));
    CUDA_TRY(cudaFuncSetAttribute(gemv_bf16_kernel<2, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  smax));
    CUDA_TRY(cudaFuncSetAttribute(gemv_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(attention_mma_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(attention_mma_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(attention_split_kernel<128, 1, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(attention_split_kernel<128, 2, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(attention_split_kernel<64, 1, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(attention_split_kernel<64, 2, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(attention_dec_kernel<128, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(attention_dec_kernel<128, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(attention_dec_kernel<64, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(attention_dec_kernel<64, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    CUDA_TRY(cudaFuncSetAttribute(kv_compact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smax));
    int occ = 0;
    CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_bf16_kernel<1>, GV_THREADS,
                                                           gemv_bf16_smem<1>()));
    ctx->occ_gemv[1] = std::max(1, occ);
    CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_bf16_kernel<2>, GV_THREADS,
                                                           gemv_bf16_smem<2>()));
    ctx->occ_gemv[2] = std::max(1, occ);
  });
  if (st != WC_OK) {
    // keep the context so the caller can read the error, but mark it unusable
    *out = ctx;
    return st;
  }
  *out = ctx;
  return WC_OK;
}

extern "C" wc_status wc_ctx_set_stream(wc_ctx* ctx, void* stream) {
  if (!ctx) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    if (ctx->own_stream) {
      CUDA_TRY(cudaStreamSynchronize(ctx->stream));
      cudaStreamDestroy(ctx->stream);
      ctx->own_stream = false;
    }
    ctx->stream = static_cast<cudaStream_t>(stream);
  });
}

extern "C" void wc_ctx_destroy(wc_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  for (auto& kv : ctx->rope) dfree(kv.second.ptr);
  dfree(ctx->d_err);
  dfree(ctx->gv_partial);
  dfree(ctx->gv_counters);
  dfree(ctx->as_part_o);
  dfree(ctx->as_part_ml);
  dfree(ctx->as_counters);
  dfree(ctx->pw_scratch);
  dfree(ctx->pw);
  dfree(ctx->qw);
  dfree(ctx->lin_xf);
  if (ctx->own_stream && ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
}

extern "C" const char* wc_last_error(const wc_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

extern "C" wc_status wc_ctx_synchronize(wc_ctx* ctx) {
  if (!ctx) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    int e = 0;
    CUDA_TRY(cudaMemcpy(&e, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
      CUDA_TRY(cudaMemset(ctx->d_err, 0, sizeof(int)));
      CUDA_TRY(cudaMemset(ctx->gv_counters, 0, sizeof(int) * ctx->gv_counters_n));
      CUDA_TRY(cudaMemset(ctx->as_counters, 0, sizeof(int) * AS_MAXHK));
      fail(WC_ERR_DEVICE, "device error flag " + std::to_string(e));
    }
  });
}

extern "C" uint64_t wc_ctx_launch_count(const wc_ctx* ctx) { return ctx ? ctx->launches : 0; }
extern "C" wc_status wc_ctx_wait_selftest(wc_ctx* ctx, int iterations) {
  if (!ctx || iterations < 1 || iterations > (1 << 20)) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    wait_selftest_kernel<<<1, 32, 0, ctx->stream>>>(ctx->d_err, uint32_t(iterations));
    check_launch(ctx, "wait self test");
  });
}

// ============================================================================ C ABI: ops

extern "C" wc_status wc_weight_create(wc_ctx* ctx, const void* data, int src_dtype, int data_on_device, int out_rows,
                                      int in_cols, int dtype, wc_weight** w) {
  if (!ctx || !w || !data || out_rows <= 0 || in_cols <= 0) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    if ((dtype != WC_F32 && dtype != WC_BF16) || (src_dtype != WC_F32 && src_dtype != WC_BF16))
      fail(WC_ERR_INVALID, "dtype must be WC_F32 or WC_BF16");
    Staged s;
    const size_t bytes = size_t(out_rows) * in_cols * dtype_size(src_dtype);
    s.dtype = src_dtype;
    if (data_on_device) {
      s.ptr = const_cast<void*>(data);
    } else {
      s.ptr = dalloc(bytes);
      CUDA_TRY(cudaMemcpy(s.ptr, data, bytes, cudaMemcpyHostToDevice));
    }
    auto* out = new wc_weight{ctx, make_lin(dtype, out_rows, {in_cols}, 1)};
    lin_put(ctx, out->lin, s, out_rows, in_cols, 0, 0, 0);
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    if (!data_on_device) dfree(s.ptr);
    *w = out;
  });
}

extern "C" void wc_weight_destroy(wc_weight* w) {
  if (!w) return;
  free_lin(w->lin);
  delete w;
}

extern "C" wc_status wc_linear(wc_ctx* ctx, const float* x, int L, int in, const wc_weight* W, float* y, int accumulate) {
  if (!ctx || !x || !W || !y || L <= 0) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    const Lin& lin = W->lin;
    if (in != lin.K) fail(WC_ERR_INVALID, "linear: input width does not match the weight");
    const bool bf16 = lin.dtype == WC_BF16;
    if (!ctx->lin_xf || ctx->lin_xf_k < in || ctx->lin_xf_bf16 != bf16) {
      CUDA_TRY(cudaStreamSynchronize(ctx->stream));
      dfree(ctx->lin_xf);
      ctx->lin_xf = xf_alloc(bf16, in);
      ctx->lin_xf_k = in;
      ctx->lin_xf_bf16 = bf16;
    } else {
      // the padding columns of a narrower input must be zero again
      CUDA_TRY(cudaMemsetAsync(ctx->lin_xf, 0, size_t(GEMV_MAXL) * xf_width(bf16, ctx->lin_xf_k) * 4, ctx->stream));
    }
    for (int r0 = 0; r0 < L; r0 += GEMV_MAXL) {
      const int rows = std::min(GEMV_MAXL, L - r0);
      PackParams pk = pack_params();
      pk.src = x + size_t(r0) * in;
      pk.ld = in;
      pk.K = in;
      pk.L = rows;
      pk.xf = ctx->lin_xf;
      launch_pack(ctx, pk, bf16, rows);
      GemvParams p = gemv_params();
      p.L = rows;
      p.L_max = rows;
      p.nseg = 1;
      p.seg[0] = xs_frag(XIn{ctx->lin_xf, nullptr, 0}, in, bf16);
      p.epi = accumulate ? EPI_ADD : EPI_STORE;
      p.y = y + size_t(r0) * lin.N;
      p.ldy = lin.N;
      p.base = p.y;
      p.ldb = lin.N;
      launch_gemv(ctx, lin, p);
    }
  });
}

extern "C" wc_status wc_rmsnorm(wc_ctx* ctx, const float* x, float* y, int rows, int d, const float* w, float eps) {
  if (!ctx || !x || !y || !w || rows <= 0 || d <= 0) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    rmsnorm_rows_kernel<<<rows, 256, 0, ctx->stream>>>(x, y, d, w, eps);
    check_launch(ctx, "rmsnorm");
  });
}

extern "C" wc_status wc_rope(wc_ctx* ctx, float* x, int L, int heads, int D, const int* positions, float base) {
  if (!ctx || !x || !positions || L <= 0 || heads <= 0 || D <= 0 || D % 2) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    RopeTable& t = rope_table(ctx, D, base, 32768);
    rope_rows_kernel<<<L, 256, 0, ctx->stream>>>(x, heads, D, positions, t.ptr, t.max_pos, ctx->d_err);
    check_launch(ctx, "rope");
  });
}

extern "C" wc_status wc_silu_mul(wc_ctx* ctx, float* gate, const float* up, int64_t n) {
  if (!ctx || !gate || !up || n < 0) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    if (n == 0) return;
    silu_mul_kernel<<<grid_for(size_t(n)), 256, 0, ctx->stream>>>(gate, up, n);
    check_launch(ctx, "silu_mul");
  });
}

extern "C" wc_status wc_softmax(wc_ctx* ctx, float* x, int n) {
  if (!ctx || !x || n <= 0) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    softmax_row_kernel<<<1, 1024, 0, ctx->stream>>>(x, n);
    check_launch(ctx, "softmax");
  });
}

extern "C" wc_status wc_argmax_rows(wc_ctx* ctx, const float* x, int rows, int n, int* out) {
  if (!ctx || !x || !out || rows <= 0 || n <= 0) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    argmax_rows_kernel<<<rows, 1024, 0, ctx->stream>>>(x, n, out);
    check_launch(ctx, "argmax");
  });
}

extern "C" wc_status wc_attention(wc_ctx* ctx, const float* q, int L, int H, int Hk, int D, const void* K,
                                  const void* V, int kv_dtype, int T, const uint8_t* mask, float* out, float scale) {
  if (!ctx || !q || !K || !V || !out || L <= 0 || H <= 0 || Hk <= 0 || D <= 0 || T <= 0) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    if (H % Hk) fail(WC_ERR_INVALID, "heads must be a multiple of kv_heads");
    const int rep = H / Hk;
    const int rows = std::max(1, ATT_MAXR / rep);
    for (int r0 = 0; r0 < L; r0 += rows) {
      const int n = std::min(rows, L - r0);
      AttnParams p = attn_params();
      p.q_ready = q + size_t(r0) * H * D;
      p.L = n;
      p.L_max = n;
      p.T_full = T;
      p.Kc = const_cast<void*>(K);
      p.Vc = const_cast<void*>(V);
      p.kv_dtype = kv_dtype;
      p.stride_h = D;
      p.stride_p = (long long)Hk * D;
      p.cap = T;
      p.H = H;
      p.Hk = Hk;
      p.D = D;
      p.mask_full = mask ? mask + size_t(r0) * T : nullptr;
      p.mask_ld = T;
      p.scale = scale;
      p.out = out + size_t(r0) * H * D;
      p.ld_out = H * D;
      p.max_pos = 1;
      launch_attention(ctx, p);
    }
  });
}

extern "C" wc_status wc_philox_uniforms(wc_ctx* ctx, uint64_t seed, uint64_t offset, int n, double* out) {
  if (!ctx || !out || n < 0) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    if (n == 0) return;
    philox_uniforms_kernel<<<(n + 255) / 256, 256, 0, ctx->stream>>>(seed, offset, n, out);
    check_launch(ctx, "philox");
  });
}

extern "C" wc_status wc_probs_from_logits(wc_ctx* ctx, const float* logits, int rows, int V, float temperature,
                                          int top_k, float top_p, float* out) {
  if (!ctx || !logits || !out || rows < 1 || V < 1) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    if (top_k < 0 || !(top_p > 0.f) || top_p > 1.f) fail(WC_ERR_INVALID, "top_k >= 0 and top_p in (0, 1]");
    struct {
      float T;
      int k;
      float p;
      int pad;
    } prm{std::max(temperature, 1e-6f), top_k, top_p, 0};
    if (ctx->pw_rows < rows) {  // scratch: parameters + per-row thresholds
      CUDA_TRY(cudaStreamSynchronize(ctx->stream));
      dfree(ctx->pw_scratch);
      ctx->pw_scratch = dalloc(16 + sizeof(RowWarp) * size_t(rows));
      ctx->pw_rows = rows;
    }
    char* sc = static_cast<char*>(ctx->pw_scratch);
    CUDA_TRY(cudaMemcpyAsync(sc, &prm, sizeof(prm), cudaMemcpyHostToDevice, ctx->stream));
    RowWarp* rw = reinterpret_cast<RowWarp*>(sc + 16);
    WarpParams w;
    std::memset(&w, 0, sizeof(w));
    w.z = logits;
    w.V = V;
    w.ld = V;
    w.temperature = reinterpret_cast<const float*>(sc);
    w.top_k = reinterpret_cast<const int*>(sc + 4);
    w.top_p = reinterpret_cast<const float*>(sc + 8);
    w.out = rw;
    launch_ex(ctx, "warp rows", warp_rows_kernel, dim3(rows), dim3(1024), 0, false, 1, w);
    warped_probs_kernel<<<dim3(std::min(148, (V + 255) / 256), rows), 256, 0, ctx->stream>>>(
        logits, V, reinterpret_cast<const float*>(sc), rw, out);
    check_launch(ctx, "probs_from_logits");
  });
}

extern "C" wc_status wc_accept_greedy(wc_ctx* ctx, const int* am, const int* tokens, const int* parents, int N,
                                      int* out_path, int* out_n, int* out_next) {
  if (!ctx || !am || !tokens || !parents || !out_path || !out_n || !out_next || N <= 0) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    accept_greedy_tree_kernel<<<1, 32, 0, ctx->stream>>>(am, tokens, parents, N, out_path, out_n, out_next,
                                                         ctx->d_err);
    check_launch(ctx, "accept_greedy");
  });
}

extern "C" wc_status wc_accept_stochastic(wc_ctx* ctx, const double* p, const double* q, int V, const int* tokens,
                                          const int* parents, int N, uint64_t seed, uint64_t offset, int* out_path,
                                          int* out_n, int* out_next, int* out_used) {
  if (!ctx || !p || !q || !tokens || !parents || !out_path || !out_n || !out_next || !out_used || N <= 0 || V <= 0)
    return WC_ERR_INVALID;
  return guard(ctx, [&] {
    if (ctx->pw_n < V) {
      CUDA_TRY(cudaStreamSynchronize(ctx->stream));
      dfree(ctx->pw);
      dfree(ctx->qw);
      ctx->pw = static_cast<double*>(dalloc(sizeof(double) * V));
      ctx->qw = static_cast<double*>(dalloc(sizeof(double) * V));
      ctx->pw_n = V;
    }
    accept_stochastic_tree_kernel<<<1, 1024, 0, ctx->stream>>>(p, q, V, tokens, parents, N, seed, offset, ctx->pw,
                                                               ctx->qw, out_path, out_n, out_next, out_used,
                                                               ctx->d_err);
    check_launch(ctx, "accept_stochastic");
  });
}

// ---- wc_accept_stochastic_noalloc: the same kernel with scratch compiled into the library,
// for callers that cannot let a verify step allocate (or free, which waits for the device).
// Two rows of WC_ACCEPT_NOALLOC_MAX_V doubles (p residual, q); each call overwrites what it reads.
static __device__ __align__(256) double g_accept_scratch[2 * WC_ACCEPT_NOALLOC_MAX_V];

namespace {
constexpr int kMaxDevices = 256;
std::mutex g_scratch_mu;
double* g_scratch_addr[kMaxDevices] = {};  // device address of g_accept_scratch per ordinal
}  // namespace

extern "C" wc_status wc_accept_stochastic_noalloc(wc_ctx* ctx, const double* p, const double* q, int V,
                                                  const int* tokens, const int* parents, int N, uint64_t seed,
                                                  uint64_t offset, int* out_path, int* out_n, int* out_next,
                                                  int* out_used) {
  if (!ctx || !p || !q || !tokens || !parents || !out_path || !out_n || !out_next || !out_used || N <= 0 || V <= 0)
    return WC_ERR_INVALID;
  return guard(ctx, [&] {
    if (V > WC_ACCEPT_NOALLOC_MAX_V)
      fail(WC_ERR_CAPACITY, "wc_accept_stochastic_noalloc: V = " + std::to_string(V) +
                                " exceeds WC_ACCEPT_NOALLOC_MAX_V = " + std::to_string(WC_ACCEPT_NOALLOC_MAX_V));
    int cur = -1;
    CUDA_TRY(cudaGetDevice(&cur));
    if (cur != ctx->device)
      fail(WC_ERR_INVALID, "wc_accept_stochastic_noalloc: make the context's device current first");
    if (cur < 0 || cur >= kMaxDevices) fail(WC_ERR_UNSUPPORTED, "device ordinal out of range");
    double* scratch = nullptr;
    {
      // one-time set-up per device, with that device current
      std::lock_guard<std::mutex> lock(g_scratch_mu);
      if (!g_scratch_addr[cur]) {
        // the look-up may load the module; that must not happen inside a stream capture
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        CUDA_TRY(cudaStreamIsCapturing(ctx->stream, &cs));
        if (cs != cudaStreamCaptureStatusNone)
          fail(WC_ERR_INVALID, "wc_accept_stochastic_noalloc: make the first call on a device before any capture");
        void* a = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&a, g_accept_scratch);
        if (e != cudaSuccess || !a)
          fail(WC_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
        g_scratch_addr[cur] = static_cast<double*>(a);
      }
      scratch = g_scratch_addr[cur];
    }
    accept_stochastic_tree_kernel<<<1, 1024, 0, ctx->stream>>>(p, q, V, tokens, parents, N, seed, offset, scratch,
                                                               scratch + WC_ACCEPT_NOALLOC_MAX_V, out_path, out_n,
                                                               out_next, out_used, ctx->d_err);
    check_launch(ctx, "accept_stochastic_noalloc");
  });
}

// ============================================================================ C ABI: KV cache

struct wc_kv {
  wc_ctx* ctx;
  int layers, Hk, D, cap, dtype;
  void* K;
  void* V;
  int n;               // host-side size for the ops / forward API
  int* keep = nullptr;  // MAXTREE ints: the compaction keep list on the device
  size_t layer_elems() const { return size_t(Hk) * cap * D; }
  void* Kl(int l) const { return static_cast<char*>(K) + size_t(l) * layer_elems() * dtype_size(dtype); }
  void* Vl(int l) const { return static_cast<char*>(V) + size_t(l) * layer_elems() * dtype_size(dtype); }
};

namespace {
wc_kv* kv_new(wc_ctx* ctx, int layers, int Hk, int D, int cap, int dtype) {
  if (layers <= 0 || Hk <= 0 || D <= 0 || cap <= 0) fail(WC_ERR_INVALID, "bad KV cache shape");
  std::unique_ptr<wc_kv, void (*)(wc_kv*)> kv(new wc_kv{ctx, layers, Hk, D, cap, dtype, nullptr, nullptr, 0},
                                              wc_kv_destroy);
  const size_t bytes = size_t(layers) * kv->layer_elems() * dtype_size(dtype);
  kv->K = dalloc(bytes);
  kv->V = dalloc(bytes);
  kv->keep = static_cast<int*>(dalloc(sizeof(int) * MAXTREE));
  CUDA_TRY(cudaMemset(kv->K, 0, bytes));
  CUDA_TRY(cudaMemset(kv->V, 0, bytes));
  return kv.release();
}
}  // namespace

extern "C" wc_status wc_kv_create(wc_ctx* ctx, int layers, int kv_heads, int head_dim, int capacity, int dtype,
                                  wc_kv** kv) {
  if (!ctx || !kv) return WC_ERR_INVALID;
  return guard(ctx, [&] { *kv = kv_new(ctx, layers, kv_heads, head_dim, capacity, dtype); });
}

extern "C" void wc_kv_destroy(wc_kv* kv) {
  if (!kv) return;
  dfree(kv->K);
  dfree(kv->V);
  dfree(kv->keep);
  delete kv;
}

extern "C" int wc_kv_size(const wc_kv* kv) { return kv ? kv->n : -1; }
extern "C" int wc_kv_capacity(const wc_kv* kv) { return kv ? kv->cap : -1; }

extern "C" wc_status wc_kv_append(wc_kv* kv, int layer, const float* k, const float* v, int L) {
  if (!kv || !k || !v || L < 0 || layer < 0 || layer >= kv->layers) return WC_ERR_INVALID;
  return guard(kv->ctx, [&] {
    if (kv->n + L > kv->cap) fail(WC_ERR_CAPACITY, "KV cache capacity exceeded");
    if (L == 0) return;
    kv_append_kernel<<<grid_for(size_t(L) * kv->Hk * kv->D), 256, 0, kv->ctx->stream>>>(
        kv->Kl(layer), kv->Vl(layer), kv->dtype, kv->Hk, kv->D, kv->cap, kv->n, k, v, L);
    check_launch(kv->ctx, "kv_append");
  });
}

extern "C" wc_status wc_kv_commit(wc_kv* kv, int L) {
  if (!kv || L < 0) return WC_ERR_INVALID;
  return guard(kv->ctx, [&] {
    if (kv->n + L > kv->cap) fail(WC_ERR_CAPACITY, "KV cache capacity exceeded");
    kv->n += L;
  });
}

extern "C" wc_status wc_kv_trim_to(wc_kv* kv, int n) {
  if (!kv || n < 0 || n > kv->cap) return WC_ERR_INVALID;
  kv->n = n;
  return WC_OK;
}

namespace {
void kv_compact_impl(wc_kv* kv, int start, const int* keep_host, int n_keep) {
  if (start < 0 || n_keep < 0 || start + n_keep > kv->cap) fail(WC_ERR_INVALID, "bad compaction range");
  for (int i = 0; i < n_keep; ++i) {
    if (keep_host[i] < i || start + keep_host[i] >= kv->cap || (i && keep_host[i] <= keep_host[i - 1]))
      fail(WC_ERR_INVALID, "keep list must be increasing, with keep[i] >= i");
  }
  bool identity = true;
  for (int i = 0; i < n_keep; ++i) identity &= keep_host[i] == i;
  if (!identity && n_keep > 0) {
    if (n_keep > MAXTREE) fail(WC_ERR_UNSUPPORTED, "keep list longer than 64");
    // stream-ordered: a later compaction's copy into kv->keep waits for this kernel; a pageable
    // source is staged by the copy call, so keep_host may be reused when it returns
    CUDA_TRY(cudaMemcpyAsync(kv->keep, keep_host, sizeof(int) * n_keep, cudaMemcpyHostToDevice, kv->ctx->stream));
    const int slabs = kv->layers * kv->Hk;
    kv_compact_kernel<<<2 * slabs, 256, size_t(n_keep) * kv->D * sizeof(float), kv->ctx->stream>>>(
        kv->K, kv->V, kv->dtype, kv->D, kv->cap, slabs, kv->keep, n_keep, start);
    check_launch(kv->ctx, "kv_compact");
  }
  kv->n = start + n_keep;
}
}  // namespace

extern "C" wc_status wc_kv_compact(wc_kv* kv, int start, const int* keep, int n_keep) {
  if (!kv || (!keep && n_keep)) return WC_ERR_INVALID;
  return guard(kv->ctx, [&] { kv_compact_impl(kv, start, keep, n_keep); });
}

extern "C" wc_status wc_kv_read(const wc_kv* kv, int layer, int T, float* k, float* v) {
  if (!kv || !k || !v || layer < 0 || layer >= kv->layers || T < 0 || T > kv->cap) return WC_ERR_INVALID;
  return guard(kv->ctx, [&] {
    if (T == 0) return;
    kv_read_kernel<<<grid_for(size_t(T) * kv->Hk * kv->D), 256, 0, kv->ctx->stream>>>(
        kv->Kl(layer), kv->Vl(layer), kv->dtype, kv->Hk, kv->D, kv->cap, T, k, v);
    check_launch(kv->ctx, "kv_read");
  });
}

// ============================================================================ models: shared pieces

namespace {

struct Rows {
  bool stable = false;  // n_dev and the cache below it were written by completed work (round graphs)
  int L = 0;
  const int* L_dev = nullptr;
  int L_max = 0;
  const int* n_dev = nullptr;
  int n_add = 0;
  const int* positions = nullptr;
  const unsigned long long* newmask = nullptr;
  bool mask_from_prefix = false;  // newmask bits count from *n_dev (drafted tree levels)
  const uint8_t* mask_full = nullptr;
  int mask_ld = 0;
};

struct Stage {
  std::map<std::string, Staged> t;
  ~Stage() { clear(); }
  void clear() {
    for (auto& kv : t) dfree(kv.second.ptr);
    t.clear();
  }
  const Staged& get(const std::string& name, std::vector<int64_t> shape) const {
    auto it = t.find(name);
    if (it == t.end()) fail(WC_ERR_IO, "missing tensor " + name);
    if (it->second.shape != shape) {
      std::string s = "tensor " + name + " has shape [";
      for (size_t i = 0; i < it->second.shape.size(); ++i) s += (i ? "," : "") + std::to_string(it->second.shape[i]);
      s += "], expected [";
      for (size_t i = 0; i < shape.size(); ++i) s += (i ? "," : "") + std::to_string(shape[i]);
      fail(WC_ERR_INVALID, s + "]");
    }
    return it->second;
  }
  bool has(const std::string& name) const { return t.count(name) > 0; }
};

void stage_put(wc_ctx* ctx, Stage& stg, const std::string& name, const void* data, int src_dtype, int on_device,
               const int64_t* shape, int ndim) {
  if (!data || !shape || ndim <= 0) fail(WC_ERR_INVALID, "bad tensor " + name);
  Staged s;
  s.shape.assign(shape, shape + ndim);
  const int64_t n = s.numel();
  if (n <= 0) fail(WC_ERR_INVALID, "empty tensor " + name);
  if (src_dtype == 2) {  // f16 -> f32 on the device
    void* tmp = dalloc(size_t(n) * 2);
    CUDA_TRY(cudaMemcpy(tmp, data, size_t(n) * 2, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
    s.ptr = dalloc(size_t(n) * 4);
    f16_to_f32_kernel<<<grid_for(size_t(n)), 256, 0, ctx->stream>>>(static_cast<uint16_t*>(tmp),
                                                                   static_cast<float*>(s.ptr), size_t(n));
    check_launch(ctx, "f16 convert");
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    dfree(tmp);
    s.dtype = 0;
  } else if (src_dtype == 0 || src_dtype == 1) {
    s.dtype = src_dtype;
    const size_t bytes = size_t(n) * dtype_size(src_dtype);
    s.ptr = dalloc(bytes);
    CUDA_TRY(cudaMemcpy(s.ptr, data, bytes, on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
  } else {
    fail(WC_ERR_INVALID, "unsupported dtype for " + name);
  }
  auto it = stg.t.find(name);
  if (it != stg.t.end()) dfree(it->second.ptr);
  stg.t[name] = s;
}

float* to_f32_vec(wc_ctx* ctx, const Staged& s) {
  const size_t n = size_t(s.numel());
  float* out = static_cast<float*>(dalloc(n * 4));
  convert_kernel<<<grid_for(n), 256, 0, ctx->stream>>>(s.ptr, s.dtype, out, 0, n);
  check_launch(ctx, "convert");
  return out;
}

void* to_dtype(wc_ctx* ctx, const Staged& s, int dtype) {
  const size_t n = size_t(s.numel());
  void* out = dalloc(n * dtype_size(dtype));
  convert_kernel<<<grid_for(n), 256, 0, ctx->stream>>>(s.ptr, s.dtype, out, dtype, n);
  check_launch(ctx, "convert");
  return out;
}

void load_dir_tensors(const std::string& dir, const std::string& only_file,
                      const std::function<void(const std::string&, const TensorView&)>& put) {
  std::vector<std::string> files;
  if (!only_file.empty()) {
    files.push_back((fs::path(dir) / only_file).string());
  } else {
    if (!fs::is_directory(dir)) fail(WC_ERR_IO, "not a directory: " + dir);
    for (auto& e : fs::directory_iterator(dir))
      if (e.path().extension() == ".safetensors") files.push_back(e.path().string());
    std::sort(files.begin(), files.end());
  }
  if (files.empty()) fail(WC_ERR_IO, "no .safetensors in " + dir);
  for (auto& f : files) {
    const std::string real = fs::is_symlink(f) ? fs::canonical(f).string() : f;
    SafetensorsFile sf(real);
    for (auto& kv : sf.tensors()) put(kv.first, kv.second);
  }
}

}  // namespace

// ============================================================================ target (Qwen3)

namespace {
struct TLayer {
  Lin qkv, o, gu, down;
  float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  float *ss_o = nullptr, *ss_d = nullptr;  // sums of squares of h after the o / down projections
};

// Where the three tap layers' outputs go: fp32 rows (taps + f * stride) and / or
// fragments times a gain (the drafter's feature norms).
struct TapOut {
  float* rows = nullptr;
  size_t stride = 0;
  uint32_t* xf[3] = {nullptr, nullptr, nullptr};
  const float* w[3] = {nullptr, nullptr, nullptr};
};
}  // namespace

struct wc_target {
  wc_ctx* ctx;
  wc_qwen3_config cfg;
  int taps[3];
  int dtype;
  bool finalized = false;
  Stage stage;
  void* embed = nullptr;  // [V][H] in dtype
  Lin head;
  float* final_norm = nullptr;
  std::vector<TLayer> layers;
  RopeTable* rope = nullptr;
  // workspace for up to GEMV_MAXL rows
  float *ws_h = nullptr, *ws_qkv = nullptr;
  uint32_t *xf_in = nullptr, *xf_post = nullptr, *xf_att = nullptr, *xf_act = nullptr, *xf_tmp = nullptr;
  float *ss_pack = nullptr, *ss_tmp = nullptr;
  unsigned long long* ws_keys = nullptr;
  int* ws_tokens = nullptr;
  wc_batch* pf = nullptr;  // tensor-core prompt forward (made at the first prefill)
};

namespace {

bool is_bf16(int dtype) { return dtype == WC_BF16; }

void target_check_cfg(const wc_qwen3_config& c) {
  if (c.hidden <= 0 || c.layers <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.head_dim <= 0 || c.intermediate <= 0 ||
      c.vocab <= 0)
    fail(WC_ERR_INVALID, "target config has non-positive sizes");
  if (c.heads % c.kv_heads) fail(WC_ERR_INVALID, "heads must be a multiple of kv_heads");
  if (c.hidden % 16 || c.head_dim % 32) fail(WC_ERR_UNSUPPORTED, "hidden must be a multiple of 16, head_dim of 32");
}

void target_set_taps(wc_target* t, const int* taps) {
  int tp[3];
  if (taps) {
    for (int i = 0; i < 3; ++i) tp[i] = taps[i];
  } else {  // python default_feature_layers / src/core/qwen3.cpp:57
    tp[0] = 2;
    tp[1] = t->cfg.layers / 2;
    tp[2] = t->cfg.layers - 3;
  }
  for (int i = 0; i < 3; ++i)
    if (tp[i] < 0 || tp[i] >= t->cfg.layers) fail(WC_ERR_INVALID, "tap layer index out of range");
  std::sort(tp, tp + 3);  // taps are emitted in ascending layer order (qwen3.cpp:103-104)
  if (tp[0] == tp[1] || tp[1] == tp[2]) fail(WC_ERR_INVALID, "tap layers must be distinct");
  for (int i = 0; i < 3; ++i) t->taps[i] = tp[i];
}

void target_finalize_impl(wc_target* t) {
  wc_ctx* ctx = t->ctx;
  const auto& c = t->cfg;
  const int H = c.hidden, D = c.head_dim, Hq = c.heads * D, Hkv = c.kv_heads * D, I = c.intermediate;
  const bool bf16 = is_bf16(t->dtype);
  const Stage& s = t->stage;
  t->embed = to_dtype(ctx, s.get("model.embed_tokens.weight", {c.vocab, H}), t->dtype);
  t->final_norm = to_f32_vec(ctx, s.get("model.norm.weight", {H}));
  const bool tied = c.tie_embeddings || !s.has("lm_head.weight");
  if (tied && !bf16) {
    if (H % 4) fail(WC_ERR_UNSUPPORTED, "fp32 hidden size must be a multiple of 4");
    t->head.w = t->embed;
    t->head.owned = false;
    t->head.dtype = WC_F32;
    t->head.N = c.vocab;
    t->head.Np = c.vocab;
    t->head.K = H;
    t->head.Kp = H;
    t->head.group = 1;
    t->head.nseg = 1;
    t->head.seg_len[0] = H;
  } else {
    const Staged& hw = tied ? s.get("model.embed_tokens.weight", {c.vocab, H}) : s.get("lm_head.weight", {c.vocab, H});
    t->head = make_lin(t->dtype, c.vocab, {H}, 1);
    lin_put(ctx, t->head, hw, c.vocab, H, 0, 0, 0);
  }
  t->layers.resize(c.layers);
  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "model.layers." + std::to_string(i) + ".";
    TLayer& L = t->layers[i];
    L.qkv = make_lin(t->dtype, Hq + 2 * Hkv, {H}, 1);
    lin_put(ctx, L.qkv, s.get(p + "self_attn.q_proj.weight", {Hq, H}), Hq, H, 0, 0, 0);
    lin_put(ctx, L.qkv, s.get(p + "self_attn.k_proj.weight", {Hkv, H}), Hkv, H, Hq, 0, 0);
    lin_put(ctx, L.qkv, s.get(p + "self_attn.v_proj.weight", {Hkv, H}), Hkv, H, Hq + Hkv, 0, 0);
    L.o = make_lin(t->dtype, H, {Hq}, 1);
    lin_put(ctx, L.o, s.get(p + "self_attn.o_proj.weight", {H, Hq}), H, Hq, 0, 0, 0);
    L.gu = make_lin(t->dtype, I, {H}, 2);
    lin_put(ctx, L.gu, s.get(p + "mlp.gate_proj.weight", {I, H}), I, H, 0, 0, 0);
    lin_put(ctx, L.gu, s.get(p + "mlp.up_proj.weight", {I, H}), I, H, 0, 0, 1);
    L.down = make_lin(t->dtype, H, {I}, 1);
    lin_put(ctx, L.down, s.get(p + "mlp.down_proj.weight", {H, I}), H, I, 0, 0, 0);
    L.in_norm = to_f32_vec(ctx, s.get(p + "input_layernorm.weight", {H}));
    L.post_norm = to_f32_vec(ctx, s.get(p + "post_attention_layernorm.weight", {H}));
    L.q_norm = to_f32_vec(ctx, s.get(p + "self_attn.q_norm.weight", {D}));
    L.k_norm = to_f32_vec(ctx, s.get(p + "self_attn.k_norm.weight", {D}));
    L.ss_o = ss_alloc(ctx);
    L.ss_d = ss_alloc(ctx);
  }
  t->rope = &rope_table(ctx, D, c.rope_theta, 32768);
  const int M = GEMV_MAXL;
  t->ws_h = static_cast<float*>(dalloc(sizeof(float) * M * H));
  t->ws_qkv = static_cast<float*>(dalloc(sizeof(float) * M * (Hq + 2 * Hkv)));
  t->xf_in = xf_alloc(bf16, H);
  t->xf_post = xf_alloc(bf16, H);
  t->xf_att = xf_alloc(bf16, Hq);
  t->xf_act = xf_alloc(bf16, I);
  t->xf_tmp = xf_alloc(bf16, H);
  t->ss_pack = ss_alloc(ctx);
  t->ss_tmp = ss_alloc(ctx);
  t->ws_keys = static_cast<unsigned long long*>(dalloc(sizeof(unsigned long long) * M));
  t->ws_tokens = static_cast<int*>(dalloc(sizeof(int) * 4096));
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  t->stage.clear();
  t->finalized = true;
}

// Embedding rows -> the residual stream h (fp32) and the first layer's input fragments
// (times its input norm gain) with their sums of squares. Tokens from `tokens`, or the
// verify input [x_n, d_1..d_K] of the round state `st`.
XIn target_embed(wc_target* t, const Rows& r, const int* tokens, RoundState* st, const int* vocab_map, float* h,
                 int* err) {
  PackParams p = pack_params();
  p.table = t->embed;
  p.table_dtype = t->dtype == WC_BF16 ? 1 : 0;
  p.tokens = tokens;
  p.st = st;
  p.vocab_map = vocab_map;
  p.vocab = t->cfg.vocab;
  p.K = t->cfg.hidden;
  p.L = r.L;
  p.L_dev = r.L_dev;
  p.w = t->layers[0].in_norm;
  p.xf = t->xf_in;
  p.ss = t->ss_pack;
  p.copy = h;
  p.err = err;
  launch_pack(t->ctx, p, is_bf16(t->dtype), r.L_max);
  return XIn{t->xf_in, t->ss_pack, 1};
}

// The layer stack on the residual stream h[L][H] in place (rows and prefix from `r`),
// starting from `in0` (layer 0's input fragments). Returns the head input: fragments of
// h times the final norm gain with the last layer's sums of squares.
XIn target_layers(wc_target* t, wc_kv* kv, const Rows& r, XIn in0, float* h, const TapOut* taps, int* err) {
  wc_ctx* ctx = t->ctx;
  const auto& c = t->cfg;
  const int H = c.hidden, D = c.head_dim, Hq = c.heads * D, Hkv = c.kv_heads * D, I = c.intermediate;
  const int ld_qkv = Hq + 2 * Hkv;
  const bool bf16 = is_bf16(t->dtype);
  XIn x = in0;
  for (int li = 0; li < c.layers; ++li) {
    const TLayer& Ly = t->layers[li];
    {
      GemvParams p = gemv_params();
      p.L = r.L;
      p.L_dev = r.L_dev;
      p.L_max = r.L_max;
      p.nseg = 1;
      p.seg[0] = xs_frag(x, H, bf16, c.eps);
      p.epi = EPI_STORE;
      p.y = t->ws_qkv;
      p.ldy = ld_qkv;
      p.err = err;
      gemv_prefetch(ctx, p, &Ly.o, &Ly.gu);  // both land while attention runs
      prof_begin(ctx, PK_QKV);
      launch_gemv(ctx, Ly.qkv, p);
      prof_end(ctx, PK_QKV);
    }
    {
      AttnParams a = attn_params();
      a.qkv = t->ws_qkv;
      a.ld_qkv = ld_qkv;
      a.q_norm = Ly.q_norm;
      a.k_norm = Ly.k_norm;
      a.eps = c.eps;
      a.rope = t->rope->ptr;
      a.max_pos = t->rope->max_pos;
      a.positions = r.positions;
      a.n_dev = r.n_dev;
      a.n_add = r.n_add;
      a.L = r.L;
      a.L_dev = r.L_dev;
      a.L_max = r.L_max;
      a.Kc = kv->Kl(li);
      a.Vc = kv->Vl(li);
      a.kv_dtype = kv->dtype;
      a.stride_h = (long long)kv->cap * D;
      a.stride_p = D;
      a.cap = kv->cap;
      a.H = c.heads;
      a.Hk = c.kv_heads;
      a.D = D;
      a.newmask = r.newmask;
      a.mask_full = r.mask_full;
      a.mask_ld = r.mask_ld;
      a.scale = 1.f / std::sqrt(float(D));
      a.xf_out = t->xf_att;
      a.xf_fp32 = bf16 ? 0 : 1;
      a.write_cache = 1;
      a.stable_prefix = r.stable ? 1 : 0;
      a.err = err;
      prof_begin(ctx, PK_ATTN);
      launch_attention(ctx, a);
      prof_end(ctx, PK_ATTN);
    }
    {
      GemvParams p = gemv_params();
      p.L = r.L;
      p.L_dev = r.L_dev;
      p.L_max = r.L_max;
      p.nseg = 1;
      p.seg[0] = xs_frag(XIn{t->xf_att, nullptr, 0}, Hq, bf16);
      p.epi = EPI_ADD;
      p.y = h;
      p.ldy = H;
      p.base = h;
      p.ldb = H;
      p.nout = 1;
      p.out[0] = XOut{t->xf_post, Ly.post_norm};
      p.ss_out = Ly.ss_o;
      p.err = err;
      prof_begin(ctx, PK_O);
      launch_gemv(ctx, Ly.o, p);
      prof_end(ctx, PK_O);
    }
    {
      GemvParams p = gemv_params();
      p.L = r.L;
      p.L_dev = r.L_dev;
      p.L_max = r.L_max;
      p.nseg = 1;
      p.seg[0] = xs_frag(XIn{t->xf_post, Ly.ss_o, gemv_parts(ctx, Ly.o, r.L_max)}, H, bf16, c.eps);
      p.epi = EPI_SWIGLU;
      p.nout = 1;
      p.out[0] = XOut{t->xf_act, nullptr};
      p.err = err;
      gemv_prefetch(ctx, p, &Ly.down);
      prof_begin(ctx, PK_GU);
      launch_gemv(ctx, Ly.gu, p);
      prof_end(ctx, PK_GU);
    }
    {
      GemvParams p = gemv_params();
      p.L = r.L;
      p.L_dev = r.L_dev;
      p.L_max = r.L_max;
      p.nseg = 1;
      p.seg[0] = xs_frag(XIn{t->xf_act, nullptr, 0}, I, bf16);
      p.epi = EPI_ADD;
      p.y = h;
      p.ldy = H;
      p.base = h;
      p.ldb = H;
      p.nout = 1;
      p.out[0] = XOut{t->xf_in, li + 1 < c.layers ? t->layers[li + 1].in_norm : t->final_norm};
      p.ss_out = Ly.ss_d;
      for (int f = 0; f < 3; ++f)
        if (taps && t->taps[f] == li) {
          if (taps->rows) {
            p.y2 = taps->rows + size_t(f) * taps->stride;
            p.ldy2 = H;
          }
          if (taps->xf[f]) p.out[p.nout++] = XOut{taps->xf[f], taps->w[f]};
        }
      p.err = err;
      gemv_prefetch(ctx, p, li + 1 < c.layers ? &t->layers[li + 1].qkv : &t->head);
      prof_begin(ctx, PK_DOWN);
      launch_gemv(ctx, Ly.down, p);
      prof_end(ctx, PK_DOWN);
    }
    x = XIn{t->xf_in, Ly.ss_d, gemv_parts(ctx, Ly.down, r.L_max)};
  }
  return x;
}

// Sums of squares of a tap layer's output, as the fuse reads them.
XIn target_tap_stats(const wc_target* t, int f, const uint32_t* xf, int L_max) {
  const TLayer& Ly = t->layers[t->taps[f]];
  return XIn{xf, Ly.ss_d, gemv_parts(t->ctx, Ly.down, L_max)};
}

// Head over `rows` rows given as fragments (times the final norm): argmax keys and,
// optionally, logits [rows][V].
void target_head(wc_target* t, XIn x, int rows, const int* L_dev, int L_max, unsigned long long* keys, float* logits,
                 int* err, const Pick* pick = nullptr) {
  GemvParams p = gemv_params();
  p.L = rows;
  p.L_dev = L_dev;
  p.L_max = L_max;
  p.nseg = 1;
  p.seg[0] = xs_frag(x, t->cfg.hidden, is_bf16(t->dtype), t->cfg.eps);
  p.epi = EPI_ARGMAX;
  p.y = logits;
  p.ldy = t->cfg.vocab;
  p.keys = keys;
  p.err = err;
  apply_pick(p, pick);
  prof_begin(t->ctx, PK_HEAD);
  launch_gemv(t->ctx, t->head, p);
  prof_end(t->ctx, PK_HEAD);
}

// Head over fp32 residual rows h[rows][H] (any row offset): re-packs them first.
void target_head_rows(wc_target* t, const float* h, int rows, unsigned long long* keys, float* logits, int* err,
                      const Pick* pick = nullptr) {
  PackParams p = pack_params();
  p.src = h;
  p.ld = t->cfg.hidden;
  p.K = t->cfg.hidden;
  p.L = rows;
  p.w = t->final_norm;
  p.xf = t->xf_tmp;
  p.ss = t->ss_tmp;
  p.err = err;
  launch_pack(t->ctx, p, is_bf16(t->dtype), rows);
  target_head(t, XIn{t->xf_tmp, t->ss_tmp, 1}, rows, nullptr, rows, keys, logits, err, pick);
}

}  // namespace

extern "C" wc_status wc_target_create(wc_ctx* ctx, const wc_qwen3_config* cfg, const int* taps, int dtype,
                                      wc_target** out) {
  if (!ctx || !cfg || !out) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    if (dtype != WC_F32 && dtype != WC_BF16) fail(WC_ERR_INVALID, "dtype must be WC_F32 or WC_BF16");
    target_check_cfg(*cfg);
    auto t = std::make_unique<wc_target>();
    t->ctx = ctx;
    t->cfg = *cfg;
    t->dtype = dtype;
    target_set_taps(t.get(), taps);
    *out = t.release();
  });
}

extern "C" wc_status wc_target_set_tensor(wc_target* t, const char* name, const void* data, int src_dtype,
                                          int on_device, const int64_t* shape, int ndim) {
  if (!t || !name) return WC_ERR_INVALID;
  return guard(t->ctx, [&] {
    if (t->finalized) fail(WC_ERR_INVALID, "target already finalized");
    stage_put(t->ctx, t->stage, name, data, src_dtype, on_device, shape, ndim);
  });
}

extern "C" wc_status wc_target_finalize(wc_target* t) {
  if (!t) return WC_ERR_INVALID;
  return guard(t->ctx, [&] {
    if (t->finalized) fail(WC_ERR_INVALID, "target already finalized");
    target_finalize_impl(t);
  });
}

namespace {
wc_qwen3_config qwen3_config_from_json(const std::string& path) {
  const JsonValue j = json_parse(read_file(path));
  wc_qwen3_config c{};
  c.hidden = int(j.at("hidden_size").num);
  c.layers = int(j.at("num_hidden_layers").num);
  c.heads = int(j.at("num_attention_heads").num);
  c.kv_heads = int(j.at("num_key_value_heads").num);
  c.head_dim = int(j.number_or("head_dim", double(c.hidden / std::max(1, c.heads))));
  c.intermediate = int(j.at("intermediate_size").num);
  c.vocab = int(j.at("vocab_size").num);
  c.eps = float(j.number_or("rms_norm_eps", 1e-6));
  c.rope_theta = float(j.number_or("rope_theta", 1e6));
  c.tie_embeddings = j.bool_or("tie_word_embeddings", false) ? 1 : 0;
  return c;
}
}  // namespace

extern "C" wc_status wc_target_load(wc_ctx* ctx, const char* dir, const int* taps, int dtype, wc_target** out) {
  if (!ctx || !dir || !out) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    const wc_qwen3_config cfg = qwen3_config_from_json((fs::path(dir) / "config.json").string());
    if (dtype != WC_F32 && dtype != WC_BF16) fail(WC_ERR_INVALID, "dtype must be WC_F32 or WC_BF16");
    target_check_cfg(cfg);
    auto t = std::make_unique<wc_target>();
    t->ctx = ctx;
    t->cfg = cfg;
    t->dtype = dtype;
    target_set_taps(t.get(), taps);
    load_dir_tensors(dir, "", [&](const std::string& name, const TensorView& v) {
      const int dt = src_dtype_code(v.dtype);
      if (dt < 0) fail(WC_ERR_IO, "unsupported dtype " + v.dtype + " for " + name);
      stage_put(ctx, t->stage, name, v.data, dt, 0, v.shape.data(), int(v.shape.size()));
    });
    target_finalize_impl(t.get());
    *out = t.release();
  });
}

extern "C" void wc_target_destroy(wc_target* t) {
  if (!t) return;
  cudaStreamSynchronize(t->ctx->stream);
  if (t->pf) wc_batch_destroy(t->pf);
  dfree(t->embed);
  free_lin(t->head);
  dfree(t->final_norm);
  for (auto& L : t->layers) {
    free_lin(L.qkv);
    free_lin(L.o);
    free_lin(L.gu);
    free_lin(L.down);
    dfree(L.in_norm);
    dfree(L.post_norm);
    dfree(L.q_norm);
    dfree(L.k_norm);
    dfree(L.ss_o);
    dfree(L.ss_d);
  }
  for (void* p : {(void*)t->ws_h, (void*)t->ws_qkv, (void*)t->xf_in, (void*)t->xf_post, (void*)t->xf_att,
                  (void*)t->xf_act, (void*)t->xf_tmp, (void*)t->ss_pack, (void*)t->ss_tmp, (void*)t->ws_keys,
                  (void*)t->ws_tokens})
    dfree(p);
  delete t;
}

extern "C" wc_status wc_target_config(const wc_target* t, wc_qwen3_config* cfg, int* taps3, int* dtype) {
  if (!t) return WC_ERR_INVALID;
  if (cfg) *cfg = t->cfg;
  if (taps3)
    for (int i = 0; i < 3; ++i) taps3[i] = t->taps[i];
  if (dtype) *dtype = t->dtype;
  return WC_OK;
}

extern "C" wc_status wc_target_make_cache(wc_target* t, int capacity, wc_kv** kv) {
  if (!t || !kv) return WC_ERR_INVALID;
  return guard(t->ctx, [&] {
    *kv = kv_new(t->ctx, t->cfg.layers, t->cfg.kv_heads, t->cfg.head_dim, capacity, t->dtype);
  });
}

extern "C" wc_status wc_target_forward(wc_target* t, wc_kv* cache, const int* tokens, int L, const int* positions,
                                       const uint8_t* mask, int logits_from, float* logits, int* argmax,
                                       float* taps) {
  if (!t || !cache || !tokens || L <= 0) return WC_ERR_INVALID;
  return guard(t->ctx, [&] {
    if (!t->finalized) fail(WC_ERR_INVALID, "target not finalized");
    const auto& c = t->cfg;
    if (cache->layers != c.layers || cache->Hk != c.kv_heads || cache->D != c.head_dim || cache->dtype != t->dtype)
      fail(WC_ERR_INVALID, "cache does not match the target");
    if (logits_from < 0 || logits_from > L) fail(WC_ERR_INVALID, "logits_from out of range");
    const int prefix = cache->n;
    if (prefix + L > cache->cap) fail(WC_ERR_CAPACITY, "KV cache capacity exceeded");
    wc_ctx* ctx = t->ctx;
    const int H = c.hidden;
    TapOut to;
    to.rows = taps;
    to.stride = size_t(L) * H;
    for (int r0 = 0; r0 < L; r0 += GEMV_MAXL) {
      const int rows = std::min(GEMV_MAXL, L - r0);
      Rows r;
      r.L = rows;
      r.L_max = rows;
      r.n_add = prefix + r0;
      r.positions = positions ? positions + r0 : nullptr;
      r.mask_full = mask ? mask + size_t(r0) * (prefix + L) : nullptr;
      r.mask_ld = prefix + L;
      const XIn in0 = target_embed(t, r, tokens + r0, nullptr, nullptr, t->ws_h, ctx->d_err);
      TapOut tc = to;
      if (taps) tc.rows = taps + size_t(r0) * H;
      const XIn hx = target_layers(t, cache, r, in0, t->ws_h, taps ? &tc : nullptr, ctx->d_err);
      const int h0 = std::max(logits_from, r0);
      if (h0 < r0 + rows && (logits || argmax)) {
        const int hr = r0 + rows - h0;
        float* lg = logits ? logits + size_t(h0 - logits_from) * c.vocab : nullptr;
        CUDA_TRY(cudaMemsetAsync(t->ws_keys, 0, sizeof(unsigned long long) * GEMV_MAXL, ctx->stream));
        if (h0 == r0) target_head(t, hx, hr, nullptr, hr, t->ws_keys, lg, ctx->d_err);
        else target_head_rows(t, t->ws_h + size_t(h0 - r0) * H, hr, t->ws_keys, lg, ctx->d_err);
        if (argmax) {
          keys_to_index_kernel<<<1, 32, 0, ctx->stream>>>(t->ws_keys, hr, nullptr, argmax + (h0 - logits_from));
          check_launch(ctx, "keys");
        }
      }
    }
    cache->n = prefix + L;
  });
}

// ============================================================================ drafter (EAGLE-3)

namespace {
struct DLayer {
  Lin qkv, o, gu, down;
  Lin qkv_main;  // layer 0 with the auxiliary table: the Q/K/V weights of the feature input alone
  float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *aux_norm = nullptr;
  float *ss_o = nullptr, *ss_d = nullptr;
};
}  // namespace

struct DrafterGemm;

struct wc_drafter {
  wc_ctx* ctx;
  wc_drafter_config cfg;
  int dtype;
  bool finalized = false;
  Stage stage;
  void* embed = nullptr;
  float* aux_inv = nullptr;  // [vocab]: 1/rms of each embedding row with the drafter eps (aux_norm)
  float* aux_table = nullptr;  // [vocab][Q+K+V]: W_aux . aux_norm(embed(t)) per token (bf16 drafters)
  Lin fc;
  float* feature_norms[GEMV_MAXSEG] = {nullptr, nullptr, nullptr};
  std::vector<DLayer> layers;
  float* norm = nullptr;
  Lin head;
  int* vocab_map = nullptr;  // restricted head row -> token id
  int* vocab_inv = nullptr;  // token id -> restricted head row or -1 (sampled decoding)
  int head_rows = 0;
  RopeTable* rope = nullptr;
  // workspace for up to GEMV_MAXL rows
  float *ws_h = nullptr, *ws_feat = nullptr, *ws_g = nullptr, *ws_qkv = nullptr;
  uint32_t *xf_feat = nullptr, *xf_post = nullptr, *xf_att = nullptr, *xf_act = nullptr, *xf_out = nullptr;
  uint32_t* xf_tap[3] = {nullptr, nullptr, nullptr};
  float *ss_feat = nullptr, *ss_g = nullptr, *ss_pack = nullptr;
  float* ss_tap[3] = {nullptr, nullptr, nullptr};
  unsigned long long* ws_keys = nullptr;
  DrafterGemm* pg = nullptr;  // tensor-core prompt pass (row-major weight copies), made on first use
};

namespace {
void drafter_build_aux_table(wc_drafter* d);

void drafter_check_cfg(const wc_drafter_config& c) {
  if (c.hidden <= 0 || c.layers <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.head_dim <= 0 || c.intermediate <= 0 ||
      c.vocab <= 0 || c.target_hidden <= 0)
    fail(WC_ERR_INVALID, "drafter config has non-positive sizes");
  if (c.num_features < 1 || c.num_features > GEMV_MAXSEG)
    fail(WC_ERR_UNSUPPORTED, "drafter num_features must be 1..3");
  if (c.heads % c.kv_heads) fail(WC_ERR_INVALID, "heads must be a multiple of kv_heads");
  if (c.hidden % 16 || c.head_dim % 32) fail(WC_ERR_UNSUPPORTED, "hidden must be a multiple of 16, head_dim of 32");
}

void drafter_finalize_impl(wc_drafter* d) {
  wc_ctx* ctx = d->ctx;
  const auto& c = d->cfg;
  const int H = c.hidden, D = c.head_dim, Hq = c.heads * D, Hkv = c.kv_heads * D, I = c.intermediate;
  const bool bf16 = is_bf16(d->dtype);
  const Stage& s = d->stage;
  d->embed = to_dtype(ctx, s.get("embed_tokens.weight", {c.vocab, H}), d->dtype);
  const int F = c.num_features, Ht = c.target_hidden;
  if (F == 1) d->fc = make_lin(d->dtype, H, {Ht}, 1);
  else if (F == 2) d->fc = make_lin(d->dtype, H, {Ht, Ht}, 1);
  else d->fc = make_lin(d->dtype, H, {Ht, Ht, Ht}, 1);
  {
    // fc.weight [H][F*Ht]: split into one part per tap column block
    const Staged& fw = s.get("fc.weight", {H, F * Ht});
    for (int f = 0; f < F; ++f) {
      Staged part;
      part.dtype = fw.dtype;
      part.shape = {H, Ht};
      const size_t es = size_t(dtype_size(fw.dtype));
      part.ptr = dalloc(size_t(H) * Ht * es);
      CUDA_TRY(cudaMemcpy2DAsync(part.ptr, Ht * es, static_cast<const char*>(fw.ptr) + f * Ht * es, size_t(F) * Ht * es,
                                 Ht * es, H, cudaMemcpyDeviceToDevice, ctx->stream));
      lin_put(ctx, d->fc, part, H, Ht, 0, f, 0);
      CUDA_TRY(cudaStreamSynchronize(ctx->stream));
      dfree(part.ptr);
    }
  }
  if (c.feature_norm)
    for (int f = 0; f < F; ++f)
      d->feature_norms[f] = to_f32_vec(ctx, s.get("feature_norms." + std::to_string(f) + ".weight", {Ht}));
  d->layers.resize(c.layers);
  for (int i = 0; i < c.layers; ++i) {
    const std::string p = "layers." + std::to_string(i) + ".";
    DLayer& L = d->layers[i];
    const bool aux = i == 0;  // layer 0 is dual-stream (drafter.cpp:64-70)
    L.qkv = aux ? make_lin(d->dtype, Hq + 2 * Hkv, {H, H}, 1) : make_lin(d->dtype, Hq + 2 * Hkv, {H}, 1);
    lin_put(ctx, L.qkv, s.get(p + "self_attn.q_proj.weight", {Hq, H}), Hq, H, 0, 0, 0);
    lin_put(ctx, L.qkv, s.get(p + "self_attn.k_proj.weight", {Hkv, H}), Hkv, H, Hq, 0, 0);
    lin_put(ctx, L.qkv, s.get(p + "self_attn.v_proj.weight", {Hkv, H}), Hkv, H, Hq + Hkv, 0, 0);
    if (aux) {
      lin_put(ctx, L.qkv, s.get(p + "self_attn.aux_q.weight", {Hq, H}), Hq, H, 0, 1, 0);
      lin_put(ctx, L.qkv, s.get(p + "self_attn.aux_k.weight", {Hkv, H}), Hkv, H, Hq, 1, 0);
      lin_put(ctx, L.qkv, s.get(p + "self_attn.aux_v.weight", {Hkv, H}), Hkv, H, Hq + Hkv, 1, 0);
      L.aux_norm = to_f32_vec(ctx, s.get(p + "aux_norm.weight", {H}));
    }
    L.o = make_lin(d->dtype, H, {Hq}, 1);
    lin_put(ctx, L.o, s.get(p + "self_attn.o_proj.weight", {H, Hq}), H, Hq, 0, 0, 0);
    L.gu = make_lin(d->dtype, I, {H}, 2);
    lin_put(ctx, L.gu, s.get(p + "mlp.gate_proj.weight", {I, H}), I, H, 0, 0, 0);
    lin_put(ctx, L.gu, s.get(p + "mlp.up_proj.weight", {I, H}), I, H, 0, 0, 1);
    L.down = make_lin(d->dtype, H, {I}, 1);
    lin_put(ctx, L.down, s.get(p + "mlp.down_proj.weight", {H, I}), H, I, 0, 0, 0);
    L.in_norm = to_f32_vec(ctx, s.get(p + "input_layernorm.weight", {H}));
    L.post_norm = to_f32_vec(ctx, s.get(p + "post_attention_layernorm.weight", {H}));
    L.q_norm = to_f32_vec(ctx, s.get(p + "self_attn.q_norm.weight", {D}));
    L.k_norm = to_f32_vec(ctx, s.get(p + "self_attn.k_norm.weight", {D}));
    L.ss_o = ss_alloc(ctx);
    L.ss_d = ss_alloc(ctx);
  }
  d->aux_inv = static_cast<float*>(dalloc(sizeof(float) * c.vocab));
  row_inv_kernel<<<(c.vocab + 7) / 8, 256, 0, ctx->stream>>>(d->embed, d->dtype == WC_BF16 ? 1 : 0, c.vocab, H, c.eps,
                                                             d->aux_inv);
  check_launch(ctx, "row_inv");
  d->norm = to_f32_vec(ctx, s.get("norm.weight", {H}));
  d->head = make_lin(d->dtype, c.vocab, {H}, 1);
  lin_put(ctx, d->head, s.get("lm_head.weight", {c.vocab, H}), c.vocab, H, 0, 0, 0);
  d->head_rows = c.vocab;
  d->rope = &rope_table(ctx, D, c.rope_theta, 32768);
  const int M = GEMV_MAXL;
  d->ws_h = static_cast<float*>(dalloc(sizeof(float) * M * H));
  d->ws_feat = static_cast<float*>(dalloc(sizeof(float) * M * H));
  d->ws_g = static_cast<float*>(dalloc(sizeof(float) * M * H));
  d->ws_qkv = static_cast<float*>(dalloc(sizeof(float) * M * (Hq + 2 * Hkv)));
  d->xf_feat = xf_alloc(bf16, H);
  d->xf_post = xf_alloc(bf16, H);
  d->xf_att = xf_alloc(bf16, Hq);
  d->xf_act = xf_alloc(bf16, I);
  d->xf_out = xf_alloc(bf16, H);
  for (int f = 0; f < 3; ++f) {
    d->xf_tap[f] = xf_alloc(bf16, Ht);
    d->ss_tap[f] = ss_alloc(ctx);
  }
  d->ss_feat = ss_alloc(ctx);
  d->ss_g = ss_alloc(ctx);
  d->ss_pack = ss_alloc(ctx);
  d->ws_keys = static_cast<unsigned long long*>(dalloc(sizeof(unsigned long long) * M));
  drafter_build_aux_table(d);
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  d->stage.clear();
  d->finalized = true;
}

// Drafter layer stack (drafter.cpp:91-136). `feat` [L][H] is the residual stream input
// (fp32) and `feat_in` its fragments times layer 0's input norm gain; layer 0 adds
// W_aux . aux_norm(embed(token)). The result h lands in h_out [L][H]. `extra` (optional)
// receives fragments of h as well (the next chain step's feature without post-norm).
// Returns the head input: fragments of h times the final norm gain, with h's sums of squares.
XIn drafter_layers(wc_drafter* d, wc_kv* kv, const Rows& r, XIn feat_in, const float* feat, const TokenSrc& tok,
                   float* h_out, const XOut* extra, int* err) {
  wc_ctx* ctx = d->ctx;
  const auto& c = d->cfg;
  const int H = c.hidden, D = c.head_dim, Hq = c.heads * D, Hkv = c.kv_heads * D, I = c.intermediate;
  const int ld_qkv = Hq + 2 * Hkv;
  const bool bf16 = is_bf16(d->dtype);
  XIn x = feat_in;
  for (int li = 0; li < c.layers; ++li) {
    const DLayer& Ly = d->layers[li];
    {
      GemvParams p = gemv_params();
      p.L = r.L;
      p.L_dev = r.L_dev;
      p.L_max = r.L_max;
      p.nseg = 1;
      p.seg[0] = xs_frag(x, H, bf16, c.eps);
      const bool table = Ly.aux_norm && d->aux_table && Ly.qkv_main.w;
      p.epi = EPI_STORE;
      if (table) {  // the token's row of the precomputed auxiliary term, added in the epilogue
        p.epi = EPI_ADD;
        p.base = d->aux_table;
        p.ldb = ld_qkv;
        p.base_tok = 1;
        p.tok = tok;
        p.tok.vocab = c.vocab;
      } else if (Ly.aux_norm) {
        p.nseg = 2;
        p.seg[1] = xs_embed(d->embed, H, bf16, Ly.aux_norm, d->aux_inv);
        p.tok = tok;
        p.tok.vocab = c.vocab;
      }
      p.y = d->ws_qkv;
      p.ldy = ld_qkv;
      p.err = err;
      gemv_prefetch(ctx, p, &Ly.o, &Ly.gu);  // both land while attention runs
      launch_gemv(ctx, table ? Ly.qkv_main : Ly.qkv, p);
    }
    {
      AttnParams a = attn_params();
      a.qkv = d->ws_qkv;
      a.ld_qkv = ld_qkv;
      a.q_norm = Ly.q_norm;
      a.k_norm = Ly.k_norm;
      a.eps = c.eps;
      a.rope = d->rope->ptr;
      a.max_pos = d->rope->max_pos;
      a.positions = r.positions;
      a.n_dev = r.n_dev;
      a.n_add = r.n_add;
      a.L = r.L;
      a.L_dev = r.L_dev;
      a.L_max = r.L_max;
      a.Kc = kv->Kl(li);
      a.Vc = kv->Vl(li);
      a.kv_dtype = kv->dtype;
      a.stride_h = (long long)kv->cap * D;
      a.stride_p = D;
      a.cap = kv->cap;
      a.H = c.heads;
      a.Hk = c.kv_heads;
      a.D = D;
      a.newmask = r.newmask;
      a.mask_from_prefix = r.mask_from_prefix ? 1 : 0;
      a.window = c.window;
      a.mask_full = r.mask_full;
      a.mask_ld = r.mask_ld;
      a.scale = 1.f / std::sqrt(float(D));
      a.xf_out = d->xf_att;
      a.xf_fp32 = bf16 ? 0 : 1;
      a.write_cache = 1;
      a.stable_prefix = r.stable ? 1 : 0;
      a.err = err;
      launch_attention(ctx, a);
    }
    {
      GemvParams p = gemv_params();
      p.L = r.L;
      p.L_dev = r.L_dev;
      p.L_max = r.L_max;
      p.nseg = 1;
      p.seg[0] = xs_frag(XIn{d->xf_att, nullptr, 0}, Hq, bf16);
      p.epi = EPI_ADD;
      p.y = h_out;
      p.ldy = H;
      p.base = li == 0 ? feat : h_out;
      p.ldb = H;
      p.nout = 1;
      p.out[0] = XOut{d->xf_post, Ly.post_norm};
      p.ss_out = Ly.ss_o;
      p.err = err;
      launch_gemv(ctx, Ly.o, p);
    }
    {
      GemvParams p = gemv_params();
      p.L = r.L;
      p.L_dev = r.L_dev;
      p.L_max = r.L_max;
      p.nseg = 1;
      p.seg[0] = xs_frag(XIn{d->xf_post, Ly.ss_o, gemv_parts(ctx, Ly.o, r.L_max)}, H, bf16, c.eps);
      p.epi = EPI_SWIGLU;
      p.nout = 1;
      p.out[0] = XOut{d->xf_act, nullptr};
      p.err = err;
      gemv_prefetch(ctx, p, &Ly.down);
      launch_gemv(ctx, Ly.gu, p);
    }
    {
      const bool last = li + 1 == c.layers;
      GemvParams p = gemv_params();
      p.L = r.L;
      p.L_dev = r.L_dev;
      p.L_max = r.L_max;
      p.nseg = 1;
      p.seg[0] = xs_frag(XIn{d->xf_act, nullptr, 0}, I, bf16);
      p.epi = EPI_ADD;
      p.y = h_out;
      p.ldy = H;
      p.base = h_out;
      p.ldb = H;
      p.nout = 1;
      p.out[0] = XOut{d->xf_out, last ? d->norm : d->layers[li + 1].in_norm};
      if (last && extra) p.out[p.nout++] = *extra;
      p.ss_out = Ly.ss_d;
      p.err = err;
      gemv_prefetch(ctx, p, last ? &d->head : &d->layers[li + 1].qkv);
      launch_gemv(ctx, Ly.down, p);
    }
    x = XIn{d->xf_out, Ly.ss_d, gemv_parts(ctx, Ly.down, r.L_max)};
  }
  return x;
}

// fuse (drafter.cpp:75-89): per-tap RMSNorm (the tap fragments are already times the
// feature norm gains), concatenated, through fc. Writes g [L][H] (fp32, the layer-0
// residual input) and its fragments times layer 0's input norm gain with sums of squares;
// returns them as the layer-0 input.
XIn drafter_fuse_impl(wc_drafter* d, const XIn* taps, int L, const int* L_dev, int L_max, float* g, int* err) {
  const auto& c = d->cfg;
  const bool bf16 = is_bf16(d->dtype);
  GemvParams p = gemv_params();
  p.L = L;
  p.L_dev = L_dev;
  p.L_max = L_max;
  p.nseg = c.num_features;
  for (int f = 0; f < c.num_features; ++f) {
    XIn tf = taps[f];
    if (!c.feature_norm) tf.ss = nullptr;
    p.seg[f] = xs_frag(tf, c.target_hidden, bf16, c.eps);
  }
  p.epi = EPI_STORE;
  p.y = g;
  p.ldy = c.hidden;
  p.nout = 1;
  p.out[0] = XOut{d->xf_feat, d->layers[0].in_norm};
  p.ss_out = d->ss_g;
  p.err = err;
  gemv_prefetch(d->ctx, p, &d->layers[0].qkv);
  launch_gemv(d->ctx, d->fc, p);
  return XIn{d->xf_feat, d->ss_g, gemv_parts(d->ctx, d->fc, L_max)};
}

// Tap rows [L][Ht] (fp32, row stride ld, tap f at + f * stride) -> tap fragments times
// the feature norm gains with their sums of squares.
void drafter_pack_taps(wc_drafter* d, const float* taps, size_t stride, int ld, int L, XIn* out, int* err) {
  for (int f = 0; f < d->cfg.num_features; ++f) {
    PackParams p = pack_params();
    p.src = taps + f * stride;
    p.ld = ld;
    p.K = d->cfg.target_hidden;
    p.L = L;
    p.w = d->cfg.feature_norm ? d->feature_norms[f] : nullptr;
    p.xf = d->xf_tap[f];
    p.ss = d->ss_tap[f];
    p.err = err;
    launch_pack(d->ctx, p, is_bf16(d->dtype), L);
    out[f] = XIn{d->xf_tap[f], d->ss_tap[f], 1};
  }
}

// fp32 rows [L][H] -> fragments times `w` (+ sums of squares) in xf / ss.
XIn drafter_pack_rows(wc_drafter* d, const float* x, int L, const float* w, uint32_t* xf, float* ss, int* err) {
  PackParams p = pack_params();
  p.src = x;
  p.ld = d->cfg.hidden;
  p.K = d->cfg.hidden;
  p.L = L;
  p.w = w;
  p.xf = xf;
  p.ss = ss;
  p.err = err;
  launch_pack(d->ctx, p, is_bf16(d->dtype), L);
  return XIn{xf, ss, 1};
}

// Head over `rows` rows of fragments `x` (seg 0; normalised by x.ss when set); the side
// job (when side_y is set) writes the next chain feature RMSNorm(h) * norm as fp32 rows and
// as fragments times layer 0's input gain, with sums of squares in ss_feat.
void drafter_head(wc_drafter* d, XIn x, int rows, unsigned long long* keys, float* logits, const float* side_src,
                  float* side_y, int* err, const Pick* pick = nullptr) {
  const bool bf16 = is_bf16(d->dtype);
  GemvParams p = gemv_params();
  p.L = rows;
  p.L_max = rows;
  p.nseg = 1;
  p.seg[0] = xs_frag(x, d->cfg.hidden, bf16, d->cfg.eps);
  p.epi = EPI_ARGMAX;
  p.y = logits;
  p.ldy = d->head_rows;
  p.keys = keys;
  if (side_y) {
    p.side_src = side_src;
    p.side_len = d->cfg.hidden;
    p.side_w = d->norm;
    p.side_y = side_y;
    p.side_out = XOut{d->xf_feat, d->layers[0].in_norm};
    p.side_ss = d->ss_feat;
  }
  p.err = err;
  apply_pick(p, pick);
  gemv_prefetch(d->ctx, p, &d->layers[0].qkv);
  prof_begin(d->ctx, PK_DRAFT_HEAD);
  launch_gemv(d->ctx, d->head, p);
  prof_end(d->ctx, PK_DRAFT_HEAD);
}

wc_drafter_config drafter_config_from_json(const std::string& path) {
  const JsonValue j = json_parse(read_file(path));
  wc_drafter_config c{};
  c.hidden = int(j.at("hidden_size").num);
  c.layers = int(j.at("num_layers").num);
  c.heads = int(j.at("num_heads").num);
  c.kv_heads = int(j.at("num_kv_heads").num);
  c.head_dim = int(j.at("head_dim").num);
  c.intermediate = int(j.at("intermediate_size").num);
  c.vocab = int(j.at("vocab_size").num);
  c.target_hidden = int(j.at("target_hidden_size").num);
  c.num_features = int(j.number_or("num_features", 3));
  c.eps = float(j.number_or("rms_norm_eps", 1e-6));
  c.rope_theta = float(j.number_or("rope_theta", 1e6));
  // drafter.cpp:36, 41 and drafter.py:55-63 reject these configurations
  if (j.str_or("residual", "feature") != "feature")
    fail(WC_ERR_UNSUPPORTED, "unsupported drafter mode in " + path);
  if (j.number_or("lowrank_rank", 0) != 0) fail(WC_ERR_UNSUPPORTED, "unsupported drafter configuration in " + path);
  c.post_norm = j.bool_or("post_norm", true) ? 1 : 0;
  c.feature_norm = j.bool_or("feature_norm", true) ? 1 : 0;
  c.window = int(j.number_or("window", 0));
  return c;
}

}  // namespace

extern "C" wc_status wc_drafter_create(wc_ctx* ctx, const wc_drafter_config* cfg, int dtype, wc_drafter** out) {
  if (!ctx || !cfg || !out) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    if (dtype != WC_F32 && dtype != WC_BF16) fail(WC_ERR_INVALID, "dtype must be WC_F32 or WC_BF16");
    drafter_check_cfg(*cfg);
    auto d = std::make_unique<wc_drafter>();
    d->ctx = ctx;
    d->cfg = *cfg;
    d->dtype = dtype;
    *out = d.release();
  });
}

extern "C" wc_status wc_drafter_set_tensor(wc_drafter* d, const char* name, const void* data, int src_dtype,
                                           int on_device, const int64_t* shape, int ndim) {
  if (!d || !name) return WC_ERR_INVALID;
  return guard(d->ctx, [&] {
    if (d->finalized) fail(WC_ERR_INVALID, "drafter already finalized");
    stage_put(d->ctx, d->stage, name, data, src_dtype, on_device, shape, ndim);
  });
}

extern "C" wc_status wc_drafter_finalize(wc_drafter* d) {
  if (!d) return WC_ERR_INVALID;
  return guard(d->ctx, [&] {
    if (d->finalized) fail(WC_ERR_INVALID, "drafter already finalized");
    drafter_finalize_impl(d);
  });
}

extern "C" wc_status wc_drafter_load(wc_ctx* ctx, const char* dir, int dtype, wc_drafter** out) {
  if (!ctx || !dir || !out) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    const wc_drafter_config cfg = drafter_config_from_json((fs::path(dir) / "config.json").string());
    if (dtype != WC_F32 && dtype != WC_BF16) fail(WC_ERR_INVALID, "dtype must be WC_F32 or WC_BF16");
    drafter_check_cfg(cfg);
    auto d = std::make_unique<wc_drafter>();
    d->ctx = ctx;
    d->cfg = cfg;
    d->dtype = dtype;
    load_dir_tensors(dir, "model.safetensors", [&](const std::string& name, const TensorView& v) {
      const int dt = src_dtype_code(v.dtype);
      if (dt < 0) fail(WC_ERR_IO, "unsupported dtype " + v.dtype + " for " + name);
      stage_put(ctx, d->stage, name, v.data, dt, 0, v.shape.data(), int(v.shape.size()));
    });
    drafter_finalize_impl(d.get());
    *out = d.release();
  });
}

namespace {
void drafter_gemm_free(wc_drafter* d);
}  // namespace

extern "C" void wc_drafter_destroy(wc_drafter* d) {
  if (!d) return;
  cudaStreamSynchronize(d->ctx->stream);
  drafter_gemm_free(d);
  dfree(d->aux_table);
  dfree(d->embed);
  dfree(d->aux_inv);
  free_lin(d->fc);
  for (auto* f : d->feature_norms) dfree(f);
  for (auto& L : d->layers) {
    free_lin(L.qkv);
    free_lin(L.qkv_main);
    free_lin(L.o);
    free_lin(L.gu);
    free_lin(L.down);
    dfree(L.in_norm);
    dfree(L.post_norm);
    dfree(L.q_norm);
    dfree(L.k_norm);
    dfree(L.aux_norm);
    dfree(L.ss_o);
    dfree(L.ss_d);
  }
  dfree(d->norm);
  free_lin(d->head);
  dfree(d->vocab_map);
  dfree(d->vocab_inv);
  for (void* p : {(void*)d->ws_h, (void*)d->ws_feat, (void*)d->ws_g, (void*)d->ws_qkv, (void*)d->xf_feat,
                  (void*)d->xf_post, (void*)d->xf_att, (void*)d->xf_act, (void*)d->xf_out, (void*)d->ss_feat,
                  (void*)d->ss_g, (void*)d->ss_pack, (void*)d->ws_keys})
    dfree(p);
  for (int f = 0; f < 3; ++f) {
    dfree(d->xf_tap[f]);
    dfree(d->ss_tap[f]);
  }
  delete d;
}

extern "C" wc_status wc_drafter_config_get(const wc_drafter* d, wc_drafter_config* cfg, int* dtype, int* head_rows) {
  if (!d) return WC_ERR_INVALID;
  if (cfg) *cfg = d->cfg;
  if (dtype) *dtype = d->dtype;
  if (head_rows) *head_rows = d->head_rows;
  return WC_OK;
}

extern "C" wc_status wc_drafter_restrict_vocab(wc_drafter* d, const int* ids, int n) {
  if (!d || !ids || n <= 0) return WC_ERR_INVALID;
  return guard(d->ctx, [&] {
    if (!d->finalized) fail(WC_ERR_INVALID, "drafter not finalized");
    if (d->vocab_map) fail(WC_ERR_INVALID, "drafter vocabulary is already restricted");
    for (int i = 0; i < n; ++i)
      if (ids[i] < 0 || ids[i] >= d->cfg.vocab) fail(WC_ERR_INVALID, "vocabulary id out of range");
    wc_ctx* ctx = d->ctx;
    int* map = static_cast<int*>(dalloc(sizeof(int) * n));
    CUDA_TRY(cudaMemcpy(map, ids, sizeof(int) * n, cudaMemcpyHostToDevice));
    // token -> row (the scatter of spec.py:239-249; a repeated id keeps its last row)
    std::vector<int> inv(size_t(d->cfg.vocab), -1);
    for (int i = 0; i < n; ++i) inv[size_t(ids[i])] = i;
    int* dinv = static_cast<int*>(dalloc(sizeof(int) * inv.size()));
    CUDA_TRY(cudaMemcpy(dinv, inv.data(), sizeof(int) * inv.size(), cudaMemcpyHostToDevice));
    Lin nh = make_lin(d->dtype, n, {d->cfg.hidden}, 1);
    if (d->dtype == WC_BF16) {
      const int KT = nh.Kp / 16;
      gather_tiled_rows_kernel<<<grid_for(size_t(nh.Np) * nh.Kp), 256, 0, ctx->stream>>>(
          static_cast<const uint16_t*>(d->head.w), KT, map, n, static_cast<uint16_t*>(nh.w));
    } else {
      gather_rows_f32_kernel<<<grid_for(size_t(n) * nh.Kp), 256, 0, ctx->stream>>>(
          static_cast<const float*>(d->head.w), nh.Kp, map, n, static_cast<float*>(nh.w));
    }
    check_launch(ctx, "restrict_vocab");
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    free_lin(d->head);  // the full head is dropped, as in drafter.py:217-229
    d->head = nh;
    d->vocab_map = map;
    d->vocab_inv = dinv;
    d->head_rows = n;
  });
}

extern "C" wc_status wc_drafter_make_cache(wc_drafter* d, int capacity, wc_kv** kv) {
  if (!d || !kv) return WC_ERR_INVALID;
  return guard(d->ctx, [&] {
    *kv = kv_new(d->ctx, d->cfg.layers, d->cfg.kv_heads, d->cfg.head_dim, capacity, d->dtype);
  });
}

extern "C" wc_status wc_drafter_fuse(wc_drafter* d, const float* taps, int L, float* g) {
  if (!d || !taps || !g || L <= 0) return WC_ERR_INVALID;
  return guard(d->ctx, [&] {
    const int Ht = d->cfg.target_hidden;
    const size_t stride = size_t(L) * Ht;
    for (int r0 = 0; r0 < L; r0 += GEMV_MAXL) {
      const int rows = std::min(GEMV_MAXL, L - r0);
      XIn tx[3];
      drafter_pack_taps(d, taps + size_t(r0) * Ht, stride, Ht, rows, tx, d->ctx->d_err);
      drafter_fuse_impl(d, tx, rows, nullptr, rows, g + size_t(r0) * d->cfg.hidden, d->ctx->d_err);
    }
  });
}

extern "C" wc_status wc_drafter_forward(wc_drafter* d, wc_kv* cache, const int* tokens, int L, const float* feat,
                                        const int* positions, const uint8_t* mask, float* hidden, float* out) {
  if (!d || !cache || !tokens || !feat || L <= 0) return WC_ERR_INVALID;
  return guard(d->ctx, [&] {
    const auto& c = d->cfg;
    if (cache->layers != c.layers || cache->Hk != c.kv_heads || cache->D != c.head_dim || cache->dtype != d->dtype)
      fail(WC_ERR_INVALID, "cache does not match the drafter");
    const int prefix = cache->n;
    if (prefix + L > cache->cap) fail(WC_ERR_CAPACITY, "KV cache capacity exceeded");
    wc_ctx* ctx = d->ctx;
    const int H = c.hidden;
    for (int r0 = 0; r0 < L; r0 += GEMV_MAXL) {
      const int rows = std::min(GEMV_MAXL, L - r0);
      Rows r;
      r.L = rows;
      r.L_max = rows;
      r.n_add = prefix + r0;
      r.positions = positions ? positions + r0 : nullptr;
      r.mask_full = mask ? mask + size_t(r0) * (prefix + L) : nullptr;
      r.mask_ld = prefix + L;
      TokenSrc tok;
      std::memset(&tok, 0, sizeof(tok));
      tok.tokens = tokens + r0;
      tok.vocab = c.vocab;
      const float* f = feat + size_t(r0) * H;
      const XIn fin = drafter_pack_rows(d, f, rows, d->layers[0].in_norm, d->xf_feat, d->ss_pack, ctx->d_err);
      drafter_layers(d, cache, r, fin, f, tok, d->ws_h, nullptr, ctx->d_err);
      if (hidden) CUDA_TRY(cudaMemcpyAsync(hidden + size_t(r0) * H, d->ws_h, sizeof(float) * rows * H,
                                           cudaMemcpyDeviceToDevice, ctx->stream));
      if (out) {
        rmsnorm_rows_kernel<<<rows, 256, 0, ctx->stream>>>(d->ws_h, out + size_t(r0) * H, H, d->norm, c.eps);
        check_launch(ctx, "rmsnorm");
      }
    }
    cache->n = prefix + L;
  });
}

extern "C" wc_status wc_drafter_logits(wc_drafter* d, const float* out, int rows, float* z) {
  if (!d || !out || !z || rows <= 0) return WC_ERR_INVALID;
  return guard(d->ctx, [&] {
    for (int r0 = 0; r0 < rows; r0 += GEMV_MAXL) {
      const int n = std::min(GEMV_MAXL, rows - r0);
      CUDA_TRY(cudaMemsetAsync(d->ws_keys, 0, sizeof(unsigned long long) * GEMV_MAXL, d->ctx->stream));
      const XIn x = drafter_pack_rows(d, out + size_t(r0) * d->cfg.hidden, n, nullptr, d->xf_out, nullptr,
                                      d->ctx->d_err);
      drafter_head(d, x, n, d->ws_keys, z + size_t(r0) * d->head_rows, nullptr, nullptr, d->ctx->d_err);
    }
  });
}

extern "C" wc_status wc_drafter_head_softmax(wc_drafter* d, const float* out, int rows, float temperature,
                                             float* probs) {
  if (!d || !out || !probs || rows <= 0) return WC_ERR_INVALID;
  if (!(temperature > 0.f)) {
    d->ctx->err = "the draft distribution needs a temperature > 0 (greedy drafting uses 1)";
    return WC_ERR_INVALID;
  }
  const wc_status st = wc_drafter_logits(d, out, rows, probs);  // logits into the output, then in place
  if (st != WC_OK) return st;
  return wc_probs_from_logits(d->ctx, probs, rows, d->head_rows, temperature, 0, 1.f, probs);
}

extern "C" wc_status wc_drafter_head_argmax(wc_drafter* d, const float* out, int rows, int* token) {
  if (!d || !out || !token || rows <= 0) return WC_ERR_INVALID;
  return guard(d->ctx, [&] {
    for (int r0 = 0; r0 < rows; r0 += GEMV_MAXL) {
      const int n = std::min(GEMV_MAXL, rows - r0);
      CUDA_TRY(cudaMemsetAsync(d->ws_keys, 0, sizeof(unsigned long long) * GEMV_MAXL, d->ctx->stream));
      const XIn x = drafter_pack_rows(d, out + size_t(r0) * d->cfg.hidden, n, nullptr, d->xf_out, nullptr,
                                      d->ctx->d_err);
      drafter_head(d, x, n, d->ws_keys, nullptr, nullptr, nullptr, d->ctx->d_err);
      keys_to_index_kernel<<<1, 32, 0, d->ctx->stream>>>(d->ws_keys, n, d->vocab_map, token + r0);
      check_launch(d->ctx, "keys");
    }
  });
}

// ============================================================================ prompt forward on the tensor cores

namespace {
// Rows [0, n) of tokens_dev (device) through every target layer as tcgen05 GEMMs over all
// rows at once, their K/V appended to `kv` after its first `start` rows, tap rows into
// `to->rows` (when set). Returns the fp32 residual row of the last token (before the final
// norm), or nullptr when the target cannot take this path (the caller then runs the decode
// kernels). Defined with the batched verification.
const float* prefill_gemm_forward(wc_target* t, wc_kv* kv, const int* tokens_dev, int n, int start, const TapOut* to);
// The drafter's prompt pass the same way (fuse, then every layer as tcgen05 GEMMs over all rows,
// causal attention, K/V appended to `kv` after `start`): tokens_dev[n] are the entries' tokens,
// taps [3][n][target hidden] (tap f at + f * tstride) their features. Returns the last row's
// residual before the final norm, or nullptr when the drafter cannot take this path.
const float* drafter_prefill_gemm(wc_drafter* d, wc_kv* kv, const int* tokens_dev, int n, int start,
                                  const float* taps, size_t tstride);
}  // namespace

// ============================================================================ sampled decoding

namespace {

// probs_from_logits (sampling.py:39-55) on the device: temperature, top-k, top-p.
bool sampling_on(const wc_sampling_params* sp) {
  if (!sp || !(sp->temperature > 0.f)) return false;
  if (sp->top_k < 0) fail(WC_ERR_INVALID, "top_k must be >= 0");
  if (!(sp->top_p > 0.f) || sp->top_p > 1.f) fail(WC_ERR_INVALID, "top_p must be in (0, 1]");
  return true;
}
bool warping_on(const wc_sampling_params* sp) { return sp && (sp->top_k > 0 || sp->top_p < 1.f); }

// RoundState's random state and warping: seed, counter base 0 (the first token's draw), T,
// top-k, top-p
void seed_rounds(wc_ctx* ctx, RoundState* st, const wc_sampling_params* sp, bool on) {
  struct {
    unsigned long long rng[2];
    float temperature;
    int top_k;
    float top_p;
    int pad;
  } v{{on ? (unsigned long long)sp->seed : 0ull, 0ull}, on ? sp->temperature : 0.f, on ? sp->top_k : 0,
      on ? sp->top_p : 1.f, 0};
  static_assert(sizeof(v) == sizeof(RoundState) - offsetof(RoundState, rng), "RoundState tail layout");
  CUDA_TRY(cudaMemcpyAsync(st->rng, &v, sizeof(v), cudaMemcpyHostToDevice, ctx->stream));
}

// A warped draw from logits rows z [rows][V] into keys[0..rows) (first token / autoregressive
// step): thresholds, then the Gumbel-max over the kept tokens (stream 0 + row).
void warped_draw(wc_ctx* ctx, RoundState* st, const float* z, int rows, int V, RowWarp* warp,
                 unsigned long long* keys) {
  WarpParams w;
  std::memset(&w, 0, sizeof(w));
  w.z = z;
  w.V = V;
  w.ld = V;
  w.temperature = &st->temperature;
  w.top_k = &st->top_k;
  w.top_p = &st->top_p;
  w.out = warp;
  w.zero_keys = keys;
  w.zero_n = rows;
  launch_ex(ctx, "warp rows", warp_rows_kernel, dim3(rows), dim3(1024), 0, true, 1, w);
  SampleRowsParams sr;
  sr.z = z;
  sr.V = V;
  sr.ld = V;
  sr.temperature = &st->temperature;
  sr.warp = warp;
  sr.rng = st->rng;
  sr.stream = 0;
  sr.keys = keys;
  launch_ex(ctx, "sample rows", sample_rows_kernel, dim3(148, rows), dim3(256), 0, true, 1, sr);
}

}  // namespace

// ============================================================================ decoder

struct wc_decoder {
  wc_ctx* ctx = nullptr;
  wc_target* t = nullptr;
  wc_drafter* d = nullptr;
  int max_ctx = 0, max_k = 0;
  wc_kv* tkv = nullptr;
  wc_kv* dkv = nullptr;
  RoundState* st = nullptr;
  int* out_dev = nullptr;
  int* out_host = nullptr;  // pinned: [n_out, tokens..., err]
  // the next round's chain root: head input and first drafter feature (fp32 + fragments)
  float *root_out = nullptr, *root_fb = nullptr;
  uint32_t *xf_root = nullptr, *xf_fb = nullptr;
  float* ss_fb = nullptr;
  float* taps = nullptr;  // prefill taps [3][n][Ht]
  int taps_n = 0;
  std::map<int, std::pair<cudaGraphExec_t, uint64_t>> graphs;
  std::map<int, std::pair<cudaGraphExec_t, uint64_t>> prof_graphs;
  std::map<int, std::unique_ptr<Profiler>> profilers;
  int host_n = 0;  // committed length mirrored on the host
  bool prefilled = false;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_ms = 0.f;
  // sampled decoding (temperature > 0, set by the prefill): the round's logits, their softmax
  // slices and the acceptance kernel's partials
  bool sampled = false;
  bool warped = false;       // top-k / top-p on the target distribution
  RowWarp* rwarp = nullptr;  // [max_k + 1] warp thresholds of the verify rows
  float* zt = nullptr;       // [max_k + 1][V] target logits of the verify rows
  float* zd = nullptr;       // [max_k][head rows] draft logits
  float2* zstats = nullptr;  // logit_stats_kernel output
  double* apart = nullptr;   // [kAcceptBlocks][3]
  unsigned* acount = nullptr;
  int nbt = 0, nbd = 0;      // softmax slices per target / draft row
  int zd_rows = 0;           // draft head rows zd was sized for
  // device draft trees (tree.cuh): node state, node features, head logits, taps of the verify rows
  TreeState* ts = nullptr;
  float* tree_fb = nullptr;     // [1 + 32][H]
  float* tree_z = nullptr;      // [TR_MAXW][head rows], allocated at the first tree round
  int tree_z_rows = 0;
  float* tree_taps = nullptr;   // [2][3][TR_MAXV][Ht]: the verify rows', then the kept rows'
  // wc_decoder_save_state snapshot
  RoundState* saved_st = nullptr;
  unsigned char* saved_root = nullptr;
  size_t root_bytes[5] = {};
  int saved_host_n = -1;
};

namespace {

constexpr int kAcceptBlocks = 148;      // acceptance draw: one slice of the vocabulary per SM
constexpr int kStatsSlice = 4096;       // logits per softmax slice
constexpr int kSampledGraphKey = 1000;  // graph key offset of sampled rounds

void launch_finish(wc_decoder* dec, const int* L_dev, int L_static, bool advance, const float* h = nullptr) {
  wc_drafter* d = dec->d;
  FinishParams f;
  std::memset(&f, 0, sizeof(f));
  f.st = dec->st;
  f.L_dev = L_dev;
  f.L_static = L_static;
  f.h = h ? h : d->ws_h;
  f.d = d->cfg.hidden;
  f.norm_w = d->norm;
  f.eps = d->cfg.eps;
  f.post_norm = d->cfg.post_norm;
  f.root_out = dec->root_out;
  f.root_fb = dec->root_fb;
  f.xf_out = dec->xf_root;
  f.xf_fb = dec->xf_fb;
  f.in_norm0 = d->layers[0].in_norm;
  f.ss_fb = dec->ss_fb;
  f.xf_width = xf_width(is_bf16(d->dtype), d->cfg.hidden);
  f.xf_fp32 = is_bf16(d->dtype) ? 0 : 1;
  f.advance_dc = advance ? 1 : 0;
  launch_ex(dec->ctx, "finish update", finish_update_kernel, dim3(1), dim3(256), 0, true, 1, f);
}

void build_round(wc_decoder* dec, int K) {
  wc_ctx* ctx = dec->ctx;
  wc_target* t = dec->t;
  wc_drafter* d = dec->d;
  RoundState* st = dec->st;
  int* err = &st->err;
  const bool post = d->cfg.post_norm != 0;
  const bool smp = dec->sampled;
  Pick pick;
  pick.temperature = &st->temperature;
  pick.rng = st->rng;
  // ---- draft chain (spec.py:344-350): K heads, K-1 drafter layer passes; sampled rounds
  // draw d_k from softmax(z_k / T) in the head's epilogue and keep z_k for the acceptance
  XIn head_in{dec->xf_root, nullptr, 0};  // root_out is already normalised
  const Lin& ld = d->layers.back().down;
  for (int k = 0; k < K; ++k) {
    const bool more = k < K - 1;
    pick.stream = k;
    // with post-norm the next feature is RMSNorm(h) * norm: the head's side job makes it
    drafter_head(d, head_in, 1, st->keys + k, smp ? dec->zd + size_t(k) * d->head_rows : nullptr,
                 (k > 0 && post && more) ? d->ws_h : nullptr, (k > 0 && post && more) ? d->ws_feat : nullptr, err,
                 smp ? &pick : nullptr);
    if (!more) break;
    XIn fin;
    const float* feat;
    if (k == 0) {
      fin = XIn{dec->xf_fb, dec->ss_fb, 1};
      feat = dec->root_fb;
    } else if (post) {
      fin = XIn{d->xf_feat, d->ss_feat, side_parts(ctx, d->head, 1)};
      feat = d->ws_feat;
    } else {
      fin = XIn{d->xf_feat, d->layers.back().ss_d, gemv_parts(ctx, ld, 1)};
      feat = d->ws_h;
    }
    Rows r;
    r.stable = true;
    r.L = 1;
    r.L_max = 1;
    r.n_dev = &st->dc_len;
    r.n_add = k;
    TokenSrc tok;
    std::memset(&tok, 0, sizeof(tok));
    tok.keys = st->keys + k;
    tok.vocab_map = d->vocab_map;
    tok.forced = st->forced + k;
    tok.vocab = d->cfg.vocab;
    const XOut extra{d->xf_feat, d->layers[0].in_norm};
    prof_begin(ctx, PK_DRAFT_LAYER);
    head_in = drafter_layers(d, dec->dkv, r, fin, feat, tok, d->ws_h, post ? nullptr : &extra, err);
    prof_end(ctx, PK_DRAFT_LAYER);
  }
  // ---- verification of [x_n, d_1..d_K] (spec.py:353-355)
  Rows rv;
  rv.stable = true;
  rv.L = K + 1;
  rv.L_max = K + 1;
  rv.n_dev = &st->n;
  const XIn in0 = target_embed(t, rv, nullptr, st, d->vocab_map, t->ws_h, err);
  TapOut to;
  for (int f = 0; f < 3; ++f) {
    to.xf[f] = d->xf_tap[f];
    to.w[f] = d->cfg.feature_norm ? d->feature_norms[f] : nullptr;
  }
  const XIn hx = target_layers(t, dec->tkv, rv, in0, t->ws_h, &to, err);
  target_head(t, hx, K + 1, nullptr, K + 1, st->keys + K, smp ? dec->zt : nullptr, err);
  // ---- acceptance + chain compaction (spec.py:357-362; sampled: spec.py:321-324 with
  // verify_tree_stochastic on the chain)
  if (smp) {
    if (dec->warped) {  // top-k / top-p thresholds of the verify rows
      WarpParams w;
      std::memset(&w, 0, sizeof(w));
      w.z = dec->zt;
      w.V = t->cfg.vocab;
      w.ld = t->cfg.vocab;
      w.temperature = &st->temperature;
      w.top_k = &st->top_k;
      w.top_p = &st->top_p;
      w.out = dec->rwarp;
      launch_ex(ctx, "warp rows", warp_rows_kernel, dim3(K + 1), dim3(1024), 0, true, 1, w);
    }
    StatsParams sp;
    sp.z1 = dec->zt;
    sp.R1 = dec->warped ? 0 : K + 1;
    sp.V1 = t->cfg.vocab;
    sp.nb1 = dec->nbt;
    sp.z2 = dec->zd;
    sp.R2 = K;
    sp.V2 = d->head_rows;
    sp.nb2 = dec->nbd;
    sp.temperature = &st->temperature;
    sp.out = dec->zstats;
    launch_ex(ctx, "logit stats", logit_stats_kernel, dim3(sp.R1 * dec->nbt + K * dec->nbd), dim3(256), 0, true, 1,
              sp);
    SampleAcceptParams ap;
    ap.st = st;
    ap.K = K;
    ap.zt = dec->zt;
    ap.V = t->cfg.vocab;
    ap.zd = dec->zd;
    ap.Vd = d->head_rows;
    ap.vocab_inv = d->vocab_inv;
    ap.stats = dec->zstats;
    ap.nbt = dec->nbt;
    ap.nbd = dec->nbd;
    ap.warp = dec->warped ? dec->rwarp : nullptr;
    ap.part = dec->apart;
    ap.counter = dec->acount;
    ap.out_host_view = dec->out_dev;
    launch_ex(ctx, "accept sampled", accept_sampled_kernel, dim3(kAcceptBlocks), dim3(256), 0, true, 1, ap);
  } else {
    launch_ex(ctx, "accept", accept_chain_kernel, dim3(1), dim3(32), 0, true, 1, st, K, (const int*)nullptr,
              dec->out_dev);
  }
  // ---- drafter update on the accepted rows (spec.py:363, 366-374)
  XIn tx[3];
  for (int f = 0; f < 3; ++f) tx[f] = target_tap_stats(t, f, d->xf_tap[f], K + 1);
  const XIn gin = drafter_fuse_impl(d, tx, K + 1, &st->L_upd, K + 1, d->ws_g, err);
  Rows ru;
  ru.stable = true;
  ru.L = K + 1;
  ru.L_dev = &st->L_upd;
  ru.L_max = K + 1;
  ru.n_dev = &st->dc_len;
  TokenSrc tok;
  std::memset(&tok, 0, sizeof(tok));
  tok.tokens = st->acc;
  tok.vocab = d->cfg.vocab;
  drafter_layers(d, dec->dkv, ru, gin, d->ws_g, tok, d->ws_h, nullptr, err);
  launch_finish(dec, &st->L_upd, K + 1, true);
}

// ---- device draft trees (tree.cuh)

struct TreeShape {
  int depth, width, budget, rows;  // rows: verify rows the graph is built for
};

// Checks a greedy tree shape against the device limits and returns its verify row count.
TreeShape tree_shape(int depth, int width, int budget) {
  if (depth < 1 || width < 1 || budget < 1) fail(WC_ERR_INVALID, "tree depth, width and budget must be >= 1");
  if (width > TR_MAXW) fail(WC_ERR_UNSUPPORTED, "tree width above 16");
  if ((depth - 1) * width > 32) fail(WC_ERR_UNSUPPORTED, "(depth - 1) * width above 32 drafted rows");
  long long nodes = 1 + width;
  for (int dd = 2; dd <= depth; ++dd) nodes += (long long)width * width;
  if (nodes > TR_MAXN) fail(WC_ERR_UNSUPPORTED, "tree of more than 128 drafted nodes");
  const int rows = int(std::min<long long>(nodes - 1, budget)) + 1;
  if (rows > TR_MAXV) fail(WC_ERR_UNSUPPORTED, "verify budget above 15 nodes (16 rows per target pass)");
  return {depth, width, budget, rows};
}

TreeStepParams tree_params(wc_decoder* dec, const TreeShape& sh) {
  wc_drafter* d = dec->d;
  TreeStepParams p;
  std::memset(&p, 0, sizeof(p));
  p.ts = dec->ts;
  p.st = dec->st;
  p.W = sh.width;
  p.budget = sh.budget;
  p.max_rows = sh.rows;
  p.z = dec->tree_z;
  p.Vh = d->head_rows;
  p.vocab_map = d->vocab_map;
  p.vocab = dec->t->cfg.vocab;
  p.root_fb = dec->root_fb;
  p.fb_store = dec->tree_fb;
  p.H = d->cfg.hidden;
  p.h = d->ws_h;
  p.norm_w = d->norm;
  p.eps = d->cfg.eps;
  p.post_norm = d->cfg.post_norm;
  p.out_host_view = dec->out_dev;
  return p;
}

// One greedy tree round: draft the tree level by level, verify it in one target pass, accept,
// compact and update the drafter on the accepted rows.
void build_tree_round(wc_decoder* dec, const TreeShape& sh) {
  wc_ctx* ctx = dec->ctx;
  wc_target* t = dec->t;
  wc_drafter* d = dec->d;
  RoundState* st = dec->st;
  TreeState* ts = dec->ts;
  int* err = &st->err;
  const int W = sh.width, N = sh.rows, H = d->cfg.hidden, Ht = t->cfg.hidden;
  TreeStepParams tp = tree_params(dec, sh);
  launch_ex(ctx, "tree begin", tree_begin_kernel, dim3(1), dim3(256), 0, true, 1, tp);
  // depth 1: the root's children from its head row
  drafter_head(d, XIn{dec->xf_root, nullptr, 0}, 1, ts->hkeys, dec->tree_z, nullptr, nullptr, err);
  tp.level = 1;
  launch_ex(ctx, "tree expand", tree_expand_kernel, dim3(1), dim3(256), 0, true, 1, tp);
  for (int lvl = 1; lvl < sh.depth; ++lvl) {
    tp.level = lvl;
    launch_ex(ctx, "tree frontier", tree_frontier_kernel, dim3(1), dim3(32), 0, true, 1, tp);
    PackParams pk = pack_params();  // the frontier's parent features: fragments x layer-0 gain, fp32 rows
    pk.src = dec->tree_fb;
    pk.row_map = ts->fr_fbrow;
    pk.ld = H;
    pk.K = H;
    pk.L = W;
    pk.L_dev = &ts->n_frontier;
    pk.w = d->layers[0].in_norm;
    pk.xf = d->xf_feat;
    pk.ss = d->ss_feat;
    pk.copy = d->ws_feat;
    pk.err = err;
    launch_pack(ctx, pk, is_bf16(d->dtype), W);
    Rows r;
    r.stable = true;
    r.L = W;
    r.L_dev = &ts->n_frontier;
    r.L_max = W;
    r.n_dev = &st->dc_len;
    r.n_add = (lvl - 1) * W;
    r.positions = ts->fr_pos;
    r.newmask = ts->fr_mask;
    r.mask_from_prefix = true;
    TokenSrc tok;
    std::memset(&tok, 0, sizeof(tok));
    tok.tokens = ts->fr_tok;
    tok.vocab = d->cfg.vocab;
    const XIn head_in = drafter_layers(d, dec->dkv, r, XIn{d->xf_feat, d->ss_feat, 1}, d->ws_feat, tok, d->ws_h,
                                       nullptr, err);
    launch_ex(ctx, "tree store fb", tree_store_fb_kernel, dim3(W), dim3(256), 0, true, 1, tp);
    drafter_head(d, head_in, W, ts->hkeys, dec->tree_z, nullptr, nullptr, err);
    tp.level = lvl + 1;
    launch_ex(ctx, "tree expand", tree_expand_kernel, dim3(W), dim3(256), 0, true, 1, tp);
  }
  launch_ex(ctx, "tree select", tree_select_kernel, dim3(1), dim3(32), 0, true, 1, tp);
  // verification of the tree in one target pass (positions n + depth, tree-mask bits)
  Rows rv;
  rv.stable = true;
  rv.L = N;
  rv.L_dev = &ts->N;
  rv.L_max = N;
  rv.n_dev = &st->n;
  rv.positions = ts->vpos;
  rv.newmask = ts->vmask;
  const XIn in0 = target_embed(t, rv, ts->vtok, nullptr, nullptr, t->ws_h, err);
  TapOut to;
  to.rows = dec->tree_taps;
  to.stride = size_t(TR_MAXV) * Ht;
  const XIn hx = target_layers(t, dec->tkv, rv, in0, t->ws_h, &to, err);
  target_head(t, hx, N, &ts->N, N, ts->vkeys, nullptr, err);
  launch_ex(ctx, "tree accept", tree_accept_kernel, dim3(1), dim3(32), 0, true, 1, tp);
  TreeCompactParams cp;
  cp.ts = ts;
  cp.st = st;
  cp.K = dec->tkv->K;
  cp.V = dec->tkv->V;
  cp.layer_elems = (long long)dec->tkv->layer_elems();
  cp.stride_h = (long long)dec->tkv->cap * dec->tkv->D;
  cp.D = dec->tkv->D;
  cp.esize = int(dtype_size(dec->tkv->dtype));
  cp.cap = dec->tkv->cap;
  launch_ex(ctx, "tree compact", tree_compact_kernel, dim3(t->cfg.layers, t->cfg.kv_heads), dim3(128), 0, true, 1,
            cp);
  TreeTapsParams tq;
  tq.ts = ts;
  tq.st = st;
  tq.in = dec->tree_taps;
  tq.out = dec->tree_taps + size_t(3) * TR_MAXV * Ht;
  tq.rows = TR_MAXV;
  tq.Ht = Ht;
  launch_ex(ctx, "tree taps", tree_taps_kernel, dim3(3, N), dim3(256), 0, true, 1, tq);
  // drafter update on the accepted rows (spec.cpp:226-233)
  XIn tx[3];
  for (int f = 0; f < 3; ++f) {
    PackParams pt = pack_params();
    pt.src = tq.out + size_t(f) * TR_MAXV * Ht;
    pt.ld = Ht;
    pt.K = Ht;
    pt.L = N;
    pt.L_dev = &st->L_upd;
    pt.w = d->cfg.feature_norm ? d->feature_norms[f] : nullptr;
    pt.xf = d->xf_tap[f];
    pt.ss = d->ss_tap[f];
    pt.err = err;
    launch_pack(ctx, pt, is_bf16(d->dtype), N);
    tx[f] = XIn{d->xf_tap[f], d->ss_tap[f], 1};
  }
  const XIn gin = drafter_fuse_impl(d, tx, N, &st->L_upd, N, d->ws_g, err);
  Rows ru;
  ru.stable = true;
  ru.L = N;
  ru.L_dev = &st->L_upd;
  ru.L_max = N;
  ru.n_dev = &st->dc_len;
  TokenSrc tok;
  std::memset(&tok, 0, sizeof(tok));
  tok.tokens = st->acc;
  tok.vocab = d->cfg.vocab;
  drafter_layers(d, dec->dkv, ru, gin, d->ws_g, tok, d->ws_h, nullptr, err);
  launch_finish(dec, &st->L_upd, N, true);
}

std::pair<cudaGraphExec_t, uint64_t>& tree_graph(wc_decoder* dec, const TreeShape& sh) {
  const int key = 1 << 20 | sh.depth << 12 | sh.width << 6 | sh.budget;
  auto it = dec->graphs.find(key);
  if (it != dec->graphs.end()) return it->second;
  wc_ctx* ctx = dec->ctx;
  if (!dec->tree_z || dec->tree_z_rows != dec->d->head_rows) {  // outside the capture
    dfree(dec->tree_z);
    dec->tree_z = static_cast<float*>(dalloc(sizeof(float) * size_t(TR_MAXW) * dec->d->head_rows));
    dec->tree_z_rows = dec->d->head_rows;
  }
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  cudaGraph_t g = nullptr;
  CUDA_TRY(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  ctx->capturing = true;
  ctx->capture_launches = 0;
  try {
    build_tree_round(dec, sh);
  } catch (...) {
    ctx->capturing = false;
    cudaStreamEndCapture(ctx->stream, &g);
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    throw;
  }
  ctx->capturing = false;
  CUDA_TRY(cudaStreamEndCapture(ctx->stream, &g));
  cudaGraphExec_t exec = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) fail(WC_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
  dec->graphs[key] = {exec, ctx->capture_launches};
  return dec->graphs[key];
}

int graph_key(const wc_decoder* dec, int K) {
  return K + (dec->sampled ? kSampledGraphKey : 0) + (dec->warped ? 2 * kSampledGraphKey : 0);
}

std::pair<cudaGraphExec_t, uint64_t>& round_graph(wc_decoder* dec, int K, bool profiled = false) {
  auto& store = profiled ? dec->prof_graphs : dec->graphs;
  const int gk = graph_key(dec, K);
  auto it = store.find(gk);
  if (it != store.end()) return it->second;
  wc_ctx* ctx = dec->ctx;
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  if (profiled) {
    dec->profilers[gk] = std::make_unique<Profiler>();
    ctx->prof = dec->profilers[gk].get();
  }
  cudaGraph_t g = nullptr;
  CUDA_TRY(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  ctx->capturing = true;
  ctx->capture_launches = 0;
  try {
    build_round(dec, K);
  } catch (...) {
    ctx->capturing = false;
    ctx->prof = nullptr;
    cudaStreamEndCapture(ctx->stream, &g);
    if (g) cudaGraphDestroy(g);
    cudaGetLastError();
    throw;
  }
  ctx->capturing = false;
  ctx->prof = nullptr;
  CUDA_TRY(cudaStreamEndCapture(ctx->stream, &g));
  cudaGraphExec_t exec = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) fail(WC_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
  store[gk] = {exec, ctx->capture_launches};
  return store[gk];
}

void check_state_error(wc_decoder* dec) {
  int e = 0;
  CUDA_TRY(cudaMemcpy(&e, &dec->st->err, sizeof(int), cudaMemcpyDeviceToHost));
  int ce = 0;
  CUDA_TRY(cudaMemcpy(&ce, dec->ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e || ce) {
    CUDA_TRY(cudaMemset(&dec->st->err, 0, sizeof(int)));
    CUDA_TRY(cudaMemset(dec->ctx->d_err, 0, sizeof(int)));
    CUDA_TRY(cudaMemset(dec->ctx->gv_counters, 0, sizeof(int) * dec->ctx->gv_counters_n));
    CUDA_TRY(cudaMemset(dec->ctx->as_counters, 0, sizeof(int) * AS_MAXHK));
    fail(WC_ERR_DEVICE, "device error flag " + std::to_string(e | ce));
  }
}

}  // namespace

extern "C" wc_status wc_decoder_create(wc_target* t, wc_drafter* d, int max_context, int max_k, wc_decoder** out) {
  if (!t || !d || !out) return WC_ERR_INVALID;
  return guard(t->ctx, [&] {
    if (t->ctx != d->ctx) fail(WC_ERR_INVALID, "target and drafter belong to different contexts");
    if (!t->finalized || !d->finalized) fail(WC_ERR_INVALID, "models not finalized");
    if (d->cfg.target_hidden != t->cfg.hidden) fail(WC_ERR_INVALID, "drafter target_hidden_size != target hidden");
    if (d->cfg.num_features != 3) fail(WC_ERR_UNSUPPORTED, "the decoder fuses exactly three target taps");
    if (t->dtype != d->dtype) fail(WC_ERR_UNSUPPORTED, "target and drafter must use the same dtype");
    if (max_k < 1 || max_k > MAXK || max_k + 1 > GEMV_MAXL) fail(WC_ERR_INVALID, "max_k must be in 1..15");
    if (max_context < 2 || max_context > 32768 - MAXK) fail(WC_ERR_INVALID, "max_context out of range");
    wc_ctx* ctx = t->ctx;
    auto dec = std::make_unique<wc_decoder>();
    dec->ctx = ctx;
    dec->t = t;
    dec->d = d;
    dec->max_k = max_k;
    dec->max_ctx = max_context;
    const int cap = max_context + std::max(max_k + 1, 33);  // room for a round's chain or tree rows
    dec->tkv = kv_new(ctx, t->cfg.layers, t->cfg.kv_heads, t->cfg.head_dim, cap, t->dtype);
    dec->dkv = kv_new(ctx, d->cfg.layers, d->cfg.kv_heads, d->cfg.head_dim, cap, d->dtype);
    dec->st = static_cast<RoundState*>(dalloc(sizeof(RoundState)));
    CUDA_TRY(cudaMemset(dec->st, 0, sizeof(RoundState)));
    std::vector<int> neg(MAXK, -1);
    CUDA_TRY(cudaMemcpy(dec->st->forced, neg.data(), sizeof(int) * MAXK, cudaMemcpyHostToDevice));
    dec->out_dev = static_cast<int*>(dalloc(sizeof(int) * (MAXK + 4)));
    CUDA_TRY(cudaMallocHost(&dec->out_host, sizeof(int) * (MAXK + 4)));
    const int H = d->cfg.hidden;
    const bool bf16 = is_bf16(d->dtype);
    dec->root_out = static_cast<float*>(dalloc(sizeof(float) * H));
    dec->root_fb = static_cast<float*>(dalloc(sizeof(float) * H));
    dec->xf_root = xf_alloc(bf16, H);
    dec->xf_fb = xf_alloc(bf16, H);
    dec->ss_fb = ss_alloc(ctx);
    dec->root_bytes[0] = sizeof(float) * H;
    dec->root_bytes[1] = sizeof(float) * H;
    dec->root_bytes[2] = size_t(GEMV_MAXL) * xf_width(bf16, H) * 4;
    dec->root_bytes[3] = dec->root_bytes[2];
    dec->root_bytes[4] = sizeof(float) * max_parts(ctx) * 16;
    {  // sampled decoding buffers
      const int V = t->cfg.vocab, Vd = d->head_rows;
      dec->nbt = (V + kStatsSlice - 1) / kStatsSlice;
      dec->nbd = (Vd + kStatsSlice - 1) / kStatsSlice;
      dec->zd_rows = Vd;
      dec->zt = static_cast<float*>(dalloc(sizeof(float) * size_t(max_k + 1) * V));
      dec->zd = static_cast<float*>(dalloc(sizeof(float) * size_t(max_k) * Vd));
      dec->zstats = static_cast<float2*>(dalloc(sizeof(float2) * size_t((max_k + 1) * dec->nbt + max_k * dec->nbd)));
      dec->apart = static_cast<double*>(dalloc(sizeof(double) * 3 * kAcceptBlocks));
      dec->rwarp = static_cast<RowWarp*>(dalloc(sizeof(RowWarp) * (MAXK + 1)));
      dec->acount = static_cast<unsigned*>(dalloc(sizeof(unsigned)));
      CUDA_TRY(cudaMemset(dec->acount, 0, sizeof(unsigned)));
    }
    dec->ts = static_cast<TreeState*>(dalloc(sizeof(TreeState)));
    CUDA_TRY(cudaMemset(dec->ts, 0, sizeof(TreeState)));
    dec->tree_fb = static_cast<float*>(dalloc(sizeof(float) * 33 * H));
    dec->tree_taps = static_cast<float*>(dalloc(sizeof(float) * 2 * 3 * TR_MAXV * t->cfg.hidden));
    CUDA_TRY(cudaEventCreate(&dec->ev0));
    CUDA_TRY(cudaEventCreate(&dec->ev1));
    *out = dec.release();
  });
}

extern "C" void wc_decoder_destroy(wc_decoder* dec) {
  if (!dec) return;
  cudaStreamSynchronize(dec->ctx->stream);
  for (auto& g : dec->graphs) cudaGraphExecDestroy(g.second.first);
  for (auto& g : dec->prof_graphs) cudaGraphExecDestroy(g.second.first);
  wc_kv_destroy(dec->tkv);
  wc_kv_destroy(dec->dkv);
  dfree(dec->st);
  dfree(dec->out_dev);
  if (dec->out_host) cudaFreeHost(dec->out_host);
  for (void* p : {(void*)dec->root_out, (void*)dec->root_fb, (void*)dec->xf_root, (void*)dec->xf_fb,
                  (void*)dec->ss_fb, (void*)dec->taps, (void*)dec->zt, (void*)dec->zd, (void*)dec->zstats,
                  (void*)dec->apart, (void*)dec->acount, (void*)dec->saved_st, (void*)dec->saved_root,
                  (void*)dec->rwarp, (void*)dec->ts, (void*)dec->tree_fb, (void*)dec->tree_z,
                  (void*)dec->tree_taps})
    dfree(p);
  if (dec->ev0) cudaEventDestroy(dec->ev0);
  if (dec->ev1) cudaEventDestroy(dec->ev1);
  delete dec;
}

namespace {

// spec.py:129-141 / spec.cpp:61-84: target forward on the prompt (taps kept), first token,
// drafter forward on prompt[1:] + [first] with the fused taps.
int decoder_prefill_impl(wc_decoder* dec, const int* prompt, int n, const wc_sampling_params* sp) {
  const bool smp = sampling_on(sp);
  if (smp && dec->d->cfg.vocab != dec->t->cfg.vocab)
    fail(WC_ERR_UNSUPPORTED, "sampled decoding needs the drafter and target vocabularies to match");
  if (dec->d->head_rows != dec->zd_rows)
    fail(WC_ERR_INVALID, "the drafter head changed after the decoder was created (restrict the vocabulary first)");
  if (n < 1) fail(WC_ERR_INVALID, "empty prompt");
  if (n + dec->max_k + 1 > dec->tkv->cap) fail(WC_ERR_CAPACITY, "prompt longer than the decoder context");
  wc_ctx* ctx = dec->ctx;
  wc_target* t = dec->t;
  wc_drafter* d = dec->d;
  const int Ht = t->cfg.hidden;
  for (int i = 0; i < n; ++i)
    if (prompt[i] < 0 || prompt[i] >= t->cfg.vocab) fail(WC_ERR_INVALID, "prompt token id out of range");
  if (dec->taps_n < n) {
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    dfree(dec->taps);
    dec->taps = static_cast<float*>(dalloc(sizeof(float) * 3 * size_t(n) * Ht));
    dec->taps_n = n;
  }
  int* d_tok = static_cast<int*>(dalloc(sizeof(int) * (n + 1)));
  struct Free {
    void* p;
    ~Free() { dfree(p); }
  } guard_free{d_tok};
  CUDA_TRY(cudaMemcpyAsync(d_tok, prompt, sizeof(int) * n, cudaMemcpyHostToDevice, ctx->stream));
  CUDA_TRY(cudaMemsetAsync(dec->st, 0, offsetof(RoundState, forced), ctx->stream));
  CUDA_TRY(cudaMemsetAsync(dec->st->keys, 0, sizeof(dec->st->keys), ctx->stream));
  seed_rounds(ctx, dec->st, sp, smp);
  int* err = &dec->st->err;
  const size_t tstride = size_t(n) * Ht;
  Pick pick;  // _sample_target (spec.py:143-147) of the first token
  pick.temperature = &dec->st->temperature;
  pick.rng = dec->st->rng;
  TapOut tg;
  tg.rows = dec->taps;
  tg.stride = tstride;
  const bool warp = smp && warping_on(sp);
  const float* last = prefill_gemm_forward(t, dec->tkv, d_tok, n, 0, &tg);
  if (last) {
    if (warp) {  // logits of the last row, then the warped draw
      target_head_rows(t, last, 1, dec->st->keys + 1, dec->zt, err);
      warped_draw(ctx, dec->st, dec->zt, 1, t->cfg.vocab, dec->rwarp, dec->st->keys);
    } else {
      target_head_rows(t, last, 1, dec->st->keys, nullptr, err, smp ? &pick : nullptr);
    }
  }
  for (int r0 = 0; r0 < n && !last; r0 += GEMV_MAXL) {
    const int rows = std::min(GEMV_MAXL, n - r0);
    Rows r;
    r.L = rows;
    r.L_max = rows;
    r.n_add = r0;
    const XIn in0 = target_embed(t, r, d_tok + r0, nullptr, nullptr, t->ws_h, err);
    TapOut to;
    to.rows = dec->taps + size_t(r0) * Ht;
    to.stride = tstride;
    target_layers(t, dec->tkv, r, in0, t->ws_h, &to, err);
    if (r0 + rows == n) {
      if (warp) {
        target_head_rows(t, t->ws_h + size_t(rows - 1) * Ht, 1, dec->st->keys + 1, dec->zt, err);
        warped_draw(ctx, dec->st, dec->zt, 1, t->cfg.vocab, dec->rwarp, dec->st->keys);
      } else {
        target_head_rows(t, t->ws_h + size_t(rows - 1) * Ht, 1, dec->st->keys, nullptr, err, smp ? &pick : nullptr);
      }
    }
  }
  int first = 0;
  {
    unsigned long long key = 0;
    CUDA_TRY(cudaMemcpyAsync(&key, dec->st->keys, sizeof(key), cudaMemcpyDeviceToHost, ctx->stream));
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    first = int(0xFFFFFFFFu - uint32_t(key & 0xFFFFFFFFull));
  }
  // drafter entries e = (token x_{e+1}, feature at e) for e = 0..n-1
  CUDA_TRY(cudaMemcpyAsync(d_tok, prompt + 1, sizeof(int) * (n - 1), cudaMemcpyHostToDevice, ctx->stream));
  CUDA_TRY(cudaMemcpyAsync(d_tok + n - 1, &first, sizeof(int), cudaMemcpyHostToDevice, ctx->stream));
  const float* dlast = drafter_prefill_gemm(d, dec->dkv, d_tok, n, 0, dec->taps, tstride);
  if (dlast) launch_finish(dec, nullptr, 1, false, dlast);
  for (int r0 = 0; r0 < n && !dlast; r0 += GEMV_MAXL) {
    const int rows = std::min(GEMV_MAXL, n - r0);
    XIn tx[3];
    drafter_pack_taps(d, dec->taps + size_t(r0) * Ht, tstride, Ht, rows, tx, err);
    const XIn gin = drafter_fuse_impl(d, tx, rows, nullptr, rows, d->ws_g, err);
    Rows r;
    r.L = rows;
    r.L_max = rows;
    r.n_add = r0;
    TokenSrc tok;
    std::memset(&tok, 0, sizeof(tok));
    tok.tokens = d_tok + r0;
    tok.vocab = d->cfg.vocab;
    drafter_layers(d, dec->dkv, r, gin, d->ws_g, tok, d->ws_h, nullptr, err);
    if (r0 + rows == n) launch_finish(dec, nullptr, rows, false);
  }
  RoundState init{};
  init.n = n;
  init.dc_len = n;
  init.x_n = first;
  CUDA_TRY(cudaMemcpyAsync(dec->st, &init, offsetof(RoundState, forced), cudaMemcpyHostToDevice, ctx->stream));
  CUDA_TRY(cudaMemsetAsync(dec->st->keys, 0, sizeof(dec->st->keys), ctx->stream));
  if (smp) {  // rounds draw from the next counter block
    const unsigned long long base = kRngRoundStride;
    CUDA_TRY(cudaMemcpyAsync(&dec->st->rng[1], &base, sizeof(base), cudaMemcpyHostToDevice, ctx->stream));
  }
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  check_state_error(dec);
  dec->host_n = n;
  dec->prefilled = true;
  dec->sampled = smp;
  dec->warped = warp;
  return first;
}

int decoder_round_impl(wc_decoder* dec, int K, int* out_tokens, bool profiled = false) {
  if (!dec->prefilled) fail(WC_ERR_INVALID, "prefill before the first round");
  if (K < 1 || K > dec->max_k) fail(WC_ERR_INVALID, "chain length outside 1..max_k");
  if (dec->host_n + K + 1 > dec->tkv->cap) fail(WC_ERR_CAPACITY, "decoder context exhausted");
  wc_ctx* ctx = dec->ctx;
  auto& g = round_graph(dec, K, profiled);
  CUDA_TRY(cudaEventRecord(dec->ev0, ctx->stream));
  CUDA_TRY(cudaGraphLaunch(g.first, ctx->stream));
  CUDA_TRY(cudaEventRecord(dec->ev1, ctx->stream));
  ctx->launches += g.second;
  CUDA_TRY(cudaMemcpyAsync(dec->out_host, dec->out_dev, sizeof(int) * (K + 2), cudaMemcpyDeviceToHost, ctx->stream));
  CUDA_TRY(cudaMemcpyAsync(dec->out_host + K + 2, &dec->st->err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));  // the round's single host synchronisation
  cudaEventElapsedTime(&dec->last_ms, dec->ev0, dec->ev1);
  if (dec->out_host[K + 2]) check_state_error(dec);
  const int m = dec->out_host[0];
  if (m < 1 || m > K + 1) fail(WC_ERR_DEVICE, "round produced an invalid token count");
  for (int i = 0; i < m; ++i) out_tokens[i] = dec->out_host[1 + i];
  dec->host_n += m;
  return m;
}

}  // namespace

namespace {
int decoder_tree_round_impl(wc_decoder* dec, int depth, int width, int budget, int* out_tokens) {
  if (!dec->prefilled) fail(WC_ERR_INVALID, "prefill before the first round");
  if (dec->sampled) fail(WC_ERR_UNSUPPORTED, "device draft trees are greedy; sampled trees are not built");
  const TreeShape sh = tree_shape(depth, width, budget);
  if (dec->host_n + std::max(sh.rows, (depth - 1) * width + width) > dec->tkv->cap)
    fail(WC_ERR_CAPACITY, "decoder context exhausted");
  wc_ctx* ctx = dec->ctx;
  auto& g = tree_graph(dec, sh);
  CUDA_TRY(cudaEventRecord(dec->ev0, ctx->stream));
  CUDA_TRY(cudaGraphLaunch(g.first, ctx->stream));
  CUDA_TRY(cudaEventRecord(dec->ev1, ctx->stream));
  ctx->launches += g.second;
  const int cnt = std::min(depth, MAXK) + 2;
  CUDA_TRY(cudaMemcpyAsync(dec->out_host, dec->out_dev, sizeof(int) * cnt, cudaMemcpyDeviceToHost, ctx->stream));
  CUDA_TRY(cudaMemcpyAsync(dec->out_host + cnt, &dec->st->err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));  // the round's single host synchronisation
  cudaEventElapsedTime(&dec->last_ms, dec->ev0, dec->ev1);
  if (dec->out_host[cnt]) check_state_error(dec);
  const int m = dec->out_host[0];
  if (m < 1 || m > depth + 1) fail(WC_ERR_DEVICE, "tree round produced an invalid token count");
  for (int i = 0; i < m; ++i) out_tokens[i] = dec->out_host[1 + i];
  dec->host_n += m;
  return m;
}
}  // namespace

extern "C" wc_status wc_decoder_tree_round(wc_decoder* dec, int depth, int width, int budget, int* out_tokens,
                                           int* out_n) {
  if (!dec || !out_tokens || !out_n) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] { *out_n = decoder_tree_round_impl(dec, depth, width, budget, out_tokens); });
}

extern "C" wc_status wc_decoder_set_forced_tree(wc_decoder* dec, const int* tokens, const int* parents, int n) {
  if (!dec) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] {
    TreeState* ts = dec->ts;
    int on = 0;
    if (tokens && parents && n > 0) {
      if (n > TR_MAXN) fail(WC_ERR_UNSUPPORTED, "forced tree of more than 128 nodes");
      if (parents[0] != -1) fail(WC_ERR_INVALID, "forced tree: node 0 is the root (parent -1)");
      for (int v = 1; v < n; ++v) {
        if (parents[v] < 0 || parents[v] >= v) fail(WC_ERR_INVALID, "forced tree: parents must precede their nodes");
        if (tokens[v] < 0 || tokens[v] >= dec->t->cfg.vocab) fail(WC_ERR_INVALID, "forced tree: token id out of range");
      }
      CUDA_TRY(cudaMemcpy(ts->f_tok, tokens, sizeof(int) * n, cudaMemcpyHostToDevice));
      CUDA_TRY(cudaMemcpy(ts->f_par, parents, sizeof(int) * n, cudaMemcpyHostToDevice));
      CUDA_TRY(cudaMemcpy(&ts->f_n, &n, sizeof(int), cudaMemcpyHostToDevice));
      on = 1;
    }
    CUDA_TRY(cudaMemcpy(&ts->forced_on, &on, sizeof(int), cudaMemcpyHostToDevice));
  });
}

extern "C" wc_status wc_decoder_tree_nodes(wc_decoder* dec, int cap, int* n_nodes, int* tokens, int* parents,
                                           int* proposals, float* proposal_logits, int* verified, int* n_verified) {
  if (!dec || cap < 0) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] {
    CUDA_TRY(cudaStreamSynchronize(dec->ctx->stream));
    TreeState* ts = dec->ts;
    int n = 0, N = 0;
    CUDA_TRY(cudaMemcpy(&n, &ts->n, sizeof(int), cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemcpy(&N, &ts->N, sizeof(int), cudaMemcpyDeviceToHost));
    n = std::max(0, std::min(n, TR_MAXN));
    N = std::max(0, std::min(N, TR_MAXV));
    if (n_nodes) *n_nodes = n;
    if (n_verified) *n_verified = N;
    const int k = std::min(n, cap);
    if (tokens) CUDA_TRY(cudaMemcpy(tokens, ts->token, sizeof(int) * k, cudaMemcpyDeviceToHost));
    if (parents) CUDA_TRY(cudaMemcpy(parents, ts->parent, sizeof(int) * k, cudaMemcpyDeviceToHost));
    if (proposals) CUDA_TRY(cudaMemcpy(proposals, ts->prop_tok, sizeof(int) * k, cudaMemcpyDeviceToHost));
    if (proposal_logits) CUDA_TRY(cudaMemcpy(proposal_logits, ts->prop_z, sizeof(float) * k, cudaMemcpyDeviceToHost));
    if (verified) CUDA_TRY(cudaMemcpy(verified, ts->vnode, sizeof(int) * std::min(N, cap), cudaMemcpyDeviceToHost));
  });
}

extern "C" wc_status wc_decoder_prefill(wc_decoder* dec, const int* prompt, int n, const wc_sampling_params* sp,
                                        int* first) {
  if (!dec || !prompt || !first) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] { *first = decoder_prefill_impl(dec, prompt, n, sp); });
}

extern "C" wc_status wc_decoder_set_forced(wc_decoder* dec, const int* forced, int k) {
  if (!dec || k < 0 || k > MAXK) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] {
    std::vector<int> f(MAXK, -1);
    for (int i = 0; i < k && forced; ++i) f[i] = forced[i];
    CUDA_TRY(cudaMemcpyAsync(dec->st->forced, f.data(), sizeof(int) * MAXK, cudaMemcpyHostToDevice, dec->ctx->stream));
    CUDA_TRY(cudaStreamSynchronize(dec->ctx->stream));
  });
}

extern "C" wc_status wc_decoder_round(wc_decoder* dec, int k, int* out_tokens, int* out_n) {
  if (!dec || !out_tokens || !out_n) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] { *out_n = decoder_round_impl(dec, k, out_tokens); });
}

extern "C" wc_status wc_decoder_generate(wc_decoder* dec, const int* prompt, int n, int max_new, int k,
                                         const wc_sampling_params* sp, const int* eos, int n_eos, int* out_tokens,
                                         int* out_n, wc_gen_stats* stats) {
  if (!dec || !prompt || !out_tokens || !out_n || max_new < 1) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] {
    wc_gen_stats s{};
    s.prompt_tokens = n;
    std::set<int> eset(eos, eos + (eos ? n_eos : 0));
    const double t0 = now_s();
    int x = decoder_prefill_impl(dec, prompt, n, sp);
    s.t_prefill = now_s() - t0;
    int m = 0;
    out_tokens[m++] = x;
    int acc[MAXK + 1];
    while (m < max_new && !eset.count(x)) {
      if (dec->host_n + k + 1 > dec->tkv->cap) fail(WC_ERR_CAPACITY, "decoder context exhausted");
      const double ta = now_s();
      const int na = decoder_round_impl(dec, k, acc);
      s.t_verify += now_s() - ta;
      s.rounds += 1;
      s.accepted += na - 1;
      s.verified += k;
      for (int i = 0; i < na; ++i) {
        out_tokens[m++] = acc[i];
        if (eset.count(acc[i]) || m >= max_new) break;
      }
      x = out_tokens[m - 1];
    }
    s.t_total = now_s() - t0;
    s.new_tokens = m;
    *out_n = m;
    if (stats) *stats = s;
  });
}

extern "C" wc_status wc_decoder_profile_round(wc_decoder* dec, int k, int* out_tokens, int* out_n, float* ms_sum,
                                             int* counts) {
  if (!dec || !out_tokens || !out_n || !ms_sum || !counts) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] {
    *out_n = decoder_round_impl(dec, k, out_tokens, true);
    Profiler* pr = dec->profilers.at(graph_key(dec, k)).get();
    for (int i = 0; i < PK_SLOTS; ++i) {
      ms_sum[i] = 0.f;
      counts[i] = 0;
    }
    for (auto& m : pr->marks) {
      float ms = 0.f;
      CUDA_TRY(cudaEventElapsedTime(&ms, m.second.first, m.second.second));
      ms_sum[m.first] += ms;
      counts[m.first] += 1;
    }
  });
}

extern "C" wc_status wc_decoder_state(const wc_decoder* dec, int* n, int* drafter_len) {
  if (!dec) return WC_ERR_INVALID;
  RoundState s;
  if (cudaMemcpy(&s, dec->st, offsetof(RoundState, tokens), cudaMemcpyDeviceToHost) != cudaSuccess) return WC_ERR_CUDA;
  if (n) *n = s.n;
  if (drafter_len) *drafter_len = s.dc_len;
  return WC_OK;
}

extern "C" wc_kv* wc_decoder_target_cache(wc_decoder* dec) { return dec ? dec->tkv : nullptr; }
extern "C" wc_kv* wc_decoder_drafter_cache(wc_decoder* dec) { return dec ? dec->dkv : nullptr; }

extern "C" wc_status wc_decoder_last_round_ms(const wc_decoder* dec, float* ms) {
  if (!dec || !ms) return WC_ERR_INVALID;
  *ms = dec->last_ms;
  return WC_OK;
}

// ---- test and measurement support: device-state snapshots and the last sampled round's logits
namespace {
void* root_buf(wc_decoder* dec, int i) {
  void* b[5] = {dec->root_out, dec->root_fb, dec->xf_root, dec->xf_fb, dec->ss_fb};
  return b[i];
}
}  // namespace

extern "C" wc_status wc_decoder_save_state(wc_decoder* dec) {
  if (!dec) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] {
    if (!dec->prefilled) fail(WC_ERR_INVALID, "prefill before saving the decoder state");
    wc_ctx* ctx = dec->ctx;
    size_t total = 0;
    for (size_t b : dec->root_bytes) total += b;
    if (!dec->saved_st) {
      dec->saved_st = static_cast<RoundState*>(dalloc(sizeof(RoundState)));
      dec->saved_root = static_cast<unsigned char*>(dalloc(total));
    }
    CUDA_TRY(cudaMemcpyAsync(dec->saved_st, dec->st, sizeof(RoundState), cudaMemcpyDeviceToDevice, ctx->stream));
    size_t off = 0;
    for (int i = 0; i < 5; ++i) {
      CUDA_TRY(cudaMemcpyAsync(dec->saved_root + off, root_buf(dec, i), dec->root_bytes[i], cudaMemcpyDeviceToDevice,
                               ctx->stream));
      off += dec->root_bytes[i];
    }
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    dec->saved_host_n = dec->host_n;
  });
}

extern "C" wc_status wc_decoder_restore_state(wc_decoder* dec) {
  if (!dec) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] {
    if (dec->saved_host_n < 0) fail(WC_ERR_INVALID, "no saved decoder state");
    wc_ctx* ctx = dec->ctx;
    // everything up to the random state; the counter base keeps running
    CUDA_TRY(cudaMemcpyAsync(dec->st, dec->saved_st, offsetof(RoundState, rng), cudaMemcpyDeviceToDevice,
                             ctx->stream));
    size_t off = 0;
    for (int i = 0; i < 5; ++i) {
      CUDA_TRY(cudaMemcpyAsync(root_buf(dec, i), dec->saved_root + off, dec->root_bytes[i], cudaMemcpyDeviceToDevice,
                               ctx->stream));
      off += dec->root_bytes[i];
    }
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    dec->host_n = dec->saved_host_n;
  });
}

extern "C" wc_status wc_decoder_round_logits(wc_decoder* dec, int k, float* zt, float* zd, int* tokens,
                                             unsigned long long* rng) {
  if (!dec) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] {
    if (!dec->sampled) fail(WC_ERR_INVALID, "the last rounds were not sampled");
    if (k < 1 || k > dec->max_k) fail(WC_ERR_INVALID, "chain length outside 1..max_k");
    wc_ctx* ctx = dec->ctx;
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    if (zt) CUDA_TRY(cudaMemcpy(zt, dec->zt, sizeof(float) * size_t(k + 1) * dec->t->cfg.vocab, cudaMemcpyDeviceToHost));
    if (zd) CUDA_TRY(cudaMemcpy(zd, dec->zd, sizeof(float) * size_t(k) * dec->d->head_rows, cudaMemcpyDeviceToHost));
    if (tokens) CUDA_TRY(cudaMemcpy(tokens, dec->st->tokens, sizeof(int) * (k + 1), cudaMemcpyDeviceToHost));
    if (rng) {
      CUDA_TRY(cudaMemcpy(rng, dec->st->rng, sizeof(unsigned long long) * 2, cudaMemcpyDeviceToHost));
      rng[1] -= kRngRoundStride;  // the base the last round drew from
    }
  });
}

extern "C" wc_status wc_decoder_draft_proposals(wc_decoder* dec, int k, int* tokens, float* logits) {
  if (!dec) return WC_ERR_INVALID;
  return guard(dec->ctx, [&] {
    if (k < 1 || k > dec->max_k) fail(WC_ERR_INVALID, "chain length outside 1..max_k");
    if (dec->sampled) fail(WC_ERR_INVALID, "sampled rounds rank perturbed logits; read wc_decoder_round_logits");
    CUDA_TRY(cudaStreamSynchronize(dec->ctx->stream));
    unsigned long long keys[MAXK];
    CUDA_TRY(cudaMemcpy(keys, dec->st->draft_keys, sizeof(unsigned long long) * k, cudaMemcpyDeviceToHost));
    for (int i = 0; i < k; ++i) {
      // argmax_key layout (common.cuh): order-preserving float bits above the inverted row index
      const uint32_t row = 0xFFFFFFFFu - uint32_t(keys[i] & 0xFFFFFFFFull);
      uint32_t u = uint32_t(keys[i] >> 32);
      u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
      int tok = int(row);
      if (dec->d->vocab_map) CUDA_TRY(cudaMemcpy(&tok, dec->d->vocab_map + row, sizeof(int), cudaMemcpyDeviceToHost));
      if (tokens) tokens[i] = tok;
      if (logits) std::memcpy(logits + i, &u, sizeof(float));
    }
  });
}

// ============================================================================ autoregressive baseline

namespace {
__global__ void ar_advance_kernel(RoundState* st, int* out) {
  if (threadIdx.x != 0) return;
  const int tok = int(argmax_key_index(st->keys[0]));
  st->x_n = tok;
  st->n += 1;
  st->keys[0] = 0ull;
  st->rng[1] += kRngRoundStride;  // sampled steps: the next step's counter block
  out[0] = tok;
}
}  // namespace

extern "C" wc_status wc_generate_autoregressive(wc_target* t, const int* prompt, int n, int max_new,
                                                const wc_sampling_params* sp, const int* eos, int n_eos,
                                                int max_context, int* out_tokens, int* out_n, wc_gen_stats* stats) {
  if (!t || !prompt || !out_tokens || !out_n || n < 1 || max_new < 1) return WC_ERR_INVALID;
  return guard(t->ctx, [&] {
    Pick pick_;
    const bool smp = sampling_on(sp);
    wc_ctx* ctx = t->ctx;
    const int Ht = t->cfg.hidden;
    const int cap = std::max(max_context, n + max_new + 1);
    wc_gen_stats s{};
    s.prompt_tokens = n;
    std::set<int> eset(eos, eos + (eos ? n_eos : 0));
    const double t0 = now_s();
    std::unique_ptr<wc_kv, void (*)(wc_kv*)> kv(kv_new(ctx, t->cfg.layers, t->cfg.kv_heads, t->cfg.head_dim, cap,
                                                      t->dtype),
                                               wc_kv_destroy);
    RoundState* st = static_cast<RoundState*>(dalloc(sizeof(RoundState)));
    int* d_tok = static_cast<int*>(dalloc(sizeof(int) * n));
    int* d_out = static_cast<int*>(dalloc(sizeof(int) * 4));
    float* h = static_cast<float*>(dalloc(sizeof(float) * GEMV_MAXL * Ht));
    const bool warp = smp && warping_on(sp);
    float* zw = warp ? static_cast<float*>(dalloc(sizeof(float) * t->cfg.vocab)) : nullptr;  // warped draws
    RowWarp* rw = warp ? static_cast<RowWarp*>(dalloc(sizeof(RowWarp))) : nullptr;
    struct FreeW {
      void* a[2];
      ~FreeW() {
        for (void* p : a) dfree(p);
      }
    } frw{{zw, rw}};
    // the step's draw: plain argmax, Gumbel-max in the head, or the warped draw from logits
    auto head_draw = [&](const float* hrow, const XIn* hx) {
      if (warp) {
        if (hx) target_head(t, *hx, 1, nullptr, 1, st->keys + 1, zw, &st->err);
        else target_head_rows(t, hrow, 1, st->keys + 1, zw, &st->err);
        warped_draw(ctx, st, zw, 1, t->cfg.vocab, rw, st->keys);
      } else if (hx) {
        target_head(t, *hx, 1, nullptr, 1, st->keys, nullptr, &st->err, smp ? &pick_ : nullptr);
      } else {
        target_head_rows(t, hrow, 1, st->keys, nullptr, &st->err, smp ? &pick_ : nullptr);
      }
    };
    cudaGraphExec_t exec = nullptr;
    struct Free {
      void* a[4];
      cudaGraphExec_t* e;
      ~Free() {
        if (*e) cudaGraphExecDestroy(*e);
        for (void* p : a) dfree(p);
      }
    } fr{{st, d_tok, d_out, h}, &exec};
    CUDA_TRY(cudaMemsetAsync(st, 0, sizeof(RoundState), ctx->stream));
    seed_rounds(ctx, st, sp, smp);
    pick_.temperature = &st->temperature;  // spec.py:377-397 samples each step from probs_from_logits
    pick_.rng = st->rng;
    CUDA_TRY(cudaMemcpyAsync(d_tok, prompt, sizeof(int) * n, cudaMemcpyHostToDevice, ctx->stream));
    for (int i = 0; i < n; ++i)
      if (prompt[i] < 0 || prompt[i] >= t->cfg.vocab) fail(WC_ERR_INVALID, "prompt token id out of range");
    const float* last = prefill_gemm_forward(t, kv.get(), d_tok, n, 0, nullptr);
    if (last) head_draw(last, nullptr);
    for (int r0 = 0; r0 < n && !last; r0 += GEMV_MAXL) {
      const int rows = std::min(GEMV_MAXL, n - r0);
      Rows r;
      r.L = rows;
      r.L_max = rows;
      r.n_add = r0;
      const XIn in0 = target_embed(t, r, d_tok + r0, nullptr, nullptr, h, &st->err);
      target_layers(t, kv.get(), r, in0, h, nullptr, &st->err);
      if (r0 + rows == n)
        head_draw(h + size_t(rows - 1) * Ht, nullptr);
    }
    // st->n = n - 1 so that the first advance makes it n while emitting the first token
    RoundState init{};
    init.n = n - 1;
    CUDA_TRY(cudaMemcpyAsync(st, &init, offsetof(RoundState, err), cudaMemcpyHostToDevice, ctx->stream));
    ar_advance_kernel<<<1, 32, 0, ctx->stream>>>(st, d_out);
    check_launch(ctx, "ar advance");
    int* hout = nullptr;
    CUDA_TRY(cudaMallocHost(&hout, sizeof(int) * 2));
    std::unique_ptr<int, cudaError_t (*)(void*)> hguard(hout, cudaFreeHost);
    CUDA_TRY(cudaMemcpyAsync(hout, d_out, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    int x = hout[0];
    s.t_prefill = now_s() - t0;
    int m = 0;
    out_tokens[m++] = x;
    uint64_t per = 0;
    while (m < max_new && !eset.count(x)) {
      if (!exec) {
        cudaGraph_t g = nullptr;
        CUDA_TRY(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
        ctx->capturing = true;
        ctx->capture_launches = 0;
        try {
          Rows r;
          r.stable = true;
          r.L = 1;
          r.L_max = 1;
          r.n_dev = &st->n;
          const XIn in0 = target_embed(t, r, nullptr, st, nullptr, h, &st->err);
          const XIn hx = target_layers(t, kv.get(), r, in0, h, nullptr, &st->err);
          head_draw(nullptr, &hx);
          ar_advance_kernel<<<1, 32, 0, ctx->stream>>>(st, d_out);
          check_launch(ctx, "ar advance");
        } catch (...) {
          ctx->capturing = false;
          cudaStreamEndCapture(ctx->stream, &g);
          if (g) cudaGraphDestroy(g);
          throw;
        }
        ctx->capturing = false;
        CUDA_TRY(cudaStreamEndCapture(ctx->stream, &g));
        const cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) fail(WC_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
        per = ctx->capture_launches;
      }
      CUDA_TRY(cudaGraphLaunch(exec, ctx->stream));
      ctx->launches += per;
      CUDA_TRY(cudaMemcpyAsync(hout, d_out, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
      CUDA_TRY(cudaMemcpyAsync(hout + 1, &st->err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
      CUDA_TRY(cudaStreamSynchronize(ctx->stream));
      if (hout[1]) {
        CUDA_TRY(cudaMemset(ctx->gv_counters, 0, sizeof(int) * ctx->gv_counters_n));
        CUDA_TRY(cudaMemset(ctx->as_counters, 0, sizeof(int) * AS_MAXHK));
        fail(WC_ERR_DEVICE, "device error flag " + std::to_string(hout[1]));
      }
      x = hout[0];
      out_tokens[m++] = x;
    }
    s.t_total = now_s() - t0;
    s.new_tokens = m;
    s.rounds = m - 1;
    *out_n = m;
    if (stats) *stats = s;
  });
}

// ============================================================================ batched tree verification

namespace {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || !p || q != cudaDriverEntryPointSuccess)
      fail(WC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D bf16 row-major [rows][K] operand, box of `box_rows` rows x 64 columns, 128-byte swizzle.
CUtensorMap tmap_bf16(const void* base, int rows, int K, int box_rows) {
  if (reinterpret_cast<uintptr_t>(base) % 16 || K % 8 || rows < 1 || K < 1)
    fail(WC_ERR_INVALID, "GEMM operand: 16-byte aligned base and K a multiple of 8 required");
  CUtensorMap m;
  const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(K) * 2};
  const cuuint32_t box[2] = {cuuint32_t(TC_BK), cuuint32_t(box_rows)};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = encode_tiled()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                                    box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail(WC_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return m;
}

bool tc_ready(wc_ctx* ctx) {
  static std::set<int> done;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(ctx->device)) return true;
  CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(gemm_tc_smem<128>())));
  CUDA_TRY(cudaFuncSetAttribute(gemm_tc_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(gemm_tc_smem<256>())));
  CUDA_TRY(cudaFuncSetAttribute(gemm_tcp_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(gemm_tc_smem<128>())));
  CUDA_TRY(cudaFuncSetAttribute(gemm_tcp_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(gemm_tc_smem<256>())));
  CUDA_TRY(cudaFuncSetAttribute(tree_attention_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(tree_attn_smem<128>())));
  CUDA_TRY(cudaFuncSetAttribute(tree_attention_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(tree_attn_smem<64>())));
  done.insert(ctx->device);
  return true;
}

// C = A . B^T on the tensor cores; A [M][K] and B [N][K] bf16 row-major behind tensor maps.
void launch_gemm_tc(wc_ctx* ctx, const CUtensorMap& ta, const CUtensorMap& tb, GemmTc p, int BN) {
  tc_ready(ctx);
  if (!p.err) p.err = ctx->d_err;
  if (p.M < 1 || p.N < 1 || p.K < 1 || p.K % TC_BK) fail(WC_ERR_INVALID, "GEMM: K must be a multiple of 64");
  if (p.epi == TC_SWIGLU && p.N % BN) fail(WC_ERR_INVALID, "GEMM SwiGLU: N must be a multiple of the tile");
  const dim3 grid((p.M + TC_BM - 1) / TC_BM, (p.N + BN - 1) / BN);
  static const bool persistent = [] {
    const char* e = std::getenv("WC_GEMM_PERSIST");
    return !e || std::atoi(e) != 0;
  }();
  if (persistent) {
    const int tiles = int(grid.x * grid.y), blocks = std::min(tiles, ctx->num_sms);
    if (BN == 256)
      launch_ex(ctx, "gemm_tcp", gemm_tcp_kernel<256>, dim3(blocks), dim3(TC_THREADS), gemm_tc_smem<256>(), true, 1,
                ta, tb, p);
    else
      launch_ex(ctx, "gemm_tcp", gemm_tcp_kernel<128>, dim3(blocks), dim3(TC_THREADS), gemm_tc_smem<128>(), true, 1,
                ta, tb, p);
  } else if (BN == 256) {
    launch_ex(ctx, "gemm_tc", gemm_tc_kernel<256>, grid, dim3(TC_THREADS), gemm_tc_smem<256>(), true, 1, ta, tb, p);
  } else {
    launch_ex(ctx, "gemm_tc", gemm_tc_kernel<128>, grid, dim3(TC_THREADS), gemm_tc_smem<128>(), true, 1, ta, tb, p);
  }
}

GemmTc gemm_tc_params(int M, int N, int K, int epi) {
  GemmTc p;
  std::memset(&p, 0, sizeof(p));
  p.M = M;
  p.N = N;
  p.K = K;
  p.epi = epi;
  return p;
}

// A GEMM weight: row-major bf16 copy of a projection, with its tensor map.
struct TcWeight {
  uint16_t* w = nullptr;
  int rows = 0, K = 0, BN = 256;
  CUtensorMap map;
};

TcWeight tc_weight_from(wc_ctx* ctx, const Lin& l, int BN) {
  if (l.dtype != WC_BF16) fail(WC_ERR_UNSUPPORTED, "batched verification needs a bf16 target");
  // several input segments read as one K when none of them is padded (the tiled layout is then
  // the same as one segment's)
  for (int sg = 0; sg < l.nseg; ++sg)
    if (l.seg_len[sg] % GV_COLS) fail(WC_ERR_UNSUPPORTED, "GEMM weight: a padded input segment");
  if (l.Kp % TC_BK) fail(WC_ERR_UNSUPPORTED, "GEMM weight: K a multiple of 64");
  TcWeight t;
  t.rows = l.group == 2 ? 2 * l.N : l.N;
  t.K = l.Kp;
  t.BN = BN;
  if (l.group == 2 && l.N % (BN / 2)) fail(WC_ERR_UNSUPPORTED, "SwiGLU GEMM weight: intermediate % (tile / 2) != 0");
  t.w = static_cast<uint16_t*>(dalloc(size_t(t.rows) * t.K * 2));
  detile_rows_kernel<<<grid_for(size_t(t.rows) * t.K), 256, 0, ctx->stream>>>(
      static_cast<const uint16_t*>(l.w), l.Kp / 16, l.group, BN / 2, t.rows, t.K, t.w);
  check_launch(ctx, "detile");
  t.map = tmap_bf16(t.w, t.rows, t.K, BN);
  return t;
}

}  // namespace

struct wc_batch {
  wc_ctx* ctx = nullptr;
  wc_target* t = nullptr;
  int B = 0, nodes_max = 0, cap = 0, M_max = 0;
  int dl = 0, dHk = 0, dD = 0;  // drafter cache shape (compacted with the target's)
  uint16_t *K = nullptr, *V = nullptr, *dK = nullptr, *dV = nullptr;
  int* lens = nullptr;
  std::vector<int> host_lens;
  struct Layer {
    TcWeight qkv, o, gu, down;
  };
  std::vector<Layer> lw;
  TcWeight head;
  float *h = nullptr, *qkv = nullptr, *logits = nullptr;
  uint16_t *a = nullptr, *q = nullptr, *att = nullptr, *act = nullptr;
  int *tok = nullptr, *par = nullptr, *dep = nullptr, *keep = nullptr, *nkeep = nullptr, *am = nullptr;
  unsigned long long* keys = nullptr;
  int maxkeep_alloc = 0;
  size_t logits_rows = 0;
  int nsplit = 1;  // attention key-range slices (WC_TA_SPLIT; one measured fastest at C5)
  bool own_kv = true;  // false: K / V belong to a single-request cache (prompt forward)
  float *part_o = nullptr, *part_ml = nullptr;
};

namespace {

size_t batch_layer_elems(const wc_batch* b) { return size_t(b->B) * b->cap * b->t->cfg.kv_heads * b->t->cfg.head_dim; }

__global__ void keys_to_ids_kernel(const unsigned long long* keys, int n, int* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = int(argmax_key_index(keys[i]));
}

__global__ void fill_normal_bf16_kernel(uint16_t* x, size_t n, uint64_t seed) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    const uint4 r = philox4x32_10(i, seed);
    // Box-Muller on two 24-bit uniforms in (0, 1)
    const float u1 = (float(r.x >> 8) + 0.5f) * (1.0f / 16777216.0f), u2 = float(r.y >> 8) * (1.0f / 16777216.0f);
    x[i] = f32_to_bf16_bits(sqrtf(-2.f * logf(u1)) * cospif(2.f * u2));
  }
}

// The verify forward of rows M = nreq * nodes (tokens / parents / depths already on the
// device): embeddings, every layer (GEMMs on the tensor cores, per-row q/k norm + RoPE +
// K/V append at slots lens[r] + i, tree attention), final norm and head (argmax keys, and
// fp32 logits when `logits` is set).
void batch_forward(wc_batch* b, int nreq, int nodes, bool logits, bool causal = false, const TapOut* taps = nullptr,
                   bool head = true) {
  wc_ctx* ctx = b->ctx;
  wc_target* t = b->t;
  const auto& c = t->cfg;
  const int M = nreq * nodes, H = c.hidden, D = c.head_dim, Hq = c.heads, Hk = c.kv_heads, I = c.intermediate;
  const int NQKV = (Hq + 2 * Hk) * D;
  int* err = ctx->d_err;
  const CUtensorMap ta_a = tmap_bf16(b->a, M, H, TC_BM);
  const CUtensorMap ta_att = tmap_bf16(b->att, M, Hq * D, TC_BM);
  const CUtensorMap ta_act = tmap_bf16(b->act, M, I, TC_BM);
  for (int l = 0; l < c.layers; ++l) {
    const TLayer& Ly = t->layers[l];
    const wc_batch::Layer& W = b->lw[l];
    RowNormParams rn;
    std::memset(&rn, 0, sizeof(rn));
    rn.x = l == 0 ? nullptr : b->h;
    rn.tokens = l == 0 ? b->tok : nullptr;
    rn.table = t->embed;
    rn.vocab = c.vocab;
    rn.h_copy = b->h;
    rn.H = H;
    rn.w = Ly.in_norm;
    rn.eps = c.eps;
    rn.out = b->a;
    rn.M = M;
    rn.err = err;
    launch_ex(ctx, "row norm", row_norm_bf16_kernel, dim3(M), dim3(256), 0, true, 1, rn);
    GemmTc g = gemm_tc_params(M, NQKV, H, TC_STORE);
    g.c = b->qkv;
    g.ldc = NQKV;
    prof_begin(ctx, PK_QKV);
    launch_gemm_tc(ctx, ta_a, W.qkv.map, g, W.qkv.BN);
    prof_end(ctx, PK_QKV);
    QkvPostParams qp;
    std::memset(&qp, 0, sizeof(qp));
    qp.qkv = b->qkv;
    qp.nodes = nodes;
    qp.Hq = Hq;
    qp.Hk = Hk;
    qp.D = D;
    qp.lens = b->lens;
    qp.depth = b->dep;
    qp.q_norm = Ly.q_norm;
    qp.k_norm = Ly.k_norm;
    qp.eps = c.eps;
    qp.rope = t->rope->ptr;
    qp.max_pos = t->rope->max_pos;
    qp.q = b->q;
    qp.K = b->K + size_t(l) * batch_layer_elems(b);
    qp.V = b->V + size_t(l) * batch_layer_elems(b);
    qp.cap = b->cap;
    qp.err = err;
    launch_ex(ctx, "qkv post", qkv_post_kernel, dim3(M), dim3(128), 0, true, 1, qp);
    TreeAttnParams ap;
    std::memset(&ap, 0, sizeof(ap));
    ap.q = b->q;
    ap.K = qp.K;
    ap.V = qp.V;
    ap.cap = b->cap;
    ap.lens = b->lens;
    ap.parents = b->par;
    ap.nodes = nodes;
    ap.Hq = Hq;
    ap.Hk = Hk;
    ap.scale = 1.f / std::sqrt(float(D));
    ap.out = b->att;
    ap.nsplit = causal ? 1 : b->nsplit;
    ap.causal = causal ? 1 : 0;
    ap.part_o = b->part_o;
    ap.part_ml = b->part_ml;
    ap.err = err;
    const int gz = causal ? (nodes + TA_MAXR / (Hq / Hk) - 1) / (TA_MAXR / (Hq / Hk)) : ap.nsplit;
    prof_begin(ctx, PK_ATTN);
    if (D == 128)
      launch_ex(ctx, "tree attention", tree_attention_kernel<128>, dim3(nreq, Hk, gz), dim3(TA_THREADS),
                tree_attn_smem<128>(), true, 1, ap);
    else
      launch_ex(ctx, "tree attention", tree_attention_kernel<64>, dim3(nreq, Hk, gz), dim3(TA_THREADS),
                tree_attn_smem<64>(), true, 1, ap);
    if (ap.nsplit > 1) {
      if (D == 128)
        launch_ex(ctx, "tree attention merge", tree_attn_merge_kernel<128>, dim3(nreq, Hk), dim3(128), 0, true, 1,
                  ap);
      else
        launch_ex(ctx, "tree attention merge", tree_attn_merge_kernel<64>, dim3(nreq, Hk), dim3(128), 0, true, 1,
                  ap);
    }
    prof_end(ctx, PK_ATTN);
    g = gemm_tc_params(M, H, Hq * D, TC_ADD);
    g.c = b->h;
    g.ldc = H;
    g.r = b->h;
    g.ldr = H;
    prof_begin(ctx, PK_O);
    launch_gemm_tc(ctx, ta_att, W.o.map, g, W.o.BN);
    prof_end(ctx, PK_O);
    rn.x = b->h;
    rn.tokens = nullptr;
    rn.w = Ly.post_norm;
    launch_ex(ctx, "row norm", row_norm_bf16_kernel, dim3(M), dim3(256), 0, true, 1, rn);
    g = gemm_tc_params(M, 2 * I, H, TC_SWIGLU);
    g.cb = b->act;
    g.ldcb = I;
    prof_begin(ctx, PK_GU);
    launch_gemm_tc(ctx, ta_a, W.gu.map, g, W.gu.BN);
    prof_end(ctx, PK_GU);
    g = gemm_tc_params(M, H, I, TC_ADD);
    g.c = b->h;
    g.ldc = H;
    g.r = b->h;
    g.ldr = H;
    prof_begin(ctx, PK_DOWN);
    launch_gemm_tc(ctx, ta_act, W.down.map, g, W.down.BN);
    prof_end(ctx, PK_DOWN);
    if (taps && taps->rows)  // block outputs of the tap layers (qwen3.cpp:103-104)
      for (int f = 0; f < 3; ++f)
        if (t->taps[f] == l)
          CUDA_TRY(cudaMemcpyAsync(taps->rows + f * taps->stride, b->h, sizeof(float) * size_t(M) * H,
                                   cudaMemcpyDeviceToDevice, ctx->stream));
  }
  if (!head) return;
  RowNormParams rn;
  std::memset(&rn, 0, sizeof(rn));
  rn.x = b->h;
  rn.H = H;
  rn.w = t->final_norm;
  rn.eps = c.eps;
  rn.out = b->a;
  rn.M = M;
  rn.err = err;
  launch_ex(ctx, "row norm", row_norm_bf16_kernel, dim3(M), dim3(256), 0, true, 1, rn);
  CUDA_TRY(cudaMemsetAsync(b->keys, 0, sizeof(unsigned long long) * M, ctx->stream));
  GemmTc g = gemm_tc_params(M, c.vocab, H, TC_ARGMAX);
  g.keys = b->keys;
  prof_begin(ctx, PK_HEAD);
  launch_gemm_tc(ctx, ta_a, b->head.map, g, b->head.BN);
  prof_end(ctx, PK_HEAD);
  if (logits) {
    g = gemm_tc_params(M, c.vocab, H, TC_STORE);
    g.c = b->logits;
    g.ldc = c.vocab;
    launch_gemm_tc(ctx, ta_a, b->head.map, g, b->head.BN);
  }
  keys_to_ids_kernel<<<(M + 255) / 256, 256, 0, ctx->stream>>>(b->keys, M, b->am);
  check_launch(ctx, "keys to ids");
}

void batch_check_tree(const int* parents, int nodes, int* depth) {
  for (int i = 0; i < nodes; ++i) {
    const int p = parents[i];
    if (i == 0 ? p != -1 : (p < 0 || p >= i)) fail(WC_ERR_INVALID, "tree parents: parents[0] = -1, 0 <= parents[i] < i");
    depth[i] = i == 0 ? 0 : depth[p] + 1;
  }
}

}  // namespace

extern "C" wc_status wc_gemm_bf16(wc_ctx* ctx, const void* A, const void* B, float* C, int M, int N, int K,
                                  const float* residual) {
  if (!ctx || !A || !B || !C || M < 1 || N < 1 || K < 1) return WC_ERR_INVALID;
  return guard(ctx, [&] {
    const CUtensorMap ta = tmap_bf16(A, M, K, TC_BM);
    const int BN = N >= 2048 ? 256 : 128;
    const CUtensorMap tb = tmap_bf16(B, N, K, BN);
    GemmTc g = gemm_tc_params(M, N, K, residual ? TC_ADD : TC_STORE);
    g.c = C;
    g.ldc = N;
    g.r = residual;
    g.ldr = N;
    launch_gemm_tc(ctx, ta, tb, g, BN);
    check_launch(ctx, "gemm_tc");
  });
}

namespace {

__global__ void iota_kernel(int* x, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = i;
}

// A batch object: GEMM weight copies and activations for max_requests x max_nodes rows, and
// (own_kv) KV arenas of `capacity` rows per request. Without own_kv it serves the prompt
// forward: one request, chain mode, K / V bound per call to a single-request cache.
wc_batch* batch_create_impl(wc_target* t, int max_requests, int max_nodes, int capacity, int drafter_layers,
                            int drafter_kv_heads, int drafter_head_dim, bool own_kv) {
  if (!t->finalized) fail(WC_ERR_INVALID, "target not finalized");
  if (t->dtype != WC_BF16) fail(WC_ERR_UNSUPPORTED, "batched verification runs bf16 targets");
  const auto& c = t->cfg;
  if (own_kv && (max_nodes > TA_MAXN || max_nodes * (c.heads / c.kv_heads) > TA_MAXR))
    fail(WC_ERR_UNSUPPORTED, "tree nodes x query heads per KV head must be <= 64");
  if (c.heads / c.kv_heads > TA_MAXR) fail(WC_ERR_UNSUPPORTED, "too many query heads per KV head");
  if (c.head_dim != 128 && c.head_dim != 64) fail(WC_ERR_UNSUPPORTED, "batched verification: head_dim 64 or 128");
  if (c.hidden % TC_BK || c.intermediate % 128 || (c.heads * c.head_dim) % TC_BK)
    fail(WC_ERR_UNSUPPORTED, "batched verification: hidden, heads x head_dim multiples of 64, intermediate of 128");
  wc_ctx* ctx = t->ctx;
  auto b = std::make_unique<wc_batch>();
  b->ctx = ctx;
  b->t = t;
  b->B = max_requests;
  b->nodes_max = max_nodes;
  b->cap = capacity;
  b->M_max = max_requests * max_nodes;
  b->own_kv = own_kv;
  b->dl = own_kv ? std::max(0, drafter_layers) : 0;
  b->dHk = drafter_kv_heads;
  b->dD = drafter_head_dim;
  if (b->dl > 0 && (b->dHk < 1 || b->dD < 1 || (b->dHk * b->dD) % 8)) fail(WC_ERR_INVALID, "drafter cache shape");
  struct Cleanup {
    wc_batch* b;
    bool armed = true;
    ~Cleanup() {
      if (armed) wc_batch_destroy(b);
    }
  } cleanup{b.get()};
  if (own_kv) {
    const size_t le = batch_layer_elems(b.get());
    b->K = static_cast<uint16_t*>(dalloc(size_t(c.layers) * le * 2));
    b->V = static_cast<uint16_t*>(dalloc(size_t(c.layers) * le * 2));
  }
  if (b->dl) {
    const size_t de = size_t(b->dl) * b->B * b->cap * b->dHk * b->dD;
    b->dK = static_cast<uint16_t*>(dalloc(de * 2));
    b->dV = static_cast<uint16_t*>(dalloc(de * 2));
  }
  b->lens = static_cast<int*>(dalloc(sizeof(int) * b->B));
  CUDA_TRY(cudaMemset(b->lens, 0, sizeof(int) * b->B));
  b->host_lens.assign(b->B, 0);
  for (const TLayer& Ly : t->layers) {
    wc_batch::Layer W;
    W.qkv = tc_weight_from(ctx, Ly.qkv, 256);
    W.o = tc_weight_from(ctx, Ly.o, 128);
    W.gu = tc_weight_from(ctx, Ly.gu, 256);
    W.down = tc_weight_from(ctx, Ly.down, 128);
    b->lw.push_back(W);
  }
  if (own_kv) b->head = tc_weight_from(ctx, t->head, 256);
  const int M = b->M_max, H = c.hidden, NQKV = (c.heads + 2 * c.kv_heads) * c.head_dim;
  b->h = static_cast<float*>(dalloc(sizeof(float) * size_t(M) * H));
  b->qkv = static_cast<float*>(dalloc(sizeof(float) * size_t(M) * NQKV));
  b->a = static_cast<uint16_t*>(dalloc(2 * size_t(M) * H));
  b->q = static_cast<uint16_t*>(dalloc(2 * size_t(M) * c.heads * c.head_dim));
  b->att = static_cast<uint16_t*>(dalloc(2 * size_t(M) * c.heads * c.head_dim));
  b->act = static_cast<uint16_t*>(dalloc(2 * size_t(M) * c.intermediate));
  for (int** pp : {&b->tok, &b->par, &b->dep, &b->am}) *pp = static_cast<int*>(dalloc(sizeof(int) * M));
  b->keys = static_cast<unsigned long long*>(dalloc(sizeof(unsigned long long) * M));
  if (!own_kv) {  // chain mode: node i sits at depth i
    iota_kernel<<<(M + 255) / 256, 256, 0, ctx->stream>>>(b->dep, M);
    check_launch(ctx, "iota");
  }
  if (const char* e = std::getenv("WC_TA_SPLIT")) b->nsplit = std::max(1, std::min(8, std::atoi(e)));
  if (own_kv && b->nsplit > 1) {
    const size_t rows = size_t(b->B) * c.kv_heads * b->nsplit * TA_MAXR;
    b->part_o = static_cast<float*>(dalloc(sizeof(float) * rows * c.head_dim));
    b->part_ml = static_cast<float*>(dalloc(sizeof(float) * rows * 2));
  }
  b->maxkeep_alloc = max_nodes;
  b->keep = static_cast<int*>(dalloc(sizeof(int) * size_t(b->B) * max_nodes));
  b->nkeep = static_cast<int*>(dalloc(sizeof(int) * b->B));
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  cleanup.armed = false;
  return b.release();
}

constexpr int kPrefillChunk = 1024;  // prompt rows per GEMM pass

bool prefill_gemm_ok(const wc_target* t) {
  static const bool on = [] {
    const char* e = std::getenv("WC_PREFILL_GEMM");
    return !e || std::atoi(e) != 0;
  }();
  const auto& c = t->cfg;
  return on && t->dtype == WC_BF16 && (c.head_dim == 128 || c.head_dim == 64) && c.hidden % TC_BK == 0 &&
         c.intermediate % 128 == 0 && (c.heads * c.head_dim) % TC_BK == 0 && c.heads / c.kv_heads <= TA_MAXR;
}

const float* prefill_gemm_forward(wc_target* t, wc_kv* kv, const int* tokens_dev, int n, int start, const TapOut* to) {
  if (!prefill_gemm_ok(t) || kv->dtype != WC_BF16 || n < 1) return nullptr;
  if (start + n > kv->cap) fail(WC_ERR_CAPACITY, "prompt longer than the cache");
  wc_ctx* ctx = t->ctx;
  if (!t->pf) t->pf = batch_create_impl(t, 1, kPrefillChunk, 0, 0, 0, 0, false);
  wc_batch* b = t->pf;
  b->K = static_cast<uint16_t*>(kv->K);  // [layer][kv_head][capacity][head_dim] = one request's arena
  b->V = static_cast<uint16_t*>(kv->V);
  b->cap = kv->cap;
  const int H = t->cfg.hidden;
  int rows = 0;
  for (int r0 = 0; r0 < n; r0 += kPrefillChunk) {
    rows = std::min(kPrefillChunk, n - r0);
    const int len = start + r0;
    CUDA_TRY(cudaMemcpyAsync(b->lens, &len, sizeof(int), cudaMemcpyHostToDevice, ctx->stream));
    CUDA_TRY(cudaMemcpyAsync(b->tok, tokens_dev + r0, sizeof(int) * rows, cudaMemcpyDeviceToDevice, ctx->stream));
    TapOut tc;
    if (to && to->rows) {
      tc.rows = to->rows + size_t(r0) * H;
      tc.stride = to->stride;
    }
    batch_forward(b, 1, rows, false, true, &tc, false);
  }
  return b->h + size_t(rows - 1) * H;
}

}  // namespace

struct DrafterGemm {
  std::vector<TcWeight> qkv, o, gu, down;
  TcWeight fc;
  int M = 0;
  float *h = nullptr, *qkv_out = nullptr;
  uint16_t *ab = nullptr, *a = nullptr, *q = nullptr, *att = nullptr, *act = nullptr;
  int *lens = nullptr, *dep = nullptr;
};

namespace {

void drafter_gemm_free(wc_drafter* d) {
  DrafterGemm* g = d->pg;
  if (!g) return;
  auto drop = [](TcWeight& w) { dfree(w.w); };
  drop(g->fc);
  for (auto* v : {&g->qkv, &g->o, &g->gu, &g->down})
    for (auto& w : *v) drop(w);
  for (void* p : {(void*)g->h, (void*)g->qkv_out, (void*)g->ab, (void*)g->a, (void*)g->q, (void*)g->att,
                  (void*)g->act, (void*)g->lens, (void*)g->dep})
    dfree(p);
  delete g;
  d->pg = nullptr;
}

bool drafter_gemm_ok(const wc_drafter* d) {
  static const bool on = [] {
    const char* e = std::getenv("WC_PREFILL_GEMM");
    return !e || std::atoi(e) != 0;
  }();
  const auto& c = d->cfg;
  return on && d->dtype == WC_BF16 && (c.head_dim == 128 || c.head_dim == 64) && c.window == 0 &&
         c.num_features == 3 && c.hidden % GV_COLS == 0 && c.target_hidden % GV_COLS == 0 &&
         c.intermediate % 128 == 0 && (c.heads * c.head_dim) % TC_BK == 0 && c.heads / c.kv_heads <= TA_MAXR;
}

const float* drafter_prefill_gemm(wc_drafter* d, wc_kv* kv, const int* tokens_dev, int n, int start,
                                  const float* taps, size_t tstride) {
  if (!drafter_gemm_ok(d) || kv->dtype != WC_BF16 || n < 1) return nullptr;
  wc_ctx* ctx = d->ctx;
  if (!tc_ready(ctx)) return nullptr;
  if (start + n > kv->cap) fail(WC_ERR_CAPACITY, "prompt longer than the drafter cache");
  const auto& c = d->cfg;
  const int H = c.hidden, Ht = c.target_hidden, D = c.head_dim, Hq = c.heads, Hk = c.kv_heads, I = c.intermediate;
  const int NQKV = (Hq + 2 * Hk) * D, rep = Hq / Hk;
  if (!d->pg) {  // row-major weight copies (made from the GEMV tiles) and activations for 1024 rows
    auto g = new DrafterGemm();
    d->pg = g;
    g->fc = tc_weight_from(ctx, d->fc, 128);
    for (const DLayer& Ly : d->layers) {
      g->qkv.push_back(tc_weight_from(ctx, Ly.qkv, 256));
      g->o.push_back(tc_weight_from(ctx, Ly.o, 128));
      g->gu.push_back(tc_weight_from(ctx, Ly.gu, 256));
      g->down.push_back(tc_weight_from(ctx, Ly.down, 128));
    }
    const int M = kPrefillChunk;
    g->M = M;
    g->h = static_cast<float*>(dalloc(sizeof(float) * size_t(M) * H));
    g->qkv_out = static_cast<float*>(dalloc(sizeof(float) * size_t(M) * NQKV));
    g->ab = static_cast<uint16_t*>(dalloc(2 * size_t(M) * 3 * Ht));
    g->a = static_cast<uint16_t*>(dalloc(2 * size_t(M) * 2 * H));
    g->q = static_cast<uint16_t*>(dalloc(2 * size_t(M) * Hq * D));
    g->att = static_cast<uint16_t*>(dalloc(2 * size_t(M) * Hq * D));
    g->act = static_cast<uint16_t*>(dalloc(2 * size_t(M) * I));
    g->lens = static_cast<int*>(dalloc(sizeof(int)));
    g->dep = static_cast<int*>(dalloc(sizeof(int) * M));
    iota_kernel<<<(M + 255) / 256, 256, 0, ctx->stream>>>(g->dep, M);
    check_launch(ctx, "iota");
  }
  DrafterGemm* g = d->pg;
  int* err = ctx->d_err;
  const size_t kv_layer = kv->layer_elems();
  int rows = 0;
  for (int r0 = 0; r0 < n; r0 += g->M) {
    rows = std::min(g->M, n - r0);
    const int M = rows;
    const int len = start + r0;
    CUDA_TRY(cudaMemcpyAsync(g->lens, &len, sizeof(int), cudaMemcpyHostToDevice, ctx->stream));
    // fuse (drafter.cpp:75-89): per-tap RMSNorm into one [M][3 Ht] row block, then fc
    RowNormParams rn;
    std::memset(&rn, 0, sizeof(rn));
    rn.H = Ht;
    rn.eps = c.eps;
    rn.M = M;
    rn.ld_out = 3 * Ht;
    rn.err = err;
    for (int f = 0; f < 3; ++f) {
      rn.x = taps + f * tstride + size_t(r0) * Ht;
      rn.w = c.feature_norm ? d->feature_norms[f] : nullptr;
      rn.out = g->ab + size_t(f) * Ht;
      if (!c.feature_norm) fail(WC_ERR_UNSUPPORTED, "tensor-core drafter prefill needs the feature norms");
      launch_ex(ctx, "row norm", row_norm_bf16_kernel, dim3(M), dim3(256), 0, true, 1, rn);
    }
    GemmTc gm = gemm_tc_params(M, H, 3 * Ht, TC_STORE);
    gm.c = g->h;
    gm.ldc = H;
    launch_gemm_tc(ctx, tmap_bf16(g->ab, M, 3 * Ht, TC_BM), g->fc.map, gm, g->fc.BN);
    for (size_t li = 0; li < d->layers.size(); ++li) {
      const DLayer& Ly = d->layers[li];
      const bool aux = Ly.aux_norm != nullptr;
      const int Kq = aux ? 2 * H : H;
      std::memset(&rn, 0, sizeof(rn));
      rn.x = g->h;
      rn.H = H;
      rn.w = Ly.in_norm;
      rn.eps = c.eps;
      rn.out = g->a;
      rn.ld_out = Kq;
      rn.M = M;
      rn.err = err;
      launch_ex(ctx, "row norm", row_norm_bf16_kernel, dim3(M), dim3(256), 0, true, 1, rn);
      if (aux) {  // the token embedding's auxiliary term beside it (drafter.cpp:110-116)
        rn.x = nullptr;
        rn.tokens = tokens_dev + r0;
        rn.table = d->embed;
        rn.vocab = c.vocab;
        rn.w = Ly.aux_norm;
        rn.out = g->a + H;
        launch_ex(ctx, "row norm", row_norm_bf16_kernel, dim3(M), dim3(256), 0, true, 1, rn);
      }
      gm = gemm_tc_params(M, NQKV, Kq, TC_STORE);
      gm.c = g->qkv_out;
      gm.ldc = NQKV;
      launch_gemm_tc(ctx, tmap_bf16(g->a, M, Kq, TC_BM), g->qkv[li].map, gm, g->qkv[li].BN);
      QkvPostParams qp;
      std::memset(&qp, 0, sizeof(qp));
      qp.qkv = g->qkv_out;
      qp.nodes = M;
      qp.Hq = Hq;
      qp.Hk = Hk;
      qp.D = D;
      qp.lens = g->lens;
      qp.depth = g->dep;
      qp.q_norm = Ly.q_norm;
      qp.k_norm = Ly.k_norm;
      qp.eps = c.eps;
      qp.rope = d->rope->ptr;
      qp.max_pos = d->rope->max_pos;
      qp.q = g->q;
      qp.K = static_cast<uint16_t*>(kv->K) + li * kv_layer;
      qp.V = static_cast<uint16_t*>(kv->V) + li * kv_layer;
      qp.cap = kv->cap;
      qp.err = err;
      launch_ex(ctx, "qkv post", qkv_post_kernel, dim3(M), dim3(128), 0, true, 1, qp);
      TreeAttnParams ap;
      std::memset(&ap, 0, sizeof(ap));
      ap.q = g->q;
      ap.K = qp.K;
      ap.V = qp.V;
      ap.cap = kv->cap;
      ap.lens = g->lens;
      ap.parents = g->dep;  // unused in causal mode
      ap.nodes = M;
      ap.Hq = Hq;
      ap.Hk = Hk;
      ap.scale = 1.f / std::sqrt(float(D));
      ap.out = g->att;
      ap.nsplit = 1;
      ap.causal = 1;
      ap.err = err;
      const int gz = (M + TA_MAXR / rep - 1) / (TA_MAXR / rep);
      if (D == 128)
        launch_ex(ctx, "tree attention", tree_attention_kernel<128>, dim3(1, Hk, gz), dim3(TA_THREADS),
                  tree_attn_smem<128>(), true, 1, ap);
      else
        launch_ex(ctx, "tree attention", tree_attention_kernel<64>, dim3(1, Hk, gz), dim3(TA_THREADS),
                  tree_attn_smem<64>(), true, 1, ap);
      gm = gemm_tc_params(M, H, Hq * D, TC_ADD);
      gm.c = g->h;
      gm.ldc = H;
      gm.r = g->h;
      gm.ldr = H;
      launch_gemm_tc(ctx, tmap_bf16(g->att, M, Hq * D, TC_BM), g->o[li].map, gm, g->o[li].BN);
      std::memset(&rn, 0, sizeof(rn));
      rn.x = g->h;
      rn.H = H;
      rn.w = Ly.post_norm;
      rn.eps = c.eps;
      rn.out = g->a;
      rn.M = M;
      rn.err = err;
      launch_ex(ctx, "row norm", row_norm_bf16_kernel, dim3(M), dim3(256), 0, true, 1, rn);
      gm = gemm_tc_params(M, 2 * I, H, TC_SWIGLU);
      gm.cb = g->act;
      gm.ldcb = I;
      launch_gemm_tc(ctx, tmap_bf16(g->a, M, H, TC_BM), g->gu[li].map, gm, g->gu[li].BN);
      gm = gemm_tc_params(M, H, I, TC_ADD);
      gm.c = g->h;
      gm.ldc = H;
      gm.r = g->h;
      gm.ldr = H;
      launch_gemm_tc(ctx, tmap_bf16(g->act, M, I, TC_BM), g->down[li].map, gm, g->down[li].BN);
    }
  }
  return g->h + size_t(rows - 1) * H;
}

// The drafter's auxiliary Q/K/V term per vocabulary token, W_aux . aux_norm(embed(t)), as an fp32
// table [vocab][Q+K+V] (two tcgen05 GEMMs over the bf16 high and low parts of the normalised
// embeddings), and the layer-0 Q/K/V weight of the feature input alone: the decode passes then
// stream half the layer-0 Q/K/V weights, without splitting K, and add the token's table row in the
// GEMV epilogue. bf16 drafters with a hidden size that is a multiple of 512; WC_AUX_TABLE=0 keeps
// the two-segment projection.
void drafter_build_aux_table(wc_drafter* d) {
  static const bool on = [] {
    const char* e = std::getenv("WC_AUX_TABLE");
    return !e || std::atoi(e) != 0;
  }();
  const auto& c = d->cfg;
  if (!on || d->aux_table || d->dtype != WC_BF16 || c.hidden % GV_COLS || d->layers.empty() ||
      !d->layers[0].aux_norm)
    return;
  wc_ctx* ctx = d->ctx;
  if (!tc_ready(ctx)) return;
  DLayer& L0 = d->layers[0];
  const int H = c.hidden, NQKV = L0.qkv.N;
  if (L0.qkv.Np != NQKV || NQKV % 256) return;
  Lin m = make_lin(WC_BF16, NQKV, {H}, 1);
  CUDA_TRY(cudaMemcpy2DAsync(m.w, size_t(H / 16) * 512, L0.qkv.w, size_t(L0.qkv.Kp / 16) * 512, size_t(H / 16) * 512,
                             size_t(L0.qkv.Np / 16), cudaMemcpyDeviceToDevice, ctx->stream));
  TcWeight B = tc_weight_from(ctx, L0.qkv, 256);  // [NQKV][2H] row-major
  float* table = static_cast<float*>(dalloc(sizeof(float) * size_t(c.vocab) * NQKV));
  constexpr int kRows = 4096;
  uint16_t* A = static_cast<uint16_t*>(dalloc(2 * size_t(kRows) * 2 * H));
  for (int r0 = 0; r0 < c.vocab; r0 += kRows) {
    const int M = std::min(kRows, c.vocab - r0);
    for (int lo = 0; lo < 2; ++lo) {
      aux_rows_kernel<<<M, 256, 0, ctx->stream>>>(static_cast<const uint16_t*>(d->embed), d->aux_inv, L0.aux_norm,
                                                  r0, H, lo, A);
      check_launch(ctx, "aux rows");
      GemmTc g = gemm_tc_params(M, NQKV, 2 * H, lo ? TC_ADD : TC_STORE);
      g.c = table + size_t(r0) * NQKV;
      g.ldc = NQKV;
      if (lo) {
        g.r = g.c;
        g.ldr = NQKV;
      }
      launch_gemm_tc(ctx, tmap_bf16(A, M, 2 * H, TC_BM), B.map, g, B.BN);
    }
  }
  CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  dfree(A);
  dfree(B.w);
  L0.qkv_main = m;
  d->aux_table = table;
}

}  // namespace

extern "C" wc_status wc_target_prompt_forward(wc_target* t, wc_kv* cache, const int* tokens_dev, int n, float* taps,
                                              float* last_hidden) {
  if (!t || !cache || !tokens_dev || n < 1) return WC_ERR_INVALID;
  return guard(t->ctx, [&] {
    if (cache->layers != t->cfg.layers || cache->Hk != t->cfg.kv_heads || cache->D != t->cfg.head_dim)
      fail(WC_ERR_INVALID, "cache shape does not match the target");
    TapOut to;
    to.rows = taps;
    to.stride = size_t(n) * t->cfg.hidden;
    const float* last = prefill_gemm_forward(t, cache, tokens_dev, n, cache->n, &to);
    if (!last) fail(WC_ERR_UNSUPPORTED, "the tensor-core prompt forward needs a bf16 target (head_dim 64 / 128)");
    if (last_hidden)
      CUDA_TRY(cudaMemcpyAsync(last_hidden, last, sizeof(float) * t->cfg.hidden, cudaMemcpyDeviceToDevice,
                               t->ctx->stream));
    cache->n += n;
    check_launch(t->ctx, "prompt forward");
  });
}

extern "C" wc_status wc_batch_create(wc_target* t, int max_requests, int max_nodes, int capacity, int drafter_layers,
                                     int drafter_kv_heads, int drafter_head_dim, wc_batch** out) {
  if (!t || !out || max_requests < 1 || max_nodes < 1 || capacity < 2) return WC_ERR_INVALID;
  return guard(t->ctx, [&] {
    *out = batch_create_impl(t, max_requests, max_nodes, capacity, drafter_layers, drafter_kv_heads, drafter_head_dim,
                             true);
  });
}

extern "C" void wc_batch_destroy(wc_batch* b) {
  if (!b) return;
  cudaStreamSynchronize(b->ctx->stream);
  for (auto& W : b->lw)
    for (TcWeight* w : {&W.qkv, &W.o, &W.gu, &W.down}) dfree(w->w);
  dfree(b->head.w);
  if (b->own_kv) {
    dfree(b->K);
    dfree(b->V);
  }
  for (void* p : {(void*)b->dK, (void*)b->dV, (void*)b->lens, (void*)b->h, (void*)b->qkv,
                  (void*)b->logits, (void*)b->a, (void*)b->q, (void*)b->att, (void*)b->act, (void*)b->tok,
                  (void*)b->par, (void*)b->dep, (void*)b->am, (void*)b->keys, (void*)b->keep, (void*)b->nkeep,
                  (void*)b->part_o, (void*)b->part_ml})
    dfree(p);
  delete b;
}

extern "C" wc_status wc_batch_set_prefix(wc_batch* b, int r, const wc_kv* src, int n) {
  if (!b || !src || r < 0 || r >= b->B || n < 0) return WC_ERR_INVALID;
  return guard(b->ctx, [&] {
    const auto& c = b->t->cfg;
    if (src->layers != c.layers || src->Hk != c.kv_heads || src->D != c.head_dim || src->dtype != WC_BF16)
      fail(WC_ERR_INVALID, "source cache shape does not match the target");
    if (n > src->cap || n + b->nodes_max > b->cap) fail(WC_ERR_CAPACITY, "prefix longer than the batch capacity");
    const int D = c.head_dim, Hk = c.kv_heads;
    for (int l = 0; l < c.layers; ++l)
      for (int hk = 0; hk < Hk; ++hk) {  // both arenas are head-major: [Hk][capacity][D] per layer
        const size_t dst = (size_t(l) * batch_layer_elems(b) + (size_t(r) * Hk + hk) * b->cap * D) * 2;
        const size_t so = size_t(hk) * src->cap * D * 2;
        CUDA_TRY(cudaMemcpyAsync(reinterpret_cast<char*>(b->K) + dst, static_cast<const char*>(src->Kl(l)) + so,
                                 size_t(n) * D * 2, cudaMemcpyDeviceToDevice, b->ctx->stream));
        CUDA_TRY(cudaMemcpyAsync(reinterpret_cast<char*>(b->V) + dst, static_cast<const char*>(src->Vl(l)) + so,
                                 size_t(n) * D * 2, cudaMemcpyDeviceToDevice, b->ctx->stream));
      }
    b->host_lens[r] = n;
    CUDA_TRY(cudaMemcpyAsync(b->lens + r, &b->host_lens[r], sizeof(int), cudaMemcpyHostToDevice, b->ctx->stream));
    CUDA_TRY(cudaStreamSynchronize(b->ctx->stream));
  });
}

extern "C" wc_status wc_batch_fill_synthetic(wc_batch* b, int nreq, int n, uint64_t seed) {
  if (!b || nreq < 1 || nreq > b->B || n < 0) return WC_ERR_INVALID;
  return guard(b->ctx, [&] {
    if (n + b->nodes_max > b->cap) fail(WC_ERR_CAPACITY, "prefix longer than the batch capacity");
    const auto& c = b->t->cfg;
    const size_t le = batch_layer_elems(b);
    fill_normal_bf16_kernel<<<148 * 8, 256, 0, b->ctx->stream>>>(b->K, size_t(c.layers) * le, seed);
    fill_normal_bf16_kernel<<<148 * 8, 256, 0, b->ctx->stream>>>(b->V, size_t(c.layers) * le, seed + 1);
    if (b->dl) {
      const size_t de = size_t(b->dl) * b->B * b->cap * b->dHk * b->dD;
      fill_normal_bf16_kernel<<<148 * 8, 256, 0, b->ctx->stream>>>(b->dK, de, seed + 2);
      fill_normal_bf16_kernel<<<148 * 8, 256, 0, b->ctx->stream>>>(b->dV, de, seed + 3);
    }
    check_launch(b->ctx, "fill");
    for (int r = 0; r < nreq; ++r) b->host_lens[r] = n;
    CUDA_TRY(cudaMemcpyAsync(b->lens, b->host_lens.data(), sizeof(int) * nreq, cudaMemcpyHostToDevice, b->ctx->stream));
    CUDA_TRY(cudaStreamSynchronize(b->ctx->stream));
  });
}

namespace {
void batch_verify_impl(wc_batch* b, int nreq, int nodes, const int* tokens, const int* parents, int* out_argmax,
                       float* out_logits);
}

extern "C" wc_status wc_batch_verify(wc_batch* b, int nreq, int nodes, const int* tokens, const int* parents,
                                     int* out_argmax, float* out_logits) {
  if (!b || nreq < 1 || nreq > b->B || nodes < 1 || nodes > b->nodes_max || !tokens || !parents || !out_argmax)
    return WC_ERR_INVALID;
  return guard(b->ctx, [&] { batch_verify_impl(b, nreq, nodes, tokens, parents, out_argmax, out_logits); });
}

extern "C" wc_status wc_batch_verify_profiled(wc_batch* b, int nreq, int nodes, const int* tokens,
                                              const int* parents, int* out_argmax, float* ms_sum, int* counts) {
  if (!b || nreq < 1 || nreq > b->B || nodes < 1 || nodes > b->nodes_max || !tokens || !parents || !out_argmax ||
      !ms_sum || !counts)
    return WC_ERR_INVALID;
  return guard(b->ctx, [&] {
    Profiler pr;
    b->ctx->prof = &pr;
    try {
      batch_verify_impl(b, nreq, nodes, tokens, parents, out_argmax, nullptr);
    } catch (...) {
      b->ctx->prof = nullptr;
      throw;
    }
    b->ctx->prof = nullptr;
    for (int i = 0; i < PK_SLOTS; ++i) {
      ms_sum[i] = 0.f;
      counts[i] = 0;
    }
    for (auto& m : pr.marks) {
      float ms = 0.f;
      CUDA_TRY(cudaEventElapsedTime(&ms, m.second.first, m.second.second));
      ms_sum[m.first] += ms;
      counts[m.first] += 1;
    }
  });
}

namespace {
void batch_verify_impl(wc_batch* b, int nreq, int nodes, const int* tokens, const int* parents, int* out_argmax,
                       float* out_logits) {
  {
    wc_ctx* ctx = b->ctx;
    const auto& c = b->t->cfg;
    const int M = nreq * nodes;
    std::vector<int> depth(M);
    for (int r = 0; r < nreq; ++r) {
      batch_check_tree(parents + size_t(r) * nodes, nodes, depth.data() + size_t(r) * nodes);
      if (b->host_lens[r] + nodes > b->cap) fail(WC_ERR_CAPACITY, "request context exhausted");
      for (int i = 0; i < nodes; ++i) {
        const int tok = tokens[size_t(r) * nodes + i];
        if (tok < 0 || tok >= c.vocab) fail(WC_ERR_INVALID, "token id out of range");
      }
    }
    if (out_logits && b->logits_rows < size_t(M)) {
      CUDA_TRY(cudaStreamSynchronize(ctx->stream));
      dfree(b->logits);
      b->logits = static_cast<float*>(dalloc(sizeof(float) * size_t(M) * c.vocab));
      b->logits_rows = M;
    }
    CUDA_TRY(cudaMemcpyAsync(b->tok, tokens, sizeof(int) * M, cudaMemcpyHostToDevice, ctx->stream));
    CUDA_TRY(cudaMemcpyAsync(b->par, parents, sizeof(int) * M, cudaMemcpyHostToDevice, ctx->stream));
    CUDA_TRY(cudaMemcpyAsync(b->dep, depth.data(), sizeof(int) * M, cudaMemcpyHostToDevice, ctx->stream));
    batch_forward(b, nreq, nodes, out_logits != nullptr);
    CUDA_TRY(cudaMemcpyAsync(out_argmax, b->am, sizeof(int) * M, cudaMemcpyDeviceToHost, ctx->stream));
    if (out_logits)
      CUDA_TRY(cudaMemcpyAsync(out_logits, b->logits, sizeof(float) * size_t(M) * c.vocab, cudaMemcpyDeviceToHost,
                               ctx->stream));
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
    int e = 0;
    CUDA_TRY(cudaMemcpy(&e, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
      CUDA_TRY(cudaMemset(ctx->d_err, 0, sizeof(int)));
      fail(WC_ERR_DEVICE, "device error flag " + std::to_string(e));
    }
  }
}
}  // namespace

extern "C" wc_status wc_batch_commit(wc_batch* b, int nreq, const int* keep, const int* n_keep, int maxkeep) {
  if (!b || nreq < 1 || nreq > b->B || !keep || !n_keep || maxkeep < 1) return WC_ERR_INVALID;
  return guard(b->ctx, [&] {
    wc_ctx* ctx = b->ctx;
    if (maxkeep > b->maxkeep_alloc) fail(WC_ERR_INVALID, "keep lists longer than the tree size");
    for (int r = 0; r < nreq; ++r) {
      const int nk = n_keep[r];
      const int* k = keep + size_t(r) * maxkeep;
      if (nk < 1 || nk > maxkeep || k[0] != 0) fail(WC_ERR_INVALID, "keep lists start at the root (0)");
      for (int i = 1; i < nk; ++i)
        if (k[i] <= k[i - 1] || k[i] >= b->nodes_max) fail(WC_ERR_INVALID, "keep indices must increase within the tree");
      if (b->host_lens[r] + k[nk - 1] >= b->cap) fail(WC_ERR_CAPACITY, "keep index beyond the capacity");
    }
    CUDA_TRY(cudaMemcpyAsync(b->keep, keep, sizeof(int) * size_t(nreq) * maxkeep, cudaMemcpyHostToDevice, ctx->stream));
    CUDA_TRY(cudaMemcpyAsync(b->nkeep, n_keep, sizeof(int) * nreq, cudaMemcpyHostToDevice, ctx->stream));
    const auto& c = b->t->cfg;
    BatchCompactParams p;
    p.K = b->K;
    p.V = b->V;
    p.layers = c.layers;
    p.B = b->B;
    p.cap = b->cap;
    p.Hk = c.kv_heads;
    p.D = c.head_dim;
    p.lens = b->lens;
    p.keep = b->keep;
    p.n_keep = b->nkeep;
    p.maxkeep = maxkeep;
    p.err = ctx->d_err;
    batch_compact_kernel<<<dim3(nreq, c.layers), 128, 0, ctx->stream>>>(p);
    if (b->dl) {
      p.K = b->dK;
      p.V = b->dV;
      p.layers = b->dl;
      p.Hk = b->dHk;
      p.D = b->dD;
      batch_compact_kernel<<<dim3(nreq, b->dl), 128, 0, ctx->stream>>>(p);
    }
    batch_commit_lens_kernel<<<(nreq + 127) / 128, 128, 0, ctx->stream>>>(b->lens, b->nkeep, nreq);
    check_launch(ctx, "batch compact");
    for (int r = 0; r < nreq; ++r) b->host_lens[r] += n_keep[r];
    CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  });
}

extern "C" wc_status wc_batch_lens(const wc_batch* b, int nreq, int* lens) {
  if (!b || !lens || nreq < 1 || nreq > b->B) return WC_ERR_INVALID;
  for (int r = 0; r < nreq; ++r) lens[r] = b->host_lens[r];
  return WC_OK;
}

extern "C" wc_status wc_batch_read_kv(wc_batch* b, int r, int layer, int n, void* k_out, void* v_out) {
  if (!b || r < 0 || r >= b->B || layer < 0 || layer >= b->t->cfg.layers || n < 0 || n > b->cap) return WC_ERR_INVALID;
  return guard(b->ctx, [&] {
    const auto& c = b->t->cfg;
    const int D = c.head_dim, Hk = c.kv_heads;
    CUDA_TRY(cudaStreamSynchronize(b->ctx->stream));
    for (int hk = 0; hk < Hk && n > 0; ++hk) {  // head-major arena -> [n][Hk][D] rows
      const size_t off = (size_t(layer) * batch_layer_elems(b) + (size_t(r) * Hk + hk) * b->cap * D) * 2;
      for (int w = 0; w < 2; ++w) {
        void* dst = w ? v_out : k_out;
        if (!dst) continue;
        CUDA_TRY(cudaMemcpy2D(static_cast<char*>(dst) + size_t(hk) * D * 2, size_t(Hk) * D * 2,
                              reinterpret_cast<char*>(w ? b->V : b->K) + off, size_t(D) * 2, size_t(D) * 2, n,
                              cudaMemcpyDeviceToHost));
      }
    }
  });
}
