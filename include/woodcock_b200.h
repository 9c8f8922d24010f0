/*
 * woodcock_b200: C ABI of the B200-native speculative-decoding round.
 *
 * Drop-in boundary for the reference's C++ core (AtomicBot-ai/woodcock,
 * include/woodcock/{ops,cache,model,drafter,sampling,spec}.h) and for its Python
 * API (python/woodcock/{target,drafter,sampling,spec}.py). Every entry point is
 * plain C: opaque handles, device or host pointers, sizes and a status code.
 *
 * Conventions
 *  - One context per GPU; a context is not thread-safe. All work is enqueued on
 *    the context's stream (set by wc_ctx_create / wc_ctx_set_stream).
 *  - Activation buffers ("_dev" pointers) are caller-owned device memory, row-major
 *    as in the reference (x[L][d], q[L][H][D], K/V[T][Hk][D], mask[L][T], 1 = visible).
 *  - The library owns weights, KV arenas and workspaces behind its handles.
 *  - No function aborts or throws: each returns wc_status; wc_last_error(ctx)
 *    describes the most recent failure. Device-side failures (bounds, timeouts)
 *    are raised through a device error word checked at the round's sync.
 *  - dtype codes: WC_F32 = 0, WC_BF16 = 1.
 */
#ifndef WOODCOCK_B200_H_
#define WOODCOCK_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WC_API __attribute__((visibility("default")))
#else
#define WC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  WC_OK = 0,
  WC_ERR_INVALID = 1,     /* bad argument: shape, dtype, token id, tap index, tree */
  WC_ERR_IO = 2,          /* file missing / unreadable / malformed safetensors or JSON */
  WC_ERR_CUDA = 3,        /* a CUDA runtime call failed */
  WC_ERR_OOM = 4,         /* device allocation failed */
  WC_ERR_CAPACITY = 5,    /* KV arena or workspace capacity exceeded */
  WC_ERR_DEVICE = 6,      /* device-side error flag raised (bounds, bounded wait expired) */
  WC_ERR_UNSUPPORTED = 7  /* configuration the reference also rejects, or not built yet */
} wc_status;

enum { WC_F32 = 0, WC_BF16 = 1 };

typedef struct wc_ctx wc_ctx;
typedef struct wc_weight wc_weight;
typedef struct wc_kv wc_kv;
typedef struct wc_target wc_target;
typedef struct wc_drafter wc_drafter;
typedef struct wc_decoder wc_decoder;

/* ------------------------------------------------------------------ context */
WC_API wc_status wc_ctx_create(int device, void* stream, wc_ctx** out);
WC_API wc_status wc_ctx_set_stream(wc_ctx* ctx, void* stream);
WC_API void wc_ctx_destroy(wc_ctx* ctx);
WC_API const char* wc_last_error(const wc_ctx* ctx);
WC_API wc_status wc_ctx_synchronize(wc_ctx* ctx);
/* number of kernels this context launched since creation (graph replays count each kernel) */
WC_API uint64_t wc_ctx_launch_count(const wc_ctx* ctx);
/* Test support, no counterpart in the reference: launches a kernel whose bounded wait (the helper
 * every pipelined kernel uses) can never be satisfied and gives up after `iterations` tries
 * (1..2^20), raising the timeout bit of the device error word; the next wc_ctx_synchronize then
 * returns WC_ERR_DEVICE and clears the word, and the context stays usable. */
WC_API wc_status wc_ctx_wait_selftest(wc_ctx* ctx, int iterations);

/* ------------------------------------------------------------------ backend ops
 * Device-pointer counterparts of woodcock::ops (include/woodcock/ops.h:11-22,
 * src/backends/cpu_ops.cpp:45-115). A wc_weight replaces woodcock::Tensor
 * (include/woodcock/weights.h:14-24): the library keeps it in its streaming layout. */

/* W[out][in] row-major from `data` (host or device, src_dtype WC_F32/WC_BF16) stored as `dtype`. */
WC_API wc_status wc_weight_create(wc_ctx* ctx, const void* data, int src_dtype, int data_on_device, int out_rows,
                           int in_cols, int dtype, wc_weight** w);
WC_API void wc_weight_destroy(wc_weight* w);
/* ops.h:12  y[L][out] (+)= x[L][in] . W^T */
WC_API wc_status wc_linear(wc_ctx* ctx, const float* x_dev, int L, int in, const wc_weight* W, float* y_dev, int accumulate);
/* ops.h:14  y = x * rsqrt(mean(x^2) + eps) * w per row of length d; x and y may alias */
WC_API wc_status wc_rmsnorm(wc_ctx* ctx, const float* x_dev, float* y_dev, int rows, int d, const float* w_dev, float eps);
/* ops.h:16  rotate-half RoPE on x[L][heads][D] at positions[L] (device) */
WC_API wc_status wc_rope(wc_ctx* ctx, float* x_dev, int L, int heads, int D, const int* positions_dev, float base);
/* ops.h:18  gate = silu(gate) * up */
WC_API wc_status wc_silu_mul(wc_ctx* ctx, float* gate_dev, const float* up_dev, int64_t n);
/* ops.h:20  q[L][H][D]; K,V [T][Hk][D] of kv_dtype; mask[L][T] or NULL; out[L][H][D] */
WC_API wc_status wc_attention(wc_ctx* ctx, const float* q_dev, int L, int H, int Hk, int D, const void* K_dev,
                       const void* V_dev, int kv_dtype, int T, const uint8_t* mask_dev, float* out_dev, float scale);
/* ops.h:22  in-place softmax of one row of n */
WC_API wc_status wc_softmax(wc_ctx* ctx, float* x_dev, int n);
/* first index of the maximum of each of `rows` rows of n (sampling.cpp:47) */
WC_API wc_status wc_argmax_rows(wc_ctx* ctx, const float* x_dev, int rows, int n, int* out_dev);

/* ------------------------------------------------------------------ KV cache
 * include/woodcock/cache.h:9-28. Fixed capacity (no reallocation: rounds are
 * graph-replayed); layout [layer][kv_head][capacity][head_dim] of `dtype`. */
WC_API wc_status wc_kv_create(wc_ctx* ctx, int layers, int kv_heads, int head_dim, int capacity, int dtype, wc_kv** kv);
WC_API void wc_kv_destroy(wc_kv* kv);
WC_API int wc_kv_size(const wc_kv* kv);
WC_API int wc_kv_capacity(const wc_kv* kv);
/* cache.h:16  k, v: [L][kv_heads][head_dim] fp32 device rows, written at [size, size+L) of `layer` */
WC_API wc_status wc_kv_append(wc_kv* kv, int layer, const float* k_dev, const float* v_dev, int L);
WC_API wc_status wc_kv_commit(wc_kv* kv, int L);   /* cache.h:17 */
WC_API wc_status wc_kv_trim_to(wc_kv* kv, int n);  /* cache.h:18 */
/* cache.h:20  keep rows start+keep[i] contiguously at start+i (keep: host array, increasing) */
WC_API wc_status wc_kv_compact(wc_kv* kv, int start, const int* keep, int n_keep);
/* copy rows [0, T) of one layer out as [T][kv_heads][head_dim] fp32 (device) */
WC_API wc_status wc_kv_read(const wc_kv* kv, int layer, int T, float* k_dev, float* v_dev);

/* ------------------------------------------------------------------ target (Qwen3)
 * include/woodcock/model.h:27-52; python/woodcock/target.py:42-116. */
typedef struct {
  int hidden, layers, heads, kv_heads, head_dim, intermediate, vocab;
  float eps, rope_theta;
  int tie_embeddings;
} wc_qwen3_config;

/* Loads HF config.json + *.safetensors from `dir`. taps: 3 block indices, or NULL for
 * the reference default (2, L/2, L-3) (src/core/qwen3.cpp:57). dtype: storage/compute dtype. */
WC_API wc_status wc_target_load(wc_ctx* ctx, const char* dir, const int* taps, int dtype, wc_target** out);
/* Empty target of `cfg`; fill with wc_target_set_tensor (HF tensor names), then wc_target_finalize. */
WC_API wc_status wc_target_create(wc_ctx* ctx, const wc_qwen3_config* cfg, const int* taps, int dtype, wc_target** out);
WC_API wc_status wc_target_set_tensor(wc_target* t, const char* name, const void* data, int src_dtype, int on_device,
                               const int64_t* shape, int ndim);
WC_API wc_status wc_target_finalize(wc_target* t);
WC_API void wc_target_destroy(wc_target* t);
WC_API wc_status wc_target_config(const wc_target* t, wc_qwen3_config* cfg, int* taps3, int* dtype);
/* KV cache shaped for this target (Qwen3::make_cache, model.h:38) */
WC_API wc_status wc_target_make_cache(wc_target* t, int capacity, wc_kv** kv);
/* model.h:37 Qwen3::forward. tokens[L] and positions[L] (NULL = cache size + i) are device
 * int32; mask_dev is [L][size+L] uint8 or NULL (causal). Outputs (each optional, device):
 * logits [L-logits_from][vocab] fp32, argmax [L-logits_from] int32, taps [3][L][hidden] fp32. */
WC_API wc_status wc_target_forward(wc_target* t, wc_kv* cache, const int* tokens_dev, int L, const int* positions_dev,
                            const uint8_t* mask_dev, int logits_from, float* logits_dev, int* argmax_dev,
                            float* taps_dev);

/* ------------------------------------------------------------------ drafter (EAGLE-3)
 * include/woodcock/drafter.h:31-58; python/woodcock/drafter.py:134-229. */
typedef struct {
  int hidden, layers, heads, kv_heads, head_dim, intermediate, vocab, target_hidden, num_features;
  float eps, rope_theta;
  int post_norm, feature_norm, window;
} wc_drafter_config;

/* config.json + model.safetensors (drafter.cpp:18-73). Rejects what the reference rejects. */
WC_API wc_status wc_drafter_load(wc_ctx* ctx, const char* dir, int dtype, wc_drafter** out);
WC_API wc_status wc_drafter_create(wc_ctx* ctx, const wc_drafter_config* cfg, int dtype, wc_drafter** out);
WC_API wc_status wc_drafter_set_tensor(wc_drafter* d, const char* name, const void* data, int src_dtype, int on_device,
                                const int64_t* shape, int ndim);
WC_API wc_status wc_drafter_finalize(wc_drafter* d);
WC_API void wc_drafter_destroy(wc_drafter* d);
WC_API wc_status wc_drafter_config_get(const wc_drafter* d, wc_drafter_config* cfg, int* dtype, int* head_rows);
/* drafter.py:217-229 restrict_vocab: keep head rows ids[0..n) (host int32, ascending not required) */
WC_API wc_status wc_drafter_restrict_vocab(wc_drafter* d, const int* ids, int n);
WC_API wc_status wc_drafter_make_cache(wc_drafter* d, int capacity, wc_kv** kv);
/* drafter.h:41 fuse: taps [num_features][L][target_hidden] -> g [L][hidden] (device fp32) */
WC_API wc_status wc_drafter_fuse(wc_drafter* d, const float* taps_dev, int L, float* g_dev);
/* drafter.h:43 forward: tokens[L], feat [L][hidden]; positions/mask as for the target.
 * hidden_dev (un-normalised residual) and out_dev (RMSNorm(h)) are [L][hidden], each optional. */
WC_API wc_status wc_drafter_forward(wc_drafter* d, wc_kv* cache, const int* tokens_dev, int L, const float* feat_dev,
                             const int* positions_dev, const uint8_t* mask_dev, float* hidden_dev, float* out_dev);
/* drafter.h:49 logits over the head rows (full vocabulary or the restricted rows) for `rows` rows */
WC_API wc_status wc_drafter_logits(wc_drafter* d, const float* out_dev, int rows, float* z_dev);
/* The draft distribution (spec.py:113-125 _draft_dist; drafter.py:204-207 logits): softmax(z / T) over the
 * head rows (the full vocabulary or the restricted rows, in row order) for `rows` rows of drafter output,
 * into probs [rows][head rows] (device fp32). T > 0; the reference drafts greedily with T = 1. */
WC_API wc_status wc_drafter_head_softmax(wc_drafter* d, const float* out_dev, int rows, float temperature,
                                         float* probs_dev);
/* fused head + argmax; token ids are mapped back through the restricted vocabulary (drafter.py:213-215) */
WC_API wc_status wc_drafter_head_argmax(wc_drafter* d, const float* out_dev, int rows, int* token_dev);

/* ------------------------------------------------------------------ acceptance
 * python/woodcock/sampling.py:60-177; src/sampling/sampling.cpp:85-141. Trees are
 * flattened: parents[0] = -1, children in node order = draw order. */
/* sampling.cpp:95-106 verify_tree_greedy on device: argmax[N], tokens[N], parents[N] device int32.
 * out_path [N] (accepted node ids, excluding the root), out_n, out_next: device int32. */
WC_API wc_status wc_accept_greedy(wc_ctx* ctx, const int* argmax_dev, const int* tokens_dev, const int* parents_dev, int N,
                           int* out_path_dev, int* out_n_dev, int* out_next_dev);
/* sampling.py:143-177 verify_tree_stochastic on device. p_dev [N][V] target probabilities, q_dev [N][V] draft
 * distributions each node's children were drawn from (rows of leaves unused), fp64. Uniforms are the
 * Philox4x32-10 stream (seed, counter offset): one per tested child with q > 0, one per final draw.
 * out_used_dev receives the number of uniforms consumed. */
WC_API wc_status wc_accept_stochastic(wc_ctx* ctx, const double* p_dev, const double* q_dev, int V, const int* tokens_dev,
                               const int* parents_dev, int N, uint64_t seed, uint64_t offset, int* out_path_dev,
                               int* out_n_dev, int* out_next_dev, int* out_used_dev);
/* The same decision as wc_accept_stochastic (same arguments, same results), for callers that must
 * not allocate device memory while they verify. No counterpart in the reference, whose sampling
 * runs on the host (python/woodcock/sampling.py, src/sampling/sampling.cpp).
 * wc_accept_stochastic keeps two scratch rows of V doubles per context and grows them with
 * cudaMalloc / cudaFree on its first call and whenever V grows. cudaFree waits for the whole
 * device, which a caller that keeps other streams busy cannot accept, and a caller that runs
 * under a device-memory budget fixed at start-up cannot let a library allocate behind its back.
 * This entry allocates nothing: its scratch is one array compiled into the library, two rows of
 * WC_ACCEPT_NOALLOC_MAX_V doubles (2.5 MiB of device memory per GPU).
 *  - V > WC_ACCEPT_NOALLOC_MAX_V returns WC_ERR_CAPACITY and launches nothing.
 *  - Nothing in the scratch has to start at zero: each call writes the rows before it reads them.
 *  - The first call on a device looks up the array's device address (cudaGetSymbolAddress), with
 *    the context's device current (otherwise WC_ERR_INVALID). Make that first call before any
 *    stream capture begins (a first call on a capturing stream returns WC_ERR_INVALID). The
 *    address is kept for the life of the process: a cudaDeviceReset between calls is not supported.
 *  - Every call on one device uses the same array. Two calls that can run at the same time
 *    (different streams, or different contexts on that device) race on it: order them on one
 *    stream, or use wc_accept_stochastic. */
#define WC_ACCEPT_NOALLOC_MAX_V 163840
WC_API wc_status wc_accept_stochastic_noalloc(wc_ctx* ctx, const double* p_dev, const double* q_dev, int V,
                                       const int* tokens_dev, const int* parents_dev, int N, uint64_t seed,
                                       uint64_t offset, int* out_path_dev, int* out_n_dev, int* out_next_dev,
                                       int* out_used_dev);
/* fp64 uniforms of the Philox stream, for the host side of tests and for draft sampling */
/* probs_from_logits (sampling.py:39-55): rows of device fp32 logits [rows][V] -> warped
 * probabilities (temperature, top_k (0 = off), top_p (1 = off)) into out [rows][V]. Ties that
 * fall exactly on the top-k / top-p cut are all kept. */
WC_API wc_status wc_probs_from_logits(wc_ctx* ctx, const float* logits, int rows, int V, float temperature,
                                      int top_k, float top_p, float* out);
WC_API wc_status wc_philox_uniforms(wc_ctx* ctx, uint64_t seed, uint64_t offset, int n, double* out_dev);

/* ------------------------------------------------------------------ speculative decoder
 * include/woodcock/spec.h:56-78; python/woodcock/spec.py:104-374. The round runs on the
 * device from one CUDA graph per (mode, k): draft chain, verification, acceptance,
 * KV compaction and the drafter update, with one host synchronisation. */
typedef struct {
  float temperature;  /* 0 = greedy */
  int top_k;          /* 0 = off */
  float top_p;        /* 1 = off */
  uint64_t seed;
} wc_sampling_params;

typedef struct {
  int prompt_tokens, new_tokens, rounds;
  long accepted, verified;
  double t_prefill, t_draft, t_verify, t_update, t_total;
} wc_gen_stats;

/* max_context: capacity of both KV arenas; max_k: largest chain length rounds may use */
WC_API wc_status wc_decoder_create(wc_target* t, wc_drafter* d, int max_context, int max_k, wc_decoder** out);
WC_API void wc_decoder_destroy(wc_decoder* dec);
/* spec.py:129-141 prefill: prompt (host int32[n]); first token returned in *first */
WC_API wc_status wc_decoder_prefill(wc_decoder* dec, const int* prompt, int n, const wc_sampling_params* sp, int* first);
/* Oracle-drafter mode (tests/test_spec_model.py:59-92 pattern): when `forced` (host int32[k]) is
 * non-NULL, draft token j is replaced by forced[j] after the drafter computed it. */
WC_API wc_status wc_decoder_set_forced(wc_decoder* dec, const int* forced, int k);
/* One chain round of length k (spec.py:331-364). Writes the accepted tokens (d_1..d_a, next)
 * to out_tokens (host, capacity k+1) and their count to *out_n. After a prefill with
 * temperature > 0 the round is sampled (spec.py:216-324 on a chain): draft d_i is drawn from
 * the drafter's softmax(z_i / T) over its head rows, the target's p = softmax(z / T) verifies
 * with verify_tree_stochastic's chain rule (sampling.py:143-187) and the next token is drawn
 * from the residual or from the bonus row. Random numbers: Philox4x32-10 keyed by sp->seed;
 * each round consumes one counter block of 2^26 (streams of 2^21: draft step i, the
 * acceptance uniforms, the residual's Gumbel noise). top_k / top_p warp the target's p as
 * probs_from_logits does (sampling.py:39-55), as one threshold per row on z / T; the draft
 * distribution uses the temperature only (spec.py:113-125). */
WC_API wc_status wc_decoder_round(wc_decoder* dec, int k, int* out_tokens, int* out_n);
/* spec.py:151-212 generate with a static chain policy of depth k (draft trees go through
 * wc_decoder_tree_round; per-round chain lengths through wc_decoder_round).
 * eos: host int32[n_eos]. out_tokens capacity max_new. */
WC_API wc_status wc_decoder_generate(wc_decoder* dec, const int* prompt, int n, int max_new, int k,
                              const wc_sampling_params* sp, const int* eos, int n_eos, int* out_tokens, int* out_n,
                              wc_gen_stats* stats);
/* A greedy draft-tree round (spec.py:216-329; src/core/spec.cpp:86-233 with StaticPolicy(depth,
 * width, budget)) on the device from one CUDA graph per shape, one host synchronisation: the
 * drafter expands the tree level by level (top-width children of the `width` most probable nodes of
 * each level, by path probability), the `budget` most probable nodes are verified in one target
 * pass with the tree mask and positions n + depth, verify_tree_greedy picks the path, the target
 * cache is compacted to it and the drafter is updated on the accepted rows. Writes d_1..d_a, next
 * to out_tokens (host, capacity depth + 1). Limits: width <= 16, (depth - 1) * width <= 32,
 * at most 128 drafted nodes and 16 verify rows; greedy decoding only (WC_ERR_UNSUPPORTED). */
WC_API wc_status wc_decoder_tree_round(wc_decoder* dec, int depth, int width, int budget, int* out_tokens,
                                       int* out_n);
/* Test support (oracle-drafter mode for trees, tests/test_spec_model.py:59-92 pattern): while set,
 * tree rounds verify this tree (host int32 tokens[n], parents[n]; node 0 is the round's root and
 * its token is ignored; parents precede their nodes) instead of the drafted one; the drafter still
 * runs over every node that has children. NULL clears it. */
WC_API wc_status wc_decoder_set_forced_tree(wc_decoder* dec, const int* tokens, const int* parents, int n);
/* Test support: the last tree round's nodes (tokens, parents, the drafter head's own argmax token
 * and logit at every node it ran on, -1 elsewhere) and the node id of each verify row. Host
 * buffers of `cap` entries; any may be NULL. */
WC_API wc_status wc_decoder_tree_nodes(wc_decoder* dec, int cap, int* n_nodes, int* tokens, int* parents,
                                       int* proposals, float* proposal_logits, int* verified, int* n_verified);
/* spec.py:377-397 / spec.cpp:282-311 autoregressive baseline through the same target kernels */
WC_API wc_status wc_generate_autoregressive(wc_target* t, const int* prompt, int n, int max_new,
                                     const wc_sampling_params* sp, const int* eos, int n_eos, int max_context,
                                     int* out_tokens, int* out_n, wc_gen_stats* stats);
/* Test and measurement support, no counterpart in the reference. save_state snapshots the
 * decoder's device state (round state, chain root) after a prefill or a round; restore_state
 * puts it back (cache rows past the snapshot are scratch and get rewritten) but keeps the
 * current random counter, so rounds replayed from one snapshot draw fresh numbers. */
WC_API wc_status wc_decoder_save_state(wc_decoder* dec);
WC_API wc_status wc_decoder_restore_state(wc_decoder* dec);
/* The last sampled round of length k: target logits [k+1][V] at [x_n, d_1..d_k], draft
 * logits [k][head_rows], the verify tokens [x_n, d_1..d_k] and rng = {seed, counter base
 * of that round}. Host buffers; any may be NULL. */
WC_API wc_status wc_decoder_round_logits(wc_decoder* dec, int k, float* zt, float* zd, int* tokens,
                                         unsigned long long* rng);
/* Test support, no counterpart in the reference: the drafter's own choice at each of the last
 * greedy round's k chain steps (head argmax mapped to a token id, and its logit), also when
 * wc_decoder_set_forced replaced the drafts. Host buffers; either may be NULL. */
WC_API wc_status wc_decoder_draft_proposals(wc_decoder* dec, int k, int* tokens, float* logits);
/* A real round (as wc_decoder_round) replayed from a second graph that records CUDA events
 * around kernels: ms_sum[i] / counts[i] is the mean device time of kernel class i, for
 * i = 0 target QKV GEMV, 1 attention, 2 o-proj, 3 gate/up, 4 down-proj, 5 target head,
 * 6 drafter head, 7 drafter layer pass (whole). Arrays of 16. */
WC_API wc_status wc_decoder_profile_round(wc_decoder* dec, int k, int* out_tokens, int* out_n, float* ms_sum,
                                          int* counts);
/* device-side state after the last round: committed length n (target cache size) and drafter cache size */
WC_API wc_status wc_decoder_state(const wc_decoder* dec, int* n, int* drafter_len);
/* copy the target KV cache of the decoder (for tests) */
WC_API wc_kv* wc_decoder_target_cache(wc_decoder* dec);
WC_API wc_kv* wc_decoder_drafter_cache(wc_decoder* dec);
/* time the last captured round on the device (CUDA events around `iters` graph replays with the
 * state restored between them is NOT done: callers time real rounds). Returns ms of last round. */
WC_API wc_status wc_decoder_last_round_ms(const wc_decoder* dec, float* ms);

/* The prefill's target pass (spec.py:129-141; Qwen3::forward over the prompt) on the tensor
 * cores: tokens_dev (device int32[n]) through every layer as tcgen05 GEMMs over all n rows,
 * causal attention, K/V appended to `cache` after its current size; taps (device fp32
 * [3][n][hidden], NULL = none) receive the tap layers' block outputs; last_hidden (device fp32
 * [hidden], NULL = none) the last row's residual before the final norm. bf16 targets with
 * head_dim 64 or 128 (WC_ERR_UNSUPPORTED otherwise). Decoder and autoregressive prefills take
 * this path when it applies (environment WC_PREFILL_GEMM=0 keeps the decode kernels). */
WC_API wc_status wc_target_prompt_forward(wc_target* t, wc_kv* cache, const int* tokens_dev, int n, float* taps,
                                          float* last_hidden);

/* ------------------------------------------------------------------ batched tree verification
 * BASELINE config C5 (no counterpart in the reference, whose decoder runs one request): B
 * independent requests, each verifying a draft token tree against its own KV arena, then
 * compacting the accepted path in place (sampling.py:118-140 tree mask and greedy rule;
 * src/cache/kv_cache.cpp:21-31 compaction). Rows are request-major; the projections are
 * tcgen05 GEMMs (bf16 in, fp32 accumulate), attention is the tree-masked prefix attention.
 * bf16 targets with head_dim 64 or 128; nodes x (heads / kv_heads) <= 64. */
typedef struct wc_batch wc_batch;
/* Row-major GEMM copies of the target's weights are made here (their bytes again). The
 * drafter cache (drafter_layers = 0: none) is only compacted alongside the target's. */
WC_API wc_status wc_batch_create(wc_target* t, int max_requests, int max_nodes, int capacity, int drafter_layers,
                                 int drafter_kv_heads, int drafter_head_dim, wc_batch** out);
WC_API void wc_batch_destroy(wc_batch* b);
/* Request r's committed prefix: rows [0, n) of a single-request bf16 target cache. */
WC_API wc_status wc_batch_set_prefix(wc_batch* b, int r, const wc_kv* src, int n);
/* Requests [0, nreq): n committed rows of seeded N(0, 1) bf16 K/V (timing workloads). */
WC_API wc_status wc_batch_fill_synthetic(wc_batch* b, int nreq, int n, uint64_t seed);
/* Verify trees of `nodes` nodes for requests [0, nreq): tokens / parents host int32
 * [nreq][nodes] (node 0 = the request's newest committed token, parents[0] = -1, parents[i] < i),
 * positions lens[r] + depth. Appends every node's K/V at rows lens[r] + i and writes the
 * target's argmax per node (host int32 [nreq][nodes]); out_logits (host fp32 [nreq * nodes][V])
 * may be NULL. */
WC_API wc_status wc_batch_verify(wc_batch* b, int nreq, int nodes, const int* tokens, const int* parents,
                                 int* out_argmax, float* out_logits);
/* wc_batch_verify with CUDA events around kernel classes (no logits): ms_sum[i] / counts[i]
 * as wc_decoder_profile_round (0 QKV GEMM, 1 tree attention, 2 O GEMM, 3 gate/up GEMM,
 * 4 down GEMM, 5 head GEMM); arrays of 16. */
WC_API wc_status wc_batch_verify_profiled(wc_batch* b, int nreq, int nodes, const int* tokens, const int* parents,
                                          int* out_argmax, float* ms_sum, int* counts);
/* Keep lists (host int32 [nreq][maxkeep], keep[r][0] = 0, increasing) with counts n_keep[r]:
 * rows lens[r] + keep[r][i] -> lens[r] + i in the target (and drafter) caches, lens[r] += n_keep[r]. */
WC_API wc_status wc_batch_commit(wc_batch* b, int nreq, const int* keep, const int* n_keep, int maxkeep);
WC_API wc_status wc_batch_lens(const wc_batch* b, int nreq, int* lens);
/* Rows [0, n) of request r's target cache at `layer` as bf16 [n][kv_heads][head_dim] (host; the arena itself
 * is head-major, [layer][request][kv_head][capacity][head_dim]). */
WC_API wc_status wc_batch_read_kv(wc_batch* b, int r, int layer, int n, void* k_out, void* v_out);
/* C[M][N] (+)= A[M][K] . B[N][K]^T on the tensor cores (tcgen05): A, B bf16 row-major device
 * pointers (16-byte aligned, K a multiple of 64), C fp32; residual (may equal C) added when set. */
WC_API wc_status wc_gemm_bf16(wc_ctx* ctx, const void* A, const void* B, float* C, int M, int N, int K,
                              const float* residual);

#ifdef __cplusplus
}
#endif

#endif /* WOODCOCK_B200_H_ */
