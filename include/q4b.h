/*
 * q4b.h — C ABI of the B200-native int4 Llama hot path (libq4b.so, sm_100a).
 *
 * Conventions for every entry point:
 *   - plain device pointers and sizes; no allocation inside a call (the caller owns all memory,
 *     including workspaces); work is ordered on the given stream (a cudaStream_t passed as
 *     q4b_stream_t, NULL = the legacy default stream); no host synchronisation, so calls can be
 *     captured in a CUDA graph;
 *   - the return value is Q4B_OK (0) or a negative Q4B_E* code; q4b_last_error() returns a
 *     thread-local message for the last failing call on that thread;
 *   - shape and alignment errors are reported before anything is launched.
 *
 * Layouts follow the reference (paths relative to the reference project):
 *   qweight [N, K/8] int32, nibble b (bits 4b..4b+3) of word j holds k = 8j + b, stored as q + 8;
 *   scales  [N, K/G] fp16 (passed as uint16_t bit patterns);        scripts/llm/llama_q4.py:25-38
 *   activations row-major [M, K]; outputs row-major [M, N].
 */
#ifndef Q4B_H
#define Q4B_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  Q4B_OK = 0,
  Q4B_EINVAL = -1,       /* bad shape, dtype, alignment or null pointer */
  Q4B_ELAUNCH = -2,      /* a kernel launch failed (cudaGetLastError) */
  Q4B_ETIMEOUT = -3,     /* a bounded device-side wait gave up */
  Q4B_ENOMEM = -4,       /* a create call could not allocate its state */
  Q4B_EUNSUPPORTED = -5, /* valid input the library does not handle */
  Q4B_ECUDA = -6,        /* another CUDA runtime error */
  Q4B_ESTATE = -7        /* object used in the wrong state */
};

enum { Q4B_F32 = 0, Q4B_F16 = 1 };

/* Epilogues of q4b_q4_linear:
 *   STORE       y[m, n] = sum_k x[m, k] W[n, k]
 *   ACCUMULATE  y[m, n] += sum_k x[m, k] W[n, k]            (residual add, llama_q4.py:233, 236)
 *   SWIGLU      W has 2*I rows (gate rows then up rows, llama_q4.py:152); y is [M, I] with
 *               y[m, i] = silu(gate_i . x_m) * (up_i . x_m)   (llama_q4.py:235-236)           */
enum { Q4B_EPI_STORE = 0, Q4B_EPI_ACCUMULATE = 1, Q4B_EPI_SWIGLU = 2 };

/* Kernel selection for q4b_q4_linear (NULL = tuned default; all fields 0 = choose automatically).
 *   kernel 1  tensor-core dequant GEMV, weights in registers (G % 128 == 0, M <= 64): warps (1..8),
 *             tiles (128-k tiles per warp in flight: 1, 2, 3, 4, 6, 8), split (k splits, >= 1)
 *   kernel 2  generic SIMT (any G % 8 == 0)
 *   kernel 3  GEMV with the weight tile staged by bulk copies (M <= 16): warps, split
 *   kernel 4  persistent GEMV, one CTA per SM, whole-row-tile ring (M == 1, G == 128): warps (1..24)
 *   kernel 5  tcgen05 int4-weight GEMM for many rows (prefill): tiles (4 or 8 row tiles of 16), split
 *   kernel 6  persistent TMA-ring GEMV (M <= 8, G == 128, K % 1024 == 0; the default for weights of
 *             40 MB and more, e.g. the lm_head), int8 tensor-core math for one x row: tiles =
 *             residency (1: one CTA per SM leaving room for the next kernel on the stream, 2: two
 *             CTAs per SM, 3: one CTA with the whole shared memory), split = 1 keeps each row pair
 *             in one CTA                                                                      */
typedef struct q4b_linear_cfg {
  int kernel;
  int warps;
  int tiles;
  int split;
} q4b_linear_cfg;

typedef void* q4b_stream_t;

/* Message of the last failing call on this thread ("" if none). */
const char* q4b_last_error(void);
/* ABI version of this header (bumped on any incompatible change). */
int q4b_abi_version(void);

/* quantize_q4 (scripts/llm/llama_q4.py:25-38), bit-exact: w [n, k] fp32 on the device ->
 * qweight [n, k/8] int32, scales [n, k/group] fp16. Needs k % group == 0 and group % 8 == 0. */
int q4b_quantize_q4(const float* w, int n, int k, int group, int32_t* qweight, uint16_t* scales,
                    q4b_stream_t stream);

/* unpack_q4 (scripts/llm/llama_q4.py:41-45), bit-exact: qweight [n, k/8] -> nibbles [n, k] uint8. */
int q4b_unpack_q4(const int32_t* qweight, int n, int k, uint8_t* nibbles, q4b_stream_t stream);

/* dequantize_q4 (scripts/llm/llama_q4.py:48-51): -> out [n, k] of out_dtype (Q4B_F32 is exact). */
int q4b_dequantize_q4(const int32_t* qweight, const uint16_t* scales, int n, int k, int group, void* out,
                      int out_dtype, q4b_stream_t stream);

/* Bytes of workspace q4b_q4_linear needs for this problem and configuration (0 if none). The
 * workspace holds split-K partial sums and per-tile arrival counters; it must be zero-filled once
 * before its first use, and every call leaves the counters at zero again. Calls that share one
 * workspace must be ordered on one stream. */
size_t q4b_q4_linear_workspace(int m, int n, int k, int group, int epilogue, const q4b_linear_cfg* cfg);

/* QLinear.forward (scripts/llm/llama_q4.py:69-90): y = x @ dequantize_q4(qweight, scales)^T with
 * fp32 accumulation, both reference forms in one call. x [m, k] of x_dtype, y of y_dtype
 * ([m, n], or [m, n/2] for Q4B_EPI_SWIGLU). With fp32 x the tensor-core kernel splits x into two
 * fp16 terms (hi + lo), so products keep ~22 bits of x. Launched with programmatic dependent launch:
 * the weight stream starts before the previous kernel on the stream has finished. */
int q4b_q4_linear(const int32_t* qweight, const uint16_t* scales, int group, const void* x, int x_dtype,
                  void* y, int y_dtype, int m, int n, int k, int epilogue, const q4b_linear_cfg* cfg,
                  void* workspace, size_t workspace_bytes, q4b_stream_t stream);

/* The kernel (1..6, see q4b_linear_cfg) q4b_q4_linear runs for this problem with 16-byte aligned
 * pointers and the workspace q4b_q4_linear_workspace asks for; or a negative Q4B_E* code. */
int q4b_q4_linear_kernel(int m, int n, int k, int group, int epilogue, int x_dtype, const q4b_linear_cfg* cfg);

/* Allocation-free variant of q4b_q4_linear (no counterpart in the reference). For callers that
 * cannot allocate device memory themselves: hosts that reach this library only through a plain C
 * FFI with no CUDA allocator of their own, plugins that must not allocate while another framework
 * owns the device memory pool, and code paths with a fixed memory budget. The split-K workspace is
 * a static 8 MiB array inside libq4b.so instead of a caller buffer (every GPU that loads the
 * library holds it until the process exits); the caller still passes x and y. Same arguments and
 * results as q4b_q4_linear with the default configuration; returns Q4B_EINVAL, before launching
 * anything, when the problem needs more than 8 MiB of workspace. The first call on a device looks
 * up the array and zeroes its counters (synchronously); make that first call before any stream
 * capture. All calls share the one array: calls that overlap on the GPU (other streams, other host
 * threads) race, so order them on one stream. Never allocates (no cudaMalloc / cudaFree). The
 * array's address and the kernels' shared-memory attributes are looked up / set once per device for
 * the life of the process: the entry point does not survive cudaDeviceReset (or any other teardown of
 * the device's primary context) within the same process. */
int q4b_q4_linear_noalloc(const int32_t* qweight, const uint16_t* scales, int group, const void* x, int x_dtype,
                          void* y, int y_dtype, int m, int n, int k, int epilogue, q4b_stream_t stream);

/* ---- fp16 GEMM (prefill; the gemm/ tuner's problem, gemm/shapes.py:1-66) --------------------- */

/* Kernel choice and schedule of q4b_gemm_f16 (the CUDA counterpart of gemm/schedule.py:43-103's
 * Schedule; all zero = the built-in default for the shape). */
typedef struct q4b_gemm_cfg {
  int kernel; /* 0 = default, 1 = tcgen05 (TMA + TMEM accumulator), 2 = CUDA-core 64x64 tiles,
                 3 = tcgen05 persistent stream-K (one CTA run of equal (tile, 64-k) units per SM
                 slot, two TMEM accumulators, part-tiles added in k order by the last contributor) */
  int bn;     /* kernels 1, 3: output tile width 64 | 128 | 256 (tile height is 128); 0 = auto */
  int stages; /* kernels 1, 3: shared-memory ring depth, 2 .. as many as fit in 200 KB; 0 = max */
  int split;  /* kernel 1: k splits (fp32 partials in the workspace); 0 = auto, 1 = none.
                 kernel 3: 0 or 1 (it balances k itself) */
} q4b_gemm_cfg;

/* Bytes of workspace q4b_gemm_f16 needs (0 if none; -1 if the problem or cfg is invalid, with
 * q4b_last_error() saying why). Same zero-fill-once rule as q4b_q4_linear_workspace. */
long long q4b_gemm_f16_workspace(int m, int n, int k, char la, char lb, const q4b_gemm_cfg* cfg);

/* C[m, n] = op(A) op(B), fp16 in and out, fp32 accumulation (gemm/shapes.py:1-6, 56-66; the
 * harness contract of gemm/harness/vk_gemm_bench.c:5-13). Layout letters as BLAS: la 'N' = A stored
 * [m][k], 'T' = stored [k][m]; lb 'N' = B stored [k][n], 'T' = stored [n][k]. C is row-major [m][n].
 * The tcgen05 kernel needs 16-byte aligned A / B and row pitches (k or m for A, n or k for B) that
 * are multiples of 8; the default falls back to kernel 2 otherwise. */
/* The schedule q4b_gemm_f16 runs for this problem and cfg (NULL = the default: for the config-2
 * shapes the schedule a search on a B200 measured fastest, q4b/gemm/tuned_b200.json; otherwise the
 * built-in plan), written to *out (kernel 1 or 2, bn, stages, split). No reference counterpart. */
int q4b_gemm_f16_plan(int m, int n, int k, char la, char lb, const q4b_gemm_cfg* cfg, q4b_gemm_cfg* out);
int q4b_gemm_f16(const void* a, const void* b, void* c, int m, int n, int k, char la, char lb,
                 const q4b_gemm_cfg* cfg, void* workspace, size_t workspace_bytes, q4b_stream_t stream);

/* ---- model pieces (scripts/llm/llama_q4.py:93-142, 199-239) ------------------------------- */

/* QEmbedding.lookup (:106-119): out[c, :] = dequantised row tokens[c] of the [vocab, dim] table, or
 * zeros for ids outside [0, vocab). tokens are device int32; out fp32 [n_tokens, dim], 16-B aligned. */
int q4b_embed_q4_lookup(const int32_t* tokens, int n_tokens, const int32_t* qweight, const uint16_t* scales,
                        int vocab, int dim, int group, float* out, q4b_stream_t stream);

/* rms_norm (:141-142): out = x * 1/sqrt(mean(x^2) + eps) * weight, fp32 [rows, dim]. */
int q4b_rmsnorm(const float* x, const float* weight, float eps, int rows, int dim, float* out, q4b_stream_t stream);

/* Bucketed GQA attention (:208-232) for n_rows query rows at positions *start + r over the fp16
 * caches [max_ctx, n_kv_heads, head_dim]: keys 0..min(L, pos+1)-1 (the causal mask key <= pos on
 * cache[:L]). q fp32 [n_rows, n_heads, head_dim] with RoPE applied; out fp32 [n_rows, n_heads *
 * head_dim]. start is a device int32. head_dim 32, 64 or 128. Few rows (n_rows * heads per KV head
 * <= 16) use the split-key form, which needs q4b_attention_workspace() bytes, zero-filled once. */
size_t q4b_attention_workspace(int n_rows, int n_heads, int n_kv_heads, int head_dim, int L);
int q4b_attention(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* start, int n_rows,
                  int n_heads, int n_kv_heads, int head_dim, int L, float* out, void* workspace,
                  size_t workspace_bytes, q4b_stream_t stream);

/* The same attention in its one-pass form for any row count (a prefill chunk, :208-232): no
 * workspace; the causal mask and bucket as q4b_attention. */
int q4b_prefill_attn(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* start,
                     int n_rows, int n_heads, int n_kv_heads, int head_dim, int L, float* out, q4b_stream_t stream);

/* The fused q|k|v projection of one layer (:204-223): rows = x [m, dim] fp32 @ wqkv^T (wqkv rows
 * q heads | k heads | v heads, int4 [(n_heads + 2 n_kv_heads) head_dim, dim/8]), RoPE on q and k
 * with the fp32 tables rope_cos / rope_sin [max_ctx, head_dim] at positions *start + r, q to
 * q_out [m, n_heads, head_dim] fp32, k and v into the fp16 caches [max_ctx, n_kv_heads, head_dim]
 * at rows *start + r (in place, :222-223). start is a device int32. Workspace as
 * q4b_q4_linear's (zero-filled once). */
size_t q4b_qkv_rope_kvwrite_workspace(int m, int dim, int n_heads, int n_kv_heads, int head_dim, int group);
int q4b_qkv_rope_kvwrite(const int32_t* qweight, const uint16_t* scales, int group, const float* x, int m, int dim,
                         int n_heads, int n_kv_heads, int head_dim, const float* rope_cos, const float* rope_sin,
                         const int32_t* start, float* q_out, uint16_t* k_cache, uint16_t* v_cache, void* workspace,
                         size_t workspace_bytes, q4b_stream_t stream);

/* SwiGLU (:235-236): out[r, i] = silu(gate_up[r, i]) * gate_up[r, inter + i] (gate rows first,
 * :152), fp32 [rows, 2 inter] -> [rows, inter]. */
int q4b_silu_mul(const float* gate_up, int rows, int inter, float* out, q4b_stream_t stream);

/* Greedy head (:238-239): *index (device int32) = the first index of the largest of logits[n]
 * (torch.argmax's tie rule). */
int q4b_argmax(const float* logits, int n, int32_t* index, q4b_stream_t stream);

/* ---- LlamaQ4 model (scripts/llm/llama_q4.py:145-243) --------------------------------------- */

typedef struct q4b_model_cfg {
  int n_layers, dim, n_heads, n_kv_heads, head_dim, inter, vocab;
  float rms_eps;
  int max_ctx;    /* KV cache rows (positions) */
  int max_chunk;  /* most rows in one step (prefill chunk) */
  int tp_rank, tp_size; /* tensor-parallel shard of this process (0, 1 on one GPU) */
} q4b_model_cfg;

/* One quantised matrix: qweight [n, k/8] int32, scales [n, k/group] fp16, device pointers. */
typedef struct q4b_qmat {
  const int32_t* qweight;
  const uint16_t* scales;
  int n, k, group;
} q4b_qmat;

/* Layer weights (:145-155) of this rank's shard: wqkv rows q|k|v of its heads, wo [dim, heads*hd],
 * wgu rows gate|up of its slice of the intermediate size, wdown [dim, inter/tp]; fp32 norm weights;
 * fp16 KV caches [max_ctx, n_kv_heads/tp, head_dim] (updated in place, :222-223). Borrowed. */
typedef struct q4b_layer_weights {
  q4b_qmat wqkv, wo, wgu, wdown;
  const float* ln_in;
  const float* ln_post;
  uint16_t* k_cache;
  uint16_t* v_cache;
} q4b_layer_weights;

typedef struct q4b_model q4b_model;

/* Allocates the model's activations and workspaces on the current device (no weights). */
int q4b_model_create(const q4b_model_cfg* cfg, q4b_model** out);
int q4b_model_set_layer(q4b_model* model, int layer, const q4b_layer_weights* weights);
/* Tied embedding / lm_head: the full [vocab, dim] table on every rank (rank r's lm_head uses rows
 * [r*vocab/tp, (r+1)*vocab/tp)); final norm weight; RoPE tables cos, sin [max_ctx, head_dim] fp32. */
int q4b_model_set_head(q4b_model* model, const q4b_qmat* embed, const float* ln_f, const float* rope_cos,
                       const float* rope_sin);
/* LlamaQ4.step (:199-239): tokens [n_tokens] device int32 at positions start.., KV written in place,
 * attention over the bucket L; the greedy token of row `last` goes to *next_token (device, may be
 * NULL) and the row's logits to logits (device fp32 [vocab], may be NULL). */
int q4b_model_step(q4b_model* model, const int32_t* tokens, int n_tokens, int start, int last, int L,
                   int32_t* next_token, float* logits, q4b_stream_t stream);
void q4b_model_destroy(q4b_model* model);
/* Which kernel runs single-token decode steps: 1 = the persistent step (one cooperative launch per
 * token, tables built on the first decode step), 0 = one kernel per projection. No reference
 * counterpart (a diagnostic of this library's decode path). */
int q4b_model_decode_path(const q4b_model* model);
/* Testing the failure path without a device fault: marks the model's persistent decode step as
 * failed, exactly as a bounded device wait that gave up does. Later decode steps do no work, the
 * runner returns Q4B_ETIMEOUT, until the model is prepared again (q4b_model_set_head or
 * q4b_model_set_layer; single GPU). No reference counterpart. */
int q4b_model_fail_decode(q4b_model* model);
/* Phase trace of the persistent decode step (no reference counterpart; a profiling aid): with a
 * device buffer of at least q4b_model_trace_events(model) uint64 set, every persistent step writes
 * %globaltimer stamps (ns) per CTA: CTA c's row starts at c * (15 * n_layers + 4); per layer l and
 * stage s (0 q|k|v, 1 attention, 2 o, 3 gate|up, 4 down) the stamps 15 l + 3 s + {0 inputs ready
 * (barrier passed or partial sums loaded), 1 x staged, 2 done}, then 15 n_layers + {0 lm_head inputs
 * ready, 1 staged, 2 done, 3 consumers start}. NULL turns the trace off. */
size_t q4b_model_trace_events(const q4b_model* model);
int q4b_model_set_trace(q4b_model* model, unsigned long long* events, size_t n_events);

/* ---- tensor parallelism (one process per GPU, NCCL loaded at run time) ---------------------- */

/* Rank 0 makes the communicator id (128 bytes) and shares it with the other ranks out of band. */
int q4b_tp_unique_id(unsigned char* id, int id_bytes);
/* Join the communicator of the model's tp_size ranks as tp_rank (collective across the ranks).
 * Afterwards each step all-reduces the wo / wdown partial outputs and gathers the per-rank argmax. */
int q4b_model_attach_tp(q4b_model* model, const unsigned char* id, int id_bytes);

/* Standalone collectives for a tensor-parallel caller outside the model (the reference runs on
 * one device; these are the exchange steps of its column / row / vocabulary splits). */
typedef struct q4b_tp q4b_tp;
/* Join a communicator of `world` ranks as `rank` (collective; id from q4b_tp_unique_id). */
int q4b_tp_init(int rank, int world, const unsigned char* id, int id_bytes, q4b_tp** out);
void q4b_tp_destroy(q4b_tp* tp);
/* In-place sum over the ranks of n elements (a row-split projection's partial outputs). */
int q4b_tp_allreduce_f16(q4b_tp* tp, void* buf, size_t n, q4b_stream_t stream);
int q4b_tp_allreduce_f32(q4b_tp* tp, float* buf, size_t n, q4b_stream_t stream);
/* Greedy head over a vocabulary split: this rank's logits[n_local] are rows index_offset.. of
 * the full vocabulary; *token (device int32, every rank) = the global first maximum. Workspace:
 * q4b_tp_argmax_workspace(tp) bytes, 8-byte aligned. */
size_t q4b_tp_argmax_workspace(const q4b_tp* tp);
int q4b_tp_argmax_gather(q4b_tp* tp, const float* logits, int n_local, int index_offset, int32_t* token,
                         void* workspace, size_t workspace_bytes, q4b_stream_t stream);

/* ---- runner (runner/llm_runner.c) ---------------------------------------------------------- */

/* Scheduler options (llm_runner.c:35-45): prefill chunk, ascending KV buckets, schedule 0 =
 * bucketed (smallest bucket >= tokens in cache) or 1 = max (always the largest); use_graphs: one
 * captured CUDA graph per (phase, bucket); warmup: untimed calls per used (phase, bucket);
 * sync_every_step: copy each decode step's inputs in and its token out and check stop ids on the
 * host (the reference's per-call protocol) instead of running decode steps back to back. */
typedef struct q4b_runner_opts {
  int chunk;
  const int32_t* buckets;
  int n_buckets;
  int schedule;
  int use_graphs;
  int warmup;
  int sync_every_step;
} q4b_runner_opts;

/* Timings of one generate call (llm_runner.c:249-262). decode_ms sums the device time of the decode
 * steps (CUDA events); decode_wall_ms is the host clock around the decode loop. */
typedef struct q4b_report {
  double warmup_ms, prefill_ms, ttft_ms, prefill_tok_s, decode_ms, decode_wall_ms, decode_tok_s;
  int prompt_tokens, new_tokens, decode_steps;
} q4b_report;

typedef struct q4b_runner q4b_runner;

/* The runner borrows the model (and its caches) for its lifetime. */
int q4b_runner_create(q4b_model* model, const q4b_runner_opts* opts, q4b_runner** out);
/* llm_runner.c:151-262: chunked prefill of prompt[n_prompt] (host ids), then greedy decode until
 * max_new tokens (the prefill token included) or a stop id; out_tokens[max_new] receives them and
 * *n_out their count. Errors as the reference: empty prompt, prompt + new > max_ctx, no bucket. */
int q4b_runner_generate(q4b_runner* runner, const int32_t* prompt, int n_prompt, int max_new, const int32_t* stop_ids,
                        int n_stop, int32_t* out_tokens, int* n_out, q4b_report* report);
/* JSON report of the last generate call, in llm_runner.c's schema (valid until the next call). */
const char* q4b_runner_report_json(q4b_runner* runner);
void q4b_runner_destroy(q4b_runner* runner);

/* Q4B_ETIMEOUT if a bounded device-side wait gave up since the last reset, else Q4B_OK. */
int q4b_device_status(int reset);

#ifdef __cplusplus
}
#endif

#endif /* Q4B_H */
