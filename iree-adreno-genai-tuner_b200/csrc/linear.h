// Internal C++ interface of the int4 linear kernels (q4_linear.cu), used by the model step.
#pragma once

#include "common.cuh"

namespace q4b {

// Epilogues beyond the public Q4B_EPI_* ones (used inside the model step).
enum : int {
  EPI_STORE = Q4B_EPI_STORE,
  EPI_ACCUMULATE = Q4B_EPI_ACCUMULATE,
  EPI_SWIGLU = Q4B_EPI_SWIGLU,
  EPI_ROPE_KV = 3,  // fused q|k|v projection: RoPE on q and k, q to q_out, k and v into the fp16 caches
  EPI_ARGMAX = 4    // lm_head: greedy argmax over the rows (first max on ties), optional logits
};

// Device-resident step state of the decode/prefill loop. Kernels read the positions from here, so
// one captured CUDA graph per (phase, bucket) serves every step.
struct DecodeState {
  int32_t start;       // position of row 0 of this step
  int32_t last;        // row whose logits / next token this step produces
  int32_t next_token;  // greedy token of the last finished step
  int32_t n_gen;       // tokens appended to the log so far
  int32_t stopped;     // 1 once a stop id was produced
  int32_t advance;     // 1: start += 1 after the step (decode)
  int32_t n_stop;
  int32_t log_cap;
  int32_t stop_ids[16];
  unsigned long long best;  // argmax accumulator: orderable(value) << 32 | (0xffffffff - index)
  unsigned int counter;     // lm_head tiles finished
  int32_t status;           // nonzero: a bounded wait gave up
};

struct LinearOp {
  const int32_t* qw = nullptr;
  const uint16_t* scales = nullptr;
  int group = 0;
  const void* x = nullptr;
  int x_dtype = Q4B_F32;
  void* y = nullptr;
  int y_dtype = Q4B_F32;
  int m = 0, n = 0, k = 0;
  int epi = EPI_STORE;
  // prologue: x row m is x[(row_sel ? *row_sel : 0) + m]; with ln_w, x := rmsnorm(x) * ln_w (fp32 x)
  const float* ln_w = nullptr;
  float eps = 0.0f;
  const int32_t* row_sel = nullptr;
  // EPI_ROPE_KV: rows [q heads | k heads | v heads] x head_dim; row m sits at position *pos0 + m
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  const int32_t* pos0 = nullptr;
  int pos_offset = 0;  // added to *pos0 (prefill chunks processed in row blocks)
  float* q_out = nullptr;
  uint16_t* k_cache = nullptr;
  uint16_t* v_cache = nullptr;
  int n_heads = 0, n_kv = 0, head_dim = 0;
  // EPI_ARGMAX (m == 1): tiles fold into state->best; with finalize the last tile publishes the token
  DecodeState* state = nullptr;
  int32_t* token_log = nullptr;
  float* logits = nullptr;
  int index_offset = 0;
  int finalize = 1;
  // kernel selection and split-K workspace (see q4b_q4_linear)
  const q4b_linear_cfg* cfg = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
};

int linear_run(const LinearOp& op, cudaStream_t st);
// Whether the default plan of an m-row call applies an RMSNorm of fp32 x itself (op.ln_w): up to 8
// rows in the GEMV's prologue, or the tcgen05 path's x split (head_dim: the RoPE epilogue's heads).
bool linear_fuses_norm(int m, int k, int group, int epi, int head_dim);
// Greedy argmax of one row (first maximum): the key (orderable value, index) and / or the index
// (idx_offset added: a vocabulary shard's first row). One CTA.
int argmax_run(const float* v, int n, int idx_offset, unsigned long long* key_out, int32_t* index_out,
               cudaStream_t st);
size_t linear_workspace(const LinearOp& op);

// Publish a greedy token into the step state (append to the log, stop ids, advance): the device
// side of runner/llm_runner.c:233-245. One thread calls it once per step.
__device__ __forceinline__ void publish_token(DecodeState* st, int32_t* token_log, int32_t token) {
  if (!st->stopped) {
    st->next_token = token;
    if (token_log && st->n_gen < st->log_cap) token_log[st->n_gen] = token;
    st->n_gen += 1;
    for (int i = 0; i < st->n_stop && i < 16; ++i)
      if (token == st->stop_ids[i]) st->stopped = 1;
  }
  if (st->advance) st->start += 1;
}

// Greedy argmax key: larger value wins, then the lower index (torch.argmax's first maximum).
__device__ __forceinline__ unsigned long long argmax_key(float v, unsigned idx) {
  unsigned b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (0xffffffffu - idx);
}
__device__ __forceinline__ unsigned argmax_index(unsigned long long key) {
  return 0xffffffffu - (unsigned)(key & 0xffffffffull);
}

unsigned linear_status(bool reset);
// Status bits of the GEMM kernels (kStatusTimeout when a bounded wait gave up).
unsigned gemm_status(bool reset);

}  // namespace q4b
