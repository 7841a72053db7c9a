// Internal interface of the embedding, RMSNorm and attention kernels (fused.cu).
#pragma once

#include "common.cuh"

namespace q4b {

struct AttnArgs {
  const float* q;         // [C, H, hd] fp32 (RoPE applied)
  const __half* k_cache;  // [max_ctx, Hkv, hd] fp16
  const __half* v_cache;
  const int32_t* pos0;    // device: position of query row 0
  int C, H, Hkv, head_dim, L;
  float scale;            // 1 / sqrt(head_dim) rounded to fp32
  float* out;             // [C, H * hd] fp32
  void* ws_base;          // decode form: counters + per-chunk partials
  size_t ws_bytes;
  unsigned* counters;
  float* ws;
  int force_prefill;      // 1: the one-pass form for any row count (no workspace)
};

constexpr size_t kCounterRegion = 4096;  // attention arrival counters (one per KV head)

int attn_decode_chunks(int L);
size_t attention_workspace(int C, int H, int Hkv, int head_dim, int L);
int attention_run(const AttnArgs& a, cudaStream_t st);
int embed_run(const int32_t* tokens, int C, const int32_t* qw, const uint16_t* scales, int vocab, int dim, int group,
              float* out, cudaStream_t st);
int rmsnorm_run(const float* x, const float* w, float eps, int rows, int dim, const int32_t* row_sel, float* out,
                cudaStream_t st);

}  // namespace q4b
