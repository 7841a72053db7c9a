// Single-op entry points of the model's fused pieces, for a caller that replaces the reference's
// step one operation at a time (scripts/llm/llama_q4.py:204-239): the q|k|v projection with RoPE and
// the KV-cache write, SwiGLU, the greedy head. The model step itself uses the same kernels with the
// operations fused into the projections' epilogues.
#include <algorithm>

#include "linear.h"

namespace q4b {

// out[r, i] = silu(gu[r, i]) * gu[r, inter + i]   (llama_q4.py:235-236; gate rows first, :152)
__global__ void silu_mul_kernel(const float* __restrict__ gu, int rows, int inter, float* __restrict__ out) {
  const long long n = (long long)rows * inter;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / inter, c = i - r * inter;
    const float g = gu[r * 2 * inter + c], u = gu[r * 2 * inter + inter + c];
    out[i] = silu(g) * u;
  }
}

// Greedy head over one logits row (llama_q4.py:238-239): the largest value, the first index on ties
// (torch.argmax). keys = orderable(value) << 32 | (0xffffffff - index) make that one max-reduction.
// One CTA of 1024 threads; idx_offset is added to the index (a vocabulary shard's first row).
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ v, int n, int idx_offset,
                                                      unsigned long long* key_out, int32_t* index_out) {
  __shared__ unsigned long long s[32];
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < n; i += blockDim.x) best = max(best, argmax_key(v[i], (unsigned)(idx_offset + i)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    best = threadIdx.x < (blockDim.x >> 5) ? s[threadIdx.x] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if (threadIdx.x == 0) {
      if (key_out) *key_out = best;
      if (index_out) *index_out = (int32_t)argmax_index(best);
    }
  }
}

int argmax_run(const float* v, int n, int idx_offset, unsigned long long* key_out, int32_t* index_out,
               cudaStream_t st) {
  argmax_kernel<<<1, 1024, 0, st>>>(v, n, idx_offset, key_out, index_out);
  return check_launch("argmax");
}

static LinearOp qkv_op(const int32_t* qweight, const uint16_t* scales, int group, const float* x, int m, int dim,
                       int n_heads, int n_kv, int head_dim, const float* rope_cos, const float* rope_sin,
                       const int32_t* start, float* q_out, uint16_t* k_cache, uint16_t* v_cache) {
  LinearOp op;
  op.qw = qweight;
  op.scales = scales;
  op.group = group;
  op.x = x;
  op.x_dtype = Q4B_F32;
  op.m = m;
  op.n = (n_heads + 2 * n_kv) * head_dim;
  op.k = dim;
  op.epi = EPI_ROPE_KV;
  op.rope_cos = rope_cos;
  op.rope_sin = rope_sin;
  op.pos0 = start;
  op.q_out = q_out;
  op.k_cache = k_cache;
  op.v_cache = v_cache;
  op.n_heads = n_heads;
  op.n_kv = n_kv;
  op.head_dim = head_dim;
  return op;
}

}  // namespace q4b

using namespace q4b;

extern "C" size_t q4b_qkv_rope_kvwrite_workspace(int m, int dim, int n_heads, int n_kv_heads, int head_dim, int group) {
  static const int dummy[4] = {0, 0, 0, 0};  // never dereferenced: planning only
  float* f = reinterpret_cast<float*>(const_cast<int*>(dummy));
  uint16_t* h = reinterpret_cast<uint16_t*>(const_cast<int*>(dummy));
  return linear_workspace(qkv_op(dummy, h, group, f, m, dim, n_heads, n_kv_heads, head_dim, f, f, dummy, f, h, h));
}

extern "C" int q4b_qkv_rope_kvwrite(const int32_t* qweight, const uint16_t* scales, int group, const float* x, int m,
                                    int dim, int n_heads, int n_kv_heads, int head_dim, const float* rope_cos,
                                    const float* rope_sin, const int32_t* start, float* q_out, uint16_t* k_cache,
                                    uint16_t* v_cache, void* workspace, size_t workspace_bytes, q4b_stream_t stream) {
  if (!qweight || !scales || !x || !rope_cos || !rope_sin || !start || !q_out || !k_cache || !v_cache || m < 1)
    return set_error(Q4B_EINVAL, "qkv_rope_kvwrite: null pointer or m < 1");
  if (n_kv_heads < 1 || n_heads % n_kv_heads || head_dim % 16)
    return set_error(Q4B_EINVAL, "qkv_rope_kvwrite: need n_heads %% n_kv_heads == 0 and head_dim %% 16 == 0");
  LinearOp op = qkv_op(qweight, scales, group, x, m, dim, n_heads, n_kv_heads, head_dim, rope_cos, rope_sin, start,
                       q_out, k_cache, v_cache);
  op.ws = workspace;
  op.ws_bytes = workspace_bytes;
  return linear_run(op, as_stream(stream));
}

extern "C" int q4b_silu_mul(const float* gate_up, int rows, int inter, float* out, q4b_stream_t stream) {
  if (!gate_up || !out || rows < 1 || inter < 1) return set_error(Q4B_EINVAL, "silu_mul: bad arguments");
  const long long n = (long long)rows * inter;
  const int grid = (int)std::min<long long>((n + 255) / 256, 148 * 16);
  silu_mul_kernel<<<grid, 256, 0, as_stream(stream)>>>(gate_up, rows, inter, out);
  return check_launch("silu_mul");
}

extern "C" int q4b_argmax(const float* logits, int n, int32_t* index, q4b_stream_t stream) {
  if (!logits || !index || n < 1) return set_error(Q4B_EINVAL, "argmax: bad arguments");
  return argmax_run(logits, n, 0, nullptr, index, as_stream(stream));
}
