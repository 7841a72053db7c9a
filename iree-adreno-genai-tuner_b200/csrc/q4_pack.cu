// int4 packing kernels: quantize_q4, unpack_q4, dequantize_q4 (scripts/llm/llama_q4.py:25-51).
//
// quantize is bit-exact with the reference: the scale is max(absmax, 1e-8f) / 7.0f with IEEE
// division, q = rintf(w / scale) (round half to even, like torch.round), clamped to [-8, 7] and
// stored as q + 8 in nibble k % 8 of word k / 8. This file must not be built with fast-math.
#include "common.cuh"

namespace q4b {

// One thread per (row, group): absmax over the group, then quantise and pack its G/8 words.
__global__ void quantize_q4_kernel(const float* __restrict__ w, int n, int k, int group,
                                   int32_t* __restrict__ qweight, __half* __restrict__ scales) {
  const int groups = k / group;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= (long long)n * groups) return;
  const int row = (int)(gid / groups), grp = (int)(gid % groups);
  const float* src = w + (size_t)row * k + (size_t)grp * group;
  float amax = 0.0f;
  for (int i = 0; i < group; ++i) amax = fmaxf(amax, fabsf(src[i]));
  const float scale = fmaxf(amax, 1e-8f) / 7.0f;
  scales[(size_t)row * groups + grp] = __float2half_rn(scale);
  int32_t* dst = qweight + (size_t)row * (k / 8) + (size_t)grp * (group / 8);
  for (int j = 0; j < group / 8; ++j) {
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      float q = rintf(__fdiv_rn(src[8 * j + b], scale));
      q = fminf(fmaxf(q, -8.0f), 7.0f);
      word |= (uint32_t)((int)q + 8) << (4 * b);
    }
    dst[j] = (int32_t)word;
  }
}

__global__ void unpack_q4_kernel(const int32_t* __restrict__ qweight, long long words, uint8_t* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= words) return;
  const int32_t w = qweight[i];
  uint2 o;
  o.x = o.y = 0;
#pragma unroll
  for (int b = 0; b < 4; ++b) o.x |= (uint32_t)((w >> (4 * b)) & 15) << (8 * b);
#pragma unroll
  for (int b = 0; b < 4; ++b) o.y |= (uint32_t)((w >> (4 * (b + 4))) & 15) << (8 * b);
  reinterpret_cast<uint2*>(out)[i] = o;
}

template <typename OutT>
__global__ void dequantize_q4_kernel(const int32_t* __restrict__ qweight, const __half* __restrict__ scales, int n,
                                     int k, int group, OutT* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // word index
  const long long words = (long long)n * (k / 8);
  if (i >= words) return;
  const int row = (int)(i / (k / 8)), j = (int)(i % (k / 8));
  const float s = __half2float(scales[(size_t)row * (k / group) + (8 * j) / group]);
  const int32_t w = qweight[i];
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const float v = (float)(((w >> (4 * b)) & 15) - 8) * s;
    if constexpr (sizeof(OutT) == 4)
      out[i * 8 + b] = v;
    else
      out[i * 8 + b] = __float2half_rn(v);
  }
}

static int grid_for(long long items, int block) { return (int)((items + block - 1) / block); }

}  // namespace q4b

using namespace q4b;

extern "C" int q4b_quantize_q4(const float* w, int n, int k, int group, int32_t* qweight, uint16_t* scales,
                               q4b_stream_t stream) {
  if (!w || !qweight || !scales) return set_error(Q4B_EINVAL, "quantize_q4: null pointer");
  if (n <= 0 || k <= 0 || group <= 0 || group % 8 || k % group)
    return set_error(Q4B_EINVAL, "quantize_q4: need k %% group == 0 and group %% 8 == 0 (n=%d k=%d group=%d)", n, k,
                     group);
  const long long items = (long long)n * (k / group);
  quantize_q4_kernel<<<grid_for(items, 128), 128, 0, as_stream(stream)>>>(w, n, k, group, qweight,
                                                                           reinterpret_cast<__half*>(scales));
  return check_launch("quantize_q4");
}

extern "C" int q4b_unpack_q4(const int32_t* qweight, int n, int k, uint8_t* nibbles, q4b_stream_t stream) {
  if (!qweight || !nibbles) return set_error(Q4B_EINVAL, "unpack_q4: null pointer");
  if (n <= 0 || k <= 0 || k % 8) return set_error(Q4B_EINVAL, "unpack_q4: need k %% 8 == 0 (k=%d)", k);
  if (!aligned(nibbles, 8)) return set_error(Q4B_EINVAL, "unpack_q4: output must be 8-byte aligned");
  const long long words = (long long)n * (k / 8);
  unpack_q4_kernel<<<grid_for(words, 256), 256, 0, as_stream(stream)>>>(qweight, words, nibbles);
  return check_launch("unpack_q4");
}

extern "C" int q4b_dequantize_q4(const int32_t* qweight, const uint16_t* scales, int n, int k, int group, void* out,
                                 int out_dtype, q4b_stream_t stream) {
  if (!qweight || !scales || !out) return set_error(Q4B_EINVAL, "dequantize_q4: null pointer");
  if (n <= 0 || k <= 0 || group <= 0 || group % 8 || k % group)
    return set_error(Q4B_EINVAL, "dequantize_q4: need k %% group == 0 and group %% 8 == 0");
  const long long words = (long long)n * (k / 8);
  const __half* s = reinterpret_cast<const __half*>(scales);
  if (out_dtype == Q4B_F32)
    dequantize_q4_kernel<float><<<grid_for(words, 256), 256, 0, as_stream(stream)>>>(qweight, s, n, k, group,
                                                                                     (float*)out);
  else if (out_dtype == Q4B_F16)
    dequantize_q4_kernel<__half><<<grid_for(words, 256), 256, 0, as_stream(stream)>>>(qweight, s, n, k, group,
                                                                                      (__half*)out);
  else
    return set_error(Q4B_EINVAL, "dequantize_q4: bad out_dtype %d", out_dtype);
  return check_launch("dequantize_q4");
}
