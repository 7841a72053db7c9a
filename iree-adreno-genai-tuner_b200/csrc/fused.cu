// Elementwise and attention kernels of the LlamaQ4 step (scripts/llm/llama_q4.py:199-239):
//   embed_q4_lookup   QEmbedding.lookup (:106-119): dequantised rows, zero for ids outside the vocab
//   rmsnorm           rms_norm (:141-142)
//   attention         GQA over the fp16 cache with the causal mask key_pos <= pos (:208-232),
//                     reading only keys that can be unmasked (< min(L, pos + 1)): masked scores are
//                     -1e30 in the reference and contribute exactly 0 after the softmax.
//     decode form   (few query rows): split over key chunks; each CTA keeps an online softmax
//                   (max, sum, weighted V) per query row; the last CTA of a KV head (arrival
//                   counter) merges the chunks in chunk order.
//     prefill form  tiled: one CTA per (KV head, 4 query rows) for all heads of a group of up to 4,
//                   K / V tiles staged once in shared memory; larger groups: one CTA per (head,
//                   query row), its keys split over 4 warps. Online softmax over the row's keys.
#include "fused.h"

namespace q4b {

// ---- embedding ----------------------------------------------------------------------------

__global__ void embed_q4_kernel(const int32_t* __restrict__ tokens, int C, const int32_t* __restrict__ qw,
                                const __half* __restrict__ scales, int vocab, int dim, int group, float* __restrict__ out) {
  griddep_launch_dependents();
  griddep_wait();
  const int c = blockIdx.x;
  const int t = tokens[c];
  const bool valid = t >= 0 && t < vocab;
  const int words = dim / 8, KG = dim / group;
  for (int w = threadIdx.x; w < words; w += blockDim.x) {
    float v[8];
    if (valid) {
      const int32_t word = qw[(size_t)t * words + w];
      const float s = __half2float(scales[(size_t)t * KG + (8 * w) / group]);
#pragma unroll
      for (int b = 0; b < 8; ++b) v[b] = (float)(((word >> (4 * b)) & 15) - 8) * s;
    } else {
#pragma unroll
      for (int b = 0; b < 8; ++b) v[b] = 0.0f;
    }
    float4* o = reinterpret_cast<float4*>(out + (size_t)c * dim + 8 * w);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// ---- rmsnorm ------------------------------------------------------------------------------

__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, float eps, int dim,
                               const int32_t* __restrict__ row_sel, float* __restrict__ out) {
  __shared__ float red[32];
  griddep_launch_dependents();
  griddep_wait();
  const int r = blockIdx.x;
  const float* xr = x + (size_t)((row_sel ? *row_sel : 0) + r) * dim;
  constexpr int kV = 4;  // float4 per thread held in registers (rows up to 4096 with 256 threads)
  if (dim % 4 == 0 && dim <= kV * 4 * (int)blockDim.x &&
      (reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) % 16 == 0) {
    // one pass: every load of the row issued before the reduction, the row kept in registers
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    float4* o4 = reinterpret_cast<float4*>(out + (size_t)r * dim);
    const int n4 = dim / 4;
    float4 v[kV];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const int j = threadIdx.x + i * blockDim.x;
      v[i] = j < n4 ? x4[j] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
      t = warp_sum(t);
      if (threadIdx.x == 0) red[0] = 1.0f / sqrtf(t / (float)dim + eps);
    }
    __syncthreads();
    const float rs = red[0];
#pragma unroll
    for (int i = 0; i < kV; ++i) {
      const int j = threadIdx.x + i * blockDim.x;
      if (j < n4) {
        const float4 g = w4[j];
        o4[j] = make_float4(v[i].x * rs * g.x, v[i].y * rs * g.y, v[i].z * rs * g.z, v[i].w * rs * g.w);
      }
    }
    return;
  }
  float ss = 0.0f;
  for (int k = threadIdx.x; k < dim; k += blockDim.x) ss += xr[k] * xr[k];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = 1.0f / sqrtf(v / (float)dim + eps);
  }
  __syncthreads();
  const float rs = red[0];
  for (int k = threadIdx.x; k < dim; k += blockDim.x) out[(size_t)r * dim + k] = xr[k] * rs * w[k];
}

// ---- attention ------------------------------------------------------------------------------

constexpr int kMaxRows = 16;  // decode form: at most this many query rows (tokens x heads per KV head)
constexpr int kChunk = 256;   // decode form: keys per CTA
constexpr int kMaxChunks = 64;  // decode form: chunks per KV head (L <= 16384)

template <int EPL>
__device__ __forceinline__ void load_half_vec(const __half* p, float (&v)[EPL]) {
  if constexpr (EPL == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    v[0] = a.x;
    v[1] = a.y;
    v[2] = b.x;
    v[3] = b.y;
  } else if constexpr (EPL == 2) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(p));
    v[0] = a.x;
    v[1] = a.y;
  } else {
#pragma unroll
    for (int e = 0; e < EPL; ++e) v[e] = __half2float(p[e]);
  }
}

// grid (Hkv, nchunk), block 256 (8 warps x 32 keys = kChunk keys per CTA). Query row r of KV head
// kvh: token c = r / g, head kvh*g + r % g; ROWS >= C * g rows.
//   Q.K: lane j owns key k0 + 32 w + j; it loads the key's whole row and dots it with every query
//        row (read from shared memory as broadcasts), so a warp covers 32 keys with no shuffles.
//   softmax: max and sum over the warp's 32 keys per query row (two shuffle reductions per row).
//   P.V: lanes own head elements (hd / 32 each); the warp's 32 V slices were loaded together with
//        the K rows, so the CTA waits for DRAM once.
// Warp partials (max, sum, weighted V) merge in shared memory. One chunk covers the context up to
// kChunk keys and writes the output directly; longer contexts merge chunk partials through the
// workspace (last CTA of a KV head, chunk order, loads issued in parallel).
template <int HD, int ROWS>
__global__ void __launch_bounds__(256) attn_decode_kernel(AttnArgs a) {
  constexpr int EPL = HD / 32;  // head elements per lane in P.V
  constexpr int KU4 = HD / 8;   // 16-byte pieces of one key row
  constexpr int NW = kChunk / 32;
  extern __shared__ __align__(16) float s_o[];  // [NW][ROWS][HD]
  __shared__ float s_q[ROWS][HD];
  __shared__ float s_m[NW][ROWS], s_l[NW][ROWS];
  __shared__ float s_M[ROWS], s_L[ROWS];
  __shared__ float s_cs[kMaxChunks][ROWS], s_lc[kMaxChunks][ROWS];
  __shared__ int s_last;
  const int kvh = blockIdx.x, chunk = blockIdx.y, nchunk = gridDim.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = a.H / a.Hkv;
  const int R = a.C * g;
  griddep_launch_dependents();
  griddep_wait();
  const int start = *a.pos0;
  const int kend = min(a.L, start + a.C);  // keys any row of this step can see
  const int k0 = chunk * kChunk, k1 = min(k0 + kChunk, kend);
  const int jbase = k0 + 32 * warp, j = jbase + lane;
  const size_t row_stride = (size_t)a.Hkv * HD;

  // all loads of this warp first: its lane's K row and the 32 V slices of its lane's elements
  uint4 kr[KU4];
  if (j < k1) {
    const uint4* kp = reinterpret_cast<const uint4*>(a.k_cache + (size_t)j * row_stride + (size_t)kvh * HD);
#pragma unroll
    for (int u = 0; u < KU4; ++u) kr[u] = kp[u];
  } else {
#pragma unroll
    for (int u = 0; u < KU4; ++u) kr[u] = make_uint4(0u, 0u, 0u, 0u);
  }
  float vv[32][EPL];
#pragma unroll
  for (int jj = 0; jj < 32; ++jj) {
    if (jbase + jj < k1)
      load_half_vec<EPL>(a.v_cache + (size_t)(jbase + jj) * row_stride + (size_t)kvh * HD + lane * EPL, vv[jj]);
    else
#pragma unroll
      for (int e = 0; e < EPL; ++e) vv[jj][e] = 0.0f;
  }
  for (int i = threadIdx.x; i < R * HD; i += blockDim.x) {
    const int r = i / HD, e = i - r * HD;
    s_q[r][e] = a.q[((size_t)(r / g) * a.H + kvh * g + r % g) * HD + e];
  }
  __syncthreads();

  // scores of this lane's key, softmax over the warp's keys, weighted V
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    if (r >= R) continue;
    float o[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[e] = 0.0f;
    float mw = -INFINITY, lw = 0.0f;
    float d = 0.0f;
#pragma unroll
    for (int u = 0; u < KU4; ++u) {
      const __half2* h2 = reinterpret_cast<const __half2*>(&kr[u]);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __half22float2(h2[t]);
        d = fmaf(s_q[r][8 * u + 2 * t], f.x, d);
        d = fmaf(s_q[r][8 * u + 2 * t + 1], f.y, d);
      }
    }
    const int nk = min(a.L, start + r / g + 1);  // keys 0..nk-1 are unmasked for this row
    const float sc = j < nk ? d * a.scale : -INFINITY;
    const float m = warp_max(sc);
    if (m != -INFINITY) {  // else no visible key for this row in this warp
      const float p = expf(sc - m);
      mw = m;
      lw = warp_sum(p);
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        const float pj = __shfl_sync(0xffffffffu, p, jj);
#pragma unroll
        for (int e = 0; e < EPL; ++e) o[e] = fmaf(pj, vv[jj][e], o[e]);
      }
    }
    if (lane == 0) {
      s_m[warp][r] = mw;
      s_l[warp][r] = lw;
    }
#pragma unroll
    for (int e = 0; e < EPL; ++e) s_o[((size_t)warp * ROWS + r) * HD + lane * EPL + e] = o[e];
  }
  __syncthreads();
  // merge the warps: this CTA's (max, sum, weighted V) per row
  if (threadIdx.x < R) {
    const int r = threadIdx.x;
    float mm = -INFINITY;
    for (int w = 0; w < NW; ++w) mm = fmaxf(mm, s_m[w][r]);
    float ll = 0.0f;
    for (int w = 0; w < NW; ++w) {
      const float cs = s_m[w][r] == -INFINITY ? 0.0f : expf(s_m[w][r] - mm);
      s_cs[w][r] = cs;
      ll += s_l[w][r] * cs;
    }
    s_M[r] = mm;
    s_L[r] = ll;
  }
  __syncthreads();
  if (nchunk == 1) {  // the whole context in this CTA: write the output
    for (int i = threadIdx.x; i < R * HD; i += blockDim.x) {
      const int r = i / HD, e = i - r * HD;
      float oo = 0.0f;
      for (int w = 0; w < NW; ++w) oo += s_o[((size_t)w * ROWS + r) * HD + e] * s_cs[w][r];
      a.out[((size_t)(r / g) * a.H + kvh * g + r % g) * HD + e] = oo / s_L[r];
    }
    return;
  }
  float* part = a.ws + ((size_t)kvh * nchunk + chunk) * R * (HD + 2);  // [R][m, l, o[HD]]
  for (int i = threadIdx.x; i < R * HD; i += blockDim.x) {
    const int r = i / HD, e = i - r * HD;
    float oo = 0.0f;
    for (int w = 0; w < NW; ++w) oo += s_o[((size_t)w * ROWS + r) * HD + e] * s_cs[w][r];
    part[r * (HD + 2) + 2 + e] = oo;
    if (e == 0) {
      part[r * (HD + 2)] = s_M[r];
      part[r * (HD + 2) + 1] = s_L[r];
    }
  }
  // the last chunk CTA of this KV head merges all chunks
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&a.counters[kvh], 1u) == (unsigned)(nchunk - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* all = a.ws + (size_t)kvh * nchunk * R * (HD + 2);
  // every chunk's (max, sum) in one parallel round of loads, then per-chunk weights
  for (int i = threadIdx.x; i < nchunk * R; i += blockDim.x) {
    const int ch = i / R, r = i - ch * R;
    s_cs[ch][r] = __ldcg(all + ((size_t)ch * R + r) * (HD + 2));
    s_lc[ch][r] = __ldcg(all + ((size_t)ch * R + r) * (HD + 2) + 1);
  }
  __syncthreads();
  if (threadIdx.x < R) {
    const int r = threadIdx.x;
    float mm = -INFINITY;
    for (int ch = 0; ch < nchunk; ++ch) mm = fmaxf(mm, s_cs[ch][r]);
    float ll = 0.0f;
    for (int ch = 0; ch < nchunk; ++ch) {
      const float mc = s_cs[ch][r];
      const float cs = mc == -INFINITY ? 0.0f : expf(mc - mm);
      ll += s_lc[ch][r] * cs;
      s_cs[ch][r] = cs;
    }
    s_L[r] = ll;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < R * HD; i += blockDim.x) {
    const int r = i / HD, e = i - r * HD;
    float oo = 0.0f;
#pragma unroll 8
    for (int ch = 0; ch < nchunk; ++ch) oo += s_cs[ch][r] * __ldcg(all + ((size_t)ch * R + r) * (HD + 2) + 2 + e);
    a.out[((size_t)(r / g) * a.H + kvh * g + r % g) * HD + e] = oo / s_L[r];
  }
  if (threadIdx.x == 0) a.counters[kvh] = 0u;
}

// grid (H, ceil(C / 4)), block 128: warp w handles query row 4 * blockIdx.y + w of head blockIdx.x.
// Keys go in blocks of 32: lane j scores key kb + j against the whole query row (read from shared
// memory as broadcasts), one max and one sum reduction per block update the online softmax, then
// P.V with lanes owning head elements (hd / 32 each) over the block's V rows, loaded together.
template <int EPL>
__global__ void __launch_bounds__(128) attn_prefill_kernel(AttnArgs a) {
  // one CTA per (head, query row): the row's visible keys go to the 4 warps by 32-key blocks (warp
  // w takes blocks w, w + 4, ...), each an online softmax; the warps' (max, sum, weighted V) merge
  // in shared memory. A row's loads are a few rounds in parallel instead of nk / 32 in sequence.
  constexpr int HD = EPL * 32, KU4 = HD / 8, NW = 4;
  __shared__ float s_q[HD];
  __shared__ float s_o[NW][HD];
  __shared__ float s_m[NW], s_l[NW];
  const int h = blockIdx.x, c = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_launch_dependents();
  griddep_wait();
  const int g = a.H / a.Hkv, kvh = h / g;
  const int start = *a.pos0;
  const int nk = min(a.L, start + c + 1);
  const float* qp = a.q + ((size_t)c * a.H + h) * HD;
  for (int e = threadIdx.x; e < HD; e += blockDim.x) s_q[e] = qp[e];
  __syncthreads();
  float o[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) o[e] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  const size_t kv_stride = (size_t)a.Hkv * HD;
  const __half* kbase = a.k_cache + (size_t)kvh * HD;
  const __half* vbase = a.v_cache + (size_t)kvh * HD + lane * EPL;
  for (int kb = 32 * warp; kb < nk; kb += 32 * NW) {
    const int j = kb + lane;
    const bool valid = j < nk;
    // this lane's key row and the block's V slices of this lane's elements, in one round
    const uint4* kp = reinterpret_cast<const uint4*>(kbase + (size_t)min(j, nk - 1) * kv_stride);
    uint4 kr[KU4];
#pragma unroll
    for (int u = 0; u < KU4; ++u) kr[u] = kp[u];
    // V slices kept as packed fp16 (EPL halves per key) until used
    __half vv[32][EPL];
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      const __half* vp = vbase + (size_t)min(kb + jj, nk - 1) * kv_stride;
      if constexpr (EPL == 4) {
        *reinterpret_cast<uint2*>(vv[jj]) = *reinterpret_cast<const uint2*>(vp);
      } else if constexpr (EPL == 2) {
        *reinterpret_cast<uint32_t*>(vv[jj]) = *reinterpret_cast<const uint32_t*>(vp);
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) vv[jj][e] = vp[e];
      }
    }
    float d = 0.0f;
#pragma unroll
    for (int u = 0; u < KU4; ++u) {
      const __half2* h2 = reinterpret_cast<const __half2*>(&kr[u]);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __half22float2(h2[t]);
        d = fmaf(s_q[8 * u + 2 * t], f.x, d);
        d = fmaf(s_q[8 * u + 2 * t + 1], f.y, d);
      }
    }
    const float sc = valid ? d * a.scale : -INFINITY;
    const float mn = fmaxf(m, warp_max(sc));  // the block's lane 0 key is always visible: mn is finite
    const float p = valid ? expf(sc - mn) : 0.0f;
    const float cs = m == -INFINITY ? 0.0f : expf(m - mn);
    l = l * cs + warp_sum(p);
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[e] *= cs;
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);  // 0 for keys past nk
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[e] = fmaf(pj, __half2float(vv[jj][e]), o[e]);
    }
    m = mn;
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) s_o[warp][lane * EPL + e] = o[e];
  __syncthreads();
  if (warp == 0) {  // merge the warps (a warp without keys has max -inf and is skipped)
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, s_m[w]);
    float L = 0.0f, acc[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[e] = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      if (s_m[w] == -INFINITY) continue;
      const float cs = expf(s_m[w] - M);
      L += s_l[w] * cs;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[e] = fmaf(s_o[w][lane * EPL + e], cs, acc[e]);
    }
    float* op = a.out + ((size_t)c * a.H + h) * HD + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) op[e] = acc[e] / L;
  }
}

// Tiled prefill form: one CTA per (KV head, block of kPfRows query rows) takes all g heads of the
// group, NQW = g kPfRows / 4 query vectors per query set; 8 warps: warp w takes query set w % 4 and
// the even (w < 4) or odd (w >= 4) 32-key tiles. Each round stages 64 keys of K and V once per CTA in
// shared memory, serving every query vector of the block (the one-row form re-reads a KV head's keys
// once per query row and head: g C times per chunk). Per tile lane j holds key kb + j: its K row is
// read from shared memory (rows padded by one word, so the 32 lanes hit 32 banks) and scored against
// the warp's query vectors in the same dimension order as the one-row form; then an online softmax
// per query vector and P V with lane l owning dimensions EPL l .. EPL l + EPL - 1. The odd-tile
// warps' (max, sum, weighted V) merge into the even ones' at the end. fp32 throughout, fp16 K / V as
// stored.
constexpr int kPfRows = 4, kPfWarps = 8;

template <int EPL, int NQW>
__global__ void __launch_bounds__(kPfWarps * 32) attn_prefill_tiled_kernel(AttnArgs a) {
  constexpr int HD = EPL * 32, HW = HD / 2 + 1, NQ = 4 * NQW;  // HW: 32-bit words per staged K row
  __shared__ __align__(16) float s_q[NQ][HD];
  __shared__ uint32_t s_k[2][32 * HW];
  __shared__ __align__(16) __half s_v[2][32][HD];
  const int kvh = blockIdx.x, c0 = blockIdx.y * kPfRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qs = warp & 3, half = warp >> 2;  // query set, tile parity
  griddep_launch_dependents();
  griddep_wait();
  const int g = a.H / a.Hkv;  // NQ / kPfRows
  const int start = *a.pos0;
  // query vector qi: row c0 + qi / g of the chunk, head kvh g + qi % g
  for (int i = threadIdx.x; i < NQ * HD; i += blockDim.x) {
    const int qi = i / HD, e = i - qi * HD, c = c0 + qi / g;
    s_q[qi][e] = c < a.C ? a.q[((size_t)c * a.H + kvh * g + qi % g) * HD + e] : 0.0f;
  }
  // this warp's query vectors qi = qs + 4 t and the keys each sees (0 for rows past the chunk)
  int lim[NQW];
#pragma unroll
  for (int t = 0; t < NQW; ++t) {
    const int c = c0 + (qs + 4 * t) / g;
    lim[t] = c < a.C ? min(a.L, start + c + 1) : 0;
  }
  const int nk = min(a.L, start + min(c0 + kPfRows, a.C));  // keys any row of the block sees
  float o[NQW][EPL], m[NQW], l[NQW];
#pragma unroll
  for (int t = 0; t < NQW; ++t) {
    m[t] = -INFINITY;
    l[t] = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[t][e] = 0.0f;
  }
  const size_t kv_stride = (size_t)a.Hkv * HD;
  const __half* kbase = a.k_cache + (size_t)kvh * HD;
  const __half* vbase = a.v_cache + (size_t)kvh * HD;
  for (int k0 = 0; k0 < nk; k0 += 64) {
    __syncthreads();  // the previous round is consumed (the first time: s_q is written)
    // stage K / V rows k0 .. k0 + 63 (rows past nk repeat row nk - 1: finite, weighted 0)
    for (int i = threadIdx.x; i < 64 * (HD / 8); i += blockDim.x) {
      const int r = i / (HD / 8), u = i - r * (HD / 8), tb = r >> 5, rr = r & 31;
      const size_t row = (size_t)min(k0 + r, nk - 1) * kv_stride + u * 8;
      const uint4 kv = *reinterpret_cast<const uint4*>(kbase + row);
      const uint4 vv = *reinterpret_cast<const uint4*>(vbase + row);
      uint32_t* kw = s_k[tb] + rr * HW + u * 4;
      kw[0] = kv.x, kw[1] = kv.y, kw[2] = kv.z, kw[3] = kv.w;
      *reinterpret_cast<uint4*>(&s_v[tb][rr][u * 8]) = vv;
    }
    __syncthreads();
    const int kb = k0 + 32 * half;
    if (kb >= nk) continue;  // (uniform per warp; the barriers above are outside this branch)
    float s[NQW];
#pragma unroll
    for (int t = 0; t < NQW; ++t) s[t] = 0.0f;
    const uint32_t* kr = s_k[half] + lane * HW;
#pragma unroll 8
    for (int u = 0; u < HD / 4; ++u) {  // dimensions 4u .. 4u + 3 of key kb + lane
      const uint32_t w0 = kr[2 * u], w1 = kr[2 * u + 1];
      const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&w0));
      const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&w1));
#pragma unroll
      for (int t = 0; t < NQW; ++t) {
        const float4 qv = *reinterpret_cast<const float4*>(&s_q[qs + 4 * t][4 * u]);
        s[t] = fmaf(qv.x, k01.x, s[t]);
        s[t] = fmaf(qv.y, k01.y, s[t]);
        s[t] = fmaf(qv.z, k23.x, s[t]);
        s[t] = fmaf(qv.w, k23.y, s[t]);
      }
    }
    float p[NQW];
    const int j = kb + lane;
#pragma unroll
    for (int t = 0; t < NQW; ++t) {
      const float sc = j < lim[t] ? s[t] * a.scale : -INFINITY;
      const float mn = fmaxf(m[t], warp_max(sc));  // -inf only while the vector has seen no key
      p[t] = j < lim[t] ? expf(sc - mn) : 0.0f;
      const float cs = m[t] == -INFINITY ? 0.0f : expf(m[t] - mn);
      l[t] = l[t] * cs + warp_sum(p[t]);
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[t][e] *= cs;
      m[t] = mn;
    }
#pragma unroll 4
    for (int jj = 0; jj < 32; ++jj) {
      float vf[EPL];
      if constexpr (EPL == 4) {
        const uint2 vw = *reinterpret_cast<const uint2*>(&s_v[half][jj][lane * 4]);
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vw.x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vw.y));
        vf[0] = v01.x, vf[1] = v01.y, vf[2] = v23.x, vf[3] = v23.y;
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) vf[e] = __half2float(s_v[half][jj][lane * EPL + e]);
      }
#pragma unroll
      for (int t = 0; t < NQW; ++t) {
        const float pj = __shfl_sync(0xffffffffu, p[t], jj);  // 0 for keys this vector does not see
#pragma unroll
        for (int e = 0; e < EPL; ++e) o[t][e] = fmaf(pj, vf[e], o[t][e]);
      }
    }
  }
  // the odd-tile warps hand (max, sum, weighted V) over through the K / V staging area
  __syncthreads();
  float* xo = reinterpret_cast<float*>(&s_v[0][0][0]);  // [4 sets][NQW][HD] (<= 2 * 32 * HD halves)
  float* xm = reinterpret_cast<float*>(s_k[0]);          // [4 sets][NQW][2]
  if (half == 1) {
#pragma unroll
    for (int t = 0; t < NQW; ++t) {
#pragma unroll
      for (int e = 0; e < EPL; ++e) xo[(qs * NQW + t) * HD + lane * EPL + e] = o[t][e];
      if (lane == 0) xm[(qs * NQW + t) * 2] = m[t], xm[(qs * NQW + t) * 2 + 1] = l[t];
    }
  }
  __syncthreads();
  if (half == 1) return;
#pragma unroll
  for (int t = 0; t < NQW; ++t) {
    const int qi = qs + 4 * t, c = c0 + qi / g;
    if (c >= a.C) continue;
    const float m1 = xm[(qs * NQW + t) * 2], l1 = xm[(qs * NQW + t) * 2 + 1];
    const float M = fmaxf(m[t], m1);  // finite: key 0 is in the even tiles and visible to every row
    const float c_0 = expf(m[t] - M), c_1 = m1 == -INFINITY ? 0.0f : expf(m1 - M);
    const float L = l[t] * c_0 + l1 * c_1;
    float* op = a.out + ((size_t)c * a.H + kvh * g + qi % g) * HD + lane * EPL;
#pragma unroll
    for (int e = 0; e < EPL; ++e) op[e] = (o[t][e] * c_0 + xo[(qs * NQW + t) * HD + lane * EPL + e] * c_1) / L;
  }
}

template <int EPL>
static cudaError_t launch_prefill_tiled(const AttnArgs& a, int g, cudaStream_t st) {
  const dim3 grid(a.Hkv, (a.C + kPfRows - 1) / kPfRows);
  switch (g) {  // g kPfRows / 4 query vectors per warp
    case 1: return launch_pdl(attn_prefill_tiled_kernel<EPL, 1>, grid, dim3(kPfWarps * 32), 0, st, a);
    case 2: return launch_pdl(attn_prefill_tiled_kernel<EPL, 2>, grid, dim3(kPfWarps * 32), 0, st, a);
    case 3: return launch_pdl(attn_prefill_tiled_kernel<EPL, 3>, grid, dim3(kPfWarps * 32), 0, st, a);
    default: return launch_pdl(attn_prefill_tiled_kernel<EPL, 4>, grid, dim3(kPfWarps * 32), 0, st, a);
  }
}

int attn_decode_chunks(int L) { return (L + kChunk - 1) / kChunk; }

template <int HD, int ROWS>
static cudaError_t launch_decode_hd(const AttnArgs& a, dim3 grid, cudaStream_t st) {
  const size_t smem = (size_t)(kChunk / 32) * ROWS * HD * sizeof(float);
  static std::atomic<unsigned long long> done;
  const cudaError_t e = set_max_dynamic_smem(attn_decode_kernel<HD, ROWS>, (int)smem, done);
  if (e != cudaSuccess) return e;
  return launch_pdl(attn_decode_kernel<HD, ROWS>, grid, dim3(256), smem, st, a);
}

template <int ROWS>
static cudaError_t launch_decode(const AttnArgs& a, dim3 grid, cudaStream_t st) {
  switch (a.head_dim) {
    case 32: return launch_decode_hd<32, ROWS>(a, grid, st);
    case 64: return launch_decode_hd<64, ROWS>(a, grid, st);
    default: return launch_decode_hd<128, ROWS>(a, grid, st);
  }
}

size_t attention_workspace(int C, int H, int Hkv, int head_dim, int L) {
  const int g = H / Hkv;
  if (C * g > kMaxRows) return 0;
  return kCounterRegion + (size_t)Hkv * attn_decode_chunks(L) * C * g * (head_dim + 2) * sizeof(float);
}

int attention_run(const AttnArgs& in, cudaStream_t st) {
  AttnArgs a = in;
  const int g = a.H / a.Hkv;
  if (a.H % a.Hkv || (a.head_dim != 32 && a.head_dim != 64 && a.head_dim != 128))
    return set_error(Q4B_EUNSUPPORTED, "attention: head_dim must be 32, 64 or 128 and H %% Hkv == 0");
  const bool decode = a.C * g <= kMaxRows && !a.force_prefill;
  if (decode && attn_decode_chunks(a.L) > kMaxChunks)
    return set_error(Q4B_EUNSUPPORTED, "attention: bucket %d above %d keys", a.L, kMaxChunks * kChunk);
  cudaError_t e;
  if (decode) {
    const size_t need = attention_workspace(a.C, a.H, a.Hkv, a.head_dim, a.L);
    if (!a.ws_base || a.ws_bytes < need)
      return set_error(Q4B_EINVAL, "attention: workspace of %zu bytes needed, %zu given", need, a.ws_bytes);
    a.counters = reinterpret_cast<unsigned*>(a.ws_base);
    a.ws = reinterpret_cast<float*>(reinterpret_cast<char*>(a.ws_base) + kCounterRegion);
    const dim3 grid(a.Hkv, attn_decode_chunks(a.L));
    const int R = a.C * g;
    e = R <= 4 ? launch_decode<4>(a, grid, st) : R <= 8 ? launch_decode<8>(a, grid, st) : launch_decode<16>(a, grid, st);
  } else if (g <= 4) {  // groups of up to 4 heads: the tiled form
    e = a.head_dim == 32   ? launch_prefill_tiled<1>(a, g, st)
        : a.head_dim == 64 ? launch_prefill_tiled<2>(a, g, st)
                           : launch_prefill_tiled<4>(a, g, st);
  } else {
    const dim3 grid(a.H, a.C);
    switch (a.head_dim) {
      case 32: e = launch_pdl(attn_prefill_kernel<1>, grid, dim3(128), 0, st, a); break;
      case 64: e = launch_pdl(attn_prefill_kernel<2>, grid, dim3(128), 0, st, a); break;
      default: e = launch_pdl(attn_prefill_kernel<4>, grid, dim3(128), 0, st, a); break;
    }
  }
  if (e != cudaSuccess) return set_error(Q4B_ELAUNCH, "attention: launch failed: %s", cudaGetErrorString(e));
  return check_launch("attention");
}

int embed_run(const int32_t* tokens, int C, const int32_t* qw, const uint16_t* scales, int vocab, int dim, int group,
              float* out, cudaStream_t st) {
  if (dim % 8 || dim % group || group % 8) return set_error(Q4B_EINVAL, "embed: bad dim/group");
  const cudaError_t e = launch_pdl(embed_q4_kernel, dim3(C), dim3(128), 0, st, tokens, C, qw,
                                   reinterpret_cast<const __half*>(scales), vocab, dim, group, out);
  if (e != cudaSuccess) return set_error(Q4B_ELAUNCH, "embed: launch failed: %s", cudaGetErrorString(e));
  return check_launch("embed");
}

int rmsnorm_run(const float* x, const float* w, float eps, int rows, int dim, const int32_t* row_sel, float* out,
                cudaStream_t st) {
  const cudaError_t e = launch_pdl(rmsnorm_kernel, dim3(rows), dim3(256), 0, st, x, w, eps, dim, row_sel, out);
  if (e != cudaSuccess) return set_error(Q4B_ELAUNCH, "rmsnorm: launch failed: %s", cudaGetErrorString(e));
  return check_launch("rmsnorm");
}

}  // namespace q4b

using namespace q4b;

extern "C" int q4b_embed_q4_lookup(const int32_t* tokens, int n_tokens, const int32_t* qweight, const uint16_t* scales,
                                   int vocab, int dim, int group, float* out, q4b_stream_t stream) {
  if (!tokens || !qweight || !scales || !out || n_tokens < 1 || vocab < 1 || dim < 8)
    return set_error(Q4B_EINVAL, "embed_q4_lookup: bad arguments");
  if (!aligned(out, 16)) return set_error(Q4B_EINVAL, "embed_q4_lookup: out must be 16-byte aligned");
  return embed_run(tokens, n_tokens, qweight, scales, vocab, dim, group, out, as_stream(stream));
}

extern "C" int q4b_rmsnorm(const float* x, const float* weight, float eps, int rows, int dim, float* out,
                           q4b_stream_t stream) {
  if (!x || !weight || !out || rows < 1 || dim < 1) return set_error(Q4B_EINVAL, "rmsnorm: bad arguments");
  return rmsnorm_run(x, weight, eps, rows, dim, nullptr, out, as_stream(stream));
}

extern "C" size_t q4b_attention_workspace(int n_rows, int n_heads, int n_kv_heads, int head_dim, int L) {
  if (n_rows < 1 || n_heads < 1 || n_kv_heads < 1 || n_heads % n_kv_heads) return 0;
  return attention_workspace(n_rows, n_heads, n_kv_heads, head_dim, L);
}

extern "C" int q4b_attention(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* start,
                             int n_rows, int n_heads, int n_kv_heads, int head_dim, int L, float* out,
                             void* workspace, size_t workspace_bytes, q4b_stream_t stream) {
  if (!q || !k_cache || !v_cache || !start || !out || n_rows < 1 || L < 1)
    return set_error(Q4B_EINVAL, "attention: bad arguments");
  AttnArgs a = {};
  a.q = q;
  a.k_cache = reinterpret_cast<const __half*>(k_cache);
  a.v_cache = reinterpret_cast<const __half*>(v_cache);
  a.pos0 = start;
  a.C = n_rows;
  a.H = n_heads;
  a.Hkv = n_kv_heads;
  a.head_dim = head_dim;
  a.L = L;
  a.scale = (float)(1.0 / sqrt((double)head_dim));  // the reference's 1 / math.sqrt(hd) in fp32
  a.out = out;
  a.ws_base = workspace;
  a.ws_bytes = workspace_bytes;
  return attention_run(a, as_stream(stream));
}

extern "C" int q4b_prefill_attn(const float* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* start,
                                int n_rows, int n_heads, int n_kv_heads, int head_dim, int L, float* out,
                                q4b_stream_t stream) {
  if (!q || !k_cache || !v_cache || !start || !out || n_rows < 1 || L < 1)
    return set_error(Q4B_EINVAL, "prefill_attn: bad arguments");
  AttnArgs a = {};
  a.q = q;
  a.k_cache = reinterpret_cast<const __half*>(k_cache);
  a.v_cache = reinterpret_cast<const __half*>(v_cache);
  a.pos0 = start;
  a.C = n_rows;
  a.H = n_heads;
  a.Hkv = n_kv_heads;
  a.head_dim = head_dim;
  a.L = L;
  a.scale = (float)(1.0 / sqrt((double)head_dim));
  a.out = out;
  a.force_prefill = 1;
  return attention_run(a, as_stream(stream));
}
