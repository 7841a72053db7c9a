// int4 weight-only linear: QLinear.forward of scripts/llm/llama_q4.py:69-90,
//
//   y[m, n] = sum_k x[m, k] * (nib(n, k) - 8) * scale(n, k / G)          (fp32 accumulation)
//
// with the model's neighbouring elementwise work fused in (prologue: RMSNorm of x,
// llama_q4.py:141-142; epilogues: residual add :233/:236, SwiGLU :235-236, RoPE + KV-cache write
// :219-223, greedy argmax :238-239).
//
// Every kernel works on tiles of 16 weight rows ("slots") x its k-range. Slot -> row maps:
//   plain/accumulate: row = 16 rt + s;   SwiGLU: s < 8 gate row 8 rt + s, s >= 8 up row I + 8 rt + s - 8;
//   RoPE: head rt / (hd/16), slots s and s + 8 hold head elements e and e + hd/2 (a rotation pair).
// Kernels:
//   1 q4_gemv_reg  G % 128 == 0, M <= 64: mma.sync m16n8k16 (fp16 operands, fp32 accumulate). Each
//                  lane keeps T 128-k tiles of rows g and g + 8 in registers (two 16-byte streaming
//                  loads per tile, 64 contiguous bytes per 4 lanes), all issued before
//                  griddepcontrol.wait. Nibbles become exact fp16 (nib - 8) with LOP3 + HSUB2/HFMA2;
//                  inside a word the k order is permuted (MMA k-slots hold nibbles b and b + 4) and x
//                  is staged in shared memory in the same order. A 128-k tile lies inside one scale
//                  group, so each tile's MMA sum is scaled once in fp32. fp32 x is split into two fp16
//                  terms (hi + lo), keeping ~22 bits of x.
//   3 q4_gemv_tma  the same math with the weight tile streamed into shared memory by the TMA engine
//                  (one bulk copy per row, one mbarrier, bounded wait), M <= 16.
//   2 q4_linear_simt any G % 8 == 0: fp32 FMAs on exactly dequantised weights (the reference's
//                  dequant + linear form).
// Split-K partials go to a workspace; the last CTA of a row tile (arrival counter) sums them in
// split order, so results are deterministic.
#include <algorithm>
#include <atomic>

#include "linear.h"
#include "q4dev.cuh"
#include "tc.cuh"

namespace q4b {

constexpr int TILE_K = 128;

struct LinArgs {
  const int32_t* qw;
  const __half* scales;
  const void* x;
  void* y;
  float* ws;
  unsigned* counters;
  int M, N, K, G, n_out;
  int KT;      // 128-k tiles
  int kps;     // tiles per split
  int nsplit;  // k splits
  int epi;
  int y_f32;
  int wstride;  // TMA kernel: bytes per staged weight row
  int x_off;    // TMA kernel: byte offset of the x staging area in dynamic shared memory
  // prologue
  const float* ln_w;
  float eps;
  const int32_t* row_sel;
  // RoPE / KV
  const float* rope_cos;
  const float* rope_sin;
  const int32_t* pos0;
  int pos_offset;
  float* q_out;
  __half* k_cache;
  __half* v_cache;
  int H, Hkv, hd;
  // argmax
  DecodeState* state;
  int32_t* token_log;
  float* logits;
  int index_offset;
  int finalize;
  int RT;  // row tiles of the whole problem (the argmax epilogue counts finished tiles)
  // kernel 6 (ring GEMV)
  int ring_slots;   // stages in the shared-memory ring
  int kc;           // stages per row tile (K / 1024)
  int split_units;  // 1: CTAs take equal runs of stages, row tiles cut between CTAs meet in ws
  int red_off;      // byte offset of the cross-warp reduction slots in dynamic shared memory
};

// status word of this file's kernels (bounded waits that gave up), read by linear_status()
__device__ unsigned g_linear_status;

// ---- PTX helpers: q4dev.cuh -------------------------------------------------------------------

__device__ __forceinline__ float load_y(const void* y, size_t i, int f32) {
  return f32 ? reinterpret_cast<const float*>(y)[i] : __half2float(reinterpret_cast<const __half*>(y)[i]);
}
__device__ __forceinline__ void store_y(void* y, size_t i, float v, int f32) {
  if (f32)
    reinterpret_cast<float*>(y)[i] = v;
  else
    reinterpret_cast<__half*>(y)[i] = __float2half_rn(v);
}

// ---- tile geometry, prologue, epilogue (shared by all kernels) ------------------------------

__device__ __forceinline__ int tile_row(const LinArgs& p, int rt, int s) {
  if (p.epi == EPI_SWIGLU) {
    const int i = min(rt * 8 + (s & 7), p.n_out - 1);
    return s < 8 ? i : p.n_out + i;
  }
  if (p.epi == EPI_ROPE_KV) {
    const int per = p.hd / 16;
    const int head = rt / per, j = rt - head * per;
    const int e = s < 8 ? j * 8 + s : p.hd / 2 + j * 8 + (s - 8);
    return min(head * p.hd + e, p.N - 1);
  }
  return min(rt * 16 + s, p.N - 1);
}

__device__ __forceinline__ int x_row(const LinArgs& p, int m) { return (p.row_sel ? *p.row_sel : 0) + m; }

// RMSNorm prologue: rs[m] = 1 / sqrt(mean(x[row m]^2) + eps) over the full row (M <= 8).
// Must be called by every thread of the CTA; ends with a barrier.
__device__ void prologue_rms(const LinArgs& p, float* rs, float* scratch) {
  const int warps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float part[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) part[m] = 0.0f;
  const int k4 = p.K / 4;
  const float* x = reinterpret_cast<const float*>(p.x);
  for (int i = threadIdx.x; i < p.M * k4; i += blockDim.x) {
    const int m = i / k4, c = i - m * k4;
    const float4 v = *reinterpret_cast<const float4*>(x + (size_t)x_row(p, m) * p.K + 4 * c);
    const float s = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
#pragma unroll
    for (int mm = 0; mm < 8; ++mm)
      if (mm == m) part[mm] += s;
  }
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const float v = warp_sum(part[m]);
    if (lane == 0) scratch[warp * 8 + m] = v;
  }
  __syncthreads();
  if (threadIdx.x < p.M) {
    float ss = 0.0f;
    for (int w = 0; w < warps; ++w) ss += scratch[w * 8 + threadIdx.x];
    rs[threadIdx.x] = 1.0f / sqrtf(ss / (float)p.K + p.eps);
  }
  __syncthreads();
}

// x value after the prologue (SIMT kernel)
__device__ __forceinline__ float x_value(const LinArgs& p, const float* rs, int m, int k, bool xf32) {
  const size_t off = (size_t)x_row(p, m) * p.K + k;
  if (p.ln_w) return reinterpret_cast<const float*>(p.x)[off] * rs[m] * p.ln_w[k];
  if (xf32) return __ldg(reinterpret_cast<const float*>(p.x) + off);
  return __half2float(reinterpret_cast<const __half*>(p.x)[off]);
}

// Stage x[:, kt0*128 : kt0*128 + nwords*8) as permuted fp16 pairs (hi, and lo for fp32 x).
template <bool XF32>
__device__ __forceinline__ void stage_x(const LinArgs& p, const float* rs, uint4* xs_hi, uint4* xs_lo, int rstride,
                                        int kt0, int nwords, int tid, int nth) {
  for (int i = tid; i < p.M * nwords; i += nth) {
    const int m = i / nwords, w = i - m * nwords;
    const int k0 = kt0 * TILE_K + 8 * w;
    const size_t kb = (size_t)x_row(p, m) * p.K + k0;
    uint4 hi;
    if constexpr (XF32) {
      float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + kb);
      float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + kb + 4);
      if (p.ln_w) {
        const float r = rs[m];
        const float4 wa = *reinterpret_cast<const float4*>(p.ln_w + k0);
        const float4 wb = *reinterpret_cast<const float4*>(p.ln_w + k0 + 4);
        a.x = a.x * r * wa.x;
        a.y = a.y * r * wa.y;
        a.z = a.z * r * wa.z;
        a.w = a.w * r * wa.w;
        b.x = b.x * r * wb.x;
        b.y = b.y * r * wb.y;
        b.z = b.z * r * wb.z;
        b.w = b.w * r * wb.w;
      }
      uint4 lo;
      split_pair(a.x, b.x, hi.x, lo.x);  // (x0, x4)
      split_pair(a.y, b.y, hi.y, lo.y);  // (x1, x5)
      split_pair(a.z, b.z, hi.z, lo.z);  // (x2, x6)
      split_pair(a.w, b.w, hi.w, lo.w);  // (x3, x7)
      xs_lo[m * rstride + xswz(w)] = lo;
    } else {
      const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p.x) + kb);
      hi.x = __byte_perm(v.x, v.z, 0x5410);
      hi.y = __byte_perm(v.x, v.z, 0x7632);
      hi.z = __byte_perm(v.y, v.w, 0x5410);
      hi.w = __byte_perm(v.y, v.w, 0x7632);
    }
    xs_hi[m * rstride + xswz(w)] = hi;
  }
}

template <bool XF32>
__device__ __forceinline__ void stage_x(const LinArgs& p, const float* rs, uint4* xs_hi, uint4* xs_lo, int rstride,
                                        int kt0, int nwords) {
  stage_x<XF32>(p, rs, xs_hi, xs_lo, rstride, kt0, nwords, (int)threadIdx.x, (int)blockDim.x);
}

// Epilogue of one finished tile: fin[m * fs + s] holds the fp32 dot product of slot s, batch row m
// (fs = 16, or 17 where a padded stride avoids shared-memory bank conflicts when it is written).
// WARP: the calling warp alone does the work (lanes 0..31); else the whole CTA. The argmax form is
// CTA-only.
template <bool WARP = false>
__device__ void epilogue_tile(const LinArgs& p, const float* fin, int rt, int* s_flag, int fs = 16) {
  const int tid = WARP ? (int)(threadIdx.x & 31) : (int)threadIdx.x;
  const int nth = WARP ? 32 : (int)blockDim.x;
  const int items = p.M * 16;
  if (p.epi == EPI_ARGMAX) {  // m == 1
    if (threadIdx.x < 16) {
      const int row = rt * 16 + threadIdx.x;
      if (row < p.N && p.logits) p.logits[row] = fin[threadIdx.x];
    }
    if (threadIdx.x == 0) {
      unsigned long long best = 0;
      for (int s = 0; s < 16; ++s) {
        const int row = rt * 16 + s;
        if (row < p.N) best = max(best, argmax_key(fin[s], (unsigned)(p.index_offset + row)));
      }
      atomicMax(&p.state->best, best);
      __threadfence();
      *s_flag = p.finalize && (atomicAdd(&p.state->counter, 1u) == (unsigned)(p.RT - 1));
      if (*s_flag) {
        __threadfence();
        const unsigned long long b = atomicExch(&p.state->best, 0ull);
        p.state->counter = 0u;
        publish_token(p.state, p.token_log, (int32_t)argmax_index(b));
      }
    }
    return;
  }
  if (p.epi == EPI_ROPE_KV) {
    const int per = p.hd / 16;
    const int head = rt / per, j = rt - head * per;
    for (int i = tid; i < p.M * 8; i += nth) {
      const int m = i >> 3, s = i & 7;
      const int e1 = j * 8 + s, e2 = p.hd / 2 + j * 8 + s;
      const float x1 = fin[m * fs + s], x2 = fin[m * fs + s + 8];
      const int pos = *p.pos0 + p.pos_offset + m;
      if (head < p.H + p.Hkv) {
        // q * cos + rotate_half(q) * sin, rotate_half(x) = cat(-x[h:], x[:h]) (llama_q4.py:195-221)
        const float* cs = p.rope_cos + (size_t)pos * p.hd;
        const float* sn = p.rope_sin + (size_t)pos * p.hd;
        const float o1 = __fadd_rn(__fmul_rn(x1, cs[e1]), __fmul_rn(-x2, sn[e1]));
        const float o2 = __fadd_rn(__fmul_rn(x2, cs[e2]), __fmul_rn(x1, sn[e2]));
        if (head < p.H) {
          float* q = p.q_out + ((size_t)m * p.H + head) * p.hd;
          q[e1] = o1;
          q[e2] = o2;
        } else {
          __half* kc = p.k_cache + ((size_t)pos * p.Hkv + (head - p.H)) * p.hd;
          kc[e1] = __float2half_rn(o1);
          kc[e2] = __float2half_rn(o2);
        }
      } else {
        __half* vc = p.v_cache + ((size_t)pos * p.Hkv + (head - p.H - p.Hkv)) * p.hd;
        vc[e1] = __float2half_rn(x1);
        vc[e2] = __float2half_rn(x2);
      }
    }
    return;
  }
  for (int i = tid; i < items; i += nth) {
    const int m = i >> 4, s = i & 15;
    if (p.epi == EPI_SWIGLU) {
      const int col = rt * 8 + s;
      if (s < 8 && col < p.n_out)
        store_y(p.y, (size_t)m * p.n_out + col, silu(fin[m * fs + s]) * fin[m * fs + s + 8], p.y_f32);
    } else {
      const int col = rt * 16 + s;
      if (col < p.N) {
        float v = fin[m * fs + s];
        const size_t o = (size_t)m * p.N + col;
        if (p.epi == EPI_ACCUMULATE) v += load_y(p.y, o, p.y_f32);
        store_y(p.y, o, v, p.y_f32);
      }
    }
  }
}

// After the MMAs: sum the warps' accumulators in shared memory (red: W * MT*8 * 16 floats, then
// fin: M*16 floats, aliasing the x staging area), finish split-K through the workspace (last CTA
// of a row tile, fixed order), then the epilogue.
template <int MT>
__device__ __forceinline__ void finish_tile(const LinArgs& p, float (&acc)[MT][4], float* red, int* s_flag, int rt,
                                            int sp) {
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  __syncthreads();
  constexpr int MP = MT * 8;
  float* fin = red + (size_t)W * MP * 16;
#pragma unroll
  for (int nt = 0; nt < MT; ++nt) {
    const int m0 = nt * 8 + 2 * t;
    red[(warp * MP + m0) * 16 + g] = acc[nt][0];
    red[(warp * MP + m0 + 1) * 16 + g] = acc[nt][1];
    red[(warp * MP + m0) * 16 + g + 8] = acc[nt][2];
    red[(warp * MP + m0 + 1) * 16 + g + 8] = acc[nt][3];
  }
  __syncthreads();
  const int items = p.M * 16;
  for (int i = threadIdx.x; i < items; i += blockDim.x) {
    const int m = i >> 4, r = i & 15;
    float v = 0.0f;
    for (int w = 0; w < W; ++w) v += red[(w * MP + m) * 16 + r];
    fin[i] = v;
  }
  __syncthreads();
  if (p.nsplit > 1) {
    const size_t NR = (size_t)p.RT * 16;
    for (int i = threadIdx.x; i < items; i += blockDim.x) {
      const int m = i >> 4, r = i & 15;
      p.ws[((size_t)sp * p.M + m) * NR + (size_t)rt * 16 + r] = fin[i];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) *s_flag = (atomicAdd(&p.counters[rt], 1u) == (unsigned)(p.nsplit - 1));
    __syncthreads();
    if (!*s_flag) return;
    __threadfence();
    for (int i = threadIdx.x; i < items; i += blockDim.x) {
      const int m = i >> 4, r = i & 15;
      float v = 0.0f;
      for (int s = 0; s < p.nsplit; ++s) v += __ldcg(p.ws + ((size_t)s * p.M + m) * NR + (size_t)rt * 16 + r);
      fin[i] = v;
    }
    if (threadIdx.x == 0) p.counters[rt] = 0u;
    __syncthreads();
  }
  epilogue_tile(p, fin, rt, s_flag);
}

// ---- kernel 1: register-staged weights ------------------------------------------------------

template <int MT, bool XF32, int T, bool ILP = false>
__global__ void __launch_bounds__(256) q4_gemv_reg(LinArgs p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ int s_flag;
  __shared__ float s_rs[8];
  __shared__ float s_scratch[64];
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rt = blockIdx.x, sp = blockIdx.y;
  const int ra = tile_row(p, rt, g), rb = tile_row(p, rt, g + 8);
  const int kt0 = sp * p.kps;
  const int kt1 = min(kt0 + p.kps, p.KT);
  const size_t row_u4 = (size_t)p.K / 32;  // 16-byte chunks per weight row
  const int KG = p.K / p.G;
  const uint4* qw4 = reinterpret_cast<const uint4*>(p.qw);

  // 1) this warp's weight tiles and scales: independent of the previous kernel, issued first
  uint4 wa[T], wb[T];
  float sa[T], sb[T];
#pragma unroll
  for (int j = 0; j < T; ++j) {
    const int kt = kt0 + warp + W * j;
    if (kt < kt1) {
      wa[j] = ld_stream_u4(qw4 + (size_t)ra * row_u4 + kt * 4 + t);
      wb[j] = ld_stream_u4(qw4 + (size_t)rb * row_u4 + kt * 4 + t);
      const int grp = (kt * TILE_K) / p.G;
      sa[j] = __half2float(p.scales[(size_t)ra * KG + grp]);
      sb[j] = __half2float(p.scales[(size_t)rb * KG + grp]);
    } else {
      wa[j] = wb[j] = make_uint4(0u, 0u, 0u, 0u);
      sa[j] = sb[j] = 0.0f;
    }
  }
  griddep_launch_dependents();
  griddep_wait();

  // 2) prologue + x staging
  if (p.ln_w) prologue_rms(p, s_rs, s_scratch);
  const int rstride = p.kps * 16 + 4;  // uint4 per staged row; +64 B keeps rows on other bank groups
  uint4* xs_hi = reinterpret_cast<uint4*>(smem_raw);
  uint4* xs_lo = xs_hi + (size_t)p.M * rstride;
  stage_x<XF32>(p, s_rs, xs_hi, xs_lo, rstride, kt0, (kt1 - kt0) * 16);
  __syncthreads();

  // 3) MMAs
  float acc[MT][4];
#pragma unroll
  for (int nt = 0; nt < MT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
  int mrow[MT];
#pragma unroll
  for (int nt = 0; nt < MT; ++nt) mrow[nt] = min(nt * 8 + g, p.M - 1) * rstride;
#pragma unroll
  for (int j = 0; j < T; ++j) {
    const int kt = kt0 + warp + W * j;
    if (kt < kt1) mma_tile<MT, XF32, ILP>(wa[j], wb[j], sa[j], sb[j], xs_hi, xs_lo, mrow, (kt - kt0) * 16 + 4 * t, acc);
  }
  finish_tile<MT>(p, acc, reinterpret_cast<float*>(smem_raw), &s_flag, rt, sp);
}

// ---- kernel 3: weights streamed into shared memory by the TMA engine ---------------------------
//
// Thread 0 issues one bulk copy per weight row of the tile (k-range x 64 B per 128-k tile) into
// shared memory, completing on one mbarrier, before griddepcontrol.wait: the weight tile is in
// flight while the previous kernel finishes and no registers hold it. The row stride in shared
// memory is padded so rows g and g + 8 of a quad land on other banks.
template <int MT, bool XF32>
__global__ void __launch_bounds__(256) q4_gemv_tma(LinArgs p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ int s_flag;
  __shared__ float s_rs[8];
  __shared__ float s_scratch[64];
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rt = blockIdx.x, sp = blockIdx.y;
  const int kt0 = sp * p.kps;
  const int kt1 = min(kt0 + p.kps, p.KT);
  const int ntile = kt1 - kt0;
  const int KG = p.K / p.G;
  unsigned char* sw = smem_raw;                                       // [16][wstride] weights
  __half* ss = reinterpret_cast<__half*>(smem_raw + 16 * p.wstride);  // [16][KG] scales
  uint4* xs_hi = reinterpret_cast<uint4*>(smem_raw + p.x_off);
  const int rstride = p.kps * 16 + 4;
  uint4* xs_lo = xs_hi + (size_t)p.M * rstride;

  // 1) bulk copies of the tile's weight rows (thread 0); scales by plain loads
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    const uint32_t wbytes = (uint32_t)ntile * 64;
    mbar_arrive_expect_tx(&bar, 16u * wbytes);
    const unsigned char* q8 = reinterpret_cast<const unsigned char*>(p.qw);
    for (int s = 0; s < 16; ++s)
      bulk_g2s(sw + s * p.wstride, q8 + (size_t)tile_row(p, rt, s) * (p.K / 2) + (size_t)kt0 * 64, wbytes, &bar);
  }
  for (int i = threadIdx.x; i < 16 * KG; i += blockDim.x) {
    const int s = i / KG, c = i - s * KG;
    ss[i] = p.scales[(size_t)tile_row(p, rt, s) * KG + c];
  }
  griddep_launch_dependents();
  griddep_wait();

  // 2) prologue + x staging
  if (p.ln_w) prologue_rms(p, s_rs, s_scratch);
  stage_x<XF32>(p, s_rs, xs_hi, xs_lo, rstride, kt0, ntile * 16);
  __syncthreads();  // also publishes the initialised barrier to every thread

  // 3) weights landed? (bounded: a copy that never completes sets a status bit instead of hanging;
  // the CTA then skips its MMAs but still arrives on the split-K counter, so the workspace counters
  // return to zero, and waits once more for the copy before exiting)
  const bool ok = mbar_wait_bounded(&bar, 0, kWaitLimitNs);
  const bool failed = __syncthreads_or(!ok);
  if (failed && threadIdx.x == 0) atomicOr(&g_linear_status, kStatusTimeout);

  // 4) MMAs from shared memory
  float acc[MT][4];
#pragma unroll
  for (int nt = 0; nt < MT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
  int mrow[MT];
#pragma unroll
  for (int nt = 0; nt < MT; ++nt) mrow[nt] = min(nt * 8 + g, p.M - 1) * rstride;
  const unsigned char* swa = sw + g * p.wstride + t * 16;
  const unsigned char* swb = sw + (g + 8) * p.wstride + t * 16;
  for (int kl = failed ? ntile : warp; kl < ntile; kl += W) {
    const int grp = ((kt0 + kl) * TILE_K) / p.G;
    const float sa = __half2float(ss[g * KG + grp]);
    const float sb = __half2float(ss[(g + 8) * KG + grp]);
    const uint4 wa = *reinterpret_cast<const uint4*>(swa + kl * 64);
    const uint4 wb = *reinterpret_cast<const uint4*>(swb + kl * 64);
    mma_tile<MT, XF32, false>(wa, wb, sa, sb, xs_hi, xs_lo, mrow, kl * 16 + 4 * t, acc);
  }
  finish_tile<MT>(p, acc, reinterpret_cast<float*>(smem_raw + p.x_off), &s_flag, rt, sp);
  if (failed && threadIdx.x == 0) mbar_wait_bounded(&bar, 0, kWaitLimitNs);
}

// ---- kernel 4: persistent, weights streamed through a TMA ring ---------------------------------
//
// For decode (M == 1, G == 128, K % 1024 == 0, K <= 8192). One CTA per SM loops over row tiles
// rt = blockIdx.x, + gridDim.x, ...; a stage is one row tile's 16 rows x SK k (SK = K up to 4096,
// else K / 2), i.e. 24 or 32 KB, kept kStreamRing stages deep. Warp 0's lanes issue the stage's
// bulk copies in parallel (lane r < 16 the weight row r, lane 16 + r its scales) onto one mbarrier
// per ring slot; the first stages are issued before griddepcontrol.wait, so the projection's
// weight stream starts while the previous kernel finishes. x is staged once per CTA. Each warp
// computes its 128-k tiles of a stage; a row tile's 16 sums are reduced across warps in shared
// memory, the residual operand is fetched when the tile starts, and the greedy-head keys are
// folded per CTA (one atomic per CTA).
constexpr int kStreamRing = 3;

__device__ __forceinline__ int stream_sk(int K) { return K <= 4096 ? K : K / 2; }

template <bool XF32>
__global__ void __launch_bounds__(768) q4_gemv_stream(LinArgs p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t full[kStreamRing];
  __shared__ float s_red[2][24][16];  // by row-tile parity: warps may finish the next tile first
  __shared__ float s_fin[16];
  __shared__ int s_flag;
  __shared__ float s_rs[8];
  __shared__ float s_scratch[64];
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int SK = stream_sk(p.K);
  const int KC = p.K / SK;            // stages per row tile
  const int TPS = SK / TILE_K;        // 128-k tiles per stage
  const int SWB = 16 * SK / 2;        // weight bytes per stage
  const int SSB = 16 * (SK / 128) * 2;  // scale bytes per stage
  const int my_tiles = (p.RT - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int nstages = my_tiles * KC;
  unsigned char* ring_w = smem_raw;
  __half* ring_s = reinterpret_cast<__half*>(smem_raw + kStreamRing * SWB);
  uint4* xs_hi = reinterpret_cast<uint4*>(smem_raw + p.x_off);
  const int rstride = p.K / 8 + 4;  // all of K is staged
  uint4* xs_lo = xs_hi + rstride;
  const unsigned char* q8 = reinterpret_cast<const unsigned char*>(p.qw);
  const int KG = p.K / 128;

  auto issue = [&](int i) {  // warp 0: stage i into ring slot i % kStreamRing
    const int slot = i % kStreamRing;
    const int rt = (int)blockIdx.x + (i / KC) * (int)gridDim.x, kc = i % KC;
    if (lane == 0) mbar_arrive_expect_tx(&full[slot], SWB + SSB);
    __syncwarp();
    const int r = lane & 15;
    const int row = tile_row(p, rt, r);
    if (lane < 16)
      bulk_g2s(ring_w + slot * SWB + r * (SK / 2), q8 + (size_t)row * (p.K / 2) + (size_t)kc * (SK / 2), SK / 2,
               &full[slot]);
    else
      bulk_g2s(ring_s + slot * (SSB / 2) + r * (SK / 128), p.scales + (size_t)row * KG + kc * (SK / 128),
               (SK / 128) * 2, &full[slot]);
  };
  if (warp == 0) {
    if (lane == 0) {
      for (int s = 0; s < kStreamRing; ++s) mbar_init(&full[s], 1);
      fence_mbar_init();
    }
    __syncwarp();
    for (int i = 0; i < kStreamRing && i < nstages; ++i) issue(i);
  }
  griddep_launch_dependents();
  griddep_wait();

  if (p.ln_w) prologue_rms(p, s_rs, s_scratch);
  stage_x<XF32>(p, s_rs, xs_hi, xs_lo, rstride, 0, p.K / 8);
  __syncthreads();

  unsigned long long best = 0;  // thread 0: this CTA's greedy-head key
  float acc[1][4] = {{0.0f, 0.0f, 0.0f, 0.0f}};
  int mrow[1];
  mrow[0] = 0;
  float yres = 0.0f;  // thread s < 16: residual operand of slot s of the current row tile
  for (int i = 0; i < nstages; ++i) {
    const int slot = i % kStreamRing;
    const int rt = (int)blockIdx.x + (i / KC) * (int)gridDim.x, kc = i % KC;
    if (kc == 0 && p.epi == EPI_ACCUMULATE && threadIdx.x < 16) {
      const int col = rt * 16 + threadIdx.x;
      yres = col < p.N ? load_y(p.y, col, p.y_f32) : 0.0f;
    }
    const bool ok = mbar_wait_bounded(&full[slot], (uint32_t)((i / kStreamRing) & 1), kWaitLimitNs);
    if (__syncthreads_or(!ok)) {
      // a copy did not land: stop consuming, let the copies in flight (stages i .. i + ring - 1)
      // finish before the CTA exits, and still fold into the argmax counter below so it completes
      if (threadIdx.x == 0) {
        atomicOr(&g_linear_status, kStatusTimeout);
        for (int j = i; j < i + kStreamRing && j < nstages; ++j)
          mbar_wait_bounded(&full[j % kStreamRing], (uint32_t)((j / kStreamRing) & 1), kWaitLimitNs);
      }
      break;
    }
    const unsigned char* sw = ring_w + slot * SWB + t * 16;
    const __half* ss = ring_s + slot * (SSB / 2);
    for (int tl = warp; tl < TPS; tl += W) {
      const uint4 wa = *reinterpret_cast<const uint4*>(sw + g * (SK / 2) + tl * 64);
      const uint4 wb = *reinterpret_cast<const uint4*>(sw + (g + 8) * (SK / 2) + tl * 64);
      const float sa = __half2float(ss[g * (SK / 128) + tl]);
      const float sb = __half2float(ss[(g + 8) * (SK / 128) + tl]);
      mma_tile<1, XF32, true>(wa, wb, sa, sb, xs_hi, xs_lo, mrow, (kc * TPS + tl) * 16 + 4 * t, acc);
    }
    if (kc == KC - 1) {  // row tile done: column 0 of the accumulators (lanes with t == 0)
      if (t == 0) {
        s_red[(i / KC) & 1][warp][g] = acc[0][0];
        s_red[(i / KC) & 1][warp][g + 8] = acc[0][2];
      }
      acc[0][0] = acc[0][1] = acc[0][2] = acc[0][3] = 0.0f;
    }
    __syncthreads();  // the slot is free again; s_red is complete
    if (warp == 0 && i + kStreamRing < nstages) issue(i + kStreamRing);
    if (kc == KC - 1) {
      if (threadIdx.x < 16) {
        float v = 0.0f;
        for (int w = 0; w < W; ++w) v += s_red[(i / KC) & 1][w][threadIdx.x];
        if (p.epi == EPI_ARGMAX) {
          const int row = rt * 16 + threadIdx.x;
          unsigned long long key = 0;
          if (row < p.N) {
            if (p.logits) p.logits[row] = v;
            key = argmax_key(v, (unsigned)(p.index_offset + row));
          }
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0x0000ffffu, key, o));
          if (threadIdx.x == 0) best = max(best, key);
        } else if (p.epi == EPI_ACCUMULATE) {
          const int col = rt * 16 + threadIdx.x;
          if (col < p.N) store_y(p.y, col, yres + v, p.y_f32);
        } else {
          s_fin[threadIdx.x] = v;
        }
      }
      if (p.epi != EPI_ARGMAX && p.epi != EPI_ACCUMULATE) {
        __syncthreads();
        epilogue_tile(p, s_fin, rt, &s_flag);
      }
    }
  }
  if (p.epi == EPI_ARGMAX && threadIdx.x == 0) {
    atomicMax(&p.state->best, best);
    __threadfence();
    if (p.finalize && atomicAdd(&p.state->counter, 1u) == gridDim.x - 1) {
      __threadfence();
      const unsigned long long b = atomicExch(&p.state->best, 0ull);
      p.state->counter = 0u;
      publish_token(p.state, p.token_log, (int32_t)argmax_index(b));
    }
  }
}

// ---- kernel 6: persistent ring GEMV ------------------------------------------------------------
//
// Decode shapes: M <= 8 rows of x, G == 128, K % 1024 == 0, no fused norm. One CTA per SM (cfg
// tiles = 2: two) with 8 consumer warps and 1 producer warp, sized so that one CTA of the next
// kernel on the stream still fits beside it: that kernel starts under programmatic dependent launch
// and fills its own ring while this one finishes.
//  - A stage is a row pair (two row tiles, 32 rows) x 1024 k: one 2-D TMA box of {128 int32 words,
//    32 rows} of int4 and one of {8 fp16 scales, 32 rows} (SwiGLU and RoPE tiles, whose rows come
//    in runs of 8, take four 8-row boxes of each), 16896 bytes completing on the slot's `full`
//    mbarrier. Few large copies per stage keep the copy engine's per-copy cost off the critical
//    path. The producer refills a slot once the 8 consumer warps have arrived on its `empty`
//    mbarrier. It never waits for the previous kernel (the weights are not that kernel's output);
//    only the consumers wait (griddepcontrol) before staging x.
//  - Consumer warp w takes 128-k tile w of both row tiles of every stage: two independent tiles per
//    barrier wait, sharing one set of x fragments, and keeps the row pair's sums in registers across
//    its stages; it releases a ring slot as soon as its share is in registers. Loop indices advance
//    by increments (no divisions in the stream loop). At a row pair's last stage of this CTA every
//    consumer writes its sums into a reduction slot and arrives on that slot's `red_full`
//    mbarrier; a separate epilogue warp adds the 8 in warp order, finishes the pair (cross-CTA
//    partials, epilogue) and frees the slot (`red_free`), off the consumers' path.
//  - CTAs take equal runs of the NRP x K/1024 stages (NRP row pairs). A row pair cut between CTAs
//    is finished by the last of them through the split-K workspace (partials added in CTA order):
//    deterministic results.
//  - Every wait is bounded. A wait that gives up sets the status bit and the abort flag; the warps
//    then finish their loops without waiting (all counters still arrive, so the workspace is left
//    clean) and the producer waits for its copies in flight before the CTA exits.
constexpr int kRingSK = 1024;
constexpr int kRingCW = kRingSK / TILE_K;  // consumer warps: one 128-k tile of each stage
constexpr int kRingThreads = (kRingCW + 2) * 32;  // + the producer warp and the epilogue warp
constexpr int kRingRed = 4;  // reduction slots (row pairs between the consumers and the epilogue warp)
constexpr int kRingRowPitch = kRingSK / 2;  // a TMA box lands rows densely
constexpr int kRingWBytes = 32 * kRingRowPitch;
constexpr int kRingSlotBytes = kRingWBytes + 32 * 16;  // + 32 rows x 8 fp16 scales (16896, 128-B multiple)
constexpr uint32_t kRingTx = kRingSlotBytes;
constexpr int kRingMaxSlots = 16;

// the CTA whose run of stages [c U / G, (c + 1) U / G) contains stage u
__device__ __forceinline__ int ring_cta_of(long long u, long long U, int G) {
  return (int)(((u + 1) * G + U - 1) / U) - 1;
}

// first weight row of run `half` (slots 0..7 or 8..15) of a SwiGLU / RoPE row tile
__device__ __forceinline__ int ring_run_row(const LinArgs& p, int rt, int half) {
  if (p.epi == EPI_SWIGLU) return half * p.n_out + rt * 8;
  const int per = p.hd / 16;
  const int head = rt / per, j = rt - head * per;
  return head * p.hd + half * (p.hd / 2) + j * 8;
}

// x row 0 (after the row select) for the int8 tile form (mma_tile_i8): per 128-k group, terms
// m = 0..2 as {even, odd} byte words at xq[m * qstride + word] (qstride = K/8 + 8 uint2, so the three
// terms' rows fall on different bank halves) and xg[group] = {X_a, X_b, X_c, sx}. Warp w of nw
// stages groups w, w + nw, ...; lane l holds k = 4l .. 4l + 3 of the group.
template <bool XF32>
__device__ void stage_x_i8(const LinArgs& p, uint2* xq, int4* xg, int qstride, int warp, int lane, int nw) {
  const int NG = p.K / 128;
  const size_t base = (size_t)x_row(p, 0) * p.K;
  for (int grp = warp; grp < NG; grp += nw) {
    const int k0 = grp * 128 + 4 * lane;
    float v[4];
    if constexpr (XF32) {
      const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + base + k0);
      v[0] = f.x, v[1] = f.y, v[2] = f.z, v[3] = f.w;
    } else {
      const uint2 h = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(p.x) + base + k0);
      const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
      const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
      v[0] = f0.x, v[1] = f0.y, v[2] = f1.x, v[3] = f1.y;
    }
    const float am = warp_max(fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
    const float sx = am > 0.0f ? am / 127.0f : 1.0f;
    int q[3][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float u = v[i] / sx;
      const float a = fminf(fmaxf(rintf(u), -127.0f), 127.0f);
      const float r = (u - a) * 254.0f;
      const float b = fminf(fmaxf(rintf(r), -127.0f), 127.0f);
      const float c = fminf(fmaxf(rintf((r - b) * 254.0f), -127.0f), 127.0f);
      q[0][i] = (int)a, q[1][i] = (int)b, q[2][i] = (int)c;
    }
    int X[3];
#pragma unroll
    for (int m = 0; m < 3; ++m) {
      int sum = q[m][0] + q[m][1] + q[m][2] + q[m][3];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      X[m] = sum;
      // k % 8 = 4 (lane & 1) + i: even bytes hold k % 8 = 0, 2, 4, 6, odd bytes 1, 3, 5, 7
      const uint32_t ev = (q[m][0] & 0xFF) | ((q[m][2] & 0xFF) << 8);
      const uint32_t od = (q[m][1] & 0xFF) | ((q[m][3] & 0xFF) << 8);
      const uint32_t mine = ev | (od << 16);
      const uint32_t other = __shfl_xor_sync(0xffffffffu, mine, 1);
      if (!(lane & 1))
        xq[(size_t)m * qstride + grp * 16 + (lane >> 1)] =
            make_uint2((mine & 0xFFFFu) | (other << 16), (mine >> 16) | (other & 0xFFFF0000u));
    }
    if (lane == 0) xg[grp] = make_int4(X[0], X[1], X[2], __float_as_int(sx));
  }
}

// One warp finishes row pair rp: per row tile the 8 warps' sums (red [kRingCW][2][M*16]) in warp
// order, the cross-CTA partials if the pair was cut (`cut`: this CTA holds only part of its stages;
// only a CTA's first and last pair can be), then the epilogue (argmax keys fold into *s_best).
__device__ void ring_finish(const LinArgs& p, const float* red, float* fin, int rp, long long U, bool cut,
                            unsigned long long* s_best, int lane) {
  const int items = p.M * 16;
  for (int i = lane; i < 2 * items; i += 32) {
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kRingCW; ++w) v += red[w * 2 * items + i];
    fin[i] = v;
  }
  __syncwarp();
  if (cut) {
    const long long ua = (long long)rp * p.kc;
    const int c0 = ring_cta_of(ua, U, gridDim.x), c1 = ring_cta_of(ua + p.kc - 1, U, gridDim.x);
    if (c1 > c0) {
      float* part = p.ws + (size_t)rp * p.kc * 2 * items;
      for (int i = lane; i < 2 * items; i += 32) part[((int)blockIdx.x - c0) * 2 * items + i] = fin[i];
      __threadfence();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(&p.counters[rp], 1u) == (unsigned)(c1 - c0);
      if (!__shfl_sync(0xffffffffu, last, 0)) return;
      __threadfence();
      for (int i = lane; i < 2 * items; i += 32) {
        float v = 0.0f;
        for (int q = 0; q <= c1 - c0; ++q) v += __ldcg(part + q * 2 * items + i);
        fin[i] = v;
      }
      if (lane == 0) p.counters[rp] = 0u;
      __syncwarp();
    }
  }
  for (int j = 0; j < 2; ++j) {
    const int rt = 2 * rp + j;
    if (rt >= p.RT) break;
    const float* f = fin + j * items;
    if (p.epi == EPI_ARGMAX) {  // m == 1
      unsigned long long key = 0ull;
      if (lane < 16) {
        const int row = rt * 16 + lane;
        if (row < p.N) {
          if (p.logits) p.logits[row] = f[lane];
          key = argmax_key(f[lane], (unsigned)(p.index_offset + row));
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
      if (lane == 0) atomicMax(s_best, key);
    } else {
      epilogue_tile<true>(p, f, rt, nullptr);
    }
  }
}

template <bool XF32, bool M1>
__global__ void __launch_bounds__(kRingThreads, 2)
    q4_gemv_ring(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap ts, LinArgs p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t full[kRingMaxSlots];
  __shared__ __align__(8) uint64_t empty[kRingMaxSlots];
  __shared__ __align__(8) uint64_t red_full[kRingRed];
  __shared__ __align__(8) uint64_t red_free[kRingRed];
  __shared__ unsigned long long s_best;
  __shared__ volatile int s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.ring_slots, KC = p.kc, nct = gridDim.x, c = blockIdx.x;
  const int NRP = (p.RT + 1) / 2;
  const long long U = (long long)NRP * KC;
  long long u0, u1;
  if (p.split_units) {
    u0 = (long long)c * U / nct;
    u1 = (long long)(c + 1) * U / nct;
  } else {
    u0 = (long long)c * NRP / nct * KC;
    u1 = (long long)(c + 1) * NRP / nct * KC;
  }
  const int n = (int)(u1 - u0);
  const int rp0 = (int)(u0 / KC), kc0 = (int)(u0 - (long long)rp0 * KC);
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRingCW);
    }
    for (int r = 0; r < kRingRed; ++r) {
      mbar_init(&red_full[r], kRingCW);
      mbar_init(&red_free[r], 1);
    }
    s_best = 0ull;
    s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  griddep_launch_dependents();
  int issued = 0;  // producer: stages whose copies were issued

  if (warp == kRingCW + 1) {
    // ---- epilogue warp: finishes this CTA's row pairs in order ----
    const int items = p.M * 16;
    float* red = reinterpret_cast<float*>(smem_raw + p.red_off);  // [kRingRed][kRingCW][2][M * 16]
    const int npairs = n > 0 ? (int)((u1 - 1) / KC) - rp0 + 1 : 0;
    const bool last_cut = n > 0 && (u1 % KC) != 0;
    for (int q = 0; q < npairs; ++q) {
      const int r = q & (kRingRed - 1);
      int ok = !s_abort;
      if (ok) ok = mbar_wait_bounded(&red_full[r], (uint32_t)((q / kRingRed) & 1), kWaitLimitNs);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && lane == 0) {
        atomicOr(&g_linear_status, kStatusTimeout);
        s_abort = 1;
      }
      // cut: the pair began in an earlier CTA, or this CTA's run ends before its last stage
      const bool cut = p.split_units && ((q == 0 && kc0 != 0) || (q == npairs - 1 && last_cut));
      float* rs = red + (size_t)r * kRingCW * 2 * items;
      ring_finish(p, rs, rs, rp0 + q, U, cut, &s_best, lane);  // sums land in warp 0's row
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_free[r]);
    }
  } else if (warp == kRingCW) {
    // ---- producer warp (lane 0 issues) ----
    const uint64_t pol = l2_policy_evict_first();
    const bool paired = p.epi == EPI_SWIGLU || p.epi == EPI_ROPE_KV;
    if (lane == 0) {
      tma_prefetch_map(&tw);
      tma_prefetch_map(&ts);
      int rp = rp0, kc = kc0, slot = 0;
      uint32_t ph = 0;  // parity of the empty phase a refill waits for
      for (int i = 0; i < n; ++i) {
        if (i >= S && !(!s_abort && mbar_wait_bounded(&empty[slot], ph, kWaitLimitNs) && !s_abort)) {
          atomicOr(&g_linear_status, kStatusTimeout);
          s_abort = 1;
          break;
        }
        unsigned char* sl = smem_raw + (size_t)slot * kRingSlotBytes;
        mbar_arrive_expect_tx(&full[slot], kRingTx);
        if (paired) {
          for (int j = 0; j < 2; ++j)
            for (int h = 0; h < 2; ++h) {
              const int row = ring_run_row(p, 2 * rp + j, h);
              tma_load_2d_hint(sl + (16 * j + 8 * h) * kRingRowPitch, &tw, kc * (kRingSK / 8), row, &full[slot], pol);
              tma_load_2d_hint(sl + kRingWBytes + (16 * j + 8 * h) * 16, &ts, kc * 4, row, &full[slot], pol);
            }
        } else {
          tma_load_2d_hint(sl, &tw, kc * (kRingSK / 8), rp * 32, &full[slot], pol);
          tma_load_2d_hint(sl + kRingWBytes, &ts, kc * 4, rp * 32, &full[slot], pol);
        }
        issued = i + 1;
        if (++kc == KC) {
          kc = 0;
          ++rp;
        }
        if (++slot == S) {
          slot = 0;
          if (i >= S) ph ^= 1u;  // refills of round r wait for the consumers' phase r - 1
        }
      }
    }
    __syncwarp();
  } else {
    // ---- consumer warps ----
    const int g = lane >> 2, t = lane & 3;
    griddep_wait();
    const int rstride = p.K / 8 + 4;
    uint4* xs_hi = reinterpret_cast<uint4*>(smem_raw + p.x_off);
    uint4* xs_lo = xs_hi + (size_t)p.M * rstride;
    const int qstride = p.K / 8 + 8;  // M1: int8 x terms
    uint2* xq = reinterpret_cast<uint2*>(smem_raw + p.x_off);
    int4* xg = reinterpret_cast<int4*>(xq + 3 * (size_t)qstride);
    if constexpr (M1)
      stage_x_i8<XF32>(p, xq, xg, qstride, warp, lane, kRingCW);
    else
      stage_x<XF32>(p, nullptr, xs_hi, xs_lo, rstride, 0, p.K / 8, (int)threadIdx.x, kRingCW * 32);
    named_bar_sync(1, kRingCW * 32);
    float* red = reinterpret_cast<float*>(smem_raw + p.red_off);  // [kRingRed][kRingCW][2][M * 16]
    const int items = p.M * 16;
    float acc[2][1][4];
    float hl[2][2];  // M1: rows g and g + 8 of both row tiles (lanes t == 0)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][0][e] = 0.0f;
      hl[j][0] = hl[j][1] = 0.0f;
    }
    int mrow[1];
    mrow[0] = min(g, p.M - 1) * rstride;
    int rp = rp0, kc = kc0, slot = 0, q = 0;
    uint32_t ph = 0;
    for (int i = 0; i < n; ++i) {
      const bool last = kc == KC - 1 || i == n - 1;
      int ok = !s_abort;
      if (ok) ok = mbar_wait_bounded(&full[slot], ph, kWaitLimitNs);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && lane == 0) {
        atomicOr(&g_linear_status, kStatusTimeout);
        s_abort = 1;
      }
      uint4 w[2][2];
      float sc[2][2];
      const unsigned char* sl = smem_raw + (size_t)slot * kRingSlotBytes;
      const __half* ss = reinterpret_cast<const __half*>(sl + kRingWBytes);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        if (ok) {
          w[j][0] = *reinterpret_cast<const uint4*>(sl + (16 * j + g) * kRingRowPitch + warp * 64 + t * 16);
          w[j][1] = *reinterpret_cast<const uint4*>(sl + (16 * j + g + 8) * kRingRowPitch + warp * 64 + t * 16);
          sc[j][0] = __half2float(ss[(16 * j + g) * 8 + warp]);
          sc[j][1] = __half2float(ss[(16 * j + g + 8) * 8 + warp]);
        } else {
          w[j][0] = w[j][1] = make_uint4(0u, 0u, 0u, 0u);
          sc[j][0] = sc[j][1] = 0.0f;
        }
      }
      __syncwarp();  // registers hold this warp's share: the slot may be refilled
      if (lane == 0) mbar_arrive(&empty[slot]);
      const int ktile = kc * kRingCW + warp;  // 128-k tile = scale group
      if constexpr (M1) {
        uint2 xv[4];
        if (g < 3) {
          const uint4* src = reinterpret_cast<const uint4*>(xq + (size_t)g * qstride + ktile * 16 + 4 * t);
          const uint4 lo = src[0], hi = src[1];
          xv[0] = make_uint2(lo.x, lo.y), xv[1] = make_uint2(lo.z, lo.w);
          xv[2] = make_uint2(hi.x, hi.y), xv[3] = make_uint2(hi.z, hi.w);
        } else {
          xv[0] = xv[1] = xv[2] = xv[3] = make_uint2(0u, 0u);
        }
        const int4 xgv = xg[ktile];
#pragma unroll
        for (int j = 0; j < 2; ++j) mma_tile_i8(w[j][0], w[j][1], sc[j][0], sc[j][1], xv, xgv, hl[j]);
      } else {
        const int wbase = ktile * 16 + 4 * t;
#pragma unroll
        for (int j = 0; j < 2; ++j)
          mma_tile<1, XF32, true>(w[j][0], w[j][1], sc[j][0], sc[j][1], xs_hi, xs_lo, mrow, wbase, acc[j]);
      }
      if (last) {
        // reduction slot of this CTA's q-th row pair; wait until the epilogue warp has read its
        // previous use (pair q - kRingRed)
        const int r = q & (kRingRed - 1);
        if (q >= kRingRed) {
          int fr = !s_abort;
          if (fr) fr = mbar_wait_bounded(&red_free[r], (uint32_t)(((q / kRingRed) - 1) & 1), kWaitLimitNs);
          if (!__all_sync(0xffffffffu, fr) && lane == 0) {
            atomicOr(&g_linear_status, kStatusTimeout);
            s_abort = 1;
          }
        }
        float* rw = red + ((size_t)r * kRingCW + warp) * 2 * items;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float* r = rw + j * items;
          if constexpr (M1) {
            if (t == 0) {
              r[g] = hl[j][0];
              r[g + 8] = hl[j][1];
            }
            hl[j][0] = hl[j][1] = 0.0f;
          } else {
            const int m0 = 2 * t;
            if (m0 < p.M) {
              r[m0 * 16 + g] = acc[j][0][0];
              r[m0 * 16 + g + 8] = acc[j][0][2];
            }
            if (m0 + 1 < p.M) {
              r[(m0 + 1) * 16 + g] = acc[j][0][1];
              r[(m0 + 1) * 16 + g + 8] = acc[j][0][3];
            }
            acc[j][0][0] = acc[j][0][1] = acc[j][0][2] = acc[j][0][3] = 0.0f;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&red_full[r]);  // release: the epilogue warp's wait sees the sums
        ++q;
      }
      if (++kc == KC) {
        kc = 0;
        ++rp;
      }
      if (++slot == S) {
        slot = 0;
        ph ^= 1u;
      }
    }
  }
  __syncthreads();
  if (warp == kRingCW && lane == 0 && s_abort) {
    // copies still in flight land in this CTA's shared memory: wait for them before exiting
    for (int i = max(0, issued - S); i < issued; ++i)
      mbar_wait_bounded(&full[i % S], (uint32_t)((i / S) & 1), kWaitLimitNs);
  }
  if (p.epi == EPI_ARGMAX && threadIdx.x == 0) {
    atomicMax(&p.state->best, s_best);
    __threadfence();
    if (p.finalize && atomicAdd(&p.state->counter, 1u) == gridDim.x - 1) {
      __threadfence();
      const unsigned long long b = atomicExch(&p.state->best, 0ull);
      p.state->counter = 0u;
      publish_token(p.state, p.token_log, (int32_t)argmax_index(b));
    }
  }
}

// ---- kernel 2: generic SIMT ---------------------------------------------------------------
//
// One CTA per 16-slot tile and all batch rows; warp w computes slots 2w and 2w + 1 with fp32 FMAs
// on (nib - 8) * scale (exact), lanes striding over the words of the row.
template <bool XF32>
__global__ void __launch_bounds__(256) q4_linear_simt(LinArgs p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ int s_flag;
  __shared__ float s_rs[8];
  __shared__ float s_scratch[64];
  float* fin = reinterpret_cast<float*>(smem_raw);  // [M][16]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rt = blockIdx.x;
  griddep_launch_dependents();
  griddep_wait();
  if (p.ln_w) prologue_rms(p, s_rs, s_scratch);
  const int KW = p.K / 8, KG = p.K / p.G;
  for (int s = 2 * warp; s < 2 * warp + 2; ++s) {
    const int row = tile_row(p, rt, s);
    for (int m0 = 0; m0 < p.M; m0 += 8) {
      const int mcount = min(8, p.M - m0);
      float acc[8];
#pragma unroll
      for (int m = 0; m < 8; ++m) acc[m] = 0.0f;
      for (int w = lane; w < KW; w += 32) {
        const int32_t word = __ldg(p.qw + (size_t)row * KW + w);
        const float sc = __half2float(p.scales[(size_t)row * KG + (8 * w) / p.G]);
        float wv[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) wv[b] = (float)(((word >> (4 * b)) & 15) - 8) * sc;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          if (m < mcount) {
            float d = 0.0f;
#pragma unroll
            for (int b = 0; b < 8; ++b) d = fmaf(wv[b], x_value(p, s_rs, m0 + m, 8 * w + b, XF32), d);
            acc[m] += d;
          }
        }
      }
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const float v = warp_sum(acc[m]);
        if (lane == 0 && m < mcount) fin[(m0 + m) * 16 + s] = v;
      }
    }
  }
  __syncthreads();
  epilogue_tile(p, fin, rt, &s_flag);
}

// ---- kernel 5: tcgen05 int4-weight GEMM (prefill, many x rows) ----------------------------------
//
// One CTA per (128 x rows, BN weight rows = BN/16 row tiles, k split). A pre-pass writes x as two
// fp16 matrices hi / lo (x = hi + lo, ~22 bits) in the nibble-permuted k order of dequant_word;
// the TMA engine streams their 128 x 64 tiles into a 128-byte-swizzled ring, hi and lo of a stage
// back to back. Raw int4 rows arrive
// by bulk copies (32 bytes per row and 64-k stage, rows picked by tile_row, so SwiGLU and RoPE
// tiles keep their row pairs); four dequant warps turn them into exact fp16 (nib - 8) tiles in the
// same swizzled K-major layout. One thread issues tcgen05.mma per stage, alternating between two TMEM
// accumulators by scale group. BN = 128: the weights are the A operand (M = 128 weight rows) and the
// stage's hi and lo x tiles together the B operand (N = 256: tokens' hi then lo), so a 64-k stage is
// 4 MMAs of N = 256 (measured: 8 MMAs of N = 128 issue at about half the tensor core's rate); the
// accumulator's TMEM lane is a weight row, its columns the tokens' hi and lo partial sums. BN = 64:
// x is A (M = 128 tokens), the weights B (N = 64), hi and lo into one accumulator. Eight epilogue
// warps read each finished group from TMEM, scale it by the group's fp16 scale and add it to fp32
// registers -- the same arithmetic as kernels 1 and 3 (per-group fp32 sum of exact products, then
// one fmaf with the scale). Split-K partials go through the workspace as in
// the other kernels; the shared epilogue_tile then handles store / accumulate / SwiGLU / RoPE+KV.
constexpr int K5_BM = 128, K5_BK = 64;
constexpr int K5_RAW = 8, K5_XS = 3, K5_DS = 3;
constexpr int K5_THREADS = 15 * 32;  // 8 epilogue, 4 dequant, 1 weight producer, 1 MMA, 1 x producer
constexpr int K5_MAX_GROUPS = 64;    // scales of up to 64 groups per CTA stay in shared memory
constexpr int K5_FS = 17;            // padded fin row stride (conflict-free column writes)

template <int BN>
struct K5 {
  static constexpr int X_BYTES = K5_BM * K5_BK * 2;  // one of hi / lo
  static constexpr int XSTAGE = 2 * X_BYTES;
  static constexpr int W_BYTES = BN * K5_BK * 2;
  static constexpr int RAW_BYTES = BN * K5_BK / 2;
  static constexpr int X_OFF = 0;
  static constexpr int W_OFF = X_OFF + K5_XS * XSTAGE;
  static constexpr int RAW_OFF = W_OFF + K5_DS * W_BYTES;
  static constexpr int SC_OFF = RAW_OFF + K5_RAW * RAW_BYTES;
  static constexpr int SMEM = SC_OFF + K5_MAX_GROUPS * BN * 2 + 1024;  // + alignment slack
  static_assert(BN * K5_BM * 4 / 16 * K5_FS <= K5_XS * XSTAGE, "final tile must fit in the x ring");
};

// Row blockIdx.x of x, RMS-normalised and scaled by ln_w, -> hi / lo fp16 in the permuted k order.
// The sum of squares runs in the order of rmsnorm_kernel's one-pass form (thread t adds float4s
// t, t + 256, ... in turn, then the warps' sums in warp order) and each value is (x rs) w as there,
// so the split sees the same fp32 values as a separate RMSNorm launch would write.
__device__ void xsplit_norm_row(const LinArgs& p, __half* xh, __half* xl) {
  __shared__ float red[32];
  const int m = blockIdx.x;
  const float* xr = reinterpret_cast<const float*>(p.x) + (size_t)x_row(p, m) * p.K;
  const float4* x4 = reinterpret_cast<const float4*>(xr);
  const int n4 = p.K / 4;
  float ss = 0.0f;
  for (int j = threadIdx.x; j < n4; j += blockDim.x) {
    const float4 v = x4[j];
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = 1.0f / sqrtf(t / (float)p.K + p.eps);
  }
  __syncthreads();
  const float rs = red[0];
  const float4* w4 = reinterpret_cast<const float4*>(p.ln_w);
  for (int w = threadIdx.x; w < p.K / 8; w += blockDim.x) {
    float4 a = x4[2 * w], b = x4[2 * w + 1];
    const float4 ga = w4[2 * w], gb = w4[2 * w + 1];
    a = make_float4(a.x * rs * ga.x, a.y * rs * ga.y, a.z * rs * ga.z, a.w * rs * ga.w);
    b = make_float4(b.x * rs * gb.x, b.y * rs * gb.y, b.z * rs * gb.z, b.w * rs * gb.w);
    uint4 hi, lo;
    split_pair(a.x, b.x, hi.x, lo.x);
    split_pair(a.y, b.y, hi.y, lo.y);
    split_pair(a.z, b.z, hi.z, lo.z);
    split_pair(a.w, b.w, hi.w, lo.w);
    *reinterpret_cast<uint4*>(xh + (size_t)m * p.K + 8 * w) = hi;
    *reinterpret_cast<uint4*>(xl + (size_t)m * p.K + 8 * w) = lo;
  }
}

// x [M, K] (fp32 or fp16, rows from x_row) -> hi / lo fp16 [M, K] in the permuted k order (fp32 x
// with ln_w: the fused RMSNorm form above)
template <bool XF32>
__global__ void __launch_bounds__(256) q4_xsplit(LinArgs p, __half* xh, __half* xl) {
  griddep_wait();
  if constexpr (XF32) {
    if (p.ln_w) {  // fused RMSNorm (rms_norm, llama_q4.py:141-142): one CTA per row, grid = M
      xsplit_norm_row(p, xh, xl);
      griddep_launch_dependents();
      return;
    }
  }
  const int kw = p.K / 8;
  const int n = p.M * kw;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int m = i / kw, w = i - m * kw;
    const size_t src = (size_t)x_row(p, m) * p.K + 8 * w;
    uint4 hi, lo = make_uint4(0, 0, 0, 0);
    if constexpr (XF32) {
      const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + src);
      const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + src + 4);
      split_pair(a.x, b.x, hi.x, lo.x);
      split_pair(a.y, b.y, hi.y, lo.y);
      split_pair(a.z, b.z, hi.z, lo.z);
      split_pair(a.w, b.w, hi.w, lo.w);
    } else {
      const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p.x) + src);
      hi.x = __byte_perm(v.x, v.z, 0x5410);
      hi.y = __byte_perm(v.x, v.z, 0x7632);
      hi.z = __byte_perm(v.y, v.w, 0x5410);
      hi.w = __byte_perm(v.y, v.w, 0x7632);
    }
    *reinterpret_cast<uint4*>(xh + (size_t)m * p.K + 8 * w) = hi;
    if constexpr (XF32) *reinterpret_cast<uint4*>(xl + (size_t)m * p.K + 8 * w) = lo;
  }
  griddep_launch_dependents();
}

// The BN weight rows of a kernel-5 CTA, as NB runs of consecutive rows (one TMA box each): row
// tiles rt0 .. rt0 + RTS - 1 hold 16 consecutive rows (store / accumulate), gate rows then the
// matching up rows (SwiGLU), or per head the first and second halves of its elements (RoPE, where
// slots s and s + 8 pair elements e and e + hd/2).
__host__ __device__ __forceinline__ int k5_nb(int epi, int RTS, int hd) {
  if (epi == EPI_SWIGLU) return 2;
  if (epi == EPI_ROPE_KV) {
    const int per = hd / 16;
    return RTS <= per ? 2 : 2 * (RTS / per);
  }
  return 1;
}
__device__ __forceinline__ int k5_run_row(const LinArgs& p, int rt0, int RTS, int b) {
  if (p.epi == EPI_SWIGLU) return (b ? p.n_out : 0) + rt0 * 8;
  if (p.epi == EPI_ROPE_KV) {
    const int per = p.hd / 16;
    if (RTS <= per) {
      const int h = rt0 / per, j0 = rt0 - h * per;
      return h * p.hd + b * (p.hd / 2) + 8 * j0;
    }
    return (rt0 / per + (b >> 1)) * p.hd + (b & 1) * (p.hd / 2);
  }
  return rt0 * 16;
}
// shared-memory weight row c -> (row tile - rt0, slot)
__device__ __forceinline__ void k5_col(const LinArgs& p, int RTS, int c, int& rtl, int& s) {
  if (p.epi == EPI_SWIGLU || p.epi == EPI_ROPE_KV) {
    const int nb = k5_nb(p.epi, RTS, p.hd), rpb = RTS * 16 / nb;
    const int b = c / rpb, cc = c - b * rpb;
    const int per = p.hd / 16;
    const int hb = (p.epi == EPI_ROPE_KV && RTS > per) ? (b >> 1) * per : 0;
    rtl = hb + (cc >> 3);
    s = (cc & 7) + 8 * (b & 1);
  } else {
    rtl = c >> 4;
    s = c & 15;
  }
}

template <int BN, bool XF32>
__global__ void __launch_bounds__(K5_THREADS, 1)
    q4_gemm_tc(const __grid_constant__ CUtensorMap txh, const __grid_constant__ CUtensorMap txl,
               const __grid_constant__ CUtensorMap tw, LinArgs p) {
  using L = K5<BN>;
  constexpr int RTS = BN / 16;  // row tiles per CTA
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t raw_full[K5_RAW], raw_empty[K5_RAW], x_full[K5_XS], x_empty[K5_XS], deq_full[K5_DS],
      deq_empty[K5_DS], acc_full[2], acc_free[2], mma_done;
  __shared__ uint32_t s_tmem;
  __shared__ int s_fail, s_flag;
  __shared__ int s_raw_n, s_x_n, s_mma_n;  // stages issued by each producer (drained on failure)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * K5_BM;
  const int rt0 = blockIdx.y * RTS;
  const int z = blockIdx.z;
  const int NG = p.K / p.G, SPG = p.G / K5_BK;
  const int g0 = (int)((long long)z * NG / p.nsplit), g1 = (int)((long long)(z + 1) * NG / p.nsplit);
  const int NGL = g1 - g0, NS = NGL * SPG;
  __half* s_sc = reinterpret_cast<__half*>(smem + L::SC_OFF);

  if (threadIdx.x == 0) {
    for (int i = 0; i < K5_RAW; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 4);
    }
    for (int i = 0; i < K5_XS; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < K5_DS; ++i) {
      mbar_init(&deq_full[i], 4);
      mbar_init(&deq_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_free[i], 8);
    }
    mbar_init(&mma_done, 1);
    s_fail = 0;
    s_raw_n = s_x_n = s_mma_n = 0;
    fence_mbar_init();
  }
  // BN = 128: weights as A, x hi | lo as B (see above); BN = 64: x as A
  constexpr bool SWAP = BN == 128;
  constexpr int XN = XF32 ? 2 * K5_BM : K5_BM;  // B rows when swapped: tokens' hi, then lo
  constexpr int ACOLS = SWAP ? XN : BN;         // TMEM columns of one group accumulator
  if (warp == 13) tmem_alloc(&s_tmem, 2 * ACOLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 12) {
    // weight producer: NB TMA boxes of raw int4 rows per 64-k stage (no dependence on the previous
    // kernel: starts before the wait)
    if (lane == 0) {
      const int nb = k5_nb(p.epi, RTS, p.hd), rpb = BN / nb;
      for (int i = 0; i < NS; ++i) {
        const int rs = i % K5_RAW, rr = i / K5_RAW;
        if (rr > 0 && !mbar_wait_bounded(&raw_empty[rs], (rr - 1) & 1, kWaitLimitNs)) {
          s_fail = 1;
          break;
        }
        mbar_arrive_expect_tx(&raw_full[rs], L::RAW_BYTES);
        const int j = g0 * SPG + i;
        uint8_t* dst = smem + L::RAW_OFF + rs * L::RAW_BYTES;
        for (int b = 0; b < nb; ++b) tma_load_2d(dst + b * rpb * 32, &tw, j * 8, k5_run_row(p, rt0, RTS, b), &raw_full[rs]);
        s_raw_n = i + 1;
      }
    }
    __syncwarp();
  } else if (warp == 8 + 4 + 2) {
    // x producer (waits for the pre-pass that wrote hi / lo)
    griddep_wait();
    if (lane == 0) {
      for (int i = 0; i < NS; ++i) {
        const int xs = i % K5_XS, xr = i / K5_XS;
        if (xr > 0 && !mbar_wait_bounded(&x_empty[xs], (xr - 1) & 1, kWaitLimitNs)) {
          s_fail = 1;
          break;
        }
        const int kx = (g0 * SPG + i) * K5_BK;
        uint8_t* dst = smem + L::X_OFF + xs * L::XSTAGE;
        mbar_arrive_expect_tx(&x_full[xs], XF32 ? L::XSTAGE : L::X_BYTES);
        tma_load_2d(dst, &txh, kx, m0, &x_full[xs]);
        if constexpr (XF32) tma_load_2d(dst + L::X_BYTES, &txl, kx, m0, &x_full[xs]);
        s_x_n = i + 1;
      }
    }
    __syncwarp();
  } else if (warp >= 8 && warp < 12) {
    // dequant warps: scales of this CTA's groups once, then exact fp16 (nib - 8) tiles
    const int t = threadIdx.x - 256;
    const int nb = k5_nb(p.epi, RTS, p.hd), rpb = BN / nb;
    for (int idx = t; idx < NGL * BN; idx += 128) {
      const int gl = idx / BN, c = idx - gl * BN;
      const int row = min(k5_run_row(p, rt0, RTS, c / rpb) + c % rpb, p.N - 1);  // rows past N are zero
      s_sc[idx] = p.scales[(size_t)row * NG + g0 + gl];
    }
    asm volatile("bar.sync 1, 384;" ::: "memory");  // scales visible to the epilogue warps
    for (int i = 0; i < NS; ++i) {
      const int rs = i % K5_RAW, ds = i % K5_DS;
      bool ok = mbar_wait_bounded(&raw_full[rs], (i / K5_RAW) & 1, kWaitLimitNs);
      if (ok && i >= K5_DS) ok = mbar_wait_bounded(&deq_empty[ds], ((i / K5_DS) - 1) & 1, kWaitLimitNs);
      if (!ok) {
        s_fail = 1;
        break;
      }
      const uint32_t* raw = reinterpret_cast<const uint32_t*>(smem + L::RAW_OFF + rs * L::RAW_BYTES);
      uint8_t* wt = smem + L::W_OFF + ds * L::W_BYTES;
#pragma unroll
      for (int v = 0; v < BN * 8 / 128; ++v) {
        const int wi = t + 128 * v;
        const int r = wi >> 3, c = wi & 7;
        const uint32_t w = raw[wi];
        uint4 o;
        o.x = hsub2_u(lop_and_or(w, 0x000F000Fu, 0x64006400u), 0x64086408u);
        o.y = hsub2_u(lop_and_or(w >> 4, 0x000F000Fu, 0x64006400u), 0x64086408u);
        o.z = hsub2_u(lop_and_or(w >> 8, 0x000F000Fu, 0x64006400u), 0x64086408u);
        o.w = hsub2_u(lop_and_or(w >> 12, 0x000F000Fu, 0x64006400u), 0x64086408u);
        *reinterpret_cast<uint4*>(wt + r * 128 + ((c ^ (r & 7)) << 4)) = o;
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&deq_full[ds]);
        mbar_arrive(&raw_empty[rs]);
      }
    }
  } else if (warp == 13) {
    if (lane == 0) {
      constexpr uint32_t idesc = SWAP ? idesc_f16_f32(BN, XN, false, false) : idesc_f16_f32(K5_BM, BN, false, false);
      for (int i = 0; i < NS; ++i) {
        const int xs = i % K5_XS, ds = i % K5_DS;
        const int gl = i / SPG, kg = i - gl * SPG, b = gl & 1;
        bool ok = true;
        if (kg == 0 && gl >= 2) ok = mbar_wait_bounded(&acc_free[b], ((gl >> 1) - 1) & 1, kWaitLimitNs);
        ok = ok && mbar_wait_bounded(&x_full[xs], (i / K5_XS) & 1, kWaitLimitNs);
        ok = ok && mbar_wait_bounded(&deq_full[ds], (i / K5_DS) & 1, kWaitLimitNs);
        if (!ok) {
          s_fail = 1;
          break;
        }
        tc_fence_after();
        const uint32_t xa = smem_u32(smem + L::X_OFF + xs * L::XSTAGE);
        const uint32_t wb = smem_u32(smem + L::W_OFF + ds * L::W_BYTES);
        const uint32_t d = tmem + b * ACOLS;
#pragma unroll
        for (int kk = 0; kk < K5_BK / 16; ++kk) {
          const uint64_t wd = sw128_desc(wb + kk * 32, 16, 1024);
          if constexpr (SWAP) {  // B spans the hi tile and the lo tile right after it (rows 128..255)
            tc_mma_f16(d, wd, sw128_desc(xa + kk * 32, 16, 1024), idesc, (kg | kk) != 0);
          } else {
            tc_mma_f16(d, sw128_desc(xa + kk * 32, 16, 1024), wd, idesc, (kg | kk) != 0);
            if constexpr (XF32) tc_mma_f16(d, sw128_desc(xa + L::X_BYTES + kk * 32, 16, 1024), wd, idesc, 1u);
          }
        }
        tc_commit(&x_empty[xs]);
        tc_commit(&deq_empty[ds]);
        if (kg == SPG - 1) tc_commit(&acc_full[b]);
        s_mma_n = i + 1;
      }
    }
    __syncwarp();
  }

  // epilogue warps: scale each finished group and accumulate in registers. Swapped: thread (warp q,
  // lane) holds weight row q * 32 + lane (its TMEM lane) for tokens [h * 64, h * 64 + 64); otherwise
  // token row q * 32 + lane for weight columns [h * BN / 2, (h + 1) * BN / 2).
  constexpr int HC = SWAP ? K5_BM / 2 : BN / 2;  // values per epilogue thread
  float acc[HC];
#pragma unroll
  for (int c = 0; c < HC; ++c) acc[c] = 0.0f;
  const int q = warp & 3, h = warp >> 2;
  if (warp < 8) {
    asm volatile("bar.sync 1, 384;" ::: "memory");
    for (int gl = 0; gl < NGL; ++gl) {
      const int b = gl & 1;
      if (!mbar_wait_bounded(&acc_full[b], (gl >> 1) & 1, kWaitLimitNs)) {
        s_fail = 1;
        break;
      }
      tc_fence_after();
      const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16) + b * ACOLS;
      if constexpr (SWAP) {
        const float sv = __half2float(s_sc[gl * BN + q * 32 + lane]);  // this weight row's group scale
#pragma unroll
        for (int cc = 0; cc < HC; cc += 16) {  // 16 columns of hi and of lo at a time (registers)
          uint32_t rh[16];
          tmem_ld_32x16(lane_base + h * HC + cc, rh);
          if constexpr (XF32) {
            uint32_t rl[16];
            tmem_ld_32x16(lane_base + K5_BM + h * HC + cc, rl);
#pragma unroll
            for (int e = 0; e < 16; ++e)
              acc[cc + e] = fmaf(sv, __uint_as_float(rh[e]) + __uint_as_float(rl[e]), acc[cc + e]);
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) acc[cc + e] = fmaf(sv, __uint_as_float(rh[e]), acc[cc + e]);
          }
        }
      } else {
        const __half* sc = s_sc + gl * BN + h * HC;
#pragma unroll
        for (int cc = 0; cc < HC; cc += 32) {
          uint32_t r[32];
          tmem_ld_32x32(lane_base + h * HC + cc, r);
#pragma unroll
          for (int e = 0; e < 32; ++e) acc[cc + e] = fmaf(__half2float(sc[cc + e]), __uint_as_float(r[e]), acc[cc + e]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_free[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (s_fail) {
    // a wait gave up: let this CTA's MMAs and copies in flight finish (bounded) before the TMEM
    // is freed and the CTA exits
    if (warp == 13 && lane == 0 && s_mma_n > 0) {
      tc_commit(&mma_done);
      mbar_wait_bounded(&mma_done, 0, kWaitLimitNs);
    }
    if (threadIdx.x == 0) {
      for (int i = max(0, s_raw_n - K5_RAW); i < s_raw_n; ++i)
        mbar_wait_bounded(&raw_full[i % K5_RAW], (uint32_t)((i / K5_RAW) & 1), kWaitLimitNs);
      for (int i = max(0, s_x_n - K5_XS); i < s_x_n; ++i)
        mbar_wait_bounded(&x_full[i % K5_XS], (uint32_t)((i / K5_XS) & 1), kWaitLimitNs);
    }
    __syncthreads();
  }
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * ACOLS);
  }
  if (s_fail) {
    if (threadIdx.x == 0) {
      atomicOr(&g_linear_status, kStatusTimeout);
      // still arrive on the split-K counter (the tile's result is void, but the counter must end
      // at zero for the next call that uses this workspace): the last arrival resets it
      if (p.nsplit > 1) {
        const size_t tile = (size_t)blockIdx.x * gridDim.y + blockIdx.y;
        if (atomicAdd(&p.counters[tile], 1u) == (unsigned)(p.nsplit - 1)) p.counters[tile] = 0u;
      }
    }
    griddep_launch_dependents();
    return;
  }
  griddep_wait();  // the epilogue reads / writes y, q_out and the caches
  // the x ring is free now: fin[rt][m][16] for this CTA's row tiles
  float* fin = reinterpret_cast<float*>(smem + L::X_OFF);
  const int m = q * 32 + lane;
  const int rows = min(K5_BM, p.M - m0);
  const int n_tiles = gridDim.y;
  if (p.nsplit == 1) {
    if (warp < 8) {
      if constexpr (SWAP) {
        int rtl, sl;
        k5_col(p, RTS, m, rtl, sl);  // m = this thread's weight row
#pragma unroll
        for (int j = 0; j < HC; ++j) fin[(rtl * K5_BM + h * HC + j) * K5_FS + sl] = acc[j];
      } else {
#pragma unroll
        for (int c = 0; c < HC; ++c) {
          int rtl, sl;
          k5_col(p, RTS, h * HC + c, rtl, sl);
          fin[(rtl * K5_BM + m) * K5_FS + sl] = acc[c];
        }
      }
    }
    __syncthreads();
  } else {
    // partial tile [128][BN] of split z, then the last CTA of the tile sums the splits in order
    const size_t tile = (size_t)blockIdx.x * n_tiles + blockIdx.y;
    const size_t tiles = (size_t)gridDim.x * n_tiles;
    if (warp < 8) {
      if constexpr (SWAP) {  // [token][weight row]: a warp writes 32 consecutive rows per token
        float* dst = p.ws + ((size_t)z * tiles + tile) * (K5_BM * BN) + (size_t)(h * HC) * BN + m;
#pragma unroll
        for (int j = 0; j < HC; ++j) dst[(size_t)j * BN] = acc[j];
      } else {
        float* dst = p.ws + ((size_t)z * tiles + tile) * (K5_BM * BN) + (size_t)m * BN + h * HC;
#pragma unroll
        for (int c = 0; c < HC; c += 4)
          *reinterpret_cast<float4*>(dst + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
      }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_flag = atomicAdd(&p.counters[tile], 1u) == (unsigned)(p.nsplit - 1);
    __syncthreads();
    if (!s_flag) {
      griddep_launch_dependents();
      return;
    }
    __threadfence();
    // four columns per thread and step, the splits' loads issued together, summed in split order
    const float4* part = reinterpret_cast<const float4*>(p.ws + (size_t)tile * (K5_BM * BN));
    const size_t zs = tiles * (K5_BM * BN) / 4;
    for (int i = threadIdx.x; i < K5_BM * BN / 4; i += blockDim.x) {
      float4 v = __ldcg(part + i);
      int sp = 1;
      for (; sp + 4 <= p.nsplit; sp += 4) {
        const float4 a0 = __ldcg(part + sp * zs + i), a1 = __ldcg(part + (sp + 1) * zs + i);
        const float4 a2 = __ldcg(part + (sp + 2) * zs + i), a3 = __ldcg(part + (sp + 3) * zs + i);
        v.x = (((v.x + a0.x) + a1.x) + a2.x) + a3.x;
        v.y = (((v.y + a0.y) + a1.y) + a2.y) + a3.y;
        v.z = (((v.z + a0.z) + a1.z) + a2.z) + a3.z;
        v.w = (((v.w + a0.w) + a1.w) + a2.w) + a3.w;
      }
      for (; sp < p.nsplit; ++sp) {
        const float4 a0 = __ldcg(part + sp * zs + i);
        v.x += a0.x;
        v.y += a0.y;
        v.z += a0.z;
        v.w += a0.w;
      }
      const int mm = (4 * i) / BN, col = 4 * i - mm * BN;
      const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int rtl, sl;
        k5_col(p, RTS, col + e, rtl, sl);
        fin[(rtl * K5_BM + mm) * K5_FS + sl] = vv[e];
      }
    }
    if (threadIdx.x == 0) p.counters[tile] = 0u;
    __syncthreads();
  }
  // rows [m0, m0 + rows) as a problem of their own for the shared epilogue
  LinArgs e = p;
  e.M = rows;
  const size_t yrow = (size_t)(p.epi == EPI_SWIGLU ? p.n_out : p.N) * (p.y_f32 ? 4 : 2);
  if (p.y) e.y = reinterpret_cast<char*>(p.y) + (size_t)m0 * yrow;
  if (p.q_out) e.q_out = p.q_out + (size_t)m0 * p.H * p.hd;
  e.pos_offset = p.pos_offset + m0;
  for (int r = 0; r < RTS; ++r) {
    if (rt0 + r >= p.RT) break;
    epilogue_tile(e, fin + (size_t)r * K5_BM * K5_FS, rt0 + r, &s_flag, K5_FS);
  }
  griddep_launch_dependents();
}

// ---- planning ------------------------------------------------------------------------------

struct Plan {
  int kernel = 2;  // 1 = register-staged MMA, 2 = SIMT, 3 = TMA-staged MMA, 4 = streaming, 5 = tcgen05 GEMM
  int W = 4, T = 1, nsplit = 1, kps = 1, MT = 1;
  int bn = 128, tiles_m = 1, tiles_n = 1;  // kernel 5
  bool ilp = false;                        // kernel 1: two accumulator chains
  int RT = 0;  // row tiles (grid.x)
  int wstride = 0, x_off = 0;
  int ring_slots = 0, occ = 1, split_units = 0, red_off = 0;  // kernel 6
  size_t smem = 0;
  size_t ws_bytes = 0;
};

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

constexpr size_t kMaxSmem = 200 * 1024;
// Workspace layout: [0, kCounterBytes) arrival counters, one per row tile, at a fixed place for
// every call (each call leaves the counters it used at zero, so calls with different plans can
// share one workspace), then the split-K partial sums of the current call.
constexpr size_t kCounterBytes = 64 * 1024;
constexpr int kMaxCounters = (int)(kCounterBytes / 4);
constexpr size_t kTmaSmemTarget = 112 * 1024;  // CTAs of two consecutive kernels fit on one SM

static int row_tiles(int N, int n_out, int epi) { return epi == EPI_SWIGLU ? (n_out + 7) / 8 : (N + 15) / 16; }

static size_t reg_smem(const Plan& pl, int M, bool xf32) {
  const size_t stage = (size_t)M * (pl.kps * 16 + 4) * 16 * (xf32 ? 2 : 1);
  const size_t red = (size_t)pl.W * pl.MT * 8 * 16 * 4 + (size_t)M * 16 * 4;
  return std::max(stage, red);
}

static size_t split_ws(const Plan& pl, int M) {
  if (pl.nsplit <= 1) return 0;
  return kCounterBytes + align_up((size_t)pl.nsplit * M * pl.RT * 16 * 4, 256);
}

static bool tiles_supported(int MT, int T) {
  if (MT <= 2) return T == 1 || T == 2 || T == 3 || T == 4 || T == 6 || T == 8;
  return T == 1 || T == 2;
}
static int round_up_tiles(int MT, int T) {
  for (int t = T; t <= 8; ++t)
    if (tiles_supported(MT, t)) return t;
  return 8;
}

static void tma_layout(Plan& pl, int M, int K, int G, bool xf32) {
  pl.wstride = pl.kps * 64 + ((pl.kps % 2 == 0) ? 64 : 0);
  pl.x_off = (int)(16 * (size_t)pl.wstride + align_up((size_t)16 * (K / G) * 2, 16));
  const size_t stage = (size_t)M * (pl.kps * 16 + 4) * 16 * (xf32 ? 2 : 1);
  const size_t red = (size_t)pl.W * pl.MT * 8 * 16 * 4 + (size_t)M * 16 * 4;
  pl.smem = pl.x_off + std::max(stage, red);
}

static int plan_tma(int M, int K, int G, bool xf32, const q4b_linear_cfg* cfg, Plan& pl) {
  pl.kernel = 3;
  const int KT = K / TILE_K;
  pl.W = cfg && cfg->warps ? cfg->warps : 4;
  if (pl.W < 1 || pl.W > 8) return set_error(Q4B_EINVAL, "q4_linear: warps must be 1..8");
  int S = cfg && cfg->split ? cfg->split : 1;
  for (;;) {
    pl.kps = (KT + S - 1) / S;
    pl.nsplit = (KT + pl.kps - 1) / pl.kps;
    tma_layout(pl, M, K, G, xf32);
    if (pl.smem <= kTmaSmemTarget || (cfg && cfg->split) || pl.kps == 1) break;
    ++S;
  }
  if (pl.smem > kMaxSmem) return set_error(Q4B_EUNSUPPORTED, "q4_linear: shared memory plan too large");
  if (pl.nsplit > 1 && pl.RT > kMaxCounters)
    return set_error(Q4B_EUNSUPPORTED, "q4_linear: split-K limited to %d row tiles", kMaxCounters);
  pl.ws_bytes = split_ws(pl, M);
  return Q4B_OK;
}

static int plan_reg(int M, int K, bool xf32, const q4b_linear_cfg* cfg, Plan& pl) {
  pl.kernel = 1;
  const int KT = K / TILE_K;
  int W = cfg && cfg->warps ? cfg->warps : 0;
  int T = cfg && cfg->tiles ? cfg->tiles : 0;
  int S = cfg && cfg->split ? cfg->split : 0;
  if (!W && !T && !S && pl.MT == 1 && KT <= 64) {
    // decode: up to 8 warps cover all of K with a few 128-k tiles in flight per warp and tile
    // row, no split-K, so the post-wait path is x staging + MMAs + one shared-memory reduction
    W = std::min(8, KT);
    T = round_up_tiles(pl.MT, (KT + W - 1) / W);
  } else if (!W && !T && !S && pl.MT >= 2) {
    // 9..32 rows: the staged x grows with the rows, so split K until a CTA holds at most 8 tiles
    // (one per warp): a small slice of x per CTA and many CTAs per SM (measured 1.1-4x faster on
    // the 3B projections than all of K in one CTA)
    W = std::min(8, KT);
    T = 1;
    S = (KT + W - 1) / W;
  }
  if (!T) T = pl.MT == 1 ? 2 : 1;
  if (!W) {
    if (S)
      W = std::min(8, (((KT + S - 1) / S) + T - 1) / T);
    else if (pl.RT >= 148 * 6) {  // plenty of row tiles: cover K within the CTA if it fits
      W = std::min(8, (KT + T - 1) / T);
      if (W * T < KT) W = 4;
    } else
      W = 4;
  }
  if (W < 1 || W > 8 || !tiles_supported(pl.MT, T))
    return set_error(Q4B_EINVAL, "q4_linear: warps must be 1..8 and tiles one of 1,2,3,4,6,8 (1,2 for m > 16)");
  const bool user_shape = cfg && (cfg->warps || cfg->split);
  for (;;) {
    const int s = S ? S : (KT + W * T - 1) / (W * T);
    pl.W = W;
    pl.T = T;
    pl.kps = (KT + s - 1) / s;
    pl.nsplit = (KT + pl.kps - 1) / pl.kps;
    if (pl.kps > W * T)
      return set_error(Q4B_EINVAL, "q4_linear: split %d leaves %d tiles per CTA > warps*tiles %d", s, pl.kps, W * T);
    pl.smem = reg_smem(pl, M, xf32);
    if (pl.smem <= kMaxSmem && (pl.nsplit == 1 || pl.RT <= kMaxCounters)) break;
    if (pl.smem <= kMaxSmem) {  // too many row tiles for the counter region: no split
      if (user_shape || (KT + T - 1) / T > 8)
        return set_error(Q4B_EUNSUPPORTED, "q4_linear: split-K limited to %d row tiles", kMaxCounters);
      W = (KT + T - 1) / T;
      S = 1;
      continue;
    }
    if (user_shape || W == 1) return set_error(Q4B_EUNSUPPORTED, "q4_linear: shared memory plan too large");
    W = W / 2;  // fewer tiles per CTA: a smaller staged slice of x
  }
  pl.ws_bytes = split_ws(pl, M);
  pl.ilp = (long long)pl.RT * pl.nsplit <= 3 * 148;  // few CTAs per SM: latency, not occupancy, limits
  return Q4B_OK;
}

constexpr int kStreamCtas = 148;  // one CTA per SM of a B200

static int plan_stream(int M, int K, bool xf32, const q4b_linear_cfg* cfg, Plan& pl) {
  pl.kernel = 4;
  pl.W = cfg && cfg->warps ? cfg->warps : 16;
  if (pl.W < 1 || pl.W > 24) return set_error(Q4B_EINVAL, "q4_linear: streaming kernel takes 1..24 warps");
  pl.nsplit = 1;
  pl.kps = K / TILE_K;
  const int SK = K <= 4096 ? K : K / 2;
  const size_t ring = (size_t)kStreamRing * (16 * SK / 2 + 16 * (SK / 128) * 2);
  pl.x_off = (int)align_up(ring, 128);
  const size_t stage = (size_t)M * (K / 8 + 4) * 16 * (xf32 ? 2 : 1);
  pl.smem = pl.x_off + stage;
  pl.ws_bytes = 0;
  return pl.smem <= kMaxSmem ? Q4B_OK : set_error(Q4B_EUNSUPPORTED, "q4_linear: streaming plan too large");
}

// kernel 5: weight rows per CTA from cfg->tiles (row tiles of 16: 4 or 8), k split at scale-group
// granularity; workspace = counters | x hi | x lo | split partials
static bool tc_ok(int M, int K, int G, int epi, bool norm) {
  (void)norm;  // the x split applies a fused RMSNorm (fp32 x, checked by validate)
  return M > 32 && G % 128 == 0 && epi != EPI_ARGMAX && K / G <= 64 * 64;
}
// RoPE tiles map onto TMA boxes of whole half-heads (row tiles per head and per CTA nest)
static bool tc_rope_ok(int epi, int hd, int bn) {
  if (epi != EPI_ROPE_KV) return true;
  const int per = hd / 16, rts = bn / 16;
  return hd % 16 == 0 && per > 0 && (per % rts == 0 || rts % per == 0);
}

static int plan_tc(int M, int K, int G, bool xf32, const q4b_linear_cfg* cfg, Plan& pl) {
  pl.kernel = 5;
  const int T = cfg && cfg->tiles ? cfg->tiles : 0;
  if (T && T != 4 && T != 8) return set_error(Q4B_EINVAL, "q4_linear: kernel 5 takes tiles 4 or 8 (64 or 128 rows)");
  const int NG = K / G;
  pl.tiles_m = (M + 127) / 128;
  int S = cfg && cfg->split ? cfg->split : 0;
  if (S < 0 || S > NG) return set_error(Q4B_EINVAL, "q4_linear: split must be in [1, %d] (scale groups)", NG);
  {
    // A 64-k stage costs about one loaded L2 round trip (~1.1 us) for its x tile whatever the tile
    // width, so the time is ~ waves x stages per CTA, plus the split-K partial tiles written and read
    // back (at ~5 TB/s): wide tiles (half the x re-reads) and a split that fills one wave of the
    // 148 SMs usually win.
    double best = 1e30;
    int best_bn = T ? T * 16 : 128, best_s = 1;
    for (int bn = 128; bn >= 64; bn -= 64) {
      if (T && bn != T * 16) continue;  // the configuration fixes the tile width
      const long long tl = (long long)pl.tiles_m * ((pl.RT + bn / 16 - 1) / (bn / 16));
      for (int s = 1; s <= NG && s <= 64; ++s) {
        if (S && s != S) continue;
        if ((NG + s - 1) / s > K5_MAX_GROUPS || (s > 1 && tl > kMaxCounters)) continue;
        const long long waves = (tl * s + 147) / 148;
        const double reduce = s > 1 ? 2.0 * s * (double)tl * K5_BM * bn * 4 / 5e12 / 1.1e-6 : 0.0;
        const double cost = (double)waves * ((NG + s - 1) / s) * (G / K5_BK) + reduce;
        if (cost < best - 1e-9) {
          best = cost;
          best_bn = bn;
          best_s = s;
        }
      }
    }
    pl.bn = best_bn;
    if (!S) S = best_s;
  }
  pl.tiles_n = (pl.RT + pl.bn / 16 - 1) / (pl.bn / 16);
  const long long tiles = (long long)pl.tiles_m * pl.tiles_n;
  while ((NG + S - 1) / S > K5_MAX_GROUPS) ++S;
  if (S > 1 && tiles > kMaxCounters)
    return set_error(Q4B_EUNSUPPORTED, "q4_linear: split-K limited to %d tiles", kMaxCounters);
  pl.nsplit = S;
  pl.kps = NG;
  pl.smem = pl.bn == 128 ? K5<128>::SMEM : K5<64>::SMEM;
  const size_t xbytes = align_up((size_t)M * K * 2, 256);
  pl.ws_bytes = kCounterBytes + (xf32 ? 2 : 1) * xbytes +
                (S > 1 ? (size_t)S * tiles * K5_BM * pl.bn * 4 : 0);
  return Q4B_OK;
}

// kernel 6: ring depth from the shared memory left beside the staged x and the reduction slots.
// Residency modes (cfg->tiles; 0 = automatic):
//   1  one CTA per SM, sized so that one CTA of the next kernel on the stream fits beside it: that
//      kernel starts under programmatic dependent launch and fills its own ring while this one runs
//      (chains of small projections)
//   2  two CTAs per SM filling it (twice the consumer warps and bytes in flight; large problems)
//   3  one CTA per SM with the whole shared memory (x too large to stage beside a deep ring)
constexpr size_t kRingSmemHalf = 104 * 1024;   // dynamic bytes of one of two CTAs on an SM
constexpr size_t kRingSmemAlone = 200 * 1024;  // dynamic bytes of a CTA alone on an SM
// The planner sends a GEMV to kernel 6 by default only when its weights exceed kRingMinBytes: below
// that a launch is dominated by its fixed path (x staging, a few stages per CTA, the finish), where
// kernel 1's many small CTAs with loads issued before the dependency wait do better (measured on the
// 3B projections: 8-26 MB faster in kernel 1, the 197 MB lm_head 1.6x faster in kernel 6).
constexpr size_t kRingMinBytes = 40u << 20;
static bool ring_ok(int M, int K, int G, int epi, bool norm) {
  return M <= 8 && G == 128 && K % kRingSK == 0 && !norm && (epi != EPI_ARGMAX || M == 1);
}
// staged x: one row as int8 terms (three rows of K/8 + 8 uint2, plus a 16-byte record per group), or
// up to 8 rows as fp16 (hi, and lo for fp32 x)
static size_t ring_xbytes(int M, int K, bool xf32) {
  if (M == 1) return (size_t)3 * (K / 8 + 8) * 8 + (size_t)(K / 128) * 16;
  return (size_t)M * (K / 8 + 4) * 16 * (xf32 ? 2 : 1);
}
static bool ring_layout(Plan& pl, int M, int K, bool xf32, int mode) {
  const size_t xb = align_up(ring_xbytes(M, K, xf32), 128);
  const size_t budget = mode == 3 ? kRingSmemAlone : kRingSmemHalf;
  const size_t reds = (size_t)kRingRed * kRingCW * 2 * M * 16 * 4;  // reduction slots
  const long long slots = xb + reds < budget ? (long long)((budget - xb - reds) / kRingSlotBytes) : 0;
  pl.ring_slots = (int)std::min<long long>(slots, kRingMaxSlots);
  pl.occ = mode == 2 ? 2 : 1;
  pl.x_off = pl.ring_slots * kRingSlotBytes;
  pl.red_off = (int)(pl.x_off + xb);
  pl.smem = pl.red_off + reds;
  return pl.ring_slots >= (mode == 3 ? 3 : 4);
}
static size_t ring_ws(const Plan& pl, int M, int K) {
  return kCounterBytes + align_up((size_t)((pl.RT + 1) / 2) * (K / kRingSK) * 2 * M * 16 * 4, 256);
}
static int plan_ring(int M, int N, int K, bool xf32, const q4b_linear_cfg* cfg, Plan& pl) {
  pl.kernel = 6;
  const int mode = cfg && cfg->tiles ? cfg->tiles : 0;
  if (mode < 0 || mode > 3) return set_error(Q4B_EINVAL, "q4_linear: kernel 6 takes tiles = 1, 2 or 3 (residency mode)");
  bool ok;
  if (mode) {
    ok = ring_layout(pl, M, K, xf32, mode);
  } else {
    ok = ring_layout(pl, M, K, xf32, 2) || ring_layout(pl, M, K, xf32, 3);
    (void)N;
  }
  if (!ok) return set_error(Q4B_EUNSUPPORTED, "q4_linear: kernel 6 ring does not fit beside x (m=%d k=%d)", M, K);
  pl.nsplit = 1;
  pl.kps = K / TILE_K;
  pl.split_units = !(cfg && cfg->split == 1) && (pl.RT + 1) / 2 <= kMaxCounters;
  pl.ws_bytes = pl.split_units ? ring_ws(pl, M, K) : 0;
  return Q4B_OK;
}

static bool stream_ok(int M, int K, int G, bool norm) {
  (void)norm;
  return M == 1 && G == 128 && K % 1024 == 0 && K <= 8192;
}

static int plan_linear(int M, int N, int K, int G, int epi, bool xf32, bool norm, const q4b_linear_cfg* cfg,
                       Plan& pl) {
  const int n_out = epi == EPI_SWIGLU ? N / 2 : N;
  const bool mma_ok = (G % TILE_K == 0) && M <= 64 && (!norm || M <= 8);
  const int want = cfg ? cfg->kernel : 0;
  pl.RT = row_tiles(N, n_out, epi);
  pl.MT = M <= 8 ? 1 : M <= 16 ? 2 : M <= 32 ? 4 : 8;
  if (want == 5) {
    if (!tc_ok(M, K, G, epi, norm) && !(M >= 1 && G % 128 == 0 && epi != EPI_ARGMAX))
      return set_error(Q4B_EUNSUPPORTED, "q4_linear: kernel 5 needs group %% 128 == 0, no argmax");
    return plan_tc(M, K, G, xf32, cfg, pl);
  }
  if (want == 0 && tc_ok(M, K, G, epi, norm)) return plan_tc(M, K, G, xf32, cfg, pl);
  if ((want == 1 || want == 3) && !mma_ok)
    return set_error(Q4B_EUNSUPPORTED, "q4_linear: tensor-core kernels need group %% 128 == 0 and m <= 64");
  if (want == 2 || (want == 0 && !mma_ok)) {
    pl.kernel = 2;
    pl.W = 8;
    pl.smem = (size_t)M * 16 * 4;
    if (pl.smem > kMaxSmem) return set_error(Q4B_EUNSUPPORTED, "q4_linear: m too large");
    return Q4B_OK;
  }
  if (want == 3) {
    if (pl.MT > 2) return set_error(Q4B_EUNSUPPORTED, "q4_linear: TMA kernel needs m <= 16");
    return plan_tma(M, K, G, xf32, cfg, pl);
  }
  if (want == 6) {
    if (!ring_ok(M, K, G, epi, norm))
      return set_error(Q4B_EUNSUPPORTED, "q4_linear: kernel 6 needs m <= 8, group 128, k %% 1024 == 0, no fused norm");
    return plan_ring(M, N, K, xf32, cfg, pl);
  }
  const bool tuned = !cfg || (!cfg->warps && !cfg->tiles && !cfg->split);
  if (want == 0 && tuned && ring_ok(M, K, G, epi, norm) && (size_t)N * K / 2 >= kRingMinBytes &&
      plan_ring(M, N, K, xf32, nullptr, pl) == Q4B_OK)
    return Q4B_OK;
  if (want == 4) {
    if (!stream_ok(M, K, G, norm))
      return set_error(Q4B_EUNSUPPORTED, "q4_linear: streaming kernel needs m == 1, group 128, k %% 1024 == 0, k <= 8192");
    return plan_stream(M, K, xf32, cfg, pl);
  }
  // the streaming kernel (4) is selectable but not the default: chained in a decode step its
  // one-CTA-per-SM ring cannot overlap the neighbouring launches and measures slower than kernel 1
  return plan_reg(M, K, xf32, cfg, pl);
}

template <typename Kern>
static cudaError_t set_smem_attr(Kern kern, std::atomic<unsigned long long>& done, int bytes = (int)kMaxSmem) {
  return set_max_dynamic_smem(kern, bytes, done);
}

// SMs of the current device (cached per device ordinal)
static int num_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  int v = cache[dev & 63].load(std::memory_order_relaxed);
  if (!v) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev & 63].store(v, std::memory_order_relaxed);
  }
  return v;
}

template <int MT, bool XF32, int T>
static cudaError_t launch_reg_t(const Plan& pl, const LinArgs& a, cudaStream_t st) {
  if constexpr (MT == 1 && (T == 3 || T == 8)) {  // the decode shapes: few-CTA launches take the ILP form
    if (pl.ilp) {
      static std::atomic<unsigned long long> done_ilp;
      cudaError_t e = set_smem_attr(q4_gemv_reg<MT, XF32, T, true>, done_ilp);
      if (e != cudaSuccess) return e;
      return launch_pdl(q4_gemv_reg<MT, XF32, T, true>, dim3(pl.RT, pl.nsplit), dim3(pl.W * 32), pl.smem, st, a);
    }
  }
  static std::atomic<unsigned long long> done;
  cudaError_t e = set_smem_attr(q4_gemv_reg<MT, XF32, T>, done);
  if (e != cudaSuccess) return e;
  return launch_pdl(q4_gemv_reg<MT, XF32, T>, dim3(pl.RT, pl.nsplit), dim3(pl.W * 32), pl.smem, st, a);
}

template <int MT, bool XF32>
static cudaError_t launch_reg_x(const Plan& pl, const LinArgs& a, cudaStream_t st) {
  if constexpr (MT <= 2) {
    switch (pl.T) {
      case 1: return launch_reg_t<MT, XF32, 1>(pl, a, st);
      case 2: return launch_reg_t<MT, XF32, 2>(pl, a, st);
      case 3: return launch_reg_t<MT, XF32, 3>(pl, a, st);
      case 4: return launch_reg_t<MT, XF32, 4>(pl, a, st);
      case 6: return launch_reg_t<MT, XF32, 6>(pl, a, st);
      default: return launch_reg_t<MT, XF32, 8>(pl, a, st);
    }
  } else {
    if (pl.T == 1) return launch_reg_t<MT, XF32, 1>(pl, a, st);
    return launch_reg_t<MT, XF32, 2>(pl, a, st);
  }
}

template <bool XF32>
static cudaError_t launch_reg(const Plan& pl, const LinArgs& a, cudaStream_t st) {
  switch (pl.MT) {
    case 1: return launch_reg_x<1, XF32>(pl, a, st);
    case 2: return launch_reg_x<2, XF32>(pl, a, st);
    case 4: return launch_reg_x<4, XF32>(pl, a, st);
    default: return launch_reg_x<8, XF32>(pl, a, st);
  }
}

template <int MT, bool XF32>
static cudaError_t launch_tma_t(const Plan& pl, const LinArgs& a, cudaStream_t st) {
  static std::atomic<unsigned long long> done;
  cudaError_t e = set_smem_attr(q4_gemv_tma<MT, XF32>, done);
  if (e != cudaSuccess) return e;
  return launch_pdl(q4_gemv_tma<MT, XF32>, dim3(pl.RT, pl.nsplit), dim3(pl.W * 32), pl.smem, st, a);
}

template <bool XF32>
static cudaError_t launch_tma(const Plan& pl, const LinArgs& a, cudaStream_t st) {
  return pl.MT == 1 ? launch_tma_t<1, XF32>(pl, a, st) : launch_tma_t<2, XF32>(pl, a, st);
}

static int validate(const LinearOp& op) {
  if (!op.qw || !op.scales || !op.x) return set_error(Q4B_EINVAL, "q4_linear: null pointer");
  if (!op.y && op.epi != EPI_ROPE_KV && op.epi != EPI_ARGMAX) return set_error(Q4B_EINVAL, "q4_linear: null pointer");
  if (op.m < 1 || op.n < 1 || op.k < 8 || op.k % 8)
    return set_error(Q4B_EINVAL, "q4_linear: bad shape m=%d n=%d k=%d", op.m, op.n, op.k);
  if (op.group < 8 || op.group % 8 || op.k % op.group)
    return set_error(Q4B_EINVAL, "q4_linear: need k %% group == 0 and group %% 8 == 0 (k=%d group=%d)", op.k,
                     op.group);
  if ((op.x_dtype != Q4B_F32 && op.x_dtype != Q4B_F16) || (op.y_dtype != Q4B_F32 && op.y_dtype != Q4B_F16))
    return set_error(Q4B_EINVAL, "q4_linear: bad dtype");
  if (op.epi < EPI_STORE || op.epi > EPI_ARGMAX) return set_error(Q4B_EINVAL, "q4_linear: bad epilogue %d", op.epi);
  if (op.epi == EPI_SWIGLU && op.n % 2) return set_error(Q4B_EINVAL, "q4_linear: SwiGLU needs an even row count");
  if (op.ln_w && (op.x_dtype != Q4B_F32 || op.k % 4))
    return set_error(Q4B_EINVAL, "q4_linear: fused RMSNorm needs fp32 x and k %% 4 == 0");
  if (op.epi == EPI_ROPE_KV &&
      (!op.rope_cos || !op.rope_sin || !op.pos0 || !op.q_out || !op.k_cache || !op.v_cache || op.head_dim % 16 ||
       op.n != (op.n_heads + 2 * op.n_kv) * op.head_dim))
    return set_error(Q4B_EINVAL, "q4_linear: bad RoPE/KV epilogue arguments");
  if (op.epi == EPI_ARGMAX && (!op.state || op.m != 1))
    return set_error(Q4B_EINVAL, "q4_linear: argmax epilogue needs a state and m == 1");
  return Q4B_OK;
}

bool linear_fuses_norm(int m, int k, int group, int epi, int head_dim) {
  return m <= 8 || (tc_ok(m, k, group, epi, true) && tc_rope_ok(epi, head_dim, 128) && tc_rope_ok(epi, head_dim, 64));
}

static int plan_op(const LinearOp& op, Plan& pl) {
  return plan_linear(op.m, op.n, op.k, op.group, op.epi, op.x_dtype == Q4B_F32, op.ln_w != nullptr, op.cfg, pl);
}

size_t linear_workspace(const LinearOp& op) {
  if (validate(op) != Q4B_OK) return 0;
  Plan a, b;
  LinearOp o = op;
  o.x_dtype = Q4B_F32;
  const size_t wa = plan_op(o, a) == Q4B_OK ? a.ws_bytes : 0;
  o.x_dtype = Q4B_F16;
  o.ln_w = nullptr;
  const size_t wb = plan_op(o, b) == Q4B_OK ? b.ws_bytes : 0;
  return std::max(wa, wb);
}

static void simt_plan(const LinearOp& op, Plan& pl) {
  pl = Plan();
  pl.RT = row_tiles(op.n, op.epi == EPI_SWIGLU ? op.n / 2 : op.n, op.epi);
  pl.kernel = 2;
  pl.W = 8;
  pl.smem = (size_t)op.m * 16 * 4;
}

int linear_run(const LinearOp& op, cudaStream_t st) {
  int rc = validate(op);
  if (rc) return rc;
  const bool xf32 = op.x_dtype == Q4B_F32;
  Plan pl;
  if ((rc = plan_op(op, pl))) return rc;
  const bool forced = op.cfg && op.cfg->kernel;
  // a fused RMSNorm over more than 8 rows runs in kernel 5's x split only (the other kernels' norm
  // prologue holds 8 rows): no fallback to another kernel for it
  const bool wide_norm = op.ln_w && op.m > 8;
  if (wide_norm && pl.kernel != 5)
    return set_error(Q4B_EINVAL, "q4_linear: fused RMSNorm over %d rows needs the tcgen05 path (group %% 128 == 0, "
                                 "m > 32)", op.m);
  if (pl.kernel != 2 && (!aligned(op.qw, 16) || !aligned(op.x, 16) || (op.ln_w && !aligned(op.ln_w, 16)) ||
                         (pl.kernel == 4 && !aligned(op.scales, 16)))) {
    if (forced || wide_norm) return set_error(Q4B_EINVAL, "q4_linear: qweight, x and ln_w must be 16-byte aligned");
    simt_plan(op, pl);
  }
  if (pl.kernel == 6 && !aligned(op.scales, 16)) {  // scale rows arrive by bulk copies
    if (forced) return set_error(Q4B_EINVAL, "q4_linear: kernel 6 needs 16-byte aligned scales");
    Plan alt;
    q4b_linear_cfg k1 = {1, 0, 0, 0};
    if (plan_linear(op.m, op.n, op.k, op.group, op.epi, xf32, op.ln_w != nullptr, &k1, alt) == Q4B_OK)
      pl = alt;
    else
      simt_plan(op, pl);
  }
  if (pl.kernel == 6 && pl.split_units && (pl.ws_bytes > op.ws_bytes || !op.ws || !aligned(op.ws, 16))) {
    pl.split_units = 0;  // whole row tiles per CTA: no workspace needed
    pl.ws_bytes = 0;
  }
  if (pl.kernel == 5 && !tc_rope_ok(op.epi, op.head_dim, pl.bn)) {
    if (forced || wide_norm)
      return set_error(Q4B_EUNSUPPORTED, "q4_linear: kernel 5 RoPE tiles need head_dim / 16 and the tile to nest");
    simt_plan(op, pl);
  }
  if (pl.kernel == 5 && (pl.ws_bytes > op.ws_bytes || !op.ws || !aligned(op.ws, 256))) {
    if (forced || wide_norm)
      return set_error(Q4B_EINVAL, "q4_linear: workspace of %zu bytes needed, %zu given", pl.ws_bytes, op.ws_bytes);
    simt_plan(op, pl);  // the x conversion and split partials need the workspace
  }
  if (pl.kernel != 2 && pl.kernel != 5 && pl.nsplit > 1 &&
      (pl.ws_bytes > op.ws_bytes || !op.ws || !aligned(op.ws, 16))) {
    if (op.cfg && op.cfg->split > 1)
      return set_error(Q4B_EINVAL, "q4_linear: workspace of %zu bytes needed, %zu given", pl.ws_bytes, op.ws_bytes);
    // no (or too little) workspace: all of K in one CTA when it fits, else the SIMT kernel
    const int KT = op.k / TILE_K;
    pl.kps = KT;
    pl.nsplit = 1;
    pl.ws_bytes = 0;
    bool ok = false;
    if (pl.kernel == 3) {
      tma_layout(pl, op.m, op.k, op.group, xf32);
      ok = pl.smem <= kMaxSmem;
    } else if (KT <= 64 && (pl.MT <= 2 || KT <= 16)) {
      pl.T = round_up_tiles(pl.MT, (KT + 7) / 8);
      pl.W = (KT + pl.T - 1) / pl.T;
      pl.smem = reg_smem(pl, op.m, xf32);
      ok = pl.W <= 8 && pl.smem <= kMaxSmem;
    }
    if (!ok) simt_plan(op, pl);
  }
  LinArgs a = {};
  a.qw = op.qw;
  a.scales = reinterpret_cast<const __half*>(op.scales);
  a.x = op.x;
  a.y = op.y;
  a.M = op.m;
  a.N = op.n;
  a.K = op.k;
  a.G = op.group;
  a.n_out = op.epi == EPI_SWIGLU ? op.n / 2 : op.n;
  a.KT = op.k / TILE_K;
  a.kps = pl.kps;
  a.nsplit = pl.nsplit;
  a.epi = op.epi;
  a.y_f32 = op.y_dtype == Q4B_F32;
  a.wstride = pl.wstride;
  a.x_off = pl.x_off;
  a.ln_w = op.ln_w;
  a.eps = op.eps;
  a.row_sel = op.row_sel;
  a.rope_cos = op.rope_cos;
  a.rope_sin = op.rope_sin;
  a.pos0 = op.pos0;
  a.pos_offset = op.pos_offset;
  a.q_out = op.q_out;
  a.k_cache = reinterpret_cast<__half*>(op.k_cache);
  a.v_cache = reinterpret_cast<__half*>(op.v_cache);
  a.H = op.n_heads;
  a.Hkv = op.n_kv;
  a.hd = op.head_dim;
  a.state = op.state;
  a.token_log = op.token_log;
  a.logits = op.logits;
  a.index_offset = op.index_offset;
  a.finalize = op.finalize;
  a.RT = pl.RT;
  if ((pl.kernel != 2 && pl.kernel != 5 && pl.nsplit > 1) || (pl.kernel == 6 && pl.split_units)) {
    a.counters = reinterpret_cast<unsigned*>(op.ws);
    a.ws = reinterpret_cast<float*>(reinterpret_cast<char*>(op.ws) + kCounterBytes);
  }
  a.ring_slots = pl.ring_slots;
  a.kc = op.k / kRingSK;
  a.split_units = pl.split_units;
  a.red_off = pl.red_off;
  cudaError_t e;
  if (pl.kernel == 5) {
    char* w = reinterpret_cast<char*>(op.ws);
    const size_t xbytes = align_up((size_t)op.m * op.k * 2, 256);
    auto* xh = reinterpret_cast<__half*>(w + kCounterBytes);
    auto* xl = reinterpret_cast<__half*>(w + kCounterBytes + xbytes);
    a.counters = reinterpret_cast<unsigned*>(w);
    a.ws = reinterpret_cast<float*>(w + kCounterBytes + (xf32 ? 2 : 1) * xbytes);
    CUtensorMap th, tl, tw;
    int rc2 = make_tmap_f16(&th, xh, op.k, op.m, op.k, K5_BM);
    if (!rc2) rc2 = make_tmap_f16(&tl, xf32 ? xl : xh, op.k, op.m, op.k, K5_BM);
    const int nb = k5_nb(op.epi, pl.bn / 16, op.head_dim);
    if (!rc2) rc2 = make_tmap_i32(&tw, op.qw, op.k / 8, op.n, op.k / 8, 8, pl.bn / nb);
    if (rc2) return rc2;
    const int chunks = op.m * (op.k / 8);
    const int pgrid = op.ln_w ? op.m : std::min((chunks + 255) / 256, 148 * 8);  // fused norm: a CTA per row
    e = xf32 ? launch_pdl(q4_xsplit<true>, dim3(pgrid), dim3(256), 0, st, a, xh, xl)
             : launch_pdl(q4_xsplit<false>, dim3(pgrid), dim3(256), 0, st, a, xh, xl);
    if (e == cudaSuccess) {
      static std::atomic<unsigned long long> d[4];
      const dim3 grid(pl.tiles_m, pl.tiles_n, pl.nsplit);
      auto go = [&](auto kern, std::atomic<unsigned long long>& done) {
        const cudaError_t r = set_smem_attr(kern, done, (int)pl.smem);
        if (r != cudaSuccess) return r;
        return launch_pdl(kern, grid, dim3(K5_THREADS), pl.smem, st, th, tl, tw, a);
      };
      if (pl.bn == 128)
        e = xf32 ? go(q4_gemm_tc<128, true>, d[0]) : go(q4_gemm_tc<128, false>, d[1]);
      else
        e = xf32 ? go(q4_gemm_tc<64, true>, d[2]) : go(q4_gemm_tc<64, false>, d[3]);
    }
  } else if (pl.kernel == 6) {
    static std::atomic<unsigned long long> d[4];
    const bool m1 = op.m == 1;
    auto kern = m1 ? (xf32 ? q4_gemv_ring<true, true> : q4_gemv_ring<false, true>)
                   : (xf32 ? q4_gemv_ring<true, false> : q4_gemv_ring<false, false>);
    // weights as int32 [n, k/8] in boxes of {128 words, 32 rows}, scales as int32 pairs [n, k/256]
    // in boxes of {4 words, 32 rows} (8-row boxes for SwiGLU / RoPE tiles); rows past n read zero
    const uint32_t box_rows = (op.epi == EPI_SWIGLU || op.epi == EPI_ROPE_KV) ? 8 : 32;
    CUtensorMap tw, ts;
    int rc2 = make_tmap_i32(&tw, op.qw, op.k / 8, op.n, op.k / 8, kRingSK / 8, box_rows);
    if (!rc2) rc2 = make_tmap_i32(&ts, op.scales, op.k / 256, op.n, op.k / 256, 4, box_rows);
    if (rc2) return rc2;
    e = set_smem_attr(kern, d[(m1 ? 0 : 2) + (xf32 ? 0 : 1)]);
    const long long pairs = (pl.RT + 1) / 2;
    const long long units = pl.split_units ? pairs * a.kc : pairs;
    const int grid = (int)std::min<long long>(units, (long long)num_sms() * pl.occ);
    if (e == cudaSuccess) e = launch_pdl(kern, dim3(grid), dim3(kRingThreads), pl.smem, st, tw, ts, a);
  } else if (pl.kernel == 4) {
    static std::atomic<unsigned long long> d0, d1;
    e = xf32 ? set_smem_attr(q4_gemv_stream<true>, d1) : set_smem_attr(q4_gemv_stream<false>, d0);
    const int grid = std::min(pl.RT, kStreamCtas);
    if (e == cudaSuccess)
      e = xf32 ? launch_pdl(q4_gemv_stream<true>, dim3(grid), dim3(pl.W * 32), pl.smem, st, a)
               : launch_pdl(q4_gemv_stream<false>, dim3(grid), dim3(pl.W * 32), pl.smem, st, a);
  } else if (pl.kernel == 3) {
    e = xf32 ? launch_tma<true>(pl, a, st) : launch_tma<false>(pl, a, st);
  } else if (pl.kernel == 1) {
    e = xf32 ? launch_reg<true>(pl, a, st) : launch_reg<false>(pl, a, st);
  } else {
    static std::atomic<unsigned long long> d0, d1;
    e = xf32 ? set_smem_attr(q4_linear_simt<true>, d1) : set_smem_attr(q4_linear_simt<false>, d0);
    if (e == cudaSuccess)
      e = xf32 ? launch_pdl(q4_linear_simt<true>, dim3(pl.RT), dim3(256), pl.smem, st, a)
               : launch_pdl(q4_linear_simt<false>, dim3(pl.RT), dim3(256), pl.smem, st, a);
  }
  if (e != cudaSuccess) return set_error(Q4B_ELAUNCH, "q4_linear: launch failed: %s", cudaGetErrorString(e));
  return check_launch("q4_linear");
}

unsigned linear_status(bool reset) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_linear_status, sizeof(v));
  if (reset && v) {
    const unsigned z = 0;
    cudaMemcpyToSymbol(g_linear_status, &z, sizeof(z));
  }
  return v;
}

}  // namespace q4b

using namespace q4b;

static LinearOp public_op(const int32_t* qweight, const uint16_t* scales, int group, const void* x, int x_dtype,
                          void* y, int y_dtype, int m, int n, int k, int epilogue, const q4b_linear_cfg* cfg,
                          void* workspace, size_t workspace_bytes) {
  LinearOp op;
  op.qw = qweight;
  op.scales = scales;
  op.group = group;
  op.x = x;
  op.x_dtype = x_dtype;
  op.y = y;
  op.y_dtype = y_dtype;
  op.m = m;
  op.n = n;
  op.k = k;
  op.epi = epilogue;
  op.cfg = cfg;
  op.ws = workspace;
  op.ws_bytes = workspace_bytes;
  return op;
}

static int validate_linear(const int32_t* qweight, const uint16_t* scales, int group, const void* x, int x_dtype,
                           void* y, int y_dtype, int m, int n, int k, int epi) {
  if (!qweight || !scales || !x || !y) return set_error(Q4B_EINVAL, "q4_linear: null pointer");
  if (epi < Q4B_EPI_STORE || epi > Q4B_EPI_SWIGLU) return set_error(Q4B_EINVAL, "q4_linear: bad epilogue %d", epi);
  return validate(public_op(qweight, scales, group, x, x_dtype, y, y_dtype, m, n, k, epi, nullptr, nullptr, 0));
}

extern "C" size_t q4b_q4_linear_workspace(int m, int n, int k, int group, int epilogue, const q4b_linear_cfg* cfg) {
  if (epilogue < Q4B_EPI_STORE || epilogue > Q4B_EPI_SWIGLU) return 0;
  static const int dummy[4] = {0, 0, 0, 0};  // never dereferenced: planning only
  return linear_workspace(public_op(dummy, reinterpret_cast<const uint16_t*>(dummy), group, dummy, Q4B_F32,
                                    const_cast<int*>(dummy), Q4B_F32, m, n, k, epilogue, cfg, nullptr, 0));
}

extern "C" int q4b_q4_linear_kernel(int m, int n, int k, int group, int epilogue, int x_dtype,
                                    const q4b_linear_cfg* cfg) {
  static const int dummy[4] = {0, 0, 0, 0};  // never dereferenced: planning only
  int rc = validate_linear(dummy, reinterpret_cast<const uint16_t*>(dummy), group, dummy, x_dtype,
                           const_cast<int*>(dummy), Q4B_F32, m, n, k, epilogue);
  if (rc) return rc;
  Plan pl;
  if ((rc = plan_linear(m, n, k, group, epilogue, x_dtype == Q4B_F32, false, cfg, pl))) return rc;
  return pl.kernel;
}

extern "C" int q4b_q4_linear(const int32_t* qweight, const uint16_t* scales, int group, const void* x, int x_dtype,
                             void* y, int y_dtype, int m, int n, int k, int epilogue, const q4b_linear_cfg* cfg,
                             void* workspace, size_t workspace_bytes, q4b_stream_t stream) {
  int rc = validate_linear(qweight, scales, group, x, x_dtype, y, y_dtype, m, n, k, epilogue);
  if (rc) return rc;
  return linear_run(
      public_op(qweight, scales, group, x, x_dtype, y, y_dtype, m, n, k, epilogue, cfg, workspace, workspace_bytes),
      as_stream(stream));
}

// ---- allocation-free variant ---------------------------------------------------------------
// q4b_q4_linear with its split-K workspace in a file-scope device array instead of a caller
// buffer, for callers that cannot allocate device memory. Host code must not pass the array's
// name to a kernel (on the host it is only a stand-in symbol): the device address is looked up
// once per device with cudaGetSymbolAddress and that pointer is what the kernels receive.
#include <mutex>

namespace q4b {
constexpr size_t kStaticScratchBytes = 8u << 20;  // 8 MiB: counters (64 KiB) + split-K partials
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
static std::mutex g_scratch_mu;
static void* g_scratch_ptr[64] = {};  // per device ordinal, filled at set-up
}  // namespace q4b

extern "C" int q4b_q4_linear_noalloc(const int32_t* qweight, const uint16_t* scales, int group, const void* x,
                                     int x_dtype, void* y, int y_dtype, int m, int n, int k, int epilogue,
                                     q4b_stream_t stream) {
  int rc = validate_linear(qweight, scales, group, x, x_dtype, y, y_dtype, m, n, k, epilogue);
  if (rc) return rc;
  const size_t need = q4b_q4_linear_workspace(m, n, k, group, epilogue, nullptr);
  if (need > kStaticScratchBytes)
    return set_error(Q4B_EINVAL, "q4_linear_noalloc: this problem needs %zu bytes of workspace, above the %zu-byte "
                     "static scratch", need, kStaticScratchBytes);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(Q4B_ECUDA, "q4_linear_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(Q4B_EUNSUPPORTED, "q4_linear_noalloc: device ordinal %d", dev);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {  // set-up, once per device, with that device current
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_static_scratch);
      if (e != cudaSuccess)
        return set_error(Q4B_ECUDA, "q4_linear_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      e = cudaMemset(p, 0, kCounterBytes);  // the arrival counters must start at zero
      if (e == cudaSuccess) e = cudaDeviceSynchronize();
      if (e != cudaSuccess)
        return set_error(Q4B_ECUDA, "q4_linear_noalloc: clearing the scratch counters: %s", cudaGetErrorString(e));
      g_scratch_ptr[dev] = p;
    }
    scratch = g_scratch_ptr[dev];
  }
  return q4b_q4_linear(qweight, scales, group, x, x_dtype, y, y_dtype, m, n, k, epilogue, nullptr, scratch,
                       kStaticScratchBytes, stream);
}
