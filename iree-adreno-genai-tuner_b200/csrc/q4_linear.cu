// int4 weight-only linear: QLinear.forward of scripts/llm/llama_q4.py:69-90.
//
//   y[m, n] = sum_k x[m, k] * (nib(n, k) - 8) * scale(n, k / G)          (fp32 accumulation)
//
// Two kernels:
//   q4_gemv_mma   G % 128 == 0, M <= 64: decode GEMV / small-M batch on the tensor cores
//                 (mma.sync m16n8k16, fp16 operands, fp32 accumulate). A warp owns a 16-row x 128-k
//                 tile; every lane issues two 16-byte streaming loads per tile (rows g and g + 8 of
//                 the tile, 64 contiguous bytes per 4 lanes), all of a warp's tiles before any math.
//                 Nibbles become fp16 (nib - 8) exactly with two LOP3 + one HSUB2/HFMA2 per pair;
//                 the k order inside a word is permuted (slots hold nibbles b and b + 4) and x is
//                 staged in shared memory in the same permuted order, so no shuffle is needed.
//                 One 128-k tile lies inside one scale group, so the tile's MMA sum is scaled once
//                 in fp32. fp32 x is split into hi + lo fp16 terms (two MMAs), keeping ~22 bits.
//                 Split-K partials go to a workspace; the last CTA of a row tile (arrival counter)
//                 sums them in a fixed order, so results are deterministic.
//   q4_linear_simt any G % 8 == 0: one warp per output row (and up to 8 batch rows), fp32 FMAs on
//                 the exactly dequantised weights (the reference's dequant + linear form).
// Both start streaming weights before griddepcontrol.wait (programmatic dependent launch), so the
// weight reads of one projection overlap the tail of the kernel before it.
#include <algorithm>

#include "common.cuh"

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
};

// ---- PTX helpers ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
  return d;
}
__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// 8 nibbles of one word -> 4 fp16 pairs of exact (nib - 8): {(n0,n4), (n1,n5), (n2,n6), (n3,n7)}.
// OR-ing a nibble into the mantissa of 1024.0 (0x6400) gives 1024 + nib; nibbles taken in place at
// bits 4..7 give 1024 + 16 nib, rescaled by an exact FMA.
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t (&o)[4]) {
  const uint32_t kMagic = 0x64006400u;   // 1024.0 | 1024.0
  const uint32_t k1032 = 0x64086408u;    // 1032.0
  const uint32_t kSixteenth = 0x2C002C00u;  // 0.0625
  const uint32_t kNeg72 = 0xD480D480u;   // -72.0
  const uint32_t w8 = w >> 8;
  o[0] = hsub2_u(lop_and_or(w, 0x000F000Fu, kMagic), k1032);
  o[1] = hfma2_u(lop_and_or(w, 0x00F000F0u, kMagic), kSixteenth, kNeg72);
  o[2] = hsub2_u(lop_and_or(w8, 0x000F000Fu, kMagic), k1032);
  o[3] = hfma2_u(lop_and_or(w8, 0x00F000F0u, kMagic), kSixteenth, kNeg72);
}

__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// fp32 pair (a, b) -> hi = fp16(a), fp16(b); lo = fp16(a - hi_a), fp16(b - hi_b)
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_half2(a, b);
  const __half2 h = *reinterpret_cast<const __half2*>(&hi);
  const float2 f = __half22float2(h);
  lo = pack_half2(a - f.x, b - f.y);
}

// staged-x word position: XOR the low two bits with bits 2..3, which spreads the 16-byte reads of
// the four lanes of a quad over distinct bank groups
__device__ __forceinline__ int xswz(int w) { return w ^ ((w >> 2) & 3); }

__device__ __forceinline__ float load_y(const void* y, size_t i, int f32) {
  return f32 ? reinterpret_cast<const float*>(y)[i] : __half2float(reinterpret_cast<const __half*>(y)[i]);
}
__device__ __forceinline__ void store_y(void* y, size_t i, float v, int f32) {
  if (f32)
    reinterpret_cast<float*>(y)[i] = v;
  else
    reinterpret_cast<__half*>(y)[i] = __float2half_rn(v);
}

// ---- tensor-core kernel --------------------------------------------------------------------

template <int MT, bool XF32, int T>
__global__ void __launch_bounds__(256) q4_gemv_mma(LinArgs p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ int s_last;
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int rt = blockIdx.x, sp = blockIdx.y;
  const bool swiglu = p.epi == Q4B_EPI_SWIGLU;

  // weight rows feeding A-fragment rows g and g + 8 (SwiGLU: gate row i and up row I + i)
  int ra, rb;
  if (swiglu) {
    const int i = min(rt * 8 + g, p.n_out - 1);
    ra = i;
    rb = p.n_out + i;
  } else {
    ra = min(rt * 16 + g, p.N - 1);
    rb = min(rt * 16 + g + 8, p.N - 1);
  }
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

  // 2) stage x[:, kt0*128 : kt1*128) as permuted fp16 pairs (hi, and lo for fp32 x)
  const int rstride = p.kps * 16 + 4;  // uint4 per staged row; +64 B keeps rows on other bank groups
  uint4* xs_hi = reinterpret_cast<uint4*>(smem_raw);
  uint4* xs_lo = xs_hi + (size_t)p.M * rstride;
  const int nwords = (kt1 - kt0) * 16;
  for (int i = threadIdx.x; i < p.M * nwords; i += blockDim.x) {
    const int m = i / nwords, w = i - m * nwords;
    const size_t kb = (size_t)m * p.K + (size_t)kt0 * TILE_K + 8 * (size_t)w;
    uint4 hi;
    if constexpr (XF32) {
      const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + kb);
      const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + kb + 4);
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
  __syncthreads();

  // 3) MMAs: per tile, part = sum over its 128 k of (nib - 8) * x; acc += scale * part
  float acc[MT][4];
#pragma unroll
  for (int nt = 0; nt < MT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
  int mrow[MT];
#pragma unroll
  for (int nt = 0; nt < MT; ++nt) mrow[nt] = min(nt * 8 + g, p.M - 1) * rstride;

#pragma unroll
  for (int j = 0; j < T; ++j) {
    const int kt = kt0 + warp + W * j;
    if (kt < kt1) {
      float part[MT][4];
#pragma unroll
      for (int nt = 0; nt < MT; ++nt) part[nt][0] = part[nt][1] = part[nt][2] = part[nt][3] = 0.0f;
      const int wbase = (kt - kt0) * 16 + 4 * t;
      const uint32_t wav[4] = {wa[j].x, wa[j].y, wa[j].z, wa[j].w};
      const uint32_t wbv[4] = {wb[j].x, wb[j].y, wb[j].z, wb[j].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t A[4], B[4];
        dequant_word(wav[q], A);
        dequant_word(wbv[q], B);
        const int ph = xswz(wbase + q);
#pragma unroll
        for (int nt = 0; nt < MT; ++nt) {
          const uint4 xh = xs_hi[mrow[nt] + ph];
          mma_16816(part[nt], A[0], B[0], A[1], B[1], xh.x, xh.y);
          mma_16816(part[nt], A[2], B[2], A[3], B[3], xh.z, xh.w);
          if constexpr (XF32) {
            const uint4 xl = xs_lo[mrow[nt] + ph];
            mma_16816(part[nt], A[0], B[0], A[1], B[1], xl.x, xl.y);
            mma_16816(part[nt], A[2], B[2], A[3], B[3], xl.z, xl.w);
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < MT; ++nt) {
        acc[nt][0] = fmaf(sa[j], part[nt][0], acc[nt][0]);
        acc[nt][1] = fmaf(sa[j], part[nt][1], acc[nt][1]);
        acc[nt][2] = fmaf(sb[j], part[nt][2], acc[nt][2]);
        acc[nt][3] = fmaf(sb[j], part[nt][3], acc[nt][3]);
      }
    }
  }

  // 4) sum the W warps' tiles in shared memory: red[warp][m][r], then fin[m][r]
  __syncthreads();
  constexpr int MP = MT * 8;
  float* red = reinterpret_cast<float*>(smem_raw);
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

  // 5) split-K: publish partials; the last CTA of this row tile sums them in split order
  if (p.nsplit > 1) {
    const size_t NR = (size_t)gridDim.x * 16;
    for (int i = threadIdx.x; i < items; i += blockDim.x) {
      const int m = i >> 4, r = i & 15;
      p.ws[((size_t)sp * p.M + m) * NR + (size_t)rt * 16 + r] = fin[i];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(&p.counters[rt], 1u) == (unsigned)(p.nsplit - 1));
    __syncthreads();
    if (!s_last) return;
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

  // 6) epilogue
  for (int i = threadIdx.x; i < items; i += blockDim.x) {
    const int m = i >> 4, r = i & 15;
    if (swiglu) {
      const int col = rt * 8 + r;
      if (r < 8 && col < p.n_out) store_y(p.y, (size_t)m * p.n_out + col, silu(fin[i]) * fin[i + 8], p.y_f32);
    } else {
      const int col = rt * 16 + r;
      if (col < p.N) {
        float v = fin[i];
        const size_t o = (size_t)m * p.N + col;
        if (p.epi == Q4B_EPI_ACCUMULATE) v += load_y(p.y, o, p.y_f32);
        store_y(p.y, o, v, p.y_f32);
      }
    }
  }
}

// ---- generic SIMT kernel -------------------------------------------------------------------

template <bool XF32>
__global__ void __launch_bounds__(256) q4_linear_simt(LinArgs p) {
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mchunks = (p.M + 7) / 8;
  const long long gw = (long long)blockIdx.x * warps + warp;
  griddep_launch_dependents();
  griddep_wait();
  if (gw >= (long long)p.n_out * mchunks) return;
  const int o = (int)(gw / mchunks), mc = (int)(gw % mchunks);
  const bool swiglu = p.epi == Q4B_EPI_SWIGLU;
  const int m0 = mc * 8, mcount = min(8, p.M - m0);
  const int KW = p.K / 8, KG = p.K / p.G;
  float acc[2][8];
#pragma unroll
  for (int r = 0; r < 2; ++r)
#pragma unroll
    for (int m = 0; m < 8; ++m) acc[r][m] = 0.0f;

  for (int w = lane; w < KW; w += 32) {
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      if (rr == 1 && !swiglu) break;
      const int row = rr == 0 ? o : p.n_out + o;
      const int32_t word = __ldg(p.qw + (size_t)row * KW + w);
      const float s = __half2float(p.scales[(size_t)row * KG + (8 * w) / p.G]);
      float wv[8];
#pragma unroll
      for (int b = 0; b < 8; ++b) wv[b] = (float)(((word >> (4 * b)) & 15) - 8) * s;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        if (m < mcount) {
          const size_t xb = (size_t)(m0 + m) * p.K + 8 * (size_t)w;
          float d = 0.0f;
#pragma unroll
          for (int b = 0; b < 8; ++b) {
            const float xv = XF32 ? __ldg(reinterpret_cast<const float*>(p.x) + xb + b)
                                  : __half2float(reinterpret_cast<const __half*>(p.x)[xb + b]);
            d = fmaf(wv[b], xv, d);
          }
          acc[rr][m] += d;
        }
      }
    }
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr)
#pragma unroll
    for (int m = 0; m < 8; ++m) acc[rr][m] = warp_sum(acc[rr][m]);
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      if (m < mcount) {
        if (swiglu) {
          store_y(p.y, (size_t)(m0 + m) * p.n_out + o, silu(acc[0][m]) * acc[1][m], p.y_f32);
        } else {
          const size_t off = (size_t)(m0 + m) * p.N + o;
          float v = acc[0][m];
          if (p.epi == Q4B_EPI_ACCUMULATE) v += load_y(p.y, off, p.y_f32);
          store_y(p.y, off, v, p.y_f32);
        }
      }
    }
  }
}

// ---- planning ------------------------------------------------------------------------------

struct Plan {
  int kernel = 2;  // 1 = mma, 2 = simt
  int W = 4, T = 1, nsplit = 1, kps = 1, MT = 1;
  int RT = 0;      // row tiles (grid.x)
  size_t smem = 0;
  size_t ws_bytes = 0;
};

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

constexpr size_t kMaxSmem = 200 * 1024;

static size_t mma_smem(const Plan& pl, int M, bool xf32) {
  const size_t stage = (size_t)M * (pl.kps * 16 + 4) * 16 * (xf32 ? 2 : 1);
  const size_t red = (size_t)pl.W * pl.MT * 8 * 16 * 4 + (size_t)M * 16 * 4;
  return std::max(stage, red);
}

// Workspace layout: [0, kCounterBytes) arrival counters, one per row tile, at a fixed place for
// every call (each call leaves the counters it used at zero, so calls with different plans can
// share one workspace), then the split-K partial sums of the current call.
constexpr size_t kCounterBytes = 64 * 1024;
constexpr int kMaxCounters = (int)(kCounterBytes / 4);

static size_t mma_ws(const Plan& pl, int M) {
  if (pl.nsplit <= 1) return 0;
  return kCounterBytes + align_up((size_t)pl.nsplit * M * pl.RT * 16 * 4, 256);
}

// Tuned default: keep ~2 KB of weights per warp in flight and enough CTAs to fill 148 SMs several
// times; prefer no split when the row tiles alone give that many CTAs.
static int plan_linear(int M, int N, int K, int G, int epi, bool xf32, const q4b_linear_cfg* cfg, Plan& pl) {
  const int n_out = epi == Q4B_EPI_SWIGLU ? N / 2 : N;
  const bool mma_ok = (G % TILE_K == 0) && M <= 64;
  const int want = cfg ? cfg->kernel : 0;
  if (want == 1 && !mma_ok)
    return set_error(Q4B_EUNSUPPORTED, "q4_linear: tensor-core kernel needs group %% 128 == 0 and m <= 64");
  if (want == 2 || (want == 0 && !mma_ok)) {
    pl.kernel = 2;
    pl.W = 8;
    return Q4B_OK;
  }
  pl.kernel = 1;
  pl.MT = M <= 8 ? 1 : M <= 16 ? 2 : M <= 32 ? 4 : 8;
  pl.RT = epi == Q4B_EPI_SWIGLU ? (n_out + 7) / 8 : (N + 15) / 16;
  const int KT = K / TILE_K;
  int W = cfg && cfg->warps ? cfg->warps : 0;
  int T = cfg && cfg->tiles ? cfg->tiles : 0;
  int S = cfg && cfg->split ? cfg->split : 0;
  if (!T) T = pl.MT == 1 ? 2 : 1;
  if (!W) {
    if (S) {
      W = std::min(8, (((KT + S - 1) / S) + T - 1) / T);
    } else if (pl.RT >= 148 * 6) {  // plenty of row tiles: cover K within the CTA if it fits
      W = std::min(8, (KT + T - 1) / T);
      if (W * T < KT) W = 4;
    } else {
      W = 4;
    }
  }
  if (W < 1 || W > 8 || T < 1 || T > 4) return set_error(Q4B_EINVAL, "q4_linear: warps must be 1..8, tiles 1..4");
  const bool user_shape = cfg && (cfg->warps || cfg->split);
  for (;;) {
    const int s = S ? S : (KT + W * T - 1) / (W * T);
    pl.W = W;
    pl.T = T;
    pl.kps = (KT + s - 1) / s;
    pl.nsplit = (KT + pl.kps - 1) / pl.kps;
    if (pl.kps > W * T)
      return set_error(Q4B_EINVAL, "q4_linear: split %d leaves %d tiles per CTA > warps*tiles %d", s, pl.kps, W * T);
    pl.smem = mma_smem(pl, M, xf32);
    if (pl.smem <= kMaxSmem && (pl.nsplit == 1 || pl.RT <= kMaxCounters)) break;
    if (pl.smem <= kMaxSmem) {  // too many row tiles for the counter region: no split
      if (user_shape || (KT + T - 1) / T > 8) return set_error(Q4B_EUNSUPPORTED, "q4_linear: split-K limited to "
                                                               "%d row tiles", kMaxCounters);
      W = (KT + T - 1) / T;
      S = 1;
      continue;
    }
    if (user_shape || W == 1) return set_error(Q4B_EUNSUPPORTED, "q4_linear: shared memory plan too large");
    W = W / 2;  // fewer tiles per CTA: a smaller staged slice of x
  }
  pl.ws_bytes = mma_ws(pl, M);
  return Q4B_OK;
}

template <int MT, bool XF32, int T>
static cudaError_t launch_mma_t(const Plan& pl, const LinArgs& a, cudaStream_t st) {
  auto kern = q4_gemv_mma<MT, XF32, T>;
  static unsigned long long attr_set = 0;  // bit per device: opt-in to large dynamic shared memory
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set >> (dev & 63) & 1ull)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    if (e != cudaSuccess) return e;
    attr_set |= 1ull << (dev & 63);
  }
  return launch_pdl(kern, dim3(pl.RT, pl.nsplit), dim3(pl.W * 32), pl.smem, st, a);
}

template <int MT, bool XF32>
static cudaError_t launch_mma_x(const Plan& pl, const LinArgs& a, cudaStream_t st) {
  switch (pl.T) {
    case 1: return launch_mma_t<MT, XF32, 1>(pl, a, st);
    case 2: return launch_mma_t<MT, XF32, 2>(pl, a, st);
    case 3: return launch_mma_t<MT, XF32, 3>(pl, a, st);
    default: return launch_mma_t<MT, XF32, 4>(pl, a, st);
  }
}

template <bool XF32>
static cudaError_t launch_mma(const Plan& pl, const LinArgs& a, cudaStream_t st) {
  switch (pl.MT) {
    case 1: return launch_mma_x<1, XF32>(pl, a, st);
    case 2: return launch_mma_x<2, XF32>(pl, a, st);
    case 4: return launch_mma_x<4, XF32>(pl, a, st);
    default: return launch_mma_x<8, XF32>(pl, a, st);
  }
}

}  // namespace q4b

using namespace q4b;

static int validate_linear(const int32_t* qweight, const uint16_t* scales, int group, const void* x, int x_dtype,
                           void* y, int y_dtype, int m, int n, int k, int epi) {
  if (!qweight || !scales || !x || !y) return set_error(Q4B_EINVAL, "q4_linear: null pointer");
  if (m < 1 || n < 1 || k < 8 || k % 8) return set_error(Q4B_EINVAL, "q4_linear: bad shape m=%d n=%d k=%d", m, n, k);
  if (group < 8 || group % 8 || k % group)
    return set_error(Q4B_EINVAL, "q4_linear: need k %% group == 0 and group %% 8 == 0 (k=%d group=%d)", k, group);
  if ((x_dtype != Q4B_F32 && x_dtype != Q4B_F16) || (y_dtype != Q4B_F32 && y_dtype != Q4B_F16))
    return set_error(Q4B_EINVAL, "q4_linear: bad dtype");
  if (epi < Q4B_EPI_STORE || epi > Q4B_EPI_SWIGLU) return set_error(Q4B_EINVAL, "q4_linear: bad epilogue %d", epi);
  if (epi == Q4B_EPI_SWIGLU && n % 2) return set_error(Q4B_EINVAL, "q4_linear: SwiGLU needs an even row count");
  return Q4B_OK;
}

extern "C" size_t q4b_q4_linear_workspace(int m, int n, int k, int group, int epilogue, const q4b_linear_cfg* cfg) {
  if (m < 1 || n < 1 || k < 8 || group < 8 || k % group || group % 8) return 0;
  Plan a, b;
  const size_t wa = plan_linear(m, n, k, group, epilogue, true, cfg, a) == Q4B_OK ? a.ws_bytes : 0;
  const size_t wb = plan_linear(m, n, k, group, epilogue, false, cfg, b) == Q4B_OK ? b.ws_bytes : 0;
  return std::max(wa, wb);
}

extern "C" int q4b_q4_linear(const int32_t* qweight, const uint16_t* scales, int group, const void* x, int x_dtype,
                             void* y, int y_dtype, int m, int n, int k, int epilogue, const q4b_linear_cfg* cfg,
                             void* workspace, size_t workspace_bytes, q4b_stream_t stream) {
  int rc = validate_linear(qweight, scales, group, x, x_dtype, y, y_dtype, m, n, k, epilogue);
  if (rc) return rc;
  const bool xf32 = x_dtype == Q4B_F32;
  Plan pl;
  if ((rc = plan_linear(m, n, k, group, epilogue, xf32, cfg, pl))) return rc;
  if (pl.kernel == 1) {
    if (!aligned(qweight, 16) || !aligned(x, 16)) {
      if (cfg && cfg->kernel == 1) return set_error(Q4B_EINVAL, "q4_linear: qweight and x must be 16-byte aligned");
      pl.kernel = 2;
      pl.W = 8;
    } else if (pl.ws_bytes > workspace_bytes || (pl.ws_bytes && !workspace) || !aligned(workspace, 16)) {
      if (cfg && cfg->split > 1)
        return set_error(Q4B_EINVAL, "q4_linear: workspace of %zu bytes needed, %zu given", pl.ws_bytes,
                         workspace_bytes);
      // no (or too little) workspace: cover K inside one CTA when possible, else the SIMT kernel
      const int KT = k / TILE_K;
      if (KT <= 32) {
        pl.T = (KT + 7) / 8;
        pl.W = (KT + pl.T - 1) / pl.T;
        pl.kps = KT;
        pl.nsplit = 1;
        pl.smem = mma_smem(pl, m, xf32);
        pl.ws_bytes = 0;
      } else {
        pl.kernel = 2;
        pl.W = 8;
      }
    }
  }
  LinArgs a;
  a.qw = qweight;
  a.scales = reinterpret_cast<const __half*>(scales);
  a.x = x;
  a.y = y;
  a.M = m;
  a.N = n;
  a.K = k;
  a.G = group;
  a.n_out = epilogue == Q4B_EPI_SWIGLU ? n / 2 : n;
  a.KT = k / TILE_K;
  a.kps = pl.kps;
  a.nsplit = pl.nsplit;
  a.epi = epilogue;
  a.y_f32 = y_dtype == Q4B_F32;
  a.ws = nullptr;
  a.counters = nullptr;
  if (pl.kernel == 1 && pl.nsplit > 1) {
    a.counters = reinterpret_cast<unsigned*>(workspace);
    a.ws = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + kCounterBytes);
  }
  cudaStream_t st = as_stream(stream);
  cudaError_t e;
  if (pl.kernel == 1) {
    e = xf32 ? launch_mma<true>(pl, a, st) : launch_mma<false>(pl, a, st);
  } else {
    const long long warps = (long long)a.n_out * ((m + 7) / 8);
    const int block = 256;
    const long long grid = (warps + 7) / 8;
    e = xf32 ? launch_pdl(q4_linear_simt<true>, dim3((unsigned)grid), dim3(block), 0, st, a)
             : launch_pdl(q4_linear_simt<false>, dim3((unsigned)grid), dim3(block), 0, st, a);
  }
  if (e != cudaSuccess) return set_error(Q4B_ELAUNCH, "q4_linear: launch failed: %s", cudaGetErrorString(e));
  return check_launch("q4_linear");
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
