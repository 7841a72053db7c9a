// Device helpers shared by the int4 kernels (q4_linear.cu, decode_mk.cu): LOP3 nibble dequant to
// exact fp16, the m16n8k16 MMA, fp32 -> (hi, lo) fp16 splitting and the staged-x swizzle.
#pragma once

#include "common.cuh"

namespace q4b {

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
  const uint32_t kMagic = 0x64006400u;      // 1024.0 | 1024.0
  const uint32_t k1032 = 0x64086408u;       // 1032.0
  const uint32_t kSixteenth = 0x2C002C00u;  // 0.0625
  const uint32_t kNeg72 = 0xD480D480u;      // -72.0
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

// One 128-k tile of MMAs: weights of rows g / g + 8 (4 words each) times staged x. ILP keeps two
// independent accumulator chains per n-tile (and two more for the lo terms) so consecutive MMAs do
// not wait on each other: faster for launches of few CTAs, but its registers cost occupancy in
// launches of many CTAs, which use the single chain.
template <int MT, bool XF32, bool ILP>
__device__ __forceinline__ void mma_tile(const uint4& wa, const uint4& wb, float sa, float sb, const uint4* xs_hi,
                                         const uint4* xs_lo, const int (&mrow)[MT], int wbase, float (&acc)[MT][4]) {
  constexpr int NC = ILP ? 2 : 1;
  float part[MT][NC][4], partl[MT][NC][4];
#pragma unroll
  for (int nt = 0; nt < MT; ++nt)
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) part[nt][c][e] = partl[nt][c][e] = 0.0f;
  const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t wbv[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t A[4], B[4];
    dequant_word(wav[q], A);
    dequant_word(wbv[q], B);
    const int ph = xswz(wbase + q);
#pragma unroll
    for (int nt = 0; nt < MT; ++nt) {
      const uint4 xh = xs_hi[mrow[nt] + ph];
      mma_16816(part[nt][0], A[0], B[0], A[1], B[1], xh.x, xh.y);
      mma_16816(part[nt][NC - 1], A[2], B[2], A[3], B[3], xh.z, xh.w);
      if constexpr (XF32) {
        const uint4 xl = xs_lo[mrow[nt] + ph];
        mma_16816(ILP ? partl[nt][0] : part[nt][0], A[0], B[0], A[1], B[1], xl.x, xl.y);
        mma_16816(ILP ? partl[nt][NC - 1] : part[nt][0], A[2], B[2], A[3], B[3], xl.z, xl.w);
      }
    }
  }
#pragma unroll
  for (int nt = 0; nt < MT; ++nt) {
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if constexpr (ILP)
        v[e] = (part[nt][0][e] + part[nt][NC - 1][e]) + (partl[nt][0][e] + partl[nt][NC - 1][e]);
      else
        v[e] = part[nt][0][e];
    }
    acc[nt][0] = fmaf(sa, v[0], acc[nt][0]);
    acc[nt][1] = fmaf(sa, v[1], acc[nt][1]);
    acc[nt][2] = fmaf(sb, v[2], acc[nt][2]);
    acc[nt][3] = fmaf(sb, v[3], acc[nt][3]);
  }
}


// M = 1 with fp32 x: x_hi and x_lo as the first two columns of the MMA's B operand (lanes of group
// g = 0 supply x_hi, g = 1 x_lo, the other columns are zero), so each m16n8k16 yields both halves'
// products -- half the MMAs of mma_tile<1, true, *>. Lanes with t == 0 end up holding, for rows g
// and g + 8, acc[0] / acc[2] (hi part) and acc[1] / acc[3] (lo part); the row's value is their sum.
__device__ __forceinline__ void mma_tile_hl(const uint4& wa, const uint4& wb, float sa, float sb, const uint4* xs_hi,
                                            const uint4* xs_lo, int g, int wbase, float (&acc)[4]) {
  float part[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
  const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t wbv[4] = {wb.x, wb.y, wb.z, wb.w};
  const uint4* xs = g == 0 ? xs_hi : xs_lo;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t A[4], B[4];
    dequant_word(wav[q], A);
    dequant_word(wbv[q], B);
    const uint4 xv = g < 2 ? xs[xswz(wbase + q)] : make_uint4(0u, 0u, 0u, 0u);
    mma_16816(part[0], A[0], B[0], A[1], B[1], xv.x, xv.y);
    mma_16816(part[1], A[2], B[2], A[3], B[3], xv.z, xv.w);
  }
  acc[0] = fmaf(sa, part[0][0] + part[1][0], acc[0]);
  acc[1] = fmaf(sa, part[0][1] + part[1][1], acc[1]);
  acc[2] = fmaf(sb, part[0][2] + part[1][2], acc[2]);
  acc[3] = fmaf(sb, part[0][3] + part[1][3], acc[3]);
}
// ---- int8 tensor-core form for one x row --------------------------------------------------------
//
// x row staged per 128-k group as three int8 terms, x ~= sx * (a + b / 254 + c / 254^2) with
// sx = max|x| / 127 over the group (a, b, c in [-127, 127]; the residual is at most
// 0.5 * sx / 254^2, about 6e-8 of the group's largest |x|). The weights enter the MMA as their
// stored biased nibbles (0..15, unsigned bytes) and the zero point comes back exactly as an integer:
// sum_k (nib - 8) q_k = sum_k nib q_k - 8 X with X = sum_k q_k of the group.
constexpr float kI8Step = 1.0f / 254.0f;
constexpr float kI8Step2 = kI8Step * kI8Step;

__device__ __forceinline__ void mma_k32_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 128-k tile (one scale group) of rows g and g + 8 against the staged int8 x terms. wa / wb: the
// lane's 4 words of rows g / g + 8 (words 4t .. 4t + 3 of the tile); xv[q]: {even, odd} bytes of
// word 4t + q for term g (lanes g >= 3 pass zeros); xg = {X_a, X_b, X_c, sx} of the group. MMA q
// covers words 4t + q: k-slots 4t + i hold nibble 2i (even bytes), k-slots 16 + 4t + i nibble 2i + 1.
// Two integer accumulator chains (q even / odd) are added exactly. Columns of the result: 0 = term
// a, 1 = term b (lanes t == 0), 2 = term c (lanes t == 1, fetched by a shuffle). Adds s * sx * the
// group's dot product to acc[0] (row g) and acc[1] (row g + 8) on lanes t == 0.
__device__ __forceinline__ void mma_tile_i8(const uint4& wa, const uint4& wb, float sa, float sb, const uint2 (&xv)[4],
                                            const int4& xg, float (&acc)[2]) {
  int d[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t wbv[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t a0 = wav[q] & 0x0F0F0F0Fu, a2 = (wav[q] >> 4) & 0x0F0F0F0Fu;
    const uint32_t a1 = wbv[q] & 0x0F0F0F0Fu, a3 = (wbv[q] >> 4) & 0x0F0F0F0Fu;
    mma_k32_u8s8(d[q & 1], a0, a1, a2, a3, xv[q].x, xv[q].y);
  }
  const int s0 = d[0][0] + d[1][0], s1 = d[0][1] + d[1][1];
  const int s2 = d[0][2] + d[1][2], s3 = d[0][3] + d[1][3];
  const int c_g = __shfl_down_sync(0xffffffffu, s0, 1);   // term c of row g (lane t + 1)
  const int c_g8 = __shfl_down_sync(0xffffffffu, s2, 1);  // term c of row g + 8
  const float sx = __int_as_float(xg.w);
  const float vg = (float)(s0 - 8 * xg.x) + (float)(s1 - 8 * xg.y) * kI8Step + (float)(c_g - 8 * xg.z) * kI8Step2;
  const float vg8 = (float)(s2 - 8 * xg.x) + (float)(s3 - 8 * xg.y) * kI8Step + (float)(c_g8 - 8 * xg.z) * kI8Step2;
  acc[0] = fmaf(sa * sx, vg, acc[0]);
  acc[1] = fmaf(sb * sx, vg8, acc[1]);
}
}  // namespace q4b
