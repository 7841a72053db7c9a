// fp16 GEMM C[M,N] = op(A) . op(B) with fp32 accumulation and fp16 output: the prefill / tuner GEMM
// of gemm/shapes.py:1-6 (BLAS layout letters: A 'N' = [M][K] row-major, 'T' = stored [K][M];
// B 'N' = [K][N] row-major, 'T' = stored [N][K], a torch Linear weight) and gemm/schedule.py's
// generated kernels, rebuilt for sm_100a.
//
// Kernel 1 (tcgen05): one 128 x BN output tile per CTA (BN = 64 / 128 / 256), K in 64-wide steps.
// TMA brings each operand tile into a 128-byte-swizzled shared-memory ring (K-major tiles for
// A 'N' / B 'T', MN-major tiles for A 'T' / B 'N': the layout letter only changes the tensor map and
// the descriptor's major bit, no transpose kernel); one thread issues tcgen05.mma (M=128, N=BN,
// K=16) into a TMEM accumulator and commits each ring slot back to the producer; all four warps
// then read TMEM (32 lanes each) and store fp16. Split-K (grid.z) writes fp32 partials to the
// workspace and the last CTA of a tile adds them in split order (deterministic) before storing.
// Kernel 2 (CUDA cores): 64 x 64 tiles for any size or alignment TMA cannot describe.
// Kernel 3 (tcgen05, persistent stream-K; opt-in): described at the kernel. Measured slower than
// kernel 1's searched schedules on every config-2 shape (one CTA's MMA stream per SM against two).
#include <mutex>

#include "tc.cuh"

namespace q4b {

namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kGemmSmemBudget = 200 * 1024;
constexpr size_t kGemmCounterBytes = 64 * 1024;  // per-tile split-K arrival counters (16384 tiles)

__device__ unsigned g_gemm_status = 0;

struct GemmArgs {
  int M, N, K;
  int kt;      // number of 64-wide k steps
  int split;   // k splits (grid.z)
  int tm, tn;  // kernel 3: output tiles along M and N
  int vec;     // C rows keep 16-byte alignment (n % 8 == 0, aligned base): vector stores
  __half* C;
  float* partial;       // split > 1: [split][tiles][128][BN] fp32
  unsigned* counters;   // split > 1: [tiles]
};

template <int BN>
struct GemmTile {
  static constexpr int A_BYTES = kBM * kBK * 2;  // 16 KB
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int MAX_STAGES = kGemmSmemBudget / STAGE;
};

__device__ __forceinline__ void store_row_f16(__half* crow, int col0, int ncols, int N, const float* v, bool vec) {
  // 32 consecutive outputs of one row; vector stores when the row pitch keeps 16-byte alignment
  if (vec && col0 + 32 <= N) {
    uint4* dst = reinterpret_cast<uint4*>(crow + col0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      __half2 h[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(v[8 * q + 2 * e], v[8 * q + 2 * e + 1]);
      dst[q] = *reinterpret_cast<uint4*>(h);
    }
  } else {
    for (int j = 0; j < 32 && j < ncols; ++j)
      if (col0 + j < N) crow[col0 + j] = __float2half_rn(v[j]);
  }
}

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(128, 1)
    gemm_f16_tc(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, GemmArgs p,
                int stages) {
  using T = GemmTile<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[T::MAX_STAGES], empty[T::MAX_STAGES], acc_full;
  __shared__ uint32_t s_tmem;
  __shared__ int s_last, s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN;
  const int z = blockIdx.z;
  const int k_begin = (int)((long long)z * p.kt / p.split), k_end = (int)((long long)(z + 1) * p.kt / p.split);
  const int nk = k_end - k_begin;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    s_fail = 0;
    fence_mbar_init();
    tma_prefetch_map(&ta);
    tma_prefetch_map(&tb);
  }
  if (warp == 0) tmem_alloc(&s_tmem, BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  griddep_wait();  // A / B may be written by the previous kernel on the stream

  if (warp == 0) {
    if (lane == 0) {
      // producer: TMA loads into the ring
      for (int it = 0; it < nk; ++it) {
        const int s = it % stages, r = it / stages;
        if (r > 0 && !mbar_wait_bounded(&empty[s], (r - 1) & 1, kWaitLimitNs)) {
          s_fail = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], T::STAGE);
        uint8_t* a = smem + s * T::STAGE;
        uint8_t* b = a + T::A_BYTES;
        const int kx = (k_begin + it) * kBK;
        if constexpr (!A_MN) {
          tma_load_2d(a, &ta, kx, m0, &full[s]);
        } else {
          tma_load_2d(a, &ta, m0, kx, &full[s]);
          tma_load_2d(a + 8192, &ta, m0 + 64, kx, &full[s]);
        }
        if constexpr (!B_MN) {
          tma_load_2d(b, &tb, kx, n0, &full[s]);
        } else {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) tma_load_2d(b + j * 8192, &tb, n0 + 64 * j, kx, &full[s]);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issue: 4 x (128 x BN x 16) per ring slot, accumulating in TMEM
      constexpr uint32_t idesc = idesc_f16_f32(kBM, BN, A_MN, B_MN);
      for (int it = 0; it < nk; ++it) {
        const int s = it % stages, r = it / stages;
        if (!mbar_wait_bounded(&full[s], r & 1, kWaitLimitNs)) {
          s_fail = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a = smem_u32(smem + s * T::STAGE), b = a + T::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          const uint64_t ad = A_MN ? sw128_desc(a + kk * 2048, 8192, 1024) : sw128_desc(a + kk * 32, 16, 1024);
          const uint64_t bd = B_MN ? sw128_desc(b + kk * 2048, 8192, 1024) : sw128_desc(b + kk * 32, 16, 1024);
          tc_mma_f16(tmem, ad, bd, idesc, (it | kk) != 0);
        }
        tc_commit(&empty[s]);  // the slot is free once these MMAs have read it
      }
      tc_commit(&acc_full);
    }
    __syncwarp();
  }

  // epilogue: warp w owns accumulator rows 32w..32w+31 (TMEM lanes), one row per thread
  if (!mbar_wait_bounded(&acc_full, 0, kWaitLimitNs)) s_fail = 1;
  __syncthreads();
  const bool ok = !s_fail;
  tc_fence_after();
  const int row = m0 + warp * 32 + lane;
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  const bool vec = p.vec != 0;
  const int tile = blockIdx.y * gridDim.x + blockIdx.x;
  if (!ok) {
    if (threadIdx.x == 0) atomicOr(&g_gemm_status, kStatusTimeout);
  } else if (p.split == 1) {
    __half* crow = p.C + (size_t)row * p.N;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32(trow + c * 32, r);
      if (row < p.M && n0 + c * 32 < p.N) store_row_f16(crow, n0 + c * 32, 32, p.N, reinterpret_cast<float*>(r), vec);
    }
  } else {
    float* mine = p.partial + ((size_t)z * gridDim.x * gridDim.y + tile) * (kBM * BN) + (size_t)(warp * 32 + lane) * BN;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32(trow + c * 32, r);
      float4* d = reinterpret_cast<float4*>(mine + c * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        d[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                           __uint_as_float(r[4 * q + 3]));
    }
    __threadfence();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
  if (p.split > 1 && ok) {
    if (threadIdx.x == 0) {
      const unsigned prev = atomicAdd(&p.counters[tile], 1u);
      s_last = prev == (unsigned)(p.split - 1);
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      const size_t zstride = (size_t)gridDim.x * gridDim.y * (kBM * BN);
      const float* base = p.partial + (size_t)tile * (kBM * BN) + (size_t)(warp * 32 + lane) * BN;
      __half* crow = p.C + (size_t)row * p.N;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.0f;
        for (int zz = 0; zz < p.split; ++zz) {
          const float4* src = reinterpret_cast<const float4*>(base + zz * zstride + c * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 t = __ldcg(src + q);
            v[4 * q] += t.x;
            v[4 * q + 1] += t.y;
            v[4 * q + 2] += t.z;
            v[4 * q + 3] += t.w;
          }
        }
        if (row < p.M && n0 + c * 32 < p.N) store_row_f16(crow, n0 + c * 32, 32, p.N, v, vec);
      }
      if (threadIdx.x == 0) p.counters[tile] = 0u;  // ready for the next call (graph replays)
    }
  }
  griddep_launch_dependents();
}

// ---- kernel 3: tcgen05, persistent stream-K ---------------------------------------------------
//
// T = tiles_m x tiles_n output tiles of 128 x BN make U = T x kt units (one 64-wide k step of one
// tile). CTA c of G takes the units [c U / G, (c + 1) U / G) in tile-major order, so every CTA
// streams the same number of operand tiles whatever T is: no partly filled last wave, and no k
// split chosen by hand. A CTA's run cuts into segments, one per tile it touches: the middle ones
// are whole tiles, stored from TMEM directly; only the first and the last can cover part of a
// tile. Warp 0 (one thread) keeps the TMA ring full across segment boundaries; warp 1 (one thread)
// issues segment s's MMAs into TMEM accumulator s % 2 and commits it; warps 2-5 (TMEM lane
// quadrants 2, 3, 0, 1) drain the other accumulator meanwhile, so one tile's epilogue runs under
// the next tile's main loop. A part-tile goes to the CTA's partial slot (2c for its first segment,
// 2c + 1 for its last) in the workspace; the last of a tile's contributors to arrive (arrival
// counter) adds the slots in k order and stores the tile, so results are deterministic.
constexpr int kSkThreads = 192;

// the CTA whose run of units [c U / G, (c + 1) U / G) contains unit u (G <= U: no run is empty)
__device__ __forceinline__ int sk_cta_of(long long u, long long U, int G) {
  return (int)(((u + 1) * G + U - 1) / U) - 1;
}

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kSkThreads, 2)
    gemm_f16_sk(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, GemmArgs p,
                int stages, int nacc) {
  using T = GemmTile<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[T::MAX_STAGES], empty[T::MAX_STAGES], acc_full[2], acc_empty[2], mma_done;
  __shared__ uint32_t s_tmem;
  __shared__ int s_last, s_issued, s_consumed;
  __shared__ volatile int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;
  const long long U = (long long)p.tm * p.tn * p.kt;
  const long long u0 = U * blockIdx.x / G, u1 = U * (blockIdx.x + 1) / G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    mbar_init(&mma_done, 1);
    s_fail = 0;
    s_issued = 0;
    s_consumed = 0;
    fence_mbar_init();
    tma_prefetch_map(&ta);
    tma_prefetch_map(&tb);
  }
  if (warp == 1) tmem_alloc(&s_tmem, nacc * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  griddep_wait();  // A / B may be written by the previous kernel on the stream

  if (warp == 0) {
    if (lane == 0) {
      // producer: the run's operand tiles, in unit order, through the ring (tile, k step, ring
      // slot and round advance by increments: no divisions on this thread's per-unit path)
      const int t0 = (int)(u0 / p.kt);
      int k = (int)(u0 - (long long)t0 * p.kt), im = t0 % p.tm, in = t0 / p.tm;
      int s = 0, r = 0;
      for (long long u = u0; u < u1; ++u) {
        if (s_fail || (r > 0 && !mbar_wait_bounded(&empty[s], (r - 1) & 1, kWaitLimitNs))) {
          s_fail = 1;
          break;
        }
        const int m0 = im * kBM, n0 = in * BN;
        mbar_arrive_expect_tx(&full[s], T::STAGE);
        uint8_t* a = smem + s * T::STAGE;
        uint8_t* b = a + T::A_BYTES;
        const int kx = k * kBK;
        if constexpr (!A_MN) {
          tma_load_2d(a, &ta, kx, m0, &full[s]);
        } else {
          tma_load_2d(a, &ta, m0, kx, &full[s]);
          tma_load_2d(a + 8192, &ta, m0 + 64, kx, &full[s]);
        }
        if constexpr (!B_MN) {
          tma_load_2d(b, &tb, kx, n0, &full[s]);
        } else {
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) tma_load_2d(b + j * 8192, &tb, n0 + 64 * j, kx, &full[s]);
        }
        s_issued = (int)(u - u0) + 1;
        if (++k == p.kt) {
          k = 0;
          if (++im == p.tm) im = 0, ++in;
        }
        if (++s == stages) s = 0, ++r;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issue: segment seg accumulates in TMEM columns [BN (seg % 2), BN (seg % 2 + 1))
      constexpr uint32_t idesc = idesc_f16_f32(kBM, BN, A_MN, B_MN);
      int i = 0, seg = 0, s = 0, r = 0;
      bool ok = true;
      for (long long u = u0; u < u1 && ok; ++seg) {
        const int t = (int)(u / p.kt), k0 = (int)(u - (long long)t * p.kt);
        const int k1 = (int)min((long long)p.kt, (long long)k0 + (u1 - u));
        const int b = nacc == 2 ? seg & 1 : 0, use = nacc == 2 ? seg >> 1 : seg;
        if (use > 0 && !mbar_wait_bounded(&acc_empty[b], (use - 1) & 1, kWaitLimitNs)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * BN);
        for (int k = k0; k < k1; ++k, ++i) {
          if (s_fail || !mbar_wait_bounded(&full[s], r & 1, kWaitLimitNs)) {
            ok = false;
            break;
          }
          s_consumed = i + 1;
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * T::STAGE), bb = a + T::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = A_MN ? sw128_desc(a + kk * 2048, 8192, 1024) : sw128_desc(a + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sw128_desc(bb + kk * 2048, 8192, 1024) : sw128_desc(bb + kk * 32, 16, 1024);
            tc_mma_f16(d, ad, bd, idesc, (k != k0 || kk != 0) ? 1u : 0u);
          }
          tc_commit(&empty[s]);  // the slot is free once these MMAs have read it
          if (++s == stages) s = 0, ++r;
        }
        if (!ok) break;
        tc_commit(&acc_full[b]);
        u += k1 - k0;
      }
      if (!ok) s_fail = 1;
      tc_commit(&mma_done);  // every MMA issued above has completed
    }
    __syncwarp();
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31, one output row per thread
    const int q = warp & 3;
    const int rloc = q * 32 + lane;
    const bool vec = p.vec != 0;
    int seg = 0;
    for (long long u = u0; u < u1; ++seg) {
      const int t = (int)(u / p.kt), k0 = (int)(u - (long long)t * p.kt);
      const int k1 = (int)min((long long)p.kt, (long long)k0 + (u1 - u));
      const bool whole = k0 == 0 && k1 == p.kt;
      const int b = nacc == 2 ? seg & 1 : 0, use = nacc == 2 ? seg >> 1 : seg;
      // lane 0 waits; the warp takes one decision (tcgen05.ld below is warp-collective)
      int okw = 0;
      if (lane == 0) {
        okw = !s_fail && mbar_wait_bounded(&acc_full[b], use & 1, kWaitLimitNs);
        if (!okw) s_fail = 1;
      }
      const bool ok = __shfl_sync(0xffffffffu, okw, 0) != 0;
      tc_fence_after();
      const int m0 = (t % p.tm) * kBM, n0 = (t / p.tm) * BN;
      const int row = m0 + rloc;
      const uint32_t trow = tmem + (uint32_t)(b * BN) + ((uint32_t)(q * 32) << 16);
      if (ok) {
        if (whole) {
          __half* crow = p.C + (size_t)row * p.N;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld_32x32(trow + c * 32, r);
            if (row < p.M && n0 + c * 32 < p.N)
              store_row_f16(crow, n0 + c * 32, 32, p.N, reinterpret_cast<float*>(r), vec);
          }
        } else {
          const int slot = 2 * (int)blockIdx.x + (u == u0 ? 0 : 1);
          float* mine = p.partial + ((size_t)slot * kBM + rloc) * BN;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld_32x32(trow + c * 32, r);
            float4* dst = reinterpret_cast<float4*>(mine + c * 32);
#pragma unroll
            for (int e = 0; e < 8; ++e)
              dst[e] = make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]),
                                   __uint_as_float(r[4 * e + 2]), __uint_as_float(r[4 * e + 3]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);  // the MMA thread may refill this accumulator
      if (!whole) {
        // arrive on the tile's counter (after a failure too, so that it ends at zero); the last
        // contributor adds every contributor's slot in k order
        const int c0 = sk_cta_of((long long)t * p.kt, U, G), c1 = sk_cta_of((long long)(t + 1) * p.kt - 1, U, G);
        __threadfence();
        named_bar_sync(1, 128);
        if (warp == 2 && lane == 0) s_last = atomicAdd(&p.counters[t], 1u) == (unsigned)(c1 - c0);
        named_bar_sync(1, 128);
        if (s_last) {
          __threadfence();
          if (!s_fail) {
            __half* crow = p.C + (size_t)row * p.N;
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
              float v[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.0f;
              for (int cb = c0; cb <= c1; cb += 4) {  // four contributors' loads in flight, then their sums
                float4 x[4][8];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const int cc = min(cb + j, c1);
                  const int first_tile = (int)((U * cc / G) / p.kt);
                  const int slot = 2 * cc + (t == first_tile ? 0 : 1);
                  const float4* src =
                      reinterpret_cast<const float4*>(p.partial + ((size_t)slot * kBM + rloc) * BN + c * 32);
#pragma unroll
                  for (int e = 0; e < 8; ++e) x[j][e] = __ldcg(src + e);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  if (cb + j > c1) break;
#pragma unroll
                  for (int e = 0; e < 8; ++e) {
                    v[4 * e] += x[j][e].x;
                    v[4 * e + 1] += x[j][e].y;
                    v[4 * e + 2] += x[j][e].z;
                    v[4 * e + 3] += x[j][e].w;
                  }
                }
              }
              if (row < p.M && n0 + c * 32 < p.N) store_row_f16(crow, n0 + c * 32, 32, p.N, v, vec);
            }
          }
          if (warp == 2 && lane == 0) p.counters[t] = 0u;  // ready for the next call (graph replays)
        }
      }
      u += k1 - k0;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (s_fail && threadIdx.x == 0) {
    // a wait gave up: the copies still in flight land before the CTA exits (bounded)
    for (int i = s_consumed; i < s_issued; ++i)
      mbar_wait_bounded(&full[i % stages], (uint32_t)((i / stages) & 1), kWaitLimitNs);
    atomicOr(&g_gemm_status, kStatusTimeout);
  }
  if (warp == 1) {
    if (lane == 0) mbar_wait_bounded(&mma_done, 0, kWaitLimitNs);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, nacc * BN);
  }
  griddep_launch_dependents();
}

// ---- kernel 2: CUDA-core tiles, any layout and alignment ----------------------------------------

template <bool A_T, bool B_T>
__global__ void __launch_bounds__(256) gemm_f16_simt(const __half* __restrict__ A, const __half* __restrict__ B,
                                                     __half* __restrict__ C, int M, int N, int K) {
  __shared__ float As[16][65];
  __shared__ float Bs[16][65];
  griddep_wait();
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 64 * 16; i += 256) {
      const int mm = i / 16, kk = i % 16;       // A element (m0+mm, k0+kk)
      const int m = m0 + mm, k = k0 + kk;
      float a = 0.f;
      if (m < M && k < K) a = __half2float(A_T ? A[(size_t)k * M + m] : A[(size_t)m * K + k]);
      As[kk][mm] = a;
      const int nn = i % 64, kb = i / 64;       // B element (k0+kb, n0+nn)
      const int n = n0 + nn, k2 = k0 + kb;
      float b = 0.f;
      if (n < N && k2 < K) b = __half2float(B_T ? B[(size_t)n * K + k2] : B[(size_t)k2 * N + n]);
      Bs[kb][nn] = b;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + ty + 16 * i, n = n0 + tx + 16 * j;
      if (m < M && n < N) C[(size_t)m * N + n] = __float2half_rn(acc[i][j]);
    }
  griddep_launch_dependents();
}

// ---- host --------------------------------------------------------------------------------------

struct GemmPlan {
  int kernel = 1, bn = 128, stages = 4, split = 1;
  int tiles_m = 0, tiles_n = 0;
  int ctas = 0;  // kernel 3: persistent CTAs
  int nacc = 2;  // kernel 3: TMEM accumulators per CTA
  size_t smem = 0, ws = 0;
};

// SMs of the current device (148 on a B200; also the planning answer without a device)
int device_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0) {
    cudaGetLastError();
    return 148;
  }
  return sms;
}

bool tma_ok(int M, int N, int K, char la, char lb) {
  const long long lda = la == 'N' ? K : M, ldb = lb == 'N' ? N : K;
  return lda % 8 == 0 && ldb % 8 == 0;
}

// The schedules the search (q4b.gemm.search on a B200, q4b/gemm/tuned_b200.json) measured fastest for
// the config-2 problems: the default plan of exactly these shapes and layouts.
struct TunedSchedule {
  int M, N, K;
  char la, lb;
  int bn, stages, split;
};
constexpr TunedSchedule kTuned[] = {
    {128, 5120, 3072, 'N', 'N', 64, 3, 3},  // B1 qkv_m128: 184 TFLOP/s
    {128, 3072, 3072, 'N', 'N', 64, 2, 3},  // B2 o_m128: 146 TFLOP/s
    {128, 16384, 3072, 'N', 'N', 128, 5, 1},  // B3 gate_up_m128: 529 TFLOP/s
    {128, 3072, 8192, 'N', 'N', 64, 5, 3},  // B4 down_m128: 230 TFLOP/s
    {2048, 5120, 3072, 'N', 'N', 256, 2, 1},  // B5 qkv_m2048: 881 TFLOP/s
    {2048, 3072, 3072, 'N', 'N', 256, 2, 1},  // B6 o_m2048: 943 TFLOP/s
    {2048, 16384, 3072, 'N', 'N', 256, 2, 1},  // B7 gate_up_m2048: 1009 TFLOP/s
    {2048, 3072, 8192, 'N', 'N', 256, 2, 1},  // B8 down_m2048: 922 TFLOP/s
};

// kernel 3: tile width (cfg or 256 once there are 8 row tiles, else 128) and ring depth (cfg, or the
// deepest that fits: one CTA per SM alternating two TMEM accumulators). A ring shallow enough for two
// CTAs on an SM (register cap 170 per thread) gives each one accumulator, the other CTA supplying the
// overlap (measured slower: B5 142 us against 95 us alone). Grid: SMs x CTAs per SM, at most one CTA
// per unit. Workspace: the per-tile counters and two partial slots [128][BN] fp32 per CTA.
int plan_sk(int M, int N, int kt, int tm, const q4b_gemm_cfg* cfg, GemmPlan& pl) {
  (void)M;
  int bn = cfg->bn ? cfg->bn : (tm >= 8 ? 256 : 128);
  if (bn != 64 && bn != 128 && bn != 256) return set_error(Q4B_EINVAL, "gemm_f16: bn is 64, 128 or 256");
  if (cfg->split > 1) return set_error(Q4B_EINVAL, "gemm_f16: kernel 3 balances k itself (split 0 or 1)");
  const int stage = (kBM + bn) * kBK * 2;
  const int max_stages = kGemmSmemBudget / stage;
  const auto per_sm = [](size_t smem) { return (int)(233472 / (smem + 2048)); };  // 228 KB an SM, 1 KB reserved per CTA
  const int stages = cfg->stages ? cfg->stages : max_stages;
  if (stages < 2 || stages > max_stages)
    return set_error(Q4B_EINVAL, "gemm_f16: stages must be in [2, %d] for bn %d", max_stages, bn);
  const int tn = (N + bn - 1) / bn;
  const long long tiles = (long long)tm * tn;
  if (tiles * 4 > (long long)kGemmCounterBytes) return set_error(Q4B_EUNSUPPORTED, "gemm_f16: too many tiles");
  pl.kernel = 3;
  pl.bn = bn;
  pl.stages = stages;
  pl.split = 1;
  pl.tiles_m = tm;
  pl.tiles_n = tn;
  pl.smem = (size_t)stages * stage + 1024;
  const int occ = std::max(1, std::min(2, per_sm(pl.smem)));
  pl.nacc = occ >= 2 ? 1 : 2;
  pl.ctas = (int)std::min<long long>(tiles * kt, (long long)device_sms() * occ);
  pl.ws = kGemmCounterBytes + (size_t)2 * pl.ctas * kBM * bn * 4;
  return Q4B_OK;
}

int plan_gemm(int M, int N, int K, char la, char lb, const q4b_gemm_cfg* cfg, GemmPlan& pl) {
  if (M <= 0 || N <= 0 || K <= 0) return set_error(Q4B_EINVAL, "gemm_f16: sizes must be positive");
  if ((la != 'N' && la != 'T') || (lb != 'N' && lb != 'T'))
    return set_error(Q4B_EINVAL, "gemm_f16: layouts are 'N' or 'T'");
  const int want = cfg ? cfg->kernel : 0;
  if (want < 0 || want > 3) return set_error(Q4B_EINVAL, "gemm_f16: kernel is 0, 1, 2 or 3");
  const bool tma = tma_ok(M, N, K, la, lb);
  if ((want == 1 || want == 3) && !tma)
    return set_error(Q4B_EUNSUPPORTED, "gemm_f16: the tcgen05 kernels need row pitches that are multiples of 8");
  if (want == 2 || !tma) {
    pl.kernel = 2;
    pl.split = 1;
    pl.smem = 0;
    pl.ws = 0;
    return Q4B_OK;
  }
  const int kt = (K + kBK - 1) / kBK;
  const int tm = (M + kBM - 1) / kBM;
  if (want == 3) return plan_sk(M, N, kt, tm, cfg, pl);
  pl.kernel = 1;
  q4b_gemm_cfg tuned = {};
  if (!cfg || (!cfg->kernel && !cfg->bn && !cfg->stages && !cfg->split)) {
    for (const TunedSchedule& t : kTuned)
      if (t.M == M && t.N == N && t.K == K && t.la == la && t.lb == lb) {
        tuned = {1, t.bn, t.stages, t.split};
        cfg = &tuned;
      }
  }
  int bn = cfg && cfg->bn ? cfg->bn : 0;
  if (bn && bn != 64 && bn != 128 && bn != 256) return set_error(Q4B_EINVAL, "gemm_f16: bn is 64, 128 or 256");
  if (!bn) {
    // widest tile that still fills the GPU, narrower tiles (and split-K below) for small problems
    bn = 256;
    while (bn > 64 && (long long)tm * ((N + bn - 1) / bn) < 148) bn /= 2;
  }
  const int tn = (N + bn - 1) / bn;
  int split = cfg && cfg->split ? cfg->split : 0;
  if (split < 0 || split > kt) return set_error(Q4B_EINVAL, "gemm_f16: split must be in [1, %d]", kt);
  if (!split) {
    split = 1;
    // fill the SMs while keeping at least 4 k steps (256 of K) per split
    while ((long long)tm * tn * split < 148 && kt / (split * 2) >= 4) split *= 2;
  }
  const int stage = (kBM + bn) * kBK * 2;
  const int max_stages = kGemmSmemBudget / stage;
  // 256-wide tiles over many row tiles: 2 stages (96 KB) leave room for two CTAs per SM, one's
  // epilogue beside the other's main loop (the search's fastest schedule for every M = 2048 shape)
  const int def_stages = (bn == 256 && tm >= 8 && max_stages >= 2) ? 2 : max_stages;
  int stages = cfg && cfg->stages ? cfg->stages : def_stages;
  if (stages < 2 || stages > max_stages)
    return set_error(Q4B_EINVAL, "gemm_f16: stages must be in [2, %d] for bn %d", max_stages, bn);
  const long long tiles = (long long)tm * tn;
  if (split > 1 && tiles * 4 > (long long)kGemmCounterBytes)
    return set_error(Q4B_EUNSUPPORTED, "gemm_f16: too many tiles for split-K");
  pl.bn = bn;
  pl.stages = stages;
  pl.split = split;
  pl.tiles_m = tm;
  pl.tiles_n = tn;
  pl.smem = (size_t)stages * stage + 1024;
  pl.ws = split > 1 ? kGemmCounterBytes + (size_t)split * tiles * kBM * bn * 4 : 0;
  return Q4B_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

template <int BN, bool A_MN, bool B_MN>
cudaError_t launch_tc(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, const GemmPlan& pl,
                      cudaStream_t st) {
  auto kern = gemm_f16_tc<BN, A_MN, B_MN>;
  static std::atomic<unsigned long long> done;  // per device: the smem attribute is set once
  const cudaError_t e = set_max_dynamic_smem(kern, kGemmSmemBudget + 1024, done);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(pl.tiles_m, pl.tiles_n, pl.split), dim3(128), pl.smem, st, ta, tb, a, pl.stages);
}

template <int BN, bool A_MN, bool B_MN>
cudaError_t launch_sk(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, const GemmPlan& pl,
                      cudaStream_t st) {
  auto kern = gemm_f16_sk<BN, A_MN, B_MN>;
  static std::atomic<unsigned long long> done;  // per device: the smem attribute is set once
  const cudaError_t e = set_max_dynamic_smem(kern, kGemmSmemBudget + 1024, done);
  if (e != cudaSuccess) return e;
  return launch_pdl(kern, dim3(pl.ctas), dim3(kSkThreads), pl.smem, st, ta, tb, a, pl.stages, pl.nacc);
}

template <int BN>
cudaError_t launch_sk_bn(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                         const GemmPlan& pl, cudaStream_t st) {
  if (!a_mn && !b_mn) return launch_sk<BN, false, false>(ta, tb, a, pl, st);
  if (!a_mn && b_mn) return launch_sk<BN, false, true>(ta, tb, a, pl, st);
  if (a_mn && !b_mn) return launch_sk<BN, true, false>(ta, tb, a, pl, st);
  return launch_sk<BN, true, true>(ta, tb, a, pl, st);
}

template <int BN>
cudaError_t launch_tc_bn(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a,
                         const GemmPlan& pl, cudaStream_t st) {
  if (!a_mn && !b_mn) return launch_tc<BN, false, false>(ta, tb, a, pl, st);
  if (!a_mn && b_mn) return launch_tc<BN, false, true>(ta, tb, a, pl, st);
  if (a_mn && !b_mn) return launch_tc<BN, true, false>(ta, tb, a, pl, st);
  return launch_tc<BN, true, true>(ta, tb, a, pl, st);
}

}  // namespace

int make_tmap_f16(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_rows) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return set_error(Q4B_EUNSUPPORTED, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(Q4B_EINVAL, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return Q4B_OK;
}

int make_tmap_i32(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld, uint32_t box_cols,
                  uint32_t box_rows) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return set_error(Q4B_EUNSUPPORTED, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_INT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(Q4B_EINVAL, "cuTensorMapEncodeTiled (int32) failed (%d)", (int)r);
  return Q4B_OK;
}

unsigned gemm_status(bool reset) {
  unsigned v = 0;
  cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(v));
  if (reset && v) {
    const unsigned zero = 0;
    cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(zero));
  }
  return v;
}

}  // namespace q4b

using namespace q4b;

extern "C" long long q4b_gemm_f16_workspace(int M, int N, int K, char la, char lb, const q4b_gemm_cfg* cfg) {
  GemmPlan pl;
  if (plan_gemm(M, N, K, la, lb, cfg, pl)) return -1;
  return (long long)pl.ws;
}

extern "C" int q4b_gemm_f16_plan(int M, int N, int K, char la, char lb, const q4b_gemm_cfg* cfg, q4b_gemm_cfg* out) {
  if (!out) return set_error(Q4B_EINVAL, "gemm_f16_plan: null output");
  GemmPlan pl;
  const int rc = plan_gemm(M, N, K, la, lb, cfg, pl);
  if (rc) return rc;
  const bool tc = pl.kernel == 1 || pl.kernel == 3;
  *out = {pl.kernel, tc ? pl.bn : 0, tc ? pl.stages : 0, pl.split};
  return Q4B_OK;
}

extern "C" int q4b_gemm_f16(const void* A, const void* B, void* C, int M, int N, int K, char la, char lb,
                            const q4b_gemm_cfg* cfg, void* workspace, size_t ws_bytes, q4b_stream_t stream) {
  clear_error();
  if (!A || !B || !C) return set_error(Q4B_EINVAL, "gemm_f16: null pointer");
  GemmPlan pl;
  int rc = plan_gemm(M, N, K, la, lb, cfg, pl);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  if (pl.kernel == 2) {
    const dim3 grid((N + 63) / 64, (M + 63) / 64);
    const auto* a = static_cast<const __half*>(A);
    const auto* b = static_cast<const __half*>(B);
    auto* c = static_cast<__half*>(C);
    cudaError_t e;
    if (la == 'N' && lb == 'N') e = launch_pdl(gemm_f16_simt<false, false>, grid, dim3(256), 0, st, a, b, c, M, N, K);
    else if (la == 'N') e = launch_pdl(gemm_f16_simt<false, true>, grid, dim3(256), 0, st, a, b, c, M, N, K);
    else if (lb == 'N') e = launch_pdl(gemm_f16_simt<true, false>, grid, dim3(256), 0, st, a, b, c, M, N, K);
    else e = launch_pdl(gemm_f16_simt<true, true>, grid, dim3(256), 0, st, a, b, c, M, N, K);
    if (e != cudaSuccess) return set_error(Q4B_ELAUNCH, "gemm_f16 (cuda cores): %s", cudaGetErrorString(e));
    return Q4B_OK;
  }
  if (!aligned(A, 16) || !aligned(B, 16)) return set_error(Q4B_EINVAL, "gemm_f16: A and B must be 16-byte aligned");
  if (pl.ws && (!workspace || ws_bytes < pl.ws || !aligned(workspace, 256)))
    return set_error(Q4B_EINVAL, "gemm_f16: needs a 256-byte aligned workspace of %zu bytes", pl.ws);
  const bool a_mn = la == 'T', b_mn = lb == 'N';
  CUtensorMap ta, tb;
  if ((rc = a_mn ? make_tmap_f16(&ta, A, M, K, M, 64) : make_tmap_f16(&ta, A, K, M, K, kBM))) return rc;
  if ((rc = b_mn ? make_tmap_f16(&tb, B, N, K, N, 64) : make_tmap_f16(&tb, B, K, N, K, pl.bn))) return rc;
  GemmArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.kt = (K + kBK - 1) / kBK;
  a.split = pl.split;
  a.tm = pl.tiles_m;
  a.tn = pl.tiles_n;
  a.vec = (N % 8 == 0) && aligned(C, 16);
  a.C = static_cast<__half*>(C);
  a.counters = pl.ws ? static_cast<unsigned*>(workspace) : nullptr;
  a.partial = pl.ws ? reinterpret_cast<float*>(static_cast<char*>(workspace) + kGemmCounterBytes) : nullptr;
  cudaError_t e;
  if (pl.kernel == 3)
    e = pl.bn == 256 ? launch_sk_bn<256>(a_mn, b_mn, ta, tb, a, pl, st)
        : pl.bn == 128 ? launch_sk_bn<128>(a_mn, b_mn, ta, tb, a, pl, st)
                       : launch_sk_bn<64>(a_mn, b_mn, ta, tb, a, pl, st);
  else
    e = pl.bn == 256 ? launch_tc_bn<256>(a_mn, b_mn, ta, tb, a, pl, st)
        : pl.bn == 128 ? launch_tc_bn<128>(a_mn, b_mn, ta, tb, a, pl, st)
                       : launch_tc_bn<64>(a_mn, b_mn, ta, tb, a, pl, st);
  if (e != cudaSuccess) return set_error(Q4B_ELAUNCH, "gemm_f16 (tcgen05): %s", cudaGetErrorString(e));
  return Q4B_OK;
}
