// Persistent decode step (one token, batch 1): the whole LlamaQ4.step of scripts/llm/llama_q4.py:
// 199-239 for C = 1 in ONE cooperative launch of one CTA per SM, instead of ~5 launches per layer.
//
// Why: at batch 1 every projection is a weight stream (1.66 GB per token for the 3B shape) and a
// chain of separate kernels pays a launch ramp, a tail and an x-staging round trip per projection.
// Here one producer warp per CTA streams this CTA's share of every projection's weights, in
// consumption order and across layer boundaries, into a shared-memory ring with TMA (never
// waiting for activations), while eight consumer warps follow through the dependency chain:
//
//   per layer  QKV  (RMSNorm of h fused into the x staging; RoPE + fp16 KV-cache write epilogue)
//              ATTN (split-key GQA over the cache: (query row, 128-key chunk) items)
//              WO   (merge of the attention partials fused into the x staging; h += o Wo^T)
//              WGU  (RMSNorm; SwiGLU epilogue into a)
//              WDOWN (h += a Wdown^T)
//   then       LM   (final RMSNorm; lm_head rows with the greedy argmax; the last CTA publishes)
//
// Stages are ordered by one arrival counter in global memory: a CTA adds 1 when it has written
// its part of a stage (after a gpu-scope fence); a stage starts once the counter reaches
// stage x CTAs. Every wait (ring slots, the counter) is bounded by %globaltimer (1 s); a wait that
// gives up raises an abort flag that every other wait also checks, the step reports Q4B_ETIMEOUT
// through the state, and the kernel returns.
//
// The arithmetic per 128-k group: q|k|v, o and down as q4_linear.cu's kernel 1 (exact fp16 (nib - 8)
// by LOP3, m16n8k16 with fp32 accumulation, x as fp16 hi + lo, one fmaf with the group scale);
// gate|up and the lm_head as the int8 form of the ring GEMV (kernel 6: biased nibbles as unsigned
// bytes in m16n8k32 MMAs against x as three int8 terms per group, zero point exact). The int8 form
// streams ~1.5x faster per slot but quantising x costs warp reductions on a stage transition's
// critical path, which pays off only for the two projections with the most weight bytes per staged x.
// Results match the per-projection path within the x-term residual (~6e-8 of a group's largest |x|)
// and fp32 summation order.
//
// Ring slots hold 32 weight rows x 1024 k (two 16-row MMA tiles per warp and slot): one 32-row TMA
// box streams at about twice the rate of a 16-row one, and two tiles per warp give the consumers
// two independent MMA chains. q|k|v items stay 16 rows (RoPE row pairs; 320 tiles balance over the
// SMs far better than 160).
#include <cuda.h>

#include <algorithm>
#include <cstddef>
#include <cstdlib>
#include <mutex>

#include "fused.h"
#include "model.h"
#include "q4dev.cuh"
#include "tc.cuh"

namespace q4b {

namespace {

constexpr int MK_CW = 8;                       // consumer warps
constexpr int MK_THREADS = (MK_CW + 1) * 32;   // + one producer warp (warp 0)
constexpr int MK_UK = 1024;                    // k per weight unit
constexpr int MK_SROWS = 32;                   // weight rows per ring slot
constexpr int MK_WBYTES = MK_SROWS * MK_UK / 2;  // 32 rows x 512 B of int4
constexpr int MK_SLOT = MK_WBYTES + MK_SROWS * 16;  // + 32 rows x 8 fp16 scales = 16896 B (132 x 128)
constexpr int MK_NSLOT = 10;                   // ring slots allocated at most (Q4B_MK_SLOTS)
constexpr int kMkDefaultSlots = 6;
constexpr int MK_MAXK = 8192;
constexpr int MK_XROW = MK_MAXK / 8 + 4;       // staged x: uint4 per 8-k word (+64 B, as kernel 1)
constexpr int MK_HD = 128;
static_assert(MK_HD <= MK_CW * 32, "one query element per consumer thread");
constexpr int MK_KCHUNK = 128;                 // keys per attention item (8 warps x 16)
constexpr int MK_MAXCH = 128;                  // attention chunks (contexts up to 16384)
constexpr int MK_ROWS = 4;                     // query rows per KV head (GQA group) at most
constexpr int MK_TB = 8;                       // tiles of one stage per batched epilogue
constexpr int MK_MAXKS = 4;                    // K splits of the o / down projections
constexpr int MK_MAXTP = 8;
constexpr int MK_MAXL = 128;                   // layers                    // tensor-parallel ranks
constexpr int MK_MAXD = 4096;                  // hidden size: at most two staged words per thread
constexpr int MK_PAD = 4;                      // partial row: m, l and two pad floats before o (16-B aligned)

enum { ST_QKV = 0, ST_ATTN = 1, ST_WO = 2, ST_WGU = 3, ST_WDOWN = 4, ST_PER_LAYER = 5 };

// Per projection: weight and scale tensor maps (global memory), rows per tile pairing, geometry.
struct MkProj {
  CUtensorMap w;   // int32 [n, k/8], box {128 words, 16 or 8 rows}
  CUtensorMap s;   // fp16 [n, k/G], box {8 groups, 16 or 8 rows}
};

struct MkArgs {
  const MkProj* proj;  // [layers * 4 + 1]: qkv, o, gu, down per layer, then the lm_head
  const q4b_layer_weights* layers;
  int n_layers;
  const int32_t* emb_qw;
  const __half* emb_s;
  const float* ln_f;
  const float* rope_cos;
  const float* rope_sin;
  int D, H, Hkv, hd, I, V;
  float eps, scale;
  int L;
  const int32_t* token;
  DecodeState* state;
  int32_t* token_log;
  float* logits;
  float* hb;     // [2][D] residual stream, ping-pong: QKV staging writes hb[1], WGU staging hb[0]
  float* psum;   // [2][tp * MK_MAXKS][D] partial sums of the o (buffer 0) / down (buffer 1) projections
  float* q;      // [H * hd]
  float* a;      // [I]
  float* part;   // attention partials [Hkv][MK_MAXCH][MK_ROWS][hd + 4]: m, l, -, -, o[hd]
  unsigned* rowcnt;  // [H] chunks of each query row done in this layer (the last one merges)
  float* attn_out;   // [H * hd] the attention output (the o projection's x)
  // [0] local stage arrivals, [1] abort (both zeroed per launch); [4] lm key arrivals of every rank,
  // [5] step epoch, [6] poison (an earlier step timed out) -- never reset by a launch
  unsigned* sync;
  // tensor parallelism: this rank of tp; the peers' psum / sync / key buffers (peer memory mapped
  // into this process; index rank = this GPU's own)
  int tp, rank, Vfull;
  float* peer_psum[MK_MAXTP];
  unsigned* peer_sync[MK_MAXTP];
  unsigned long long* peer_keys[MK_MAXTP];
  unsigned long long* keys;  // [tp] this rank's copy of every rank's best argmax key
  // limit of every wait: 1 s on one GPU; longer with peers, whose launches may start later
  unsigned long long wait_ns;
  // phase trace (null = off): per CTA mk_trace_stride(n_layers) %globaltimer stamps, see trace_ev
  unsigned long long* trace;
  // ring slots in use (<= MK_NSLOT): fewer slots bound how far the weight stream runs ahead of the
  // consumers, and with it the traffic queued ahead of a stage transition's latency-bound loads
  int nslot;
  // how a norm learns that the o / down partial sums of every CTA (and rank) are complete:
  // 0 = every thread polls its words' layer-parity tags; 1 = one thread per CTA waits on the
  // row-split arrival counter (sync[7]) and the words are then loaded once
  int split_sync;
  // 1: the o projection's weights are requested only once the layer's attention is over (see
  // producer_gate); 0: right after the q|k|v weights, during attention
  int gate_o;
};

// Trace events of a CTA: per layer l and stage s (0 q|k|v, 1 attention, 2 o, 3 gate|up, 4 down),
// 15 l + 3 s + {0: inputs ready (barrier passed / partial sums loaded), 1: x staged, 2: done}; then
// 15 L + {0: lm_head inputs ready, 1: staged, 2: done, 3: consumers start}.
__device__ __forceinline__ void trace_ev(const MkArgs& a, int e) {
  if (a.trace && e >= 0 && threadIdx.x == 32)
    a.trace[(size_t)blockIdx.x * mk_trace_stride(a.n_layers) + e] = globaltimer_ns();
}

// Attention scratch of one item (row 0 for a one-row item, rows 0 .. g - 1 for a long-context item
// of a KV head's group); shares shared memory with the staged x, which is free between the q|k|v
// projection (its last reads end before the stage arrival) and the o projection's staging.
struct MkAttn {
  float q[MK_ROWS][MK_HD];
  float o[MK_CW][MK_ROWS][MK_HD];
  float m[MK_CW][MK_ROWS], l[MK_CW][MK_ROWS], cs[MK_CW][MK_ROWS];
};
struct MkX {
  uint4 hi[MK_XROW];  // word w of x as fp16 hi / lo pairs at xswz(w)
  uint4 lo[MK_XROW];
};
// int8 form of a normed x (gate|up, lm_head: K = D): three terms as {even, odd} byte words per 8-k
// word, rows 2 words (16 B = 4 banks) longer than D / 8 so the terms' rows fall on different banks
constexpr int MK_QSTRIDE = MK_MAXD / 8 + 2;
struct MkXq {
  uint2 q[3 * MK_QSTRIDE];  // term m of word w at q[m * MK_QSTRIDE + w]
  int4 g[MK_MAXD / 128];    // per 128-k group: {X_a, X_b, X_c, sx bits}
};

struct MkSmem {
  union {
    MkX x;
    MkXq xq;
    MkAttn att;
  } u;
  float red[MK_TB][MK_CW][MK_SROWS];  // per-warp partial sums of up to MK_TB items of one stage
  float scratch[64];
  float rope_c[MK_HD], rope_s[MK_HD];  // RoPE rows of this step's position
  unsigned long long best[MK_CW];
  // per layer: KV cache and norm weight pointers (read once at kernel start, not chased through
  // the layer table in global memory at every use)
  __half* kcache[MK_MAXL];
  __half* vcache[MK_MAXL];
  const float* ln_in[MK_MAXL];
  const float* ln_post[MK_MAXL];
  uint64_t full[MK_NSLOT], empty[MK_NSLOT];
  int abort_flag;
  unsigned tagbase;  // epoch * n_layers: partial sums of layer l carry parity (tagbase + l) & 1
  int last;
  int att_last;
  // last: a launch allocates only the slots it uses (MkArgs::nslot), leaving the rest of the SM's
  // 256 KB of L1 + shared memory to the L1 cache
  alignas(1024) uint8_t ring[MK_NSLOT][MK_SLOT];
};
// dynamic shared memory of a launch with `nslot` ring slots (+1 KB for the 1024-byte alignment)
static size_t mk_smem_bytes(int nslot) { return offsetof(MkSmem, ring) + (size_t)nslot * MK_SLOT + 1024; }

// dynamic shared memory of the kernel (+1 KB for the 1024-byte alignment) within the 227 KB an SM
// gives one CTA
static_assert(sizeof(MkSmem) + 1024 <= 227 * 1024, "persistent decode: shared memory over 227 KB");

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(MK_CW * 32) : "memory"); }
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t n) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(n) : "memory");
}

// Sum over the consumer threads (256); every consumer thread gets the total.
__device__ float consumer_sum(float v, float* scratch) {
  const int ct = threadIdx.x - 32, w = ct >> 5, lane = ct & 31;
  v = warp_sum(v);
  if (lane == 0) scratch[w] = v;
  consumer_sync();
  float t = 0.0f;
#pragma unroll
  for (int i = 0; i < MK_CW; ++i) t += scratch[i];
  consumer_sync();
  return t;
}

// Abort of the step: every wait of every rank sees the flag; the model is poisoned (sync[6], never
// reset by a launch): partial sums of the failed step may carry the tags the retry would accept, so
// later launches do no work and report the failure until the host prepares the model again.
__device__ void raise_abort(const MkArgs& a, MkSmem& sm) {
  sm.abort_flag = 1;
  for (int r = 0; r < a.tp; ++r) {
    atomicExch_system(a.peer_sync[r] + 1, 1u);
    atomicExch_system(a.peer_sync[r] + 6, 1u);
  }
  a.state->status = 1;
}

// Stage-start wait (first consumer thread spins, bounded; then the consumer warps sync).
__device__ bool stage_wait(const MkArgs& a, MkSmem& sm, unsigned target) {
  if (threadIdx.x == 32) {
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
      // sync[0] (arrivals) and sync[1] (abort) in one acquire load
      unsigned long long both;
      asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(both) : "l"(a.sync) : "memory");
      if ((unsigned)both >= target) break;
      if (both >> 32) {
        sm.abort_flag = 1;
        break;
      }
      if (globaltimer_ns() - t0 > a.wait_ns) {
        raise_abort(a, sm);
        break;
      }
    }
  }
  consumer_sync();
  return !sm.abort_flag;
}
// Row-split completion (split_sync 1): this CTA's o / down partial sums, stored to every rank, happen
// before one release add on every rank's counter sync[7] (never reset: targets grow by the step epoch).
__device__ void split_arrive(const MkArgs& a) {
  if (a.split_sync != 1) return;
  consumer_sync();
  if (threadIdx.x == 32) {
    if (a.tp > 1) {
      for (int r = 0; r < a.tp; ++r)
        asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(a.peer_sync[r] + 7) : "memory");
    } else {
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.sync + 7) : "memory");
    }
  }
}

// Stage-end arrival: all consumer writes of this stage happen before the gpu-scope release.
__device__ void stage_arrive(const MkArgs& a) {
  consumer_sync();
  if (threadIdx.x == 32)  // release: cumulative over the CTA's writes ordered by the barrier above
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(a.sync) : "memory");
}

// The o / down partial sums carry their layer's parity in the lowest mantissa bit (one ulp, far
// below the 1e-3 tolerance of the path): the next norm's staging polls the partials themselves until
// every word it needs shows the parity of the layer it expects, on this GPU or pushed by a peer, so no
// grid-wide (or cross-GPU) barrier separates a row-split projection from the next RMSNorm. A slot is
// rewritten once per layer and every CTA reads every slot before it can write the next layer's value
// (each needs all the previous partials first), so one bit tells the two candidates apart.
__device__ __forceinline__ float tag_value(float v, unsigned tag) {
  return __uint_as_float((__float_as_uint(v) & ~1u) | tag);
}
__device__ __forceinline__ bool tags_match(const float4& q, unsigned tag) {
  return ((__float_as_uint(q.x) & __float_as_uint(q.y) & __float_as_uint(q.z) & __float_as_uint(q.w) & 1u) == tag) &&
         (((__float_as_uint(q.x) | __float_as_uint(q.y) | __float_as_uint(q.z) | __float_as_uint(q.w)) & 1u) == tag);
}
// Loads that must see other SMs' (and, with peers, other GPUs') recent stores: L2, not L1.
__device__ __forceinline__ float4 ld_fresh4(const float* p, bool sys) {
  float4 v;
  if (sys)
    asm volatile("ld.relaxed.sys.global.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
  else
    asm volatile("ld.relaxed.gpu.global.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p)
                 : "memory");
  return v;
}

// Projection of a stage: item geometry. An item is a run of rows (16 or 32) over a range of 1024-k
// units; each unit of an item is one ring slot.
struct ProjGeo {
  int K, RT, NU;  // reduction dim, row items, 1024-k units per item
  bool paired;    // two runs of rows per item (SwiGLU gate | up, RoPE element halves)
  int KS;         // K splits: work items are (row item, unit range); partial sums go to psum
  int rows;       // weight rows per item: 16 (one MMA tile) or 32 (two)
};
__host__ __device__ __forceinline__ int k_splits(int nu) {
  for (int k = MK_MAXKS; k > 1; --k)
    if (nu % k == 0) return k;
  return 1;
}
// The o / down projections have D / 32 row items (96 for the 3B shape), too few to balance over
// the SMs; splitting their K gives several smaller items per CTA. Their partial sums are added to
// the residual stream in fixed order by the next stage's x staging.
__device__ __forceinline__ ProjGeo geo(const MkArgs& a, int st) {
  switch (st) {
    case ST_QKV: return {a.D, (a.H + 2 * a.Hkv) * a.hd / 16, a.D / MK_UK, true, 1, 16};
    case ST_WO: {
      const int nu = (a.H * a.hd + MK_UK - 1) / MK_UK;  // a TP shard may end inside a unit: zero-filled
      return {a.H * a.hd, a.D / 32, nu, false, k_splits(nu), 32};
    }
    case ST_WGU: return {a.D, a.I / 16, a.D / MK_UK, true, 1, 32};
    case ST_WDOWN: {
      const int nu = (a.I + MK_UK - 1) / MK_UK;
      return {a.I, a.D / 32, nu, false, k_splits(nu), 32};
    }
    default: return {a.D, a.V / 32, a.D / MK_UK, false, 1, 32};  // lm_head
  }
}
// first weight row of run b (0 / 1) of a paired item: gate | up rows [16 rt, 16 rt + 16) (slot rows
// 0..15 / 16..31), or the RoPE halves e = 8 j .. 8 j + 7 and e + hd / 2 of a head (slot rows 0..7 / 8..15)
__device__ __forceinline__ int pair_row(const MkArgs& a, int st, int rt, int b) {
  if (st == ST_WGU) return (b ? a.I : 0) + rt * 16;
  const int per = a.hd / 16, head = rt / per, j = rt - head * per;  // RoPE
  return head * a.hd + b * (a.hd / 2) + 8 * j;
}

// ---- producer --------------------------------------------------------------------------------

__device__ bool produce_stage(const MkArgs& a, MkSmem& sm, const MkProj& pj, int st, unsigned& seq) {
  const ProjGeo gp = geo(a, st);
  tma_prefetch_map(&pj.w);
  tma_prefetch_map(&pj.s);
  const int upi = gp.NU / gp.KS;  // units per item
  const int half = gp.rows / 2;   // rows of one run of a paired item
  const uint64_t pol = l2_policy_evict_first();  // weights are read once per token
  for (int it = blockIdx.x; it < gp.RT * gp.KS; it += gridDim.x) {
    const int rt = it / gp.KS, ks = it - rt * gp.KS;
    for (int u = ks * upi; u < (ks + 1) * upi; ++u, ++seq) {
      const int slot = seq % a.nslot, round = seq / a.nslot;
      if (round > 0 && !mbar_wait_bounded(&sm.empty[slot], (round - 1) & 1, a.wait_ns)) return false;
      if (sm.abort_flag) return false;
      uint8_t* dst = sm.ring[slot];
      mbar_arrive_expect_tx(&sm.full[slot], gp.rows * (MK_UK / 2 + 16));
      if (gp.paired) {
        const int r0 = pair_row(a, st, rt, 0), r1 = pair_row(a, st, rt, 1);
        tma_load_2d_hint(dst, &pj.w, u * (MK_UK / 8), r0, &sm.full[slot], pol);
        tma_load_2d_hint(dst + half * (MK_UK / 2), &pj.w, u * (MK_UK / 8), r1, &sm.full[slot], pol);
        tma_load_2d_hint(dst + MK_WBYTES, &pj.s, u * 4, r0, &sm.full[slot], pol);
        tma_load_2d_hint(dst + MK_WBYTES + half * 16, &pj.s, u * 4, r1, &sm.full[slot], pol);
      } else {
        tma_load_2d_hint(dst, &pj.w, u * (MK_UK / 8), rt * gp.rows, &sm.full[slot], pol);
        tma_load_2d_hint(dst + MK_WBYTES, &pj.s, u * 4, rt * gp.rows, &sm.full[slot], pol);
      }
    }
  }
  return true;
}

// The o projection's weights are requested once the layer's attention stage is over: attention is a
// few dependent KV-cache loads per item, and a weight stream requested at the same moment (a full
// ring on every SM) queues ahead of them in HBM. The o weights (a sixth of a layer) then stream in
// while the attention output is merged.
__device__ bool producer_gate(const MkArgs& a, MkSmem& sm, unsigned target) {
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire(&a.sync[0]) < target) {
    __nanosleep(64);
    if (sm.abort_flag || ld_acquire(&a.sync[1])) return false;
    if (globaltimer_ns() - t0 > a.wait_ns) return false;
  }
  return true;
}

// ---- consumers: x staging --------------------------------------------------------------------

// x[8 w .. 8 w + 7] (fp32) -> hi / lo fp16 pairs of word w in the permuted order of dequant_word
// (x = hi + lo to ~22 bits; mma_tile_hl takes hi and lo as two columns of one MMA)
__device__ __forceinline__ void stage_word(MkSmem& sm, int w, const float (&v)[8]) {
  uint4 hi, lo;
  split_pair(v[0], v[4], hi.x, lo.x);
  split_pair(v[1], v[5], hi.y, lo.y);
  split_pair(v[2], v[6], hi.z, lo.z);
  split_pair(v[3], v[7], hi.w, lo.w);
  sm.u.x.hi[xswz(w)] = hi;
  sm.u.x.lo[xswz(w)] = lo;
}

// Rounding to the nearest integer (ties to even) by adding 1.5 * 2^23: for |u| < 2^22 the sum's low
// mantissa bits hold round(u) in two's complement, so its low byte is the int8 byte of round(u) and
// (sum bits - 0x4B400000) is round(u) as an int; sum - 1.5 * 2^23 is round(u) as a float.
constexpr float kRoundMagic = 12582912.0f;
constexpr uint32_t kRoundBits = 0x4B400000u;

// x[8 w .. 8 w + 7] (fp32) -> word w of the int8 form (MkXq): x ~= sx (a + b / 254 + c / 254^2) per
// 128-k group with sx = max |x| / 127, the form of q4dev.cuh's mma_tile_i8. A group is 16 words held
// by the 16 lanes of a half warp (the whole warp calls this together), whose shuffles give the
// group's max |x| and term sums X. Byte i of the even word is k = 8 w + 2 i, of the odd word
// k = 8 w + 2 i + 1 (the nibble order of the weights' byte masks).
__device__ __forceinline__ void stage_word_i8(MkSmem& sm, int w, const float (&v)[8]) {
  float am = 0.0f;
#pragma unroll
  for (int b = 0; b < 8; ++b) am = fmaxf(am, fabsf(v[b]));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  const float sx = am > 0.0f ? am / 127.0f : 1.0f;
  const float inv = am > 0.0f ? 127.0f / am : 1.0f;
  uint32_t f[3][8];              // bit patterns of round(.) + magic: low byte = the int8 term
  uint32_t pab = 0u, pc = 0u;    // this word's term sums: a + 65536 b (fields recovered below), c
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float u = fminf(fmaxf(v[i] * inv, -127.0f), 127.0f);
    const float ra = __fadd_rn(u, kRoundMagic);
    const float r = (u - __fsub_rn(ra, kRoundMagic)) * 254.0f;
    const float rb = __fadd_rn(r, kRoundMagic);
    const float rc = __fadd_rn((r - __fsub_rn(rb, kRoundMagic)) * 254.0f, kRoundMagic);
    f[0][i] = __float_as_uint(ra), f[1][i] = __float_as_uint(rb), f[2][i] = __float_as_uint(rc);
    pab += (f[0][i] - kRoundBits) + (f[1][i] - kRoundBits) * 65536u;  // mod 2^32
    pc += f[2][i] - kRoundBits;
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) {
    pab += __shfl_xor_sync(0xffffffffu, pab, o);
    pc += __shfl_xor_sync(0xffffffffu, pc, o);
  }
  // |group sums| <= 128 * 127 < 2^15: the low field of the packed a | b sum is exact as int16
  const int Xa = (int)(short)(pab & 0xFFFFu);
  const int Xb = ((int)pab - Xa) >> 16;
#pragma unroll
  for (int m = 0; m < 3; ++m) {
    const uint32_t ev = __byte_perm(__byte_perm(f[m][0], f[m][2], 0x0040), __byte_perm(f[m][4], f[m][6], 0x0040), 0x5410);
    const uint32_t od = __byte_perm(__byte_perm(f[m][1], f[m][3], 0x0040), __byte_perm(f[m][5], f[m][7], 0x0040), 0x5410);
    sm.u.xq.q[m * MK_QSTRIDE + w] = make_uint2(ev, od);
  }
  if ((threadIdx.x & 15) == 0) sm.u.xq.g[w >> 4] = make_int4(Xa, Xb, (int)pc, __float_as_int(sx));
}

// The residual stream before a norm at word w: the first layer's h is the embedding row of the token
// (QEmbedding.lookup, llama_q4.py:106-119); later it is h + the K-split partial sums of the o / down
// projection of every rank (added in rank, then split order). Returns whether every partial carries
// the expected layer-parity tag.
__device__ __forceinline__ bool norm_src(const MkArgs& a, int w, bool embed, int token, const float* hsrc,
                                         const float* psrc, int nparts, unsigned tag, float (&v)[8]) {
  if (embed) {
    const int words = a.D / 8;
    const bool ok = token >= 0 && token < a.Vfull;
    const int32_t word = ok ? a.emb_qw[(size_t)token * words + w] : 0;
    const float s = ok ? __half2float(a.emb_s[(size_t)token * (a.D / 128) + (8 * w) / 128]) : 0.0f;
#pragma unroll
    for (int b = 0; b < 8; ++b) v[b] = (float)(((word >> (4 * b)) & 15) - 8) * s;
    return true;
  }
  const float4 p0 = __ldcg(reinterpret_cast<const float4*>(hsrc + 8 * w));
  const float4 p1 = __ldcg(reinterpret_cast<const float4*>(hsrc + 8 * w) + 1);
  v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
  v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
  float d[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  bool fresh = true;
  const bool sys = a.tp > 1;
  for (int r = 0; r < a.tp; ++r) {  // every rank's partials, rank order then split order
    const float* pr = psrc + (size_t)r * MK_MAXKS * a.D + 8 * w;
    float4 q0[MK_MAXKS], q1[MK_MAXKS];
#pragma unroll
    for (int k = 0; k < MK_MAXKS; ++k) {
      if (k < nparts) {
        q0[k] = ld_fresh4(pr + (size_t)k * a.D, sys);
        q1[k] = ld_fresh4(pr + (size_t)k * a.D + 4, sys);
      }
    }
#pragma unroll
    for (int k = 0; k < MK_MAXKS; ++k) {
      if (k < nparts) {
        fresh = fresh && tags_match(q0[k], tag) && tags_match(q1[k], tag);
        d[0] += q0[k].x; d[1] += q0[k].y; d[2] += q0[k].z; d[3] += q0[k].w;
        d[4] += q1[k].x; d[5] += q1[k].y; d[6] += q1[k].z; d[7] += q1[k].w;
      }
    }
  }
#pragma unroll
  for (int b = 0; b < 8; ++b) v[b] += d[b];
  return fresh;
}

// This thread's (at most two) words of a norm weight: loaded before the stage's data arrives.
__device__ __forceinline__ void norm_weights(const MkArgs& a, const float* lnw, float (&lw)[2][8]) {
  const int ct = threadIdx.x - 32;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int w = ct + i * (MK_CW * 32);
    if (w < a.D / 8) {
      const float4 w0 = *reinterpret_cast<const float4*>(lnw + 8 * w);
      const float4 w1 = *reinterpret_cast<const float4*>(lnw + 8 * w + 4);
      lw[i][0] = w0.x; lw[i][1] = w0.y; lw[i][2] = w0.z; lw[i][3] = w0.w;
      lw[i][4] = w1.x; lw[i][5] = w1.y; lw[i][6] = w1.z; lw[i][7] = w1.w;
    }
  }
}

// x = rmsnorm(h + partials) * w (rms_norm, llama_q4.py:141-142). With hdst the updated residual
// stream is also written (each word by one CTA) to the other ping-pong buffer. Each thread reloads
// its words until their partial sums carry the expected tag (bounded; a timeout aborts the step), or
// with split_sync 1 loads them once after the row-split counter reached split_target.
__device__ void stage_norm(const MkArgs& a, MkSmem& sm, const float (&lw)[2][8], bool embed, int token,
                           const float* hsrc, const float* psrc, int nparts, unsigned tag, float* hdst,
                           unsigned split_target, int ev_ready, bool i8) {
  const int ct = threadIdx.x - 32;
  const int words = a.D / 8;
  float v[2][8];
  float ss = 0.0f;
  uint64_t t0 = 0;
  const bool counted = a.split_sync == 1 && !embed;
  if (counted) {  // every CTA of every rank has stored its partial sums: then one round of loads
    if (threadIdx.x == 32) {
      t0 = globaltimer_ns();
      for (;;) {
        unsigned c;
        if (a.tp > 1)
          asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(c) : "l"(a.sync + 7) : "memory");
        else
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(c) : "l"(a.sync + 7) : "memory");
        if ((int)(c - split_target) >= 0) break;
        if (globaltimer_ns() - t0 > a.wait_ns || *(volatile unsigned*)&a.sync[1]) {
          raise_abort(a, sm);
          break;
        }
      }
    }
    consumer_sync();
  }
  for (int tries = 0;; ++tries) {
    bool fresh = true;
#pragma unroll
    for (int i = 0; i < 2; ++i) {  // one round: every load before any store
      const int w = ct + i * (MK_CW * 32);
      if (w < words) fresh = norm_src(a, w, embed, token, hsrc, psrc, nparts, tag, v[i]) && fresh;
    }
    if (fresh || counted) break;
    if (tries == 0) t0 = globaltimer_ns();
    if (globaltimer_ns() - t0 > a.wait_ns || *(volatile unsigned*)&a.sync[1]) {
      raise_abort(a, sm);
      break;
    }
  }
  trace_ev(a, ev_ready);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int w = ct + i * (MK_CW * 32);
    if (w < words) {
#pragma unroll
      for (int b = 0; b < 8; ++b) ss += v[i][b] * v[i][b];
      if (hdst && w % (int)gridDim.x == (int)blockIdx.x) {
        float4* hp = reinterpret_cast<float4*>(hdst + 8 * w);
        hp[0] = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
        hp[1] = make_float4(v[i][4], v[i][5], v[i][6], v[i][7]);
      }
    }
  }
  const float tot = consumer_sum(ss, sm.scratch);
  const float rs = 1.0f / sqrtf(tot / (float)a.D + a.eps);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int w = ct + i * (MK_CW * 32);
    if (w < words) {
      float x[8];
#pragma unroll
      for (int b = 0; b < 8; ++b) x[b] = v[i][b] * rs * lw[i][b];
      if (i8)  // (w < words is uniform over each warp: D / 8 is a multiple of 32)
        stage_word_i8(sm, w, x);
      else
        stage_word(sm, w, x);
    }
  }
}

// x = src[0, K) plain (the attention output, the SwiGLU output), zeros up to the next 1024-k unit (a
// tensor-parallel shard may end inside one; its weights and scales there are zero-filled).
__device__ void stage_plain(const MkArgs& a, MkSmem& sm, const float* src, int K) {
  constexpr int kPer = MK_MAXK / 8 / (MK_CW * 32);  // words per thread at most
  const int ct = threadIdx.x - 32;
  const int words = K / 8, padded = (K + MK_UK - 1) / MK_UK * (MK_UK / 8);
  float4 p[kPer][2];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {  // one round: every load before any conversion
    const int w = ct + i * (MK_CW * 32);
    p[i][0] = p[i][1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (w < words) {
      p[i][0] = __ldcg(reinterpret_cast<const float4*>(src + 8 * w));
      p[i][1] = __ldcg(reinterpret_cast<const float4*>(src + 8 * w) + 1);
    }
  }
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int w = ct + i * (MK_CW * 32);
    if (w < padded) {
      const float v[8] = {p[i][0].x, p[i][0].y, p[i][0].z, p[i][0].w, p[i][1].x, p[i][1].y, p[i][1].z, p[i][1].w};
      stage_word(sm, w, v);
    }
  }
}


// ---- consumers: projections ------------------------------------------------------------------

// Epilogue of output s of an item. q|k|v (16 rows): v0 / v1 = rows s / s + 8 (RoPE halves e, e + hd/2);
// gate|up (32 rows): v0 / v1 = rows s / s + 16 (gate, up); o / down: v0 = row s of the item's 32.
__device__ void item_epilogue(const MkArgs& a, MkSmem& sm, int st, int layer, int rt, int ks, int s, float v0,
                              float v1, int pos) {
  if (st == ST_QKV) {
    const int per = a.hd / 16, head = rt / per, jj = rt - head * per;
    const int e1 = jj * 8 + s, e2 = a.hd / 2 + jj * 8 + s;
    if (head < a.H + a.Hkv) {
      // q * cos + rotate_half(q) * sin, rotate_half(x) = cat(-x[h:], x[:h]) (llama_q4.py:195-221)
      const float o1 = __fadd_rn(__fmul_rn(v0, sm.rope_c[e1]), __fmul_rn(-v1, sm.rope_s[e1]));
      const float o2 = __fadd_rn(__fmul_rn(v1, sm.rope_c[e2]), __fmul_rn(v0, sm.rope_s[e2]));
      if (head < a.H) {
        a.q[head * a.hd + e1] = o1;
        a.q[head * a.hd + e2] = o2;
      } else {
        __half* kc = sm.kcache[layer] + ((size_t)pos * a.Hkv + (head - a.H)) * a.hd;
        kc[e1] = __float2half_rn(o1);
        kc[e2] = __float2half_rn(o2);
      }
    } else {
      __half* vc = sm.vcache[layer] + ((size_t)pos * a.Hkv + (head - a.H - a.Hkv)) * a.hd;
      vc[e1] = __float2half_rn(v0);
      vc[e2] = __float2half_rn(v1);
    }
  } else if (st == ST_WGU) {
    a.a[rt * 16 + s] = silu(v0) * v1;
  } else {  // WO / WDOWN: this rank's K-split partial sums, pushed to every rank (added to h there by
            // the next norm's staging, in rank and split order)
    const size_t off = ((size_t)(st == ST_WDOWN) * a.tp * MK_MAXKS + (size_t)a.rank * MK_MAXKS + ks) * a.D + rt * 32;
    const float tv = tag_value(v0, (sm.tagbase + (unsigned)layer) & 1u);
    for (int r = 0; r < a.tp; ++r) a.peer_psum[r][off + s] = tv;
  }
}

// K split across the consumer warps: warp w takes the 128-k group w of every 1024-k unit of an item
// (a run of 16 or 32 rows and a range of its units); per slot it loads its share of the NT 16-row
// tiles into registers, releases the slot and runs NT independent MMA chains. The per-warp sums of
// up to MK_TB items are reduced and finished together (one barrier pair per batch); `fin(j, it, s, v0,
// v1)` finishes output s of the batch's item j (item index it).
template <int NT, bool I8, typename Fin>
__device__ bool consume_items(const MkArgs& a, MkSmem& sm, const ProjGeo& gp, unsigned& seq, Fin fin) {
  const int ct = threadIdx.x - 32, w = ct >> 5, lane = ct & 31;
  const int g = lane >> 2, t = lane & 3;
  const int upi = gp.NU / gp.KS;
  const int nitems = gp.RT * gp.KS;
  const int nmine = nitems > (int)blockIdx.x ? (nitems - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  // outputs per item and the row distance of a paired output's second value
  const int nout = gp.paired ? gp.rows / 2 : gp.rows, pair = gp.rows / 2;
  unsigned slot = seq % a.nslot, round = seq / a.nslot;  // advanced with seq (no division per slot)
  for (int b0 = 0; b0 < nmine; b0 += MK_TB) {
    const int nb = min(MK_TB, nmine - b0);
    for (int j = 0; j < nb; ++j) {
      const int it = blockIdx.x + (b0 + j) * gridDim.x;
      const int ks = it % gp.KS;
      float acc[NT][4];
#pragma unroll
      for (int jj = 0; jj < NT; ++jj) acc[jj][0] = acc[jj][1] = acc[jj][2] = acc[jj][3] = 0.0f;
      for (int u = ks * upi; u < (ks + 1) * upi; ++u, ++seq) {
        if (!mbar_wait_bounded(&sm.full[slot], round & 1, a.wait_ns)) {
          sm.abort_flag = 1;
          return false;
        }
        const uint8_t* sl = sm.ring[slot];
        const __half* sc = reinterpret_cast<const __half*>(sl + MK_WBYTES);
        uint4 wa[NT], wb[NT];
        float sa[NT], sb[NT];
#pragma unroll
        for (int jj = 0; jj < NT; ++jj) {
          wa[jj] = *reinterpret_cast<const uint4*>(sl + (16 * jj + g) * 512 + w * 64 + t * 16);
          wb[jj] = *reinterpret_cast<const uint4*>(sl + (16 * jj + g + 8) * 512 + w * 64 + t * 16);
          sa[jj] = __half2float(sc[(16 * jj + g) * 8 + w]);
          sb[jj] = __half2float(sc[(16 * jj + g + 8) * 8 + w]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_cnt(&sm.empty[slot], 1);
        if constexpr (I8) {
          const int ktile = u * 8 + w;  // 128-k group = scale group
          uint2 xv[4];
          if (g < 3) {
            const uint4* src = reinterpret_cast<const uint4*>(sm.u.xq.q + g * MK_QSTRIDE + ktile * 16 + 4 * t);
            const uint4 lo = src[0], hi = src[1];
            xv[0] = make_uint2(lo.x, lo.y), xv[1] = make_uint2(lo.z, lo.w);
            xv[2] = make_uint2(hi.x, hi.y), xv[3] = make_uint2(hi.z, hi.w);
          } else {
            xv[0] = xv[1] = xv[2] = xv[3] = make_uint2(0u, 0u);
          }
          const int4 xg = sm.u.xq.g[ktile];
#pragma unroll
          for (int jj = 0; jj < NT; ++jj) {
            float hl[2] = {0.0f, 0.0f};
            mma_tile_i8(wa[jj], wb[jj], sa[jj], sb[jj], xv, xg, hl);
            acc[jj][0] += hl[0];  // rows g / g + 8 (lanes t == 0); columns 1 / 3 stay zero
            acc[jj][2] += hl[1];
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < NT; ++jj)
            mma_tile_hl(wa[jj], wb[jj], sa[jj], sb[jj], sm.u.x.hi, sm.u.x.lo, g, u * 128 + w * 16 + 4 * t, acc[jj]);
        }
        if (++slot == (unsigned)a.nslot) slot = 0, ++round;
      }
      if (t == 0) {  // columns 0 / 1: the x_hi / x_lo products of rows g and g + 8 of each tile
#pragma unroll
        for (int jj = 0; jj < NT; ++jj) {
          sm.red[j][w][16 * jj + g] = acc[jj][0] + acc[jj][1];
          sm.red[j][w][16 * jj + g + 8] = acc[jj][2] + acc[jj][3];
        }
      }
    }
    consumer_sync();
    for (int i = ct; i < nb * nout; i += MK_CW * 32) {
      const int j = i / nout, sl = i - j * nout;
      float v0 = 0.0f, v1 = 0.0f;
#pragma unroll
      for (int k = 0; k < MK_CW; ++k) {
        v0 += sm.red[j][k][sl];
        if (gp.paired) v1 += sm.red[j][k][sl + pair];
      }
      fin(j, blockIdx.x + (b0 + j) * gridDim.x, sl, v0, v1);
    }
    consumer_sync();
  }
  return true;
}

__device__ bool consume_stage(const MkArgs& a, MkSmem& sm, int st, int layer, unsigned& seq, int pos) {
  const ProjGeo gp = geo(a, st);
  const auto fin = [&](int, int it, int s, float v0, float v1) {
    item_epilogue(a, sm, st, layer, it / gp.KS, it % gp.KS, s, v0, v1, pos);
  };
  // gate|up reads the int8 form of its normed x; the other projections fp16 hi / lo
  if (st == ST_WGU) return consume_items<2, true>(a, sm, gp, seq, fin);
  return gp.rows == 16 ? consume_items<1, false>(a, sm, gp, seq, fin) : consume_items<2, false>(a, sm, gp, seq, fin);
}

// lm_head: 32-row items finished with logits (optional) and greedy argmax keys; the CTA's best key
// goes to the step state, the last CTA publishes the token (first maximum on ties, like torch.argmax).
__device__ bool consume_lm(const MkArgs& a, MkSmem& sm, unsigned& seq, unsigned epoch) {
  const ProjGeo gp = geo(a, ST_PER_LAYER);
  const int ct = threadIdx.x - 32, w = ct >> 5, lane = ct & 31;
  unsigned long long best = 0ull;
  const auto fin = [&](int, int it, int s, float v, float) {
    const int row = it * 32 + s;
    if (a.logits) a.logits[row] = v;
    best = max(best, argmax_key(v, (unsigned)(a.rank * a.V + row)));
  };
  if (!consume_items<2, true>(a, sm, gp, seq, fin)) return false;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
  if (lane == 0) sm.best[w] = best;
  consumer_sync();
  if (ct == 0) {
    unsigned long long b = 0ull;
    for (int k = 0; k < MK_CW; ++k) b = max(b, sm.best[k]);
    atomicMax(&a.state->best, b);
    __threadfence();
    sm.last = atomicAdd(&a.state->counter, 1u) == gridDim.x - 1;
    if (sm.last) {
      __threadfence();
      unsigned long long bb = atomicExch(&a.state->best, 0ull);
      a.state->counter = 0u;
      if (a.tp > 1) {
        // every rank's best key to every rank, then the largest (vocab rows are split by rank)
        for (int r = 0; r < a.tp; ++r) a.peer_keys[r][a.rank] = bb;
        __threadfence_system();
        for (int r = 0; r < a.tp; ++r)
          asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(a.peer_sync[r] + 4) : "memory");
        const unsigned target = (epoch + 1) * (unsigned)a.tp;  // epoch-based: never reset
        const uint64_t t0 = globaltimer_ns();
        for (;;) {
          unsigned v;
          asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a.sync + 4) : "memory");
          if ((int)(v - target) >= 0) break;
          if (globaltimer_ns() - t0 > a.wait_ns) {
            a.state->status = 1;
            break;
          }
        }
        bb = 0ull;
        for (int r = 0; r < a.tp; ++r) bb = max(bb, *(volatile unsigned long long*)&a.keys[r]);
      }
      publish_token(a.state, a.token_log, (int32_t)argmax_index(bb));
      a.sync[5] += 1u;  // this rank's step epoch (every rank runs every step)
    }
  }
  return true;
}


// Attention item (query row r of KV head kvh's group, keys [128 ch, 128 ch + 128) of ctx): the
// chunk's (max, sum, weighted V) for that row -- the online-softmax pieces of attn_decode_kernel.
// One row per item spreads a layer's attention over three times as many CTAs as one item per KV
// head (the rows of a group share K and V, which L2 serves again).
__device__ void attn_item(const MkArgs& a, MkSmem& sm, int layer, int kvh, int ch, int r, int ctx, int nch) {
  constexpr int HD = MK_HD, EPL = HD / 32, KW = MK_KCHUNK / MK_CW;  // KW keys per warp (16)
  const int ct = threadIdx.x - 32, w = ct >> 5, lane = ct & 31;
  const int kk = lane >> 1, hh = lane & 1;  // scores: two lanes per key, alternate 16-byte pieces
  const int g = a.H / a.Hkv;
  const __half* kc = sm.kcache[layer];
  const __half* vc = sm.vcache[layer];
  const size_t row_stride = (size_t)a.Hkv * HD;
  const int k0 = ch * MK_KCHUNK, k1 = min(k0 + MK_KCHUNK, ctx);
  const int jbase = k0 + KW * w, j = jbase + kk;
  // one round of loads: the query row (one element per thread, to shared memory), this lane's
  // 4 elements of every V row of the warp's keys (8 bytes per key) and its half of its key's K row
  // (pieces 2i + hh of 16 bytes, so a load instruction reads 32 contiguous bytes of 16 rows)
  const float qv = ct < HD ? __ldcg(a.q + ((size_t)kvh * g + r) * HD + ct) : 0.0f;
  uint2 vv[KW];
#pragma unroll
  for (int jj = 0; jj < KW; ++jj) {
    const int key = min(jbase + jj, k1 - 1);
    vv[jj] = __ldcg(reinterpret_cast<const uint2*>(vc + (size_t)key * row_stride + (size_t)kvh * HD + lane * EPL));
  }
  const uint4* kp = reinterpret_cast<const uint4*>(kc + (size_t)min(j, k1 - 1) * row_stride + (size_t)kvh * HD);
  uint4 kr[HD / 16];
#pragma unroll
  for (int i = 0; i < HD / 16; ++i) kr[i] = __ldcg(kp + 2 * i + hh);
  if (ct < HD) sm.u.att.q[0][ct] = qv;
  consumer_sync();
  float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
  for (int i = 0; i < HD / 16; ++i) {
    const __half2* h2 = reinterpret_cast<const __half2*>(&kr[i]);
    const float* qp = &sm.u.att.q[0][8 * (2 * i + hh)];
#pragma unroll
    for (int tt = 0; tt < 4; ++tt) {
      const float2 f = __half22float2(h2[tt]);
      d0 = fmaf(qp[2 * tt], f.x, d0);
      d1 = fmaf(qp[2 * tt + 1], f.y, d1);
    }
  }
  float d = d0 + d1;
  d += __shfl_xor_sync(0xffffffffu, d, 1);
  const float sc = j < k1 ? d * a.scale : -INFINITY;
  const float m = warp_max(sc);  // each key twice: the maximum is the same
  float o[EPL] = {0.0f, 0.0f, 0.0f, 0.0f};
  float lw = 0.0f;
  if (m != -INFINITY) {
    const float p = expf(sc - m);  // 0 for keys past the chunk: their V slices are never used
    lw = warp_sum(hh == 0 ? p : 0.0f);
#pragma unroll
    for (int jj = 0; jj < KW; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, 2 * jj);
      const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&vv[jj].x));
      const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&vv[jj].y));
      o[0] = fmaf(pj, v0.x, o[0]);
      o[1] = fmaf(pj, v0.y, o[1]);
      o[2] = fmaf(pj, v1.x, o[2]);
      o[3] = fmaf(pj, v1.y, o[3]);
    }
  }
  if (lane == 0) {
    sm.u.att.m[w][0] = m;
    sm.u.att.l[w][0] = lw;
  }
  *reinterpret_cast<float4*>(&sm.u.att.o[w][0][lane * EPL]) = make_float4(o[0], o[1], o[2], o[3]);
  consumer_sync();
  // merge the warps into this chunk's partial for row r
  float* part = a.part + (((size_t)kvh * MK_MAXCH + ch) * MK_ROWS + r) * (HD + MK_PAD);
  if (ct == 0) {
    float M = -INFINITY;
    for (int i = 0; i < MK_CW; ++i) M = fmaxf(M, sm.u.att.m[i][0]);
    float l = 0.0f;
    for (int i = 0; i < MK_CW; ++i) {
      const float cs = sm.u.att.m[i][0] == -INFINITY ? 0.0f : expf(sm.u.att.m[i][0] - M);
      sm.u.att.cs[i][0] = cs;
      l += sm.u.att.l[i][0] * cs;
    }
    part[0] = M;
    part[1] = l;
  }
  consumer_sync();
  for (int e = ct; e < HD; e += MK_CW * 32) {
    float v = 0.0f;
    for (int k = 0; k < MK_CW; ++k) v += sm.u.att.o[k][0][e] * sm.u.att.cs[k][0];
    part[MK_PAD + e] = v;
  }
  // the CTA that completes a query row's chunks merges them (max, sum, weighted V, online over the
  // chunks) into the attention output, so the o projection stages x with one plain round of loads
  const int hq = kvh * g + r;
  consumer_sync();
  if (ct == 0) {
    __threadfence();
    sm.att_last = atomicAdd(&a.rowcnt[hq], 1u) == (unsigned)(nch - 1);
  }
  consumer_sync();
  if (!sm.att_last) return;
  __threadfence();
  if (ct < HD) {
    const float* base = a.part + ((size_t)kvh * MK_MAXCH * MK_ROWS + r) * (HD + MK_PAD);
    float M = -INFINITY, L = 0.0f, v = 0.0f;
    for (int c0 = 0; c0 < nch; c0 += 4) {
      float2 ml[4];
      float ov[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {  // one round of loads per four chunks
        if (c0 + k < nch) {
          const float* pc = base + (size_t)(c0 + k) * MK_ROWS * (HD + MK_PAD);
          ml[k] = __ldcg(reinterpret_cast<const float2*>(pc));
          ov[k] = __ldcg(pc + MK_PAD + ct);
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (c0 + k < nch && ml[k].x != -INFINITY) {
          if (ml[k].x > M) {  // rescale what was merged so far to the new maximum
            const float rs = M == -INFINITY ? 0.0f : expf(M - ml[k].x);
            L *= rs;
            v *= rs;
            M = ml[k].x;
          }
          const float cs = expf(ml[k].x - M);
          L += ml[k].y * cs;
          v += cs * ov[k];
        }
      }
    }
    a.attn_out[(size_t)hq * HD + ct] = v / L;
  }
  if (ct == 0) a.rowcnt[hq] = 0u;  // the next layer's items start after the next stage barrier
}

// Long-context attention item (many chunks): all nr = g query rows of KV head kvh's group against
// keys [128 ch, 128 ch + 128), sharing one round of K and V loads; the rows' chunk partials as in
// attn_item, and the CTA completing the group's chunks (a counter on the group's first row) merges
// all its rows. Only the long-bucket instantiation of the step kernel contains it, so the registers
// it needs stay out of the short-bucket kernel.
__device__ void attn_group_item(const MkArgs& a, MkSmem& sm, int layer, int kvh, int ch, int r0, int nr, int ctx,
                                int nch) {
  constexpr int HD = MK_HD, EPL = HD / 32, KW = MK_KCHUNK / MK_CW;  // KW keys per warp (16)
  const int ct = threadIdx.x - 32, w = ct >> 5, lane = ct & 31;
  const int kk = lane >> 1, hh = lane & 1;  // scores: two lanes per key, alternate 16-byte pieces
  const int g = a.H / a.Hkv;
  const __half* kc = sm.kcache[layer];
  const __half* vc = sm.vcache[layer];
  const size_t row_stride = (size_t)a.Hkv * HD;
  const int k0 = ch * MK_KCHUNK, k1 = min(k0 + MK_KCHUNK, ctx);
  const int jbase = k0 + KW * w, j = jbase + kk;
  // one round of loads: the query rows (one element per thread and row, to shared memory), this
  // lane's 4 elements of every V row of the warp's keys (8 bytes per key) and its half of its key's K
  // row (pieces 2i + hh of 16 bytes, so a load instruction reads 32 contiguous bytes of 16 rows)
  if (ct < HD) {
#pragma unroll 1
    for (int rr = 0; rr < nr; ++rr) sm.u.att.q[rr][ct] = __ldcg(a.q + ((size_t)kvh * g + r0 + rr) * HD + ct);
  }
  uint2 vv[KW];
#pragma unroll
  for (int jj = 0; jj < KW; ++jj) {
    const int key = min(jbase + jj, k1 - 1);
    vv[jj] = __ldcg(reinterpret_cast<const uint2*>(vc + (size_t)key * row_stride + (size_t)kvh * HD + lane * EPL));
  }
  const uint4* kp = reinterpret_cast<const uint4*>(kc + (size_t)min(j, k1 - 1) * row_stride + (size_t)kvh * HD);
  uint4 kr[HD / 16];
#pragma unroll
  for (int i = 0; i < HD / 16; ++i) kr[i] = __ldcg(kp + 2 * i + hh);
  consumer_sync();
#pragma unroll 1
  for (int rr = 0; rr < nr; ++rr) {  // uniform over the CTA
    float d0 = 0.0f, d1 = 0.0f;
#pragma unroll
    for (int i = 0; i < HD / 16; ++i) {
      const __half2* h2 = reinterpret_cast<const __half2*>(&kr[i]);
      const float* qp = &sm.u.att.q[rr][8 * (2 * i + hh)];
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        const float2 f = __half22float2(h2[tt]);
        d0 = fmaf(qp[2 * tt], f.x, d0);
        d1 = fmaf(qp[2 * tt + 1], f.y, d1);
      }
    }
    float d = d0 + d1;
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    const float sc = j < k1 ? d * a.scale : -INFINITY;
    const float m = warp_max(sc);  // each key twice: the maximum is the same
    float o[EPL] = {0.0f, 0.0f, 0.0f, 0.0f};
    float lw = 0.0f;
    if (m != -INFINITY) {
      const float p = expf(sc - m);  // 0 for keys past the chunk: their V slices are never used
      lw = warp_sum(hh == 0 ? p : 0.0f);
#pragma unroll
      for (int jj = 0; jj < KW; ++jj) {
        const float pj = __shfl_sync(0xffffffffu, p, 2 * jj);
        const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&vv[jj].x));
        const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&vv[jj].y));
        o[0] = fmaf(pj, v0.x, o[0]);
        o[1] = fmaf(pj, v0.y, o[1]);
        o[2] = fmaf(pj, v1.x, o[2]);
        o[3] = fmaf(pj, v1.y, o[3]);
      }
    }
    if (lane == 0) {
      sm.u.att.m[w][rr] = m;
      sm.u.att.l[w][rr] = lw;
    }
    *reinterpret_cast<float4*>(&sm.u.att.o[w][rr][lane * EPL]) = make_float4(o[0], o[1], o[2], o[3]);
  }
  consumer_sync();
  // merge the warps into this chunk's partial for each row
  if (ct < nr) {
    const int rr = ct;
    float* part = a.part + (((size_t)kvh * MK_MAXCH + ch) * MK_ROWS + r0 + rr) * (HD + MK_PAD);
    float M = -INFINITY;
    for (int i = 0; i < MK_CW; ++i) M = fmaxf(M, sm.u.att.m[i][rr]);
    float l = 0.0f;
    for (int i = 0; i < MK_CW; ++i) {
      const float cs = sm.u.att.m[i][rr] == -INFINITY ? 0.0f : expf(sm.u.att.m[i][rr] - M);
      sm.u.att.cs[i][rr] = cs;
      l += sm.u.att.l[i][rr] * cs;
    }
    part[0] = M;
    part[1] = l;
  }
  consumer_sync();
  for (int idx = ct; idx < nr * HD; idx += MK_CW * 32) {
    const int rr = idx / HD, e = idx - rr * HD;
    float v = 0.0f;
    for (int k = 0; k < MK_CW; ++k) v += sm.u.att.o[k][rr][e] * sm.u.att.cs[k][rr];
    a.part[(((size_t)kvh * MK_MAXCH + ch) * MK_ROWS + r0 + rr) * (HD + MK_PAD) + MK_PAD + e] = v;
  }
  // the CTA that completes the rows' chunks merges them (max, sum, weighted V, online over the
  // chunks) into the attention output, so the o projection stages x with one plain round of loads
  const int cnt = kvh * g + r0;
  consumer_sync();
  if (ct == 0) {
    __threadfence();
    sm.att_last = atomicAdd(&a.rowcnt[cnt], 1u) == (unsigned)(nch - 1);
  }
  consumer_sync();
  if (!sm.att_last) return;
  __threadfence();
  for (int idx = ct; idx < nr * HD; idx += MK_CW * 32) {
    const int rr = idx / HD, e = idx - rr * HD;
    const float* base = a.part + ((size_t)kvh * MK_MAXCH * MK_ROWS + r0 + rr) * (HD + MK_PAD);
    float M = -INFINITY, L = 0.0f, v = 0.0f;
    for (int c0 = 0; c0 < nch; c0 += 4) {
      float2 ml[4];
      float ov[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {  // one round of loads per four chunks
        if (c0 + k < nch) {
          const float* pc = base + (size_t)(c0 + k) * MK_ROWS * (HD + MK_PAD);
          ml[k] = __ldcg(reinterpret_cast<const float2*>(pc));
          ov[k] = __ldcg(pc + MK_PAD + e);
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (c0 + k < nch && ml[k].x != -INFINITY) {
          if (ml[k].x > M) {  // rescale what was merged so far to the new maximum
            const float rs = M == -INFINITY ? 0.0f : expf(M - ml[k].x);
            L *= rs;
            v *= rs;
            M = ml[k].x;
          }
          const float cs = expf(ml[k].x - M);
          L += ml[k].y * cs;
          v += cs * ov[k];
        }
      }
    }
    a.attn_out[(size_t)(kvh * g + r0 + rr) * HD + e] = v / L;
  }
  if (ct == 0) a.rowcnt[cnt] = 0u;  // the next layer's items start after the next stage barrier
}

// One CTA of 9 warps per SM: a sub-partition holds 3 of the warps (16,384 registers each), so a
// thread gets at most 168 registers.
template <bool GROUPED>
__global__ void __launch_bounds__(MK_THREADS, 1) decode_step_kernel(MkArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  MkSmem& sm = *reinterpret_cast<MkSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < MK_NSLOT; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], MK_CW);
    }
    // a poisoned model (an earlier step of it timed out) does no work and reports the failure again
    sm.abort_flag = *(volatile unsigned*)&a.sync[6] ? 1 : 0;
    if (sm.abort_flag) a.state->status = 1;
    sm.tagbase = *(volatile unsigned*)&a.sync[5] * (unsigned)a.n_layers;  // tag parity of layer 0
    fence_mbar_init();
  }
  __syncthreads();
  const int pos = a.state->start;
  const int token = *a.token;
  const unsigned epoch = *(volatile unsigned*)&a.sync[5];
  const int ctx = min(a.L, pos + 1);
  const int nch = (ctx + MK_KCHUNK - 1) / MK_KCHUNK;

  if (warp == 0) {
    // producer: every projection's weights for this CTA, in consumption order
    unsigned seq = 0;
    if (lane == 0) {
      bool ok = true;
      // projections in consumption order: per layer q|k|v, o, gate|up, down; then the lm_head
      const int nproj = 4 * a.n_layers + 1;
      const auto kind = [&](int i) {
        constexpr int per_layer[4] = {ST_QKV, ST_WO, ST_WGU, ST_WDOWN};
        return i == 4 * a.n_layers ? (int)ST_PER_LAYER : per_layer[i & 3];
      };
      for (int i = 0; i < nproj && ok; ++i) {
        // local stage arrivals: q|k|v, attention, gate|up per layer (n CTAs each)
        if (kind(i) == ST_WO && a.gate_o) ok = producer_gate(a, sm, (3u * (i >> 2) + 2u) * gridDim.x);
        ok = ok && produce_stage(a, sm, a.proj[i], kind(i), seq);
      }
      if (!ok) raise_abort(a, sm);
    }
    __syncwarp();
    return;
  }

  {
    const int ct = threadIdx.x - 32;
    for (int e = ct; e < a.hd; e += MK_CW * 32) {
      sm.rope_c[e] = a.rope_cos[(size_t)pos * a.hd + e];
      sm.rope_s[e] = a.rope_sin[(size_t)pos * a.hd + e];
    }
    for (int l = ct; l < a.n_layers; l += MK_CW * 32) {
      sm.kcache[l] = reinterpret_cast<__half*>(a.layers[l].k_cache);
      sm.vcache[l] = reinterpret_cast<__half*>(a.layers[l].v_cache);
      sm.ln_in[l] = a.layers[l].ln_in;
      sm.ln_post[l] = a.layers[l].ln_post;
    }
    if (blockIdx.x == 0)  // row counters of the attention merge (left non-zero only by an aborted launch)
      for (int i = ct; i < a.H; i += MK_CW * 32) a.rowcnt[i] = 0u;
    consumer_sync();
  }
  trace_ev(a, 15 * a.n_layers + 3);
  unsigned seq = 0;
  unsigned stage = 0;
  const unsigned n = gridDim.x;
  const int nwo = geo(a, ST_WO).KS, nwd = geo(a, ST_WDOWN).KS;  // partial sums the norms add
  const float* pwo = a.psum;                                      // o partials of every rank
  const float* pwd = a.psum + (size_t)a.tp * MK_MAXKS * a.D;      // down partials of every rank
  bool ok = !sm.abort_flag;  // a poisoned model (an earlier step timed out) does no work
  float lw[2][8];  // the next norm's weights
  // row-split arrival counter: this step's c-th completion (layer c / 2; o for odd c, down for even
  // c > 0) is reached at split0 + c * per
  const unsigned per = n * (unsigned)a.tp;
  const unsigned split0 = epoch * 2u * (unsigned)a.n_layers * per;
  for (int l = 0; l < a.n_layers && ok; ++l) {
    // QKV (x from the previous layer's down partials of every rank, tagged with that layer's parity)
    norm_weights(a, sm.ln_in[l], lw);
    stage_norm(a, sm, lw, l == 0, token, a.hb, pwd, nwd, (sm.tagbase + l + 1) & 1u, a.hb + a.D,
               split0 + 2u * (unsigned)l * per, 15 * l + 0, false);
    consumer_sync();
    trace_ev(a, 15 * l + 1);
    ok = consume_stage(a, sm, ST_QKV, l, seq, pos);
    trace_ev(a, 15 * l + 2);
    stage_arrive(a);
    ++stage;
    if (!ok) break;
    // attention
    if (!(ok = stage_wait(a, sm, stage * n))) break;
    trace_ev(a, 15 * l + 3);
    trace_ev(a, 15 * l + 4);
    const int g = a.H / a.Hkv;
    if (GROUPED && a.H * nch > 2 * (int)gridDim.x) {  // long context: (KV head, chunk) items of g rows
      for (int it = blockIdx.x; it < a.Hkv * nch; it += gridDim.x) {
        const int kvh = it / nch, ch = it - kvh * nch;
        attn_group_item(a, sm, l, kvh, ch, 0, g, ctx, nch);
        consumer_sync();
      }
    } else {
      for (int it = blockIdx.x; it < a.H * nch; it += gridDim.x) {  // (query row, chunk) items
        const int hq = it / nch, ch = it - hq * nch;
        attn_item(a, sm, l, hq / g, ch, hq % g, ctx, nch);
        consumer_sync();
      }
    }
    trace_ev(a, 15 * l + 5);
    stage_arrive(a);
    ++stage;
    // WO
    if (!(ok = stage_wait(a, sm, stage * n))) break;
    trace_ev(a, 15 * l + 6);
    stage_plain(a, sm, a.attn_out, a.H * a.hd);
    consumer_sync();
    trace_ev(a, 15 * l + 7);
    ok = consume_stage(a, sm, ST_WO, l, seq, pos);
    trace_ev(a, 15 * l + 8);
    if (!ok || sm.abort_flag) break;
    split_arrive(a);
    // WGU (x from every rank's o partials of this layer)
    norm_weights(a, sm.ln_post[l], lw);
    stage_norm(a, sm, lw, false, token, a.hb + a.D, pwo, nwo, (sm.tagbase + l) & 1u, a.hb,
               split0 + (2u * (unsigned)l + 1u) * per, 15 * l + 9, true);
    consumer_sync();
    trace_ev(a, 15 * l + 10);
    ok = consume_stage(a, sm, ST_WGU, l, seq, pos);
    trace_ev(a, 15 * l + 11);
    stage_arrive(a);
    ++stage;
    if (!ok) break;
    // WDOWN
    if (!(ok = stage_wait(a, sm, stage * n))) break;
    trace_ev(a, 15 * l + 12);
    stage_plain(a, sm, a.a, a.I);
    consumer_sync();
    trace_ev(a, 15 * l + 13);
    ok = consume_stage(a, sm, ST_WDOWN, l, seq, pos) && !sm.abort_flag;
    trace_ev(a, 15 * l + 14);
    if (ok) split_arrive(a);
  }
  if (ok) {
    norm_weights(a, a.ln_f, lw);
    stage_norm(a, sm, lw, false, token, a.hb, pwd, nwd, (sm.tagbase + a.n_layers + 1) & 1u, nullptr,
               split0 + 2u * (unsigned)a.n_layers * per, 15 * a.n_layers + 0, true);
    consumer_sync();
    trace_ev(a, 15 * a.n_layers + 1);
    ok = !sm.abort_flag && consume_lm(a, sm, seq, epoch);
    trace_ev(a, 15 * a.n_layers + 2);
  }
  if (!ok && threadIdx.x == 32) raise_abort(a, sm);
}

}  // namespace

// ---- host ----------------------------------------------------------------------------------------

// Shapes of this rank's shard the kernel takes (H, Hkv, I, V are per rank; an o / down shard may end
// inside a 1024-k unit, whose rest the TMA zero-fills).
static bool mk_shapes_ok(const Model& m) {
  return m.cfg.tp_size <= MK_MAXTP && (int)m.layers.size() <= MK_MAXL && (m.cfg.tp_size == 1 || m.comm) && m.hd == MK_HD && m.H % m.Hkv == 0 &&
         m.H / m.Hkv <= MK_ROWS && m.H <= 32 && m.D <= MK_MAXD && m.D % MK_UK == 0 && (m.H * m.hd) % 128 == 0 &&
         m.I % 128 == 0 && m.I <= MK_MAXK && m.H * m.hd <= MK_MAXK && m.V % 32 == 0 &&
         m.cfg.max_ctx <= MK_MAXCH * MK_KCHUNK;
}

// The persistent kernel is the decode path where its shapes allow; Q4B_PERSISTENT=0 selects the
// per-projection kernels instead (read on every step)
static bool persistent_enabled() {
  const char* e = std::getenv("Q4B_PERSISTENT");
  return !(e && e[0] == '0');
}

// Tensor maps and the layer table on the device; needs every weight set and no stream capture.
int Model::mk_prepare() {
  if (mk_ready) return Q4B_OK;
  if (!mk_shapes_ok(*this)) return set_error(Q4B_EUNSUPPORTED, "persistent decode: unsupported shape");
  int rc = check_ready();
  if (rc) return rc;
  const auto groups_ok = [](const q4b_qmat& w) { return w.group == 128; };
  for (const auto& L : layers)
    if (!groups_ok(L.wqkv) || !groups_ok(L.wo) || !groups_ok(L.wgu) || !groups_ok(L.wdown))
      return set_error(Q4B_EUNSUPPORTED, "persistent decode: group 128 only");
  if (embed.group != 128) return set_error(Q4B_EUNSUPPORTED, "persistent decode: group 128 only");
  std::vector<MkProj> proj(layers.size() * 4 + 1);
  mk_scale_pad.resize(proj.size(), nullptr);
  // scales: fp16 [n, k/G]; the int32 tensor-map helper describes a row as k/G/2 int32 pairs (the box
  // is 8 groups = 4 pairs = 16 bytes). A tensor map's row stride is a multiple of 16 bytes, so a
  // shard whose scale rows are not (a tensor-parallel o / down shard: k/G = 12 or 6 or 3) is read
  // from a copy with rows padded by zero scales to a multiple of 8 groups.
  // box rows: one run of a paired item (8 for the RoPE halves, 16 for gate | up) or a whole 32-row item
  auto mk = [&](size_t i, const q4b_qmat& w, int box_rows) {
    MkProj& p = proj[i];
    int r = make_tmap_i32(&p.w, w.qweight, w.k / 8, w.n, w.k / 8, MK_UK / 8, box_rows);
    if (r) return r;
    const int groups = w.k / w.group;
    if (groups % 8 == 0) return make_tmap_i32(&p.s, w.scales, groups / 2, w.n, groups / 2, 4, box_rows);
    const int padded = (groups + 7) / 8 * 8;
    if (!mk_scale_pad[i] && (r = alloc(&mk_scale_pad[i], sizeof(__half) * (size_t)w.n * padded, true))) return r;
    cudaError_t e = cudaMemcpy2D(mk_scale_pad[i], sizeof(__half) * padded, w.scales, sizeof(__half) * groups,
                                 sizeof(__half) * groups, w.n, cudaMemcpyDeviceToDevice);
    if (e != cudaSuccess) return set_error(Q4B_ECUDA, "persistent decode: scale copy: %s", cudaGetErrorString(e));
    return make_tmap_i32(&p.s, mk_scale_pad[i], (groups + 1) / 2, w.n, padded / 2, 4, box_rows);
  };
  for (size_t l = 0; l < layers.size(); ++l) {
    if ((rc = mk(4 * l + 0, layers[l].wqkv, 8))) return rc;
    if ((rc = mk(4 * l + 1, layers[l].wo, 32))) return rc;
    if ((rc = mk(4 * l + 2, layers[l].wgu, 16))) return rc;
    if ((rc = mk(4 * l + 3, layers[l].wdown, 32))) return rc;
  }
  q4b_qmat head = embed;  // this rank's vocab rows of the tied table
  head.qweight = embed.qweight + (size_t)cfg.tp_rank * V * (D / 8);
  head.scales = embed.scales + (size_t)cfg.tp_rank * V * (D / embed.group);
  head.n = V;
  if ((rc = mk(4 * layers.size(), head, 32))) return rc;
  if (!mk_proj && (rc = alloc(&mk_proj, sizeof(MkProj) * proj.size(), false))) return rc;
  if (!mk_layers && (rc = alloc(&mk_layers, sizeof(q4b_layer_weights) * layers.size(), false))) return rc;
  if (!mk_part && (rc = alloc((void**)&mk_part, sizeof(float) * Hkv * MK_MAXCH * MK_ROWS * (hd + MK_PAD), true))) return rc;
  if (!mk_rows && (rc = alloc((void**)&mk_rows, sizeof(unsigned) * H, true))) return rc;
  if (!mk_attn && (rc = alloc((void**)&mk_attn, sizeof(float) * H * hd, true))) return rc;
  const int t = cfg.tp_size;
  // sync words [0, 8) and the argmax keys at byte 64; residual ping-pong + every rank's partials
  if (!mk_sync && (rc = alloc((void**)&mk_sync, 256, true))) return rc;
  const size_t psum_bytes = sizeof(float) * 2 * (size_t)t * MK_MAXKS * D;
  if (!mk_h) {
    if ((rc = alloc((void**)&mk_h, sizeof(float) * 2 * D + psum_bytes, true))) return rc;
    // partial-sum tags: layer 0 of epoch 0 expects parity 0, so every slot starts with parity 1
    if (cudaMemset(mk_h + 2 * D, 0x01, psum_bytes) != cudaSuccess) return set_error(Q4B_ECUDA, "persistent decode: init");
  }
  if (t == 1) {  // a poisoned model (a step timed out) is cleared: slots get the parity the next layer 0 does not expect
    unsigned w[8];
    if (cudaMemcpy(w, mk_sync, sizeof(w), cudaMemcpyDeviceToHost) != cudaSuccess)
      return set_error(Q4B_ECUDA, "persistent decode: state read");
    if (w[6]) {  // back to the state of a new model: epoch 0, tags of parity 1, no row-split arrivals
      if (cudaMemset(mk_h + 2 * D, 0x01, psum_bytes) != cudaSuccess ||
          cudaMemset(mk_sync + 5, 0, 3 * sizeof(unsigned)) != cudaSuccess)
        return set_error(Q4B_ECUDA, "persistent decode: reset");
    }
  }
  if ((int)mk_peer_h.size() != t || (int)mk_peer_sync.size() != t) {  // once: the buffers live as long as the model
    mk_peer_h.assign(t, nullptr);
    mk_peer_sync.assign(t, nullptr);
    mk_peer_h[cfg.tp_rank] = mk_h;
    mk_peer_sync[cfg.tp_rank] = mk_sync;
    if (t > 1) {  // every peer's buffers mapped into this process (NVLink peer memory)
      if ((rc = tp_map_peers(mk_h, reinterpret_cast<void**>(mk_peer_h.data()))) ||
          (rc = tp_map_peers(mk_sync, reinterpret_cast<void**>(mk_peer_sync.data())))) {
        mk_peer_h.clear();
        mk_peer_sync.clear();
        return rc;
      }
    }
  }
  cudaError_t e = cudaMemcpy(mk_proj, proj.data(), sizeof(MkProj) * proj.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = cudaMemcpy(mk_layers, layers.data(), sizeof(q4b_layer_weights) * layers.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return set_error(Q4B_ECUDA, "persistent decode: table upload: %s", cudaGetErrorString(e));
  int dev = 0, sms = 0, per = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // 6 of the 10 slots by default: a deeper ring keeps more weight traffic queued ahead of each stage
  // transition's latency-bound loads (measured: 40.4 us per 3B layer with 6 slots, 42.2 with 10)
  mk_nslot = kMkDefaultSlots;
  if (const char* v = std::getenv("Q4B_MK_SLOTS")) mk_nslot = std::max(2, std::min(MK_NSLOT, std::atoi(v)));
  const size_t smem = mk_smem_bytes(mk_nslot);
  for (int grouped = 0; grouped < 2 && e == cudaSuccess; ++grouped) {
    auto kern = grouped ? decode_step_kernel<true> : decode_step_kernel<false>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, MK_THREADS, smem);
    if (per < 1) break;
  }
  if (e != cudaSuccess || per < 1)
    return set_error(Q4B_EUNSUPPORTED, "persistent decode: kernel does not fit an SM (%s)", cudaGetErrorString(e));
  mk_ctas = sms;
  // ring depth (above) and row-split synchronisation: tuning knobs Q4B_MK_SLOTS, Q4B_MK_SPLIT_SYNC
  mk_gate_o = 1;
  if (const char* e = std::getenv("Q4B_MK_GATE_O")) mk_gate_o = std::atoi(e) != 0;
  mk_split_sync = 0;
  if (const char* e = std::getenv("Q4B_MK_SPLIT_SYNC")) mk_split_sync = std::atoi(e) == 1 ? 1 : 0;
  mk_ready = true;
  return Q4B_OK;
}

// Marks the persistent step failed, as a timed-out wait does (sync[6]): the failure path without a
// device fault. Single-GPU models are cleared by preparing them again.
int Model::mk_poison() {
  if (!mk_ready) {
    const int rc = mk_prepare();
    if (rc) return rc;
  }
  const unsigned one = 1u;
  if (cudaMemcpy(mk_sync + 6, &one, sizeof(one), cudaMemcpyHostToDevice) != cudaSuccess)
    return set_error(Q4B_ECUDA, "persistent decode: poison");
  return Q4B_OK;
}

bool Model::mk_usable(int C, cudaStream_t st) {
  if (C != 1 || !persistent_enabled() || !mk_shapes_ok(*this)) return false;
  if (mk_ready) return true;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return false;
  if (mk_prepare() != Q4B_OK) {
    clear_error();
    return false;
  }
  return true;
}

int Model::mk_forward(const int32_t* toks, int L, float* logits, int32_t* token_log, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(mk_sync, 0, 2 * sizeof(unsigned), st);
  if (e != cudaSuccess) return set_error(Q4B_ECUDA, "persistent decode: reset: %s", cudaGetErrorString(e));
  MkArgs a = {};
  a.proj = reinterpret_cast<const MkProj*>(mk_proj);
  a.layers = reinterpret_cast<const q4b_layer_weights*>(mk_layers);
  a.n_layers = (int)layers.size();
  a.emb_qw = embed.qweight;
  a.emb_s = reinterpret_cast<const __half*>(embed.scales);
  a.ln_f = ln_f;
  a.rope_cos = rope_cos;
  a.rope_sin = rope_sin;
  a.D = D;
  a.H = H;
  a.Hkv = Hkv;
  a.hd = hd;
  a.I = I;
  a.V = V;
  a.eps = cfg.rms_eps;
  a.scale = (float)(1.0 / sqrt((double)hd));
  a.L = L;
  a.token = toks;
  a.state = state;
  a.token_log = token_log;
  a.logits = logits;
  a.hb = mk_h;
  a.psum = mk_h + 2 * D;
  a.tp = cfg.tp_size;
  a.rank = cfg.tp_rank;
  a.Vfull = cfg.vocab;
  for (int r = 0; r < cfg.tp_size; ++r) {
    a.peer_psum[r] = mk_peer_h[r] + 2 * D;
    a.peer_sync[r] = mk_peer_sync[r];
    a.peer_keys[r] = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(mk_peer_sync[r]) + 64);
  }
  a.keys = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(mk_sync) + 64);
  a.wait_ns = cfg.tp_size > 1 ? 5 * kWaitLimitNs : kWaitLimitNs;
  a.q = q;
  a.a = this->a;
  a.part = mk_part;
  a.rowcnt = mk_rows;
  a.attn_out = mk_attn;
  a.sync = mk_sync;
  a.trace = mk_trace_cap >= (size_t)mk_ctas * mk_trace_stride(a.n_layers) ? mk_trace : nullptr;
  a.nslot = mk_nslot;
  a.split_sync = mk_split_sync;
  a.gate_o = mk_gate_o;
  cudaLaunchConfig_t cfgl = {};
  cfgl.gridDim = dim3(mk_ctas);
  cfgl.blockDim = dim3(MK_THREADS);
  cfgl.dynamicSmemBytes = mk_smem_bytes(mk_nslot);
  cfgl.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfgl.attrs = attr;
  cfgl.numAttrs = 1;
  // grouped (KV head, chunk) attention items only where the bucket reaches them: a step of this
  // bucket attends over at most L keys, so H * ceil(L / 128) > 2 * CTAs for some position
  const bool grouped = (long long)a.H * ((L + MK_KCHUNK - 1) / MK_KCHUNK) > 2LL * mk_ctas;
  e = grouped ? cudaLaunchKernelEx(&cfgl, decode_step_kernel<true>, a) : cudaLaunchKernelEx(&cfgl, decode_step_kernel<false>, a);
  if (e != cudaSuccess) return set_error(Q4B_ELAUNCH, "persistent decode: launch: %s", cudaGetErrorString(e));
  return check_launch("persistent decode");
}

}  // namespace q4b
