// Internal model object behind the q4b_model_* C ABI (model.cu), also used by the runner.
#pragma once

#include <vector>

#include "linear.h"

struct ncclComm;

namespace q4b {

// Stamps per CTA of the persistent decode step's phase trace (15 per layer, then 4).
__host__ __device__ inline int mk_trace_stride(int n_layers) { return 15 * n_layers + 4; }

struct Model {
  q4b_model_cfg cfg{};
  int H = 0, Hkv = 0, I = 0, V = 0, D = 0, hd = 0;  // per-rank (sharded) sizes
  std::vector<q4b_layer_weights> layers;
  q4b_qmat embed{};
  const float* ln_f = nullptr;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  // owned device memory
  DecodeState* state = nullptr;
  int32_t* tokens = nullptr;
  float *h = nullptr, *xn = nullptr, *q = nullptr, *o = nullptr, *a = nullptr, *y = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  void* attn_ws = nullptr;
  size_t attn_ws_bytes = 0;
  std::vector<void*> owned;
  // persistent decode step (decode_mk.cu): tensor maps + layer table on the device
  void* mk_proj = nullptr;
  void* mk_layers = nullptr;
  float* mk_part = nullptr;
  unsigned* mk_sync = nullptr;
  unsigned* mk_rows = nullptr;  // attention row counters [H]
  float* mk_attn = nullptr;     // attention output [H * hd]
  float* mk_h = nullptr;  // residual ping-pong [2][D] + every rank's o / down partials [2][tp][3][D]
  std::vector<float*> mk_peer_h;        // per rank: its mk_h mapped here (own rank: mk_h)
  std::vector<unsigned*> mk_peer_sync;  // per rank: its mk_sync mapped here
  std::vector<void*> mk_mapped;         // peer mappings to close
  std::vector<void*> mk_scale_pad;      // per projection: scale rows padded to 16 bytes (or null)
  int tp_map_peers(void* local, void** peers);
  int mk_ctas = 0;
  int mk_nslot = 0;        // ring slots the persistent step uses
  int mk_split_sync = 0;   // 0: tag-polled partial sums, 1: row-split arrival counter
  int mk_gate_o = 1;       // o weights requested after the layer's attention (Q4B_MK_GATE_O)
  unsigned long long* mk_trace = nullptr;  // caller's phase-trace buffer (q4b_model_set_trace) or null
  size_t mk_trace_cap = 0;
  bool mk_ready = false;
  int mk_prepare();
  int mk_poison();
  bool mk_usable(int C, cudaStream_t st);
  int mk_forward(const int32_t* toks, int L, float* logits, int32_t* token_log, cudaStream_t st);
  // tensor parallelism (tp.cu)
  ncclComm* comm = nullptr;
  unsigned long long* gather = nullptr;  // [tp_size] per-rank argmax keys

  ~Model();
  int alloc(void** p, size_t bytes, bool zero);
  int init(const q4b_model_cfg& c);
  int check_ready() const;
  int forward(const int32_t* toks, int C, int L, float* logits, int32_t* token_log, cudaStream_t st);
  int residual_linear(const q4b_qmat& w, const float* x, int k, int C, cudaStream_t st);
  // rows of a chunk per projection call: up to 64 for the register-staged MMA kernel, the whole
  // chunk once it is large enough for the tcgen05 GEMM (more than 32 rows)
  static int row_block(int C) { return C > 32 ? C : 64; }
  int step(const int32_t* toks, int C, int start, int last, int L, int32_t* next, float* logits, cudaStream_t st);
  int tp_allreduce_add(int C, cudaStream_t st);
  int tp_finish_argmax(int32_t* token_log, cudaStream_t st);
  void tp_release();
};

}  // namespace q4b
