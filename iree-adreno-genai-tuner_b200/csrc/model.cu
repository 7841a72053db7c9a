// LlamaQ4.step (scripts/llm/llama_q4.py:199-239) as a sequence of fused kernels on one stream.
//
// Per decoder layer (rows C of the step; fp32 residual stream h like the reference):
//   1. wqkv   x = rmsnorm(h) * ln_in (fused prologue, C <= 8; a separate rmsnorm kernel above),
//             epilogue: RoPE on q and k, q -> q buffer, k and v -> fp16 caches at rows start + c
//   2. attention over the cache (decode: split over keys; prefill: per query row)
//   3. wo     h += o @ Wo^T            (tensor parallel: partial -> allreduce -> residual add)
//   4. wgu    x = rmsnorm(h) * ln_post, epilogue silu(gate) * up -> a
//   5. wdown  h += a @ Wdown^T
// then lm_head over rmsnorm(h[last]) * ln_f with a greedy argmax epilogue that publishes the
// token into the device step state (next token, token log, stop ids, position advance).
// The model owns only its activations and workspaces; weights and KV caches are borrowed.
#include <cstring>
#include <new>
#include <vector>

#include "fused.h"
#include "linear.h"
#include "model.h"

namespace q4b {

static int cuda_err(cudaError_t e, const char* what) {
  return e == cudaSuccess ? Q4B_OK : set_error(Q4B_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

__global__ void set_state_kernel(DecodeState* st, int start, int last, int advance) {
  st->start = start;
  st->last = last;
  st->advance = advance;
}

static LinearOp qop(const q4b_qmat& w, int m, const void* x, void* y, int epi) {
  LinearOp op;
  op.qw = w.qweight;
  op.scales = w.scales;
  op.group = w.group;
  op.n = w.n;
  op.k = w.k;
  op.m = m;
  op.x = x;
  op.x_dtype = Q4B_F32;
  op.y = y;
  op.y_dtype = Q4B_F32;
  op.epi = epi;
  return op;
}

Model::~Model() {
  tp_release();
  for (void* p : owned) cudaFree(p);
}

int Model::alloc(void** p, size_t bytes, bool zero) {
  cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
  if (e != cudaSuccess) return set_error(Q4B_ENOMEM, "model: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  owned.push_back(*p);
  if (zero) {
    e = cudaMemset(*p, 0, bytes ? bytes : 16);
    if (e != cudaSuccess) return cuda_err(e, "model: cudaMemset");
  }
  return Q4B_OK;
}

int Model::init(const q4b_model_cfg& c) {
  cfg = c;
  const int t = c.tp_size;
  if (c.n_layers < 1 || c.dim < 8 || c.n_heads < 1 || c.n_kv_heads < 1 || c.head_dim < 16 || c.inter < 8 ||
      c.vocab < 1 || c.max_ctx < 1 || c.max_chunk < 1 || t < 1 || c.tp_rank < 0 || c.tp_rank >= t)
    return set_error(Q4B_EINVAL, "model: bad configuration");
  if (c.n_heads % c.n_kv_heads || c.n_heads % t || c.n_kv_heads % t || c.inter % t || c.vocab % t)
    return set_error(Q4B_EINVAL, "model: heads, KV heads, intermediate and vocab must divide by tp_size %d", t);
  H = c.n_heads / t;
  Hkv = c.n_kv_heads / t;
  I = c.inter / t;
  V = c.vocab / t;
  D = c.dim;
  hd = c.head_dim;
  layers.assign(c.n_layers, q4b_layer_weights{});
  const int Cm = c.max_chunk;
  int rc;
  if ((rc = alloc((void**)&state, sizeof(DecodeState), true))) return rc;
  if ((rc = alloc((void**)&tokens, sizeof(int32_t) * Cm, true))) return rc;
  if ((rc = alloc((void**)&h, sizeof(float) * Cm * D, true))) return rc;
  if ((rc = alloc((void**)&xn, sizeof(float) * Cm * std::max(D, I), true))) return rc;
  if ((rc = alloc((void**)&q, sizeof(float) * Cm * H * hd, true))) return rc;
  if ((rc = alloc((void**)&o, sizeof(float) * Cm * H * hd, true))) return rc;
  if ((rc = alloc((void**)&a, sizeof(float) * Cm * I, true))) return rc;
  if ((rc = alloc((void**)&y, sizeof(float) * Cm * D, true))) return rc;
  // split-K workspace: the largest any projection plan of this model asks for
  size_t need = 0;
  const int ms[] = {1, 2, 4, 8, 16, 32, 64, Cm};
  q4b_qmat shapes[5] = {{nullptr, nullptr, (H + 2 * Hkv) * hd, D, 128}, {nullptr, nullptr, D, H * hd, 128},
                        {nullptr, nullptr, 2 * I, D, 128}, {nullptr, nullptr, D, I, 128},
                        {nullptr, nullptr, V, D, 128}};
  static const int32_t dummy[4] = {0, 0, 0, 0};
  for (const q4b_qmat& s : shapes)
    for (int m : ms) {
      if (m > Cm && m != 1) continue;  // (Cm: the whole chunk in one tcgen05 GEMM)
      q4b_qmat w = s;
      w.qweight = dummy;
      w.scales = reinterpret_cast<const uint16_t*>(dummy);
      if (w.k % 128) w.group = 8;
      LinearOp op = qop(w, m, dummy, const_cast<int32_t*>(dummy), EPI_STORE);
      need = std::max(need, linear_workspace(op));
    }
  ws_bytes = need + (1 << 20);
  if ((rc = alloc(&ws, ws_bytes, true))) return rc;
  attn_ws_bytes = 0;  // decode-form attention partials for every row count that uses that form
  for (int cc = 1; cc <= Cm && cc * (H / Hkv) <= 16; ++cc)
    attn_ws_bytes = std::max(attn_ws_bytes, attention_workspace(cc, H, Hkv, hd, c.max_ctx));
  if ((rc = alloc(&attn_ws, attn_ws_bytes, true))) return rc;
  return cudaDeviceSynchronize() == cudaSuccess ? Q4B_OK : cuda_err(cudaGetLastError(), "model: init");
}

int Model::check_ready() const {
  for (size_t i = 0; i < layers.size(); ++i)
    if (!layers[i].wqkv.qweight || !layers[i].k_cache)
      return set_error(Q4B_ESTATE, "model: layer %zu has no weights or caches", i);
  if (!embed.qweight || !ln_f || !rope_cos) return set_error(Q4B_ESTATE, "model: head weights not set");
  return Q4B_OK;
}

// The kernels of one step; positions come from the device step state.
int Model::forward(const int32_t* toks, int C, int L, float* logits, int32_t* token_log, cudaStream_t st) {
  int rc;
  if (C < 1 || C > cfg.max_chunk) return set_error(Q4B_EINVAL, "model: %d rows, max_chunk %d", C, cfg.max_chunk);
  if (L < 1 || L > cfg.max_ctx) return set_error(Q4B_EINVAL, "model: bucket %d outside 1..max_ctx %d", L, cfg.max_ctx);
  if ((rc = check_ready())) return rc;
  if (mk_usable(C, st)) return mk_forward(toks, L, logits, token_log, st);
  if ((rc = embed_run(toks, C, embed.qweight, embed.scales, cfg.vocab, D, embed.group, h, st))) return rc;
  const int* start = &state->start;
  for (size_t li = 0; li < layers.size(); ++li) {
    const q4b_layer_weights& Lw = layers[li];
    // 1. q|k|v projection with RoPE and the cache write
    for (int r0 = 0; r0 < C; r0 += row_block(C)) {
      const int m = std::min(row_block(C), C - r0);
      const float* xin = h + (size_t)r0 * D;
      // RMSNorm inside the projection's own launch where its plan has one (the GEMV prologue up to
      // 8 rows, the tcgen05 path's x split), else a separate launch
      const bool fuse_norm = linear_fuses_norm(m, Lw.wqkv.k, Lw.wqkv.group, EPI_ROPE_KV, hd) && aligned(Lw.ln_in, 16) &&
                             aligned(xin, 16);
      if (!fuse_norm) {
        if ((rc = rmsnorm_run(h + (size_t)r0 * D, Lw.ln_in, cfg.rms_eps, m, D, nullptr, xn, st))) return rc;
        xin = xn;
      }
      LinearOp op = qop(Lw.wqkv, m, xin, nullptr, EPI_ROPE_KV);
      if (fuse_norm) {
        op.ln_w = Lw.ln_in;
        op.eps = cfg.rms_eps;
      }
      op.rope_cos = rope_cos;
      op.rope_sin = rope_sin;
      op.pos0 = start;
      op.pos_offset = r0;
      op.q_out = q + (size_t)r0 * H * hd;
      op.k_cache = Lw.k_cache;
      op.v_cache = Lw.v_cache;
      op.n_heads = H;
      op.n_kv = Hkv;
      op.head_dim = hd;
      op.ws = ws;
      op.ws_bytes = ws_bytes;
      if ((rc = linear_run(op, st))) return rc;
    }
    // 2. attention
    AttnArgs at = {};
    at.q = q;
    at.k_cache = reinterpret_cast<const __half*>(Lw.k_cache);
    at.v_cache = reinterpret_cast<const __half*>(Lw.v_cache);
    at.pos0 = start;
    at.C = C;
    at.H = H;
    at.Hkv = Hkv;
    at.head_dim = hd;
    at.L = L;
    at.scale = (float)(1.0 / sqrt((double)hd));
    at.out = o;
    at.ws_base = attn_ws;
    at.ws_bytes = attn_ws_bytes;
    if ((rc = attention_run(at, st))) return rc;
    // 3. h += o Wo^T
    if ((rc = residual_linear(Lw.wo, o, H * hd, C, st))) return rc;
    // 4. a = silu(gate) * up of rmsnorm(h)
    for (int r0 = 0; r0 < C; r0 += row_block(C)) {
      const int m = std::min(row_block(C), C - r0);
      const float* xin = h + (size_t)r0 * D;
      const bool fuse_norm =
          linear_fuses_norm(m, Lw.wgu.k, Lw.wgu.group, EPI_SWIGLU, hd) && aligned(Lw.ln_post, 16) && aligned(xin, 16);
      if (!fuse_norm) {
        if ((rc = rmsnorm_run(h + (size_t)r0 * D, Lw.ln_post, cfg.rms_eps, m, D, nullptr, xn, st))) return rc;
        xin = xn;
      }
      LinearOp op = qop(Lw.wgu, m, xin, a + (size_t)r0 * I, EPI_SWIGLU);
      if (fuse_norm) {
        op.ln_w = Lw.ln_post;
        op.eps = cfg.rms_eps;
      }
      op.ws = ws;
      op.ws_bytes = ws_bytes;
      if ((rc = linear_run(op, st))) return rc;
    }
    // 5. h += a Wdown^T
    if ((rc = residual_linear(Lw.wdown, a, I, C, st))) return rc;
  }
  // lm_head over rmsnorm(h[last]) * ln_f, greedy argmax (first max) published into the state
  q4b_qmat head = embed;
  head.qweight = embed.qweight + (size_t)cfg.tp_rank * V * (D / 8);
  head.scales = embed.scales + (size_t)cfg.tp_rank * V * (D / embed.group);
  head.n = V;
  // the final norm of the one selected row, once (the lm_head has thousands of CTAs; a fused
  // prologue would re-read and re-reduce the row in every one of them)
  if ((rc = rmsnorm_run(h, ln_f, cfg.rms_eps, 1, D, &state->last, xn, st))) return rc;
  LinearOp op = qop(head, 1, xn, nullptr, EPI_ARGMAX);
  op.state = state;
  op.token_log = token_log;
  op.logits = logits;
  op.index_offset = cfg.tp_rank * V;
  op.finalize = cfg.tp_size == 1;
  op.ws = ws;
  op.ws_bytes = ws_bytes;
  if ((rc = linear_run(op, st))) return rc;
  if (cfg.tp_size > 1) return tp_finish_argmax(token_log, st);
  return Q4B_OK;
}

// h[:C] += x[:C] W^T; under tensor parallelism the rank's partial is all-reduced first.
int Model::residual_linear(const q4b_qmat& w, const float* x, int k, int C, cudaStream_t st) {
  int rc;
  (void)k;
  for (int r0 = 0; r0 < C; r0 += row_block(C)) {
    const int m = std::min(row_block(C), C - r0);
    const bool tp = cfg.tp_size > 1;
    LinearOp op = qop(w, m, x + (size_t)r0 * w.k, tp ? (void*)(y + (size_t)r0 * D) : (void*)(h + (size_t)r0 * D),
                      tp ? EPI_STORE : EPI_ACCUMULATE);
    op.ws = ws;
    op.ws_bytes = ws_bytes;
    if ((rc = linear_run(op, st))) return rc;
  }
  if (cfg.tp_size > 1) return tp_allreduce_add(C, st);
  return Q4B_OK;
}

int Model::step(const int32_t* toks, int C, int start, int last, int L, int32_t* next, float* logits,
                cudaStream_t st) {
  if (!toks) return set_error(Q4B_EINVAL, "model_step: null tokens");
  if (start < 0 || start + C > cfg.max_ctx || last < 0 || last >= C)
    return set_error(Q4B_EINVAL, "model_step: start %d + rows %d outside max_ctx %d or last %d outside the rows",
                     start, C, cfg.max_ctx, last);
  set_state_kernel<<<1, 1, 0, st>>>(state, start, last, 0);
  int rc = check_launch("model_step");
  if (rc) return rc;
  if ((rc = forward(toks, C, L, logits, nullptr, st))) return rc;
  if (next) {
    const cudaError_t e = cudaMemcpyAsync(next, &state->next_token, sizeof(int32_t), cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_err(e, "model_step: copy next token");
  }
  return Q4B_OK;
}

}  // namespace q4b

using namespace q4b;

extern "C" int q4b_model_create(const q4b_model_cfg* cfg, q4b_model** out) {
  if (!cfg || !out) return set_error(Q4B_EINVAL, "model_create: null argument");
  *out = nullptr;
  Model* m = new (std::nothrow) Model();
  if (!m) return set_error(Q4B_ENOMEM, "model_create: out of host memory");
  const int rc = m->init(*cfg);
  if (rc) {
    delete m;
    return rc;
  }
  *out = reinterpret_cast<q4b_model*>(m);
  return Q4B_OK;
}

extern "C" int q4b_model_set_layer(q4b_model* model, int layer, const q4b_layer_weights* w) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m || !w || layer < 0 || layer >= (int)m->layers.size()) return set_error(Q4B_EINVAL, "model_set_layer: bad layer");
  const int D = m->D, hd = m->hd;
  const auto ok = [](const q4b_qmat& q, int n, int k) {
    return q.qweight && q.scales && q.n == n && q.k == k && q.group >= 8 && q.group % 8 == 0 && k % q.group == 0;
  };
  if (!ok(w->wqkv, (m->H + 2 * m->Hkv) * hd, D) || !ok(w->wo, D, m->H * hd) || !ok(w->wgu, 2 * m->I, D) ||
      !ok(w->wdown, D, m->I))
    return set_error(Q4B_EINVAL, "model_set_layer: projection shapes do not match the (sharded) config");
  if (!w->ln_in || !w->ln_post || !w->k_cache || !w->v_cache)
    return set_error(Q4B_EINVAL, "model_set_layer: null norm weight or cache");
  m->layers[layer] = *w;
  m->mk_ready = false;
  return Q4B_OK;
}

extern "C" int q4b_model_set_head(q4b_model* model, const q4b_qmat* embed, const float* ln_f, const float* rope_cos,
                                  const float* rope_sin) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m || !embed || !ln_f || !rope_cos || !rope_sin || !embed->qweight || !embed->scales)
    return set_error(Q4B_EINVAL, "model_set_head: null argument");
  if (embed->n != m->cfg.vocab || embed->k != m->D || embed->group < 8 || m->D % embed->group)
    return set_error(Q4B_EINVAL, "model_set_head: embedding must be the full [vocab, dim] table");
  m->embed = *embed;
  m->ln_f = ln_f;
  m->rope_cos = rope_cos;
  m->rope_sin = rope_sin;
  m->mk_ready = false;
  return Q4B_OK;
}

extern "C" int q4b_model_step(q4b_model* model, const int32_t* tokens, int n_tokens, int start, int last, int L,
                              int32_t* next_token, float* logits, q4b_stream_t stream) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m) return set_error(Q4B_EINVAL, "model_step: null model");
  return m->step(tokens, n_tokens, start, last, L, next_token, logits, as_stream(stream));
}

extern "C" void q4b_model_destroy(q4b_model* model) { delete reinterpret_cast<Model*>(model); }

extern "C" int q4b_model_fail_decode(q4b_model* model) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m) return set_error(Q4B_EINVAL, "model_fail_decode: null model");
  if (!m->mk_usable(1, nullptr)) return set_error(Q4B_EUNSUPPORTED, "model_fail_decode: no persistent decode step");
  return m->mk_poison();
}

extern "C" int q4b_model_decode_path(const q4b_model* model) {
  const Model* m = reinterpret_cast<const Model*>(model);
  return m && m->mk_ready ? 1 : 0;
}

extern "C" size_t q4b_model_trace_events(const q4b_model* model) {
  const Model* m = reinterpret_cast<const Model*>(model);
  if (!m) return 0;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  return (size_t)sms * mk_trace_stride((int)m->layers.size());
}

extern "C" int q4b_model_set_trace(q4b_model* model, unsigned long long* events, size_t n_events) {
  Model* m = reinterpret_cast<Model*>(model);
  if (!m) return set_error(Q4B_EINVAL, "model_set_trace: null model");
  if (events && (n_events < q4b_model_trace_events(model) || reinterpret_cast<uintptr_t>(events) % 8))
    return set_error(Q4B_EINVAL, "model_set_trace: %zu events, 8-byte aligned, needed", q4b_model_trace_events(model));
  m->mk_trace = events;
  m->mk_trace_cap = events ? n_events : 0;
  return Q4B_OK;
}

extern "C" int q4b_device_status(int reset) {
  const unsigned v = linear_status(reset != 0) | gemm_status(reset != 0);
  return v ? Q4B_ETIMEOUT : Q4B_OK;
}
