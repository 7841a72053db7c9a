// Generation runner: the scheduler of runner/llm_runner.c:143-262 over the native model, with one
// captured CUDA graph per (phase, bucket) instead of one compiled IREE function per bucket.
//
//   pick_bucket       smallest bucket >= needed, or the largest under schedule "max" (:143-149)
//   prefill           chunks at start = 0, C, 2C, ... padded with zeros, L = pick_bucket(start + C),
//                     last = rows - 1 (:205-223)
//   decode            the prefill token counts towards max_new; stop after a stop id; L =
//                     pick_bucket(pos + 1); stop when no bucket fits (:225-246)
//   warm-up           each used (phase, bucket) once before timing, like the reference (:175-203)
//   report            the JSON object of :249-262
// Decode steps are device-resident: the graph reads the token and position from the model's step
// state and its argmax epilogue writes the next token, appends it to a device log, checks the stop
// ids and advances the position, so steps run back to back without host round trips. With
// sync_every_step the runner instead copies each step's inputs in and the token out and checks
// stop ids on the host, the per-call protocol of the reference (:91-141).
#include <algorithm>
#include <chrono>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <map>
#include <new>
#include <string>
#include <vector>

#include "model.h"

namespace q4b {

struct Runner {
  Model* model = nullptr;
  q4b_runner_opts opts{};
  std::vector<int> buckets;
  cudaStream_t stream = nullptr;
  std::map<std::pair<int, int>, cudaGraphExec_t> graphs;  // (phase 0 prefill / 1 decode, L)
  // pinned staging; every asynchronous copy of one generate call reads its own slot, so the host
  // never rewrites a buffer a pending copy still reads
  int32_t* h_tokens = nullptr;     // [max_ctx + chunk]: chunk s at offset s
  DecodeState* h_state = nullptr;  // [n_slots] step states
  int32_t* h_next = nullptr;       // first token read back after the prefill
  int n_slots = 0, slot = 0;
  int32_t* d_log = nullptr;
  int log_cap = 0;
  std::vector<cudaEvent_t> events;
  std::string report;

  ~Runner() {
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
    for (cudaEvent_t e : events) cudaEventDestroy(e);
    if (h_tokens) cudaFreeHost(h_tokens);
    if (h_state) cudaFreeHost(h_state);
    if (h_next) cudaFreeHost(h_next);
    if (d_log) cudaFree(d_log);
    if (stream) cudaStreamDestroy(stream);
  }

  int pick_bucket(int needed) const {
    if (opts.schedule == 1) return buckets.back();
    for (int b : buckets)
      if (b >= needed) return b;
    return -1;
  }

  int ensure_events(size_t n) {
    while (events.size() < n) {
      cudaEvent_t e;
      if (cudaEventCreate(&e) != cudaSuccess) return set_error(Q4B_ECUDA, "runner: cudaEventCreate");
      events.push_back(e);
    }
    return Q4B_OK;
  }

  // the step for (phase, L): prefill reads tokens from the model's token buffer, decode reads the
  // last token from the state; both take positions from the state
  int record_step(int phase, int L) {
    if (phase == 0) return model->forward(model->tokens, opts.chunk, L, nullptr, nullptr, stream);
    return model->forward(&model->state->next_token, 1, L, nullptr, d_log, stream);
  }

  int launch_step(int phase, int L) {
    if (!opts.use_graphs) return record_step(phase, L);
    auto key = std::make_pair(phase, L);
    auto it = graphs.find(key);
    if (it == graphs.end()) {
      cudaGraph_t g = nullptr;
      cudaError_t e = cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal);
      if (e != cudaSuccess) return set_error(Q4B_ECUDA, "runner: begin capture: %s", cudaGetErrorString(e));
      const int rc = record_step(phase, L);
      e = cudaStreamEndCapture(stream, &g);
      if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
      }
      if (e != cudaSuccess) return set_error(Q4B_ECUDA, "runner: end capture: %s", cudaGetErrorString(e));
      cudaGraphExec_t ge = nullptr;
      e = cudaGraphInstantiate(&ge, g, 0);
      cudaGraphDestroy(g);
      if (e != cudaSuccess) return set_error(Q4B_ECUDA, "runner: instantiate: %s", cudaGetErrorString(e));
      it = graphs.emplace(key, ge).first;
    }
    const cudaError_t e = cudaGraphLaunch(it->second, stream);
    return e == cudaSuccess ? Q4B_OK : set_error(Q4B_ECUDA, "runner: graph launch: %s", cudaGetErrorString(e));
  }

  DecodeState* new_state() {
    DecodeState* st = &h_state[slot++ % n_slots];
    memset(st, 0, sizeof(DecodeState));
    return st;
  }

  int put_state(const DecodeState* src) {
    const cudaError_t e =
        cudaMemcpyAsync(model->state, src, offsetof(DecodeState, best), cudaMemcpyHostToDevice, stream);
    return e == cudaSuccess ? Q4B_OK : set_error(Q4B_ECUDA, "runner: state copy: %s", cudaGetErrorString(e));
  }

  int generate(const int32_t* prompt, int n, int max_new, const int32_t* stops, int n_stop, int32_t* out, int* n_out,
               q4b_report* rep);
};

static double ms_between(cudaEvent_t a, cudaEvent_t b) {
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, a, b);
  return ms;
}

int Runner::generate(const int32_t* prompt, int n, int max_new, const int32_t* stops, int n_stop, int32_t* out,
                     int* n_out, q4b_report* rep) {
  using clk = std::chrono::steady_clock;
  const int C = opts.chunk;
  const int max_ctx = model->cfg.max_ctx;
  if (!prompt || !out || !n_out) return set_error(Q4B_EINVAL, "runner_generate: null argument");
  if (n <= 0) return set_error(Q4B_EINVAL, "runner_generate: empty prompt");
  if (max_new < 1) return set_error(Q4B_EINVAL, "runner_generate: max_new must be >= 1");
  if (n_stop < 0 || n_stop > 16) return set_error(Q4B_EINVAL, "runner_generate: at most 16 stop ids");
  if (n + max_new > max_ctx || (n + C - 1) / C * C > max_ctx)
    return set_error(Q4B_EINVAL, "runner_generate: prompt %d + new %d exceeds max_ctx %d", n, max_new, max_ctx);
  int rc;
  if ((rc = model->check_ready())) return rc;
  model->mk_usable(1, stream);  // persistent decode tables are built here, before any graph capture
  if ((rc = ensure_events(2 * ((n + C - 1) / C + max_new) + 4))) return rc;
  // functions the schedule will use (:181-189)
  std::vector<int> used_prefill, used_decode;
  for (int s = 0; s < n; s += C) {
    const int L = pick_bucket(s + C);
    if (L < 0) return set_error(Q4B_EINVAL, "runner_generate: no bucket >= %d", s + C);
    if (std::find(used_prefill.begin(), used_prefill.end(), L) == used_prefill.end()) used_prefill.push_back(L);
  }
  for (int pos = n; pos < n + max_new - 1; ++pos) {
    const int L = pick_bucket(pos + 1);
    if (L >= 0 && std::find(used_decode.begin(), used_decode.end(), L) == used_decode.end()) used_decode.push_back(L);
  }
  // warm-up: zeros at position 0 (writes KV rows [0, C) that the prefill overwrites, like the
  // reference); graphs are captured on first use here, outside the timed region
  const auto t_warm0 = clk::now();
  if (cudaStreamSynchronize(stream) != cudaSuccess) return set_error(Q4B_ECUDA, "runner: stream");
  // a failure recorded by an earlier request is not this one's (a poisoned persistent step sets it again)
  if (cudaMemset(&model->state->status, 0, sizeof(int32_t)) != cudaSuccess)
    return set_error(Q4B_ECUDA, "runner: state reset");
  slot = 0;
  memset(h_tokens, 0, sizeof(int32_t) * C);
  const DecodeState* zero_state = new_state();
  for (int w = 0; w < std::max(1, opts.warmup); ++w) {
    for (int L : used_prefill) {
      if (cudaMemcpyAsync(model->tokens, h_tokens, sizeof(int32_t) * C, cudaMemcpyHostToDevice, stream) != cudaSuccess)
        return set_error(Q4B_ECUDA, "runner: token copy");
      if ((rc = put_state(zero_state)) || (rc = launch_step(0, L))) return rc;
    }
    for (int L : used_decode) {
      if ((rc = put_state(zero_state)) || (rc = launch_step(1, L))) return rc;
    }
  }
  if (cudaStreamSynchronize(stream) != cudaSuccess)
    return set_error(Q4B_ECUDA, "runner: warm-up: %s", cudaGetErrorString(cudaGetLastError()));
  slot = 0;
  const double warm_ms = std::chrono::duration<double, std::milli>(clk::now() - t_warm0).count();

  // ---- prefill (:205-223) ----
  std::vector<std::pair<int, double>> chunk_ms, step_ms;
  std::vector<int> chunk_L, step_L;
  int ev = 0;
  const auto t_pre0 = clk::now();
  cudaEventRecord(events[ev++], stream);
  for (int s = 0; s < n; s += C) {
    const int m = std::min(C, n - s);
    int32_t* chunk = h_tokens + s;
    memset(chunk, 0, sizeof(int32_t) * C);
    memcpy(chunk, prompt + s, sizeof(int32_t) * m);
    DecodeState* stt = new_state();
    stt->start = s;
    stt->last = m - 1;
    if (cudaMemcpyAsync(model->tokens, chunk, sizeof(int32_t) * C, cudaMemcpyHostToDevice, stream) != cudaSuccess)
      return set_error(Q4B_ECUDA, "runner: token copy");
    const int L = pick_bucket(s + C);
    if ((rc = put_state(stt)) || (rc = launch_step(0, L))) return rc;
    cudaEventRecord(events[ev++], stream);
    chunk_L.push_back(L);
  }
  if (cudaMemcpyAsync(h_next, &model->state->next_token, sizeof(int32_t), cudaMemcpyDeviceToHost, stream) !=
          cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return set_error(Q4B_ECUDA, "runner: prefill: %s", cudaGetErrorString(cudaGetLastError()));
  const int32_t first = *h_next;
  const double prefill_ms = std::chrono::duration<double, std::milli>(clk::now() - t_pre0).count();
  for (size_t i = 0; i < chunk_L.size(); ++i) chunk_ms.push_back({chunk_L[i], ms_between(events[i], events[i + 1])});

  // ---- decode (:225-246) ----
  int n_gen = 1;
  out[0] = first;
  bool stopped = false;
  for (int i = 0; i < n_stop; ++i) stopped |= first == stops[i];
  const int ev0 = ev;
  const auto t_dec0 = clk::now();
  int steps = 0;
  if (!stopped && max_new > 1) {
    DecodeState* d0 = new_state();
    d0->start = n;
    d0->last = 0;
    d0->next_token = first;
    d0->advance = 1;
    d0->n_stop = n_stop;
    d0->log_cap = max_new - 1;
    for (int i = 0; i < n_stop; ++i) d0->stop_ids[i] = stops[i];
    if ((rc = put_state(d0))) return rc;
    cudaEventRecord(events[ev++], stream);
    int pos = n;
    while (n_gen + steps < max_new) {
      const int L = pick_bucket(pos + 1);
      if (L < 0) break;
      if (opts.sync_every_step) {
        // the reference's per-call protocol: inputs in, token out, stop check on the host
        DecodeState* ds = new_state();
        *ds = *d0;
        ds->start = pos;
        ds->next_token = out[n_gen + steps - 1];
        if ((rc = put_state(ds))) return rc;
      }
      if ((rc = launch_step(1, L))) return rc;
      cudaEventRecord(events[ev++], stream);
      step_L.push_back(L);
      ++steps;
      ++pos;
      if (opts.sync_every_step) {
        if (cudaMemcpyAsync(h_next, &model->state->next_token, sizeof(int32_t), cudaMemcpyDeviceToHost, stream) !=
                cudaSuccess ||
            cudaStreamSynchronize(stream) != cudaSuccess)
          return set_error(Q4B_ECUDA, "runner: decode step: %s", cudaGetErrorString(cudaGetLastError()));
        const int32_t tok = *h_next;
        out[n_gen + steps - 1] = tok;
        bool stop = false;
        for (int i = 0; i < n_stop; ++i) stop |= tok == stops[i];
        if (stop) break;
      }
    }
    if (cudaStreamSynchronize(stream) != cudaSuccess)
      return set_error(Q4B_ECUDA, "runner: decode: %s", cudaGetErrorString(cudaGetLastError()));
    int32_t dstat = 0;  // the persistent decode step records a bounded wait that gave up here
    if (cudaMemcpy(&dstat, &model->state->status, sizeof(dstat), cudaMemcpyDeviceToHost) != cudaSuccess)
      return set_error(Q4B_ECUDA, "runner: state read");
    if (dstat) return set_error(Q4B_ETIMEOUT, "runner: a decode step gave up a bounded device wait");
    if (!opts.sync_every_step) {
      DecodeState fin;
      if (cudaMemcpy(&fin, model->state, sizeof(DecodeState), cudaMemcpyDeviceToHost) != cudaSuccess ||
          cudaMemcpy(out + 1, d_log, sizeof(int32_t) * std::min(fin.n_gen, max_new - 1), cudaMemcpyDeviceToHost) !=
              cudaSuccess)
        return set_error(Q4B_ECUDA, "runner: token log copy");
      steps = std::min(steps, fin.n_gen);  // steps after a stop id produced nothing
    }
  }
  const double decode_wall_ms = std::chrono::duration<double, std::milli>(clk::now() - t_dec0).count();
  double decode_ms = 0.0;
  for (int i = 0; i < (int)step_L.size(); ++i) {
    const double t = ms_between(events[ev0 + i], events[ev0 + i + 1]);
    if (i < steps) step_ms.push_back({step_L[i], t});
    if (i < steps) decode_ms += t;
  }
  n_gen += steps;
  *n_out = n_gen;
  const int st = linear_status(true);
  if (st) return set_error(Q4B_ETIMEOUT, "runner: a bounded device wait gave up");

  // ---- report (:249-262) ----
  if (rep) {
    rep->warmup_ms = warm_ms;
    rep->prefill_ms = prefill_ms;
    rep->ttft_ms = prefill_ms;
    rep->prefill_tok_s = n / (prefill_ms / 1e3);
    rep->decode_ms = decode_ms;
    rep->decode_wall_ms = decode_wall_ms;
    rep->decode_steps = steps;
    rep->decode_tok_s = steps > 0 ? steps / (decode_ms / 1e3) : 0.0;
    rep->prompt_tokens = n;
    rep->new_tokens = n_gen;
  }
  char buf[256];
  std::string js;
  snprintf(buf, sizeof(buf), "{\"schedule\":\"%s\",\"chunk\":%d,\"prompt_tokens\":%d,\"new_tokens\":%d,",
           opts.schedule == 1 ? "max" : "bucketed", C, n, n_gen);
  js += buf;
  snprintf(buf, sizeof(buf), "\"warmup_ms\":%.1f,\"prefill_ms\":%.1f,\"prefill_tok_s\":%.2f,\"ttft_ms\":%.1f,", warm_ms,
           prefill_ms, n / (prefill_ms / 1e3), prefill_ms);
  js += buf;
  snprintf(buf, sizeof(buf), "\"decode_ms\":%.3f,\"decode_steps\":%d,\"decode_tok_s\":%.2f,", decode_ms, steps,
           steps > 0 ? steps / (decode_ms / 1e3) : 0.0);
  js += buf;
  js += "\"chunks\":[";
  for (size_t i = 0; i < chunk_ms.size(); ++i) {
    snprintf(buf, sizeof(buf), "%s[%d,%.3f]", i ? "," : "", chunk_ms[i].first, chunk_ms[i].second);
    js += buf;
  }
  js += "],\"steps\":[";
  for (size_t i = 0; i < step_ms.size(); ++i) {
    snprintf(buf, sizeof(buf), "%s[%d,%.4f]", i ? "," : "", step_ms[i].first, step_ms[i].second);
    js += buf;
  }
  js += "],\"tokens\":[";
  for (int i = 0; i < n_gen; ++i) {
    snprintf(buf, sizeof(buf), "%s%d", i ? "," : "", out[i]);
    js += buf;
  }
  js += "]}";
  report = js;
  return Q4B_OK;
}

}  // namespace q4b

using namespace q4b;

extern "C" int q4b_runner_create(q4b_model* model, const q4b_runner_opts* opts, q4b_runner** out) {
  if (!model || !opts || !out) return set_error(Q4B_EINVAL, "runner_create: null argument");
  *out = nullptr;
  Model* m = reinterpret_cast<Model*>(model);
  if (opts->n_buckets < 1 || opts->n_buckets > 16 || !opts->buckets)
    return set_error(Q4B_EINVAL, "runner_create: 1..16 buckets");
  if (opts->chunk < 1 || opts->chunk > m->cfg.max_chunk)
    return set_error(Q4B_EINVAL, "runner_create: chunk %d outside 1..max_chunk %d", opts->chunk, m->cfg.max_chunk);
  if (opts->schedule != 0 && opts->schedule != 1) return set_error(Q4B_EINVAL, "runner_create: schedule 0 or 1");
  for (int i = 0; i < opts->n_buckets; ++i) {
    if (opts->buckets[i] < 1 || opts->buckets[i] > m->cfg.max_ctx || (i && opts->buckets[i] <= opts->buckets[i - 1]))
      return set_error(Q4B_EINVAL, "runner_create: buckets must ascend within 1..max_ctx");
  }
  Runner* r = new (std::nothrow) Runner();
  if (!r) return set_error(Q4B_ENOMEM, "runner_create: host memory");
  r->model = m;
  r->opts = *opts;
  r->buckets.assign(opts->buckets, opts->buckets + opts->n_buckets);
  r->opts.buckets = nullptr;
  // the token log holds up to max_ctx tokens and is never reallocated (captured graphs point at it)
  r->log_cap = m->cfg.max_ctx;
  r->n_slots = m->cfg.max_ctx + 64;
  if (cudaStreamCreateWithFlags(&r->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMallocHost(&r->h_tokens, sizeof(int32_t) * (m->cfg.max_ctx + opts->chunk)) != cudaSuccess ||
      cudaMallocHost(&r->h_state, sizeof(DecodeState) * r->n_slots) != cudaSuccess ||
      cudaMallocHost(&r->h_next, sizeof(int32_t)) != cudaSuccess ||
      cudaMalloc(&r->d_log, sizeof(int32_t) * r->log_cap) != cudaSuccess) {
    delete r;
    return set_error(Q4B_ENOMEM, "runner_create: stream / pinned buffers");
  }
  *out = reinterpret_cast<q4b_runner*>(r);
  return Q4B_OK;
}

extern "C" int q4b_runner_generate(q4b_runner* runner, const int32_t* prompt, int n_prompt, int max_new,
                                   const int32_t* stop_ids, int n_stop, int32_t* out_tokens, int* n_out,
                                   q4b_report* report) {
  Runner* r = reinterpret_cast<Runner*>(runner);
  if (!r) return set_error(Q4B_EINVAL, "runner_generate: null runner");
  return r->generate(prompt, n_prompt, max_new, stop_ids, n_stop, out_tokens, n_out, report);
}

extern "C" const char* q4b_runner_report_json(q4b_runner* runner) {
  Runner* r = reinterpret_cast<Runner*>(runner);
  return r ? r->report.c_str() : "";
}

extern "C" void q4b_runner_destroy(q4b_runner* runner) { delete reinterpret_cast<Runner*>(runner); }
