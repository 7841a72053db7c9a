// gemm_bench: the CUDA counterpart of the gemm tuner's on-device harness
// (gemm/harness/vk_gemm_bench.c:1-13, 389-492). Same files, same protocol, same output:
//
//   manifest line   <name> <shape_dir> <candidate>          ('#' starts a comment)
//   candidate       <kernel>:<key=value,...>, kernel 1 = tcgen05, 2 = CUDA cores, 3 = tcgen05
//                   persistent stream-K, e.g. 1:bn=128,stages=6,split=2   or   3:bn=256,stages=4   or   2:
//                   (keys: bn, stages, split; 0 / absent = auto)
//   shape_dir       meta.txt "M N K LA LB TOL" (TOL < 0: no check); A.bin, B.bin fp16 in the stored
//                   layout of the BLAS letters; Cref.bin fp32 row-major M x N (absent if TOL < 0)
//   per candidate   poison C with 0xFF bytes (fp16 NaN), run once, max|C - Cref| / max|Cref| against
//                   TOL; warm up (--warmup-ms before the first candidate, 50 ms before the others);
//                   time `iters` back-to-back calls per rep with CUDA events (iters from a one-call
//                   estimate and --target-ms, 1..2000), median and minimum of --reps reps
//   output          {"name","ok","err","us","us_min","iters","reps"} per candidate, or
//                   {"name","ok":false,"error":...}; a sticky CUDA error prints "device_lost" and
//                   exits 3, the way the reference reports VK_ERROR_DEVICE_LOST.
//
// --cold: flush L2 (a 256 MB write) before every timed call and time each call alone (events
// around the GEMM only), for problems whose operands would otherwise stay in the 126 MB L2.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "q4b.h"

namespace {

struct Shape {
  std::string dir;
  int M = 0, N = 0, K = 0;
  char la = 'N', lb = 'N';
  double tol = -1;
  std::vector<float> cref;
  void *A = nullptr, *B = nullptr, *C = nullptr;
  size_t c_bytes = 0;
};

std::string g_cur;
double g_warmup_ms = 500;

double now_ms() {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

void fail_line(const std::string& name, const std::string& why) {
  printf("{\"name\":\"%s\",\"ok\":false,\"error\":\"%s\"}\n", name.c_str(), why.c_str());
  fflush(stdout);
}

// A CUDA error that leaves the context unusable ends the process (exit 3), like device_lost.
bool cuda_ok(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return true;
  fprintf(stderr, "%s: %s\n", what, cudaGetErrorString(e));
  if (cudaPeekAtLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    fail_line(g_cur, "device_lost");
    exit(3);
  }
  return false;
}

bool read_file(const std::string& path, std::vector<char>& out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  out.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  return true;
}

void free_shape(Shape& s) {
  cudaFree(s.A);
  cudaFree(s.B);
  cudaFree(s.C);
  s = Shape();
}

bool load_shape(const std::string& dir, Shape& s) {
  if (s.dir == dir) return true;
  free_shape(s);
  std::ifstream meta(dir + "/meta.txt");
  if (!meta) return false;
  meta >> s.M >> s.N >> s.K >> s.la >> s.lb >> s.tol;
  if (!meta || s.M <= 0 || s.N <= 0 || s.K <= 0) return false;
  std::vector<char> a, b;
  const size_t a_bytes = (size_t)s.M * s.K * 2, b_bytes = (size_t)s.K * s.N * 2;
  if (!read_file(dir + "/A.bin", a) || a.size() != a_bytes) return false;
  if (!read_file(dir + "/B.bin", b) || b.size() != b_bytes) return false;
  if (s.tol >= 0) {
    std::vector<char> c;
    if (!read_file(dir + "/Cref.bin", c) || c.size() != (size_t)s.M * s.N * 4) return false;
    s.cref.resize((size_t)s.M * s.N);
    memcpy(s.cref.data(), c.data(), c.size());
  }
  s.c_bytes = (size_t)s.M * s.N * 2;
  if (!cuda_ok(cudaMalloc(&s.A, a_bytes), "cudaMalloc A") || !cuda_ok(cudaMalloc(&s.B, b_bytes), "cudaMalloc B") ||
      !cuda_ok(cudaMalloc(&s.C, s.c_bytes), "cudaMalloc C"))
    return false;
  if (!cuda_ok(cudaMemcpy(s.A, a.data(), a_bytes, cudaMemcpyHostToDevice), "copy A") ||
      !cuda_ok(cudaMemcpy(s.B, b.data(), b_bytes, cudaMemcpyHostToDevice), "copy B"))
    return false;
  s.dir = dir;
  return true;
}

bool parse_candidate(const std::string& text, q4b_gemm_cfg& cfg) {
  cfg = q4b_gemm_cfg{};
  const size_t colon = text.find(':');
  if (colon == std::string::npos) return false;
  cfg.kernel = atoi(text.substr(0, colon).c_str());
  std::stringstream rest(text.substr(colon + 1));
  std::string kv;
  while (std::getline(rest, kv, ',')) {
    if (kv.empty()) continue;
    const size_t eq = kv.find('=');
    if (eq == std::string::npos) return false;
    const std::string k = kv.substr(0, eq);
    const int v = atoi(kv.c_str() + eq + 1);
    if (k == "bn") cfg.bn = v;
    else if (k == "stages") cfg.stages = v;
    else if (k == "split") cfg.split = v;
    else return false;
  }
  return cfg.kernel >= 1 && cfg.kernel <= 3;
}

struct Runner {
  Shape* s;
  q4b_gemm_cfg cfg;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  int call() {
    return q4b_gemm_f16(s->A, s->B, s->C, s->M, s->N, s->K, s->la, s->lb, &cfg, ws, ws_bytes, nullptr);
  }
};

void run_candidate(const std::string& name, const std::string& dir, const std::string& cand, Shape& s,
                   double target_ms, int reps, bool cold, void* flush, size_t flush_bytes) {
  g_cur = name;
  if (!load_shape(dir, s)) {
    s.dir.clear();
    fail_line(name, "shape load failed");
    return;
  }
  Runner r{&s, {}};
  if (!parse_candidate(cand, r.cfg)) return fail_line(name, "bad candidate");
  const long long ws = q4b_gemm_f16_workspace(s.M, s.N, s.K, s.la, s.lb, &r.cfg);
  if (ws < 0) return fail_line(name, std::string("rejected: ") + q4b_last_error());
  if (ws > 0) {
    if (!cuda_ok(cudaMalloc(&r.ws, (size_t)ws), "cudaMalloc ws")) return fail_line(name, "workspace");
    cuda_ok(cudaMemset(r.ws, 0, (size_t)ws), "memset ws");
    r.ws_bytes = (size_t)ws;
  }
  // correctness: poison C, run once, compare
  cuda_ok(cudaMemset(s.C, 0xFF, s.c_bytes), "poison C");
  if (r.call() != Q4B_OK) {
    fail_line(name, std::string("launch: ") + q4b_last_error());
    cudaFree(r.ws);
    return;
  }
  cuda_ok(cudaDeviceSynchronize(), "first run");
  double err = -1;
  bool ok = true;
  if (s.tol >= 0) {
    std::vector<__half> c((size_t)s.M * s.N);
    cuda_ok(cudaMemcpy(c.data(), s.C, s.c_bytes, cudaMemcpyDeviceToHost), "read C");
    double maxref = 1e-6, maxerr = 0;
    for (float v : s.cref) maxref = std::max(maxref, (double)std::fabs(v));
    for (size_t i = 0; i < c.size(); ++i) {
      const double e = std::fabs((double)__half2float(c[i]) - s.cref[i]);
      if (!(e == e)) {
        maxerr = INFINITY;
        break;
      }
      maxerr = std::max(maxerr, e);
    }
    err = maxerr / maxref;
    ok = err <= s.tol;
    if (!std::isfinite(err)) err = 1e30;
  }
  // warm-up: keep the GPU busy before timing
  static bool warmed = false;
  const double t0 = now_ms(), budget = warmed ? 50.0 : g_warmup_ms;
  while (now_ms() - t0 < budget) {
    r.call();
    cuda_ok(cudaDeviceSynchronize(), "warm-up");
  }
  warmed = true;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  auto time_calls = [&](int iters) -> double {
    if (!cold) {
      cudaEventRecord(e0);
      for (int i = 0; i < iters; ++i) r.call();
      cudaEventRecord(e1);
      cuda_ok(cudaEventSynchronize(e1), "timing");
      float ms = 0;
      cudaEventElapsedTime(&ms, e0, e1);
      return ms * 1e3 / iters;
    }
    double total = 0;
    for (int i = 0; i < iters; ++i) {
      cudaMemsetAsync(flush, i & 0xFF, flush_bytes);
      cudaEventRecord(e0);
      r.call();
      cudaEventRecord(e1);
      cuda_ok(cudaEventSynchronize(e1), "timing");
      float ms = 0;
      cudaEventElapsedTime(&ms, e0, e1);
      total += ms * 1e3;
    }
    return total / iters;
  };
  const double one = time_calls(1);
  if (one > 100e3) reps = 1;
  int iters = (int)(target_ms * 1e3 / (one > 1 ? one : 1));
  iters = std::min(std::max(iters, 1), 2000);
  reps = std::min(std::max(reps, 1), 64);
  std::vector<double> t(reps);
  for (int i = 0; i < reps; ++i) t[i] = time_calls(iters);
  std::sort(t.begin(), t.end());
  printf("{\"name\":\"%s\",\"ok\":%s,\"err\":%.3e,\"us\":%.3f,\"us_min\":%.3f,\"iters\":%d,\"reps\":%d}\n", name.c_str(),
         ok ? "true" : "false", err, t[reps / 2], t[0], iters, reps);
  fflush(stdout);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(r.ws);
  if (q4b_device_status(1) != Q4B_OK) fprintf(stderr, "%s: a bounded device wait timed out\n", name.c_str());
}

}  // namespace

int main(int argc, char** argv) {
  const char* manifest = nullptr;
  double target_ms = 30;
  int reps = 5;
  bool cold = false;
  for (int i = 1; i < argc; ++i) {
    if (!strncmp(argv[i], "--manifest=", 11)) manifest = argv[i] + 11;
    else if (!strncmp(argv[i], "--target-ms=", 12)) target_ms = atof(argv[i] + 12);
    else if (!strncmp(argv[i], "--reps=", 7)) reps = atoi(argv[i] + 7);
    else if (!strncmp(argv[i], "--warmup-ms=", 12)) g_warmup_ms = atof(argv[i] + 12);
    else if (!strcmp(argv[i], "--cold")) cold = true;
  }
  if (!manifest) {
    fprintf(stderr, "usage: %s --manifest=FILE [--target-ms=30] [--reps=5] [--warmup-ms=500] [--cold]\n", argv[0]);
    return 2;
  }
  std::ifstream f(manifest);
  if (!f) {
    fprintf(stderr, "no manifest %s\n", manifest);
    return 2;
  }
  void* flush = nullptr;
  const size_t flush_bytes = 256u << 20;
  if (cold && !cuda_ok(cudaMalloc(&flush, flush_bytes), "cudaMalloc flush")) return 1;
  Shape s;
  std::string line;
  while (std::getline(f, line)) {
    std::stringstream ls(line);
    std::string name, dir, cand;
    if (!(ls >> name) || name[0] == '#') continue;
    if (!(ls >> dir >> cand)) {
      fail_line(name, "bad manifest line");
      continue;
    }
    run_candidate(name, dir, cand, s, target_ms, reps, cold, flush, flush_bytes);
  }
  free_shape(s);
  cudaFree(flush);
  return 0;
}
