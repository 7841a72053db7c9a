/*
 * CPU restatement of the reference's int4 decode GEMV, for the tests and the CPU timing legs of
 * bench.py only (never on the product path).
 *
 * QLinear._gemv_fused (scripts/llm/llama_q4.py:74-90): with q the packed int32 weights viewed as
 * [N, K/G, G/8] and nibble b of word w holding k = 8w + b (stored q + 8, llama_q4.py:34-37),
 *
 *     y[n] = sum_g s[n, g] * sum_{w, b} x[g, 8w + b] * (((q[n, g, w] >> 4b) & 15) - 8)
 *
 * in fp32 (the reference folds the scale into every term before one sum; here each group's sum is
 * scaled once, the same value up to fp32 rounding). Rows are split over one pthread per CPU this
 * process may run on.
 *
 *   gcc -O3 -march=x86-64-v3 -pthread -shared -fPIC q4_cpu.c -o libq4cpu.so
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdint.h>
#include <string.h>

/* IEEE binary16 bit pattern -> float (normal, subnormal, zero, inf, nan) */
static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t exp = (h >> 10) & 31, man = h & 1023;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: man * 2^-24 */
      float f = (float)man * (1.0f / 16777216.0f);
      memcpy(&bits, &f, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

int q4cpu_threads(void) {
  cpu_set_t set;
  if (sched_getaffinity(0, sizeof(set), &set) == 0) {
    const int c = CPU_COUNT(&set);
    if (c > 0) return c > 64 ? 64 : c;
  }
  return 1;
}

static void gemv_rows(const int32_t* qweight, const uint16_t* scales, int r0, int r1, int k, int group,
                      const float* x, float* y) {
  const int words = k / 8, wpg = group / 8, ng = k / group;
  for (int r = r0; r < r1; ++r) {
    const uint32_t* q = (const uint32_t*)qweight + (size_t)r * words;
    const uint16_t* s = scales + (size_t)r * ng;
    float total = 0.0f;
    for (int g = 0; g < ng; ++g) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int w = g * wpg; w < (g + 1) * wpg; ++w) {
        const uint32_t v = q[w];
        const float* xx = x + 8 * (size_t)w;
        for (int b = 0; b < 8; ++b) acc[b] += xx[b] * (float)((int)((v >> (4 * b)) & 15u) - 8);
      }
      const float a = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
      total += half_to_float(s[g]) * a;
    }
    y[r] = total;
  }
}

typedef struct {
  const int32_t* qweight;
  const uint16_t* scales;
  int r0, r1, k, group;
  const float* x;
  float* y;
} job_t;

static void* gemv_job(void* arg) {
  const job_t* j = (const job_t*)arg;
  gemv_rows(j->qweight, j->scales, j->r0, j->r1, j->k, j->group, j->x, j->y);
  return 0;
}

/* y[n] = int4 GEMV of one x row, as above. group % 8 == 0, k % group == 0. */
void q4cpu_gemv(const int32_t* qweight, const uint16_t* scales, int n, int k, int group, const float* x, float* y) {
  int t = q4cpu_threads();
  if (t > n) t = n;
  pthread_t th[64];
  int made[64] = {0};
  job_t jobs[64];
  for (int i = 0; i < t; ++i)
    jobs[i] = (job_t){qweight, scales, (int)((long long)n * i / t), (int)((long long)n * (i + 1) / t), k, group, x, y};
  for (int i = 1; i < t; ++i) {
    made[i] = pthread_create(&th[i], 0, gemv_job, &jobs[i]) == 0;
    if (!made[i]) gemv_job(&jobs[i]); /* no thread: this one does the rows */
  }
  gemv_job(&jobs[0]);
  for (int i = 1; i < t; ++i)
    if (made[i]) pthread_join(th[i], 0);
}

/* The greedy head's argmax with the first maximum on ties (torch.argmax, llama_q4.py:238-239). */
int q4cpu_argmax(const float* v, int n) {
  int best = 0;
  for (int i = 1; i < n; ++i)
    if (v[i] > v[best]) best = i;
  return best;
}
