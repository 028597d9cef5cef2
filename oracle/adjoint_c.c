/* CPU restatement of the clean Picard adjoint in C (float32, pthreads over entries).
 *
 * TEST INFRASTRUCTURE ONLY: the compiled CPU baseline that bench.py times beside
 * the GPU adjoint (the configs[3] micro-benchmark), at one thread and at every
 * host core, and that tests/test_oracle_cpu.py checks against the float64 numpy
 * oracle (oracle/deq_oracle.py: adjoint).  Nothing in aideen_b200/ links or loads it.
 *
 * It restates staged_adjoint_picard_clean.wgsl:143-248 (the clean step without
 * Anderson mixing): per (token, slot) entry with pre = branch + h*,
 *   rms = sqrt(mean(pre^2) + 1e-6), inv = 1 / max(rms, 1e-6),
 *   den = max(d * rms^3, 1e-6),
 *   v' = rhs + beta * (NS * inv * v - pre * (sum(v * NS * pre) / den)) + (1 - beta) * v,
 * starting from v = rhs, for `iters` iterations; then
 *   g_pre = beta * (NS * inv * v - pre * (sum(v * NS * pre) / den)).
 * The step is diagonal plus rank one, so each iteration is one dot product and
 * one fused update over d: a = beta * NS * inv + (1 - beta), w = beta * NS * pre,
 * v' = rhs + a * v - ((w . v) / den) * pre.
 *
 * Layouts: hstar, branch, rhs_slot, v, g_pre are [N][h][d]; rhs_tok is [N][d]
 * (added to every slot scaled by 1/h) or NULL; NS is [d].
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdlib.h>
#include <unistd.h>

#if defined(__x86_64__) && defined(__GNUC__) && !defined(__clang__)
/* one binary for any x86-64 host: the loader picks the widest vector ISA present */
#define CLONES __attribute__((target_clones("avx512f", "avx2", "default")))
#else
#define CLONES
#endif

CLONES
static void adjoint_entry(const float *restrict hs, const float *restrict br, const float *restrict rs,
                          const float *restrict rt, float inv_h, const float *restrict NS, int d, int iters,
                          float beta, float *restrict pre, float *restrict a, float *restrict w,
                          float *restrict rhs, float *restrict v, float *restrict g) {
  float ss = 0.f;
#pragma omp simd reduction(+ : ss)
  for (int j = 0; j < d; ++j) {
    const float p = br[j] + hs[j];
    pre[j] = p;
    ss += p * p;
  }
  const float r = sqrtf(ss / (float)d + 1e-6f);
  const float inv = 1.f / fmaxf(r, 1e-6f);
  const float den = fmaxf((float)d * r * r * r, 1e-6f);
  const float ninv_den = -1.f / den;
  for (int j = 0; j < d; ++j) {
    a[j] = beta * NS[j] * inv + (1.f - beta);
    w[j] = beta * NS[j] * pre[j];
    float b = rs ? rs[j] : 0.f;
    if (rt) b += inv_h * rt[j];
    rhs[j] = b;
    v[j] = b;
  }
  for (int k = 0; k < iters; ++k) {
    float c = 0.f;
#pragma omp simd reduction(+ : c)
    for (int j = 0; j < d; ++j) c += w[j] * v[j];
    const float nc = c * ninv_den;
#pragma omp simd
    for (int j = 0; j < d; ++j) v[j] = rhs[j] + a[j] * v[j] + nc * pre[j];
  }
  float c = 0.f;
#pragma omp simd reduction(+ : c)
  for (int j = 0; j < d; ++j) c += w[j] * v[j];
  const float nc = c * ninv_den;
  if (g)
    for (int j = 0; j < d; ++j) g[j] = (a[j] - (1.f - beta)) * v[j] + nc * pre[j];
}

typedef struct {
  const float *hstar, *branch, *rhs_slot, *rhs_tok, *NS;
  int h, d, iters;
  float beta;
  float *v, *g;
  long e0, e1;
  int bad;
} job_t;

static void *run_job(void *arg) {
  job_t *j = (job_t *)arg;
  float *buf = (float *)malloc(sizeof(float) * 4 * (size_t)j->d);
  if (!buf) {
    j->bad = 1;
    return NULL;
  }
  for (long e = j->e0; e < j->e1; ++e) {
    const long n = e / j->h;
    const size_t o = (size_t)e * j->d;
    adjoint_entry(j->hstar + o, j->branch + o, j->rhs_slot ? j->rhs_slot + o : NULL,
                  j->rhs_tok ? j->rhs_tok + (size_t)n * j->d : NULL, 1.f / (float)j->h, j->NS, j->d, j->iters,
                  j->beta, buf, buf + j->d, buf + 2 * j->d, buf + 3 * j->d, j->v + o, j->g ? j->g + o : NULL);
  }
  free(buf);
  return NULL;
}

/* Returns 0, or -1 for a bad argument or a failed allocation / thread start.
 * threads <= 0: one thread per online host core.  Entries are split into
 * contiguous ranges, one per thread. */
int oracle_adjoint_c(const float *hstar, const float *branch, const float *rhs_slot, const float *rhs_tok,
                     const float *NS, int N, int h, int d, int iters, float beta, float *v_out,
                     float *gpre_out, int threads) {
  if (N < 0 || h <= 0 || d <= 0 || iters < 0 || !hstar || !branch || !NS || !v_out) return -1;
  if (threads <= 0) threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (threads < 1) threads = 1;
  const long E = (long)N * h;
  if (threads > E) threads = E > 0 ? (int)E : 1;
  job_t *jobs = (job_t *)calloc((size_t)threads, sizeof(job_t));
  pthread_t *tid = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
  if (!jobs || !tid) {
    free(jobs);
    free(tid);
    return -1;
  }
  int bad = 0, started = 0;
  for (int t = 0; t < threads; ++t) {
    job_t *j = &jobs[t];
    j->hstar = hstar; j->branch = branch; j->rhs_slot = rhs_slot; j->rhs_tok = rhs_tok; j->NS = NS;
    j->h = h; j->d = d; j->iters = iters; j->beta = beta; j->v = v_out; j->g = gpre_out;
    j->e0 = E * t / threads;
    j->e1 = E * (t + 1) / threads;
  }
  /* thread 0's range runs on the calling thread */
  for (int t = 1; t < threads; ++t) {
    if (pthread_create(&tid[t], NULL, run_job, &jobs[t]) != 0) {
      bad = 1;
      break;
    }
    started = t;
  }
  if (!bad) run_job(&jobs[0]);
  for (int t = 1; t <= started; ++t) pthread_join(tid[t], NULL);
  for (int t = 0; t < threads; ++t) bad |= jobs[t].bad;
  free(jobs);
  free(tid);
  return bad ? -1 : 0;
}
