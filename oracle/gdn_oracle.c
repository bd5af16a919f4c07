/*
 * gdn_oracle.c -- CPU oracle for the gated delta rule.  TEST INFRASTRUCTURE ONLY: loaded by
 * tests/, __graft_entry__.smoke() and bench.py's CPU legs as the checker, never by the
 * product library.
 *
 * A float64 restatement of the per-token recurrence archbench uses as ground truth,
 * archbench/layers/nsgdn.py:408-417 (nsgdn_ref), extended by an initial state and a final
 * state output:
 *     S = exp(la_t) S;  r = v_t - S k_t;  S += r u_t^T;  y_t = S q_t      (nsgdn.py:413-416)
 * with u_t = beta_t k_t when no write vector is given (the plain GDN write direction,
 * nsgdn.py:69).  Parallel over (b, h) with pthreads; each (b, h) is one sequential chain.
 * Pinned against archbench's own outputs by tests/test_oracle.py.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>

typedef struct {
  const float *q, *k, *u, *beta, *v, *la;
  const double* s0;
  double *y, *s_out;
  int64_t B, T, H, DK, DV;
  int64_t next; /* next (b, h) to claim */
  pthread_mutex_t lock;
  int failed;
} job_t;

static void run_head(job_t* J, int64_t bh, double* S, double* w) {
  const int64_t T = J->T, H = J->H, DK = J->DK, DV = J->DV;
  int64_t b = bh / H, h = bh % H;
  if (J->s0)
    memcpy(S, J->s0 + bh * DV * DK, sizeof(double) * DV * DK);
  else
    memset(S, 0, sizeof(double) * DV * DK);
  for (int64_t t = 0; t < T; ++t) {
    int64_t tok = (b * T + t) * H + h;
    const float* qt = J->q + tok * DK;
    const float* kt = J->k + tok * DK;
    const float* vt = J->v + tok * DV;
    double a = exp((double)J->la[tok]);
    if (J->u) {
      for (int64_t j = 0; j < DK; ++j) w[j] = (double)J->u[tok * DK + j];
    } else {
      double bt = (double)J->beta[tok];
      for (int64_t j = 0; j < DK; ++j) w[j] = bt * (double)kt[j];
    }
    double* yt = J->y + tok * DV;
    for (int64_t i = 0; i < DV; ++i) {
      double* Si = S + i * DK;
      double sk = 0.0;
      for (int64_t j = 0; j < DK; ++j) {
        Si[j] *= a;
        sk += Si[j] * (double)kt[j];
      }
      double r = (double)vt[i] - sk;
      double sq = 0.0;
      for (int64_t j = 0; j < DK; ++j) {
        Si[j] += r * w[j];
        sq += Si[j] * (double)qt[j];
      }
      yt[i] = sq;
    }
  }
  if (J->s_out) memcpy(J->s_out + bh * DV * DK, S, sizeof(double) * DV * DK);
}

static void* worker(void* arg) {
  job_t* J = (job_t*)arg;
  double* S = (double*)malloc(sizeof(double) * J->DV * J->DK);
  double* w = (double*)malloc(sizeof(double) * J->DK);
  if (!S || !w) {
    pthread_mutex_lock(&J->lock);
    J->failed = 1;
    pthread_mutex_unlock(&J->lock);
  } else {
    for (;;) {
      pthread_mutex_lock(&J->lock);
      int64_t bh = J->next++;
      pthread_mutex_unlock(&J->lock);
      if (bh >= J->B * J->H) break;
      run_head(J, bh, S, w);
    }
  }
  free(S);
  free(w);
  return NULL;
}

/* Inputs are float32 (already rounded to the kernel's input dtype), contiguous
 * [B][T][H][D]; la and beta are (B, T, H).  s0 and s_out are (B, H, DV, DK) float64; s0 may
 * be NULL (zero state).  y is [B][T][H][DV] float64.  `nthreads` <= 0 means one thread.
 * Returns 0, or -1 on bad arguments or allocation failure. */
int gdn_oracle_recurrence(const float* q, const float* k, const float* u, const float* beta,
                          const float* v, const float* la, const double* s0, double* y,
                          double* s_out, int64_t B, int64_t T, int64_t H, int64_t DK,
                          int64_t DV, int nthreads) {
  if (!q || !k || !v || !la || !y || (!u && !beta)) return -1;
  if (B <= 0 || T < 0 || H <= 0 || DK <= 0 || DV <= 0) return -1;
  job_t J = {q, k, u, beta, v, la, s0, y, s_out, B, T, H, DK, DV, 0,
             PTHREAD_MUTEX_INITIALIZER, 0};
  int n = nthreads > 0 ? nthreads : 1;
  if (n > B * H) n = (int)(B * H);
  if (n > 256) n = 256;
  pthread_t th[256];
  int started = 0;
  for (int i = 1; i < n; ++i)
    if (pthread_create(&th[started], NULL, worker, &J) == 0) ++started;
  worker(&J);
  for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
  return J.failed ? -1 : 0;
}
