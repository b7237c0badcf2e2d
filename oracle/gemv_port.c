/* C restatement of the reference's int8 GEMV, for checking and CPU timing.
 *
 * TEST INFRASTRUCTURE ONLY (tests/, smoke(), bench.py's CPU baseline).
 *
 *   gemv_port_i8_i8 : acc[o] = sum_i w[o,i] * x[i] in int32, exact -- the
 *                     integer core of rtl/gemv_i8.sv:13-76 as restated in
 *                     numpy by scripts/export_gemv_tv.py:49; optionally the
 *                     dequant y = acc * sx * sw[o] (export_gemv_tv.py:50).
 *   gemv_port_i8_f32: y[o] = (sum_i float(w[o,i]) * x[i]) * s[o], accumulated
 *                     left to right in fp32 like hls/src/gemv.hpp:28-42.
 * Rows are split across `threads` pthreads; each row's sum is sequential, so
 * the result does not depend on the thread count.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>

typedef struct {
  int32_t* acc; float* y; const int8_t* w; const float* sw; const int8_t* xi;
  const float* xf; float sx; long n0, n1, k; int kind;
} job_t;

static void* run(void* p) {
  job_t* j = (job_t*)p;
  for (long o = j->n0; o < j->n1; ++o) {
    const int8_t* row = j->w + o * j->k;
    if (j->kind == 0) {
      int32_t a = 0;
      for (long i = 0; i < j->k; ++i) a += (int32_t)row[i] * (int32_t)j->xi[i];
      if (j->acc) j->acc[o] = a;
      if (j->y) j->y[o] = ((float)a * j->sx) * j->sw[o];
    } else {
      float a = 0.0f;
      for (long i = 0; i < j->k; ++i) a += (float)row[i] * j->xf[i];
      j->y[o] = a * j->sw[o];
    }
  }
  return NULL;
}

static void split(job_t proto, long n, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  job_t jobs[256];
  int started = 0;
  for (int t = 0; t < threads; ++t) {
    jobs[t] = proto;
    jobs[t].n0 = n * t / threads;
    jobs[t].n1 = n * (t + 1) / threads;
    if (t == threads - 1 || pthread_create(&tid[t], NULL, run, &jobs[t]) != 0) {
      run(&jobs[t]);
    } else {
      ++started;
      continue;
    }
  }
  for (int t = 0; t < started; ++t) pthread_join(tid[t], NULL);
}

void gemv_port_i8_i8(int32_t* acc, float* y, const int8_t* w, const float* sw,
                     const int8_t* x, float sx, long n, long k, int threads) {
  job_t p = {acc, y, w, sw, x, NULL, sx, 0, 0, k, 0};
  split(p, n, threads);
}

void gemv_port_i8_f32(float* y, const int8_t* w, const float* s, const float* x,
                      long n, long k, int threads) {
  job_t p = {NULL, y, w, s, NULL, x, 0.0f, 0, 0, k, 1};
  split(p, n, threads);
}
