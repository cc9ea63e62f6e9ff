/*
 * q4_cpu_baseline.c -- the timed CPU baseline for bench.py (reference arm and
 * cpu_baseline leg).  TEST/BENCH INFRASTRUCTURE ONLY, never part of the
 * product.
 *
 * It restates the reference's CPU semantics for the operator (QLin::
 * cpu_dequant + linear, engine/src/qwen35.rs:327-352 and dequant_affine
 * :110-134): each weight is dequantised to bf16 (q * s + b, rounded to nearest
 * even) and the products are accumulated in f32.  The reference's own CPU
 * path cannot serve: it is Rust + candle (no toolchain here) and panics for
 * out >= 2 (qwen35.rs:6876-6880).  Work is split over output rows across
 * threads; each group's 64 weights are decoded once and reused for all m
 * activation rows, with 16 independent f32 accumulators per row so the
 * compiler vectorises the inner loop.
 */
#include "q4_oracle.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_rne(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  memcpy(&v, &u, 4);
  return v;
}

typedef struct {
  const uint32_t *wq;
  const uint16_t *sb;
  int sb_dtype, out, in, m;
  const float *x;
  float *y;
  int r0, r1;
} base_job;

#define MAXM 64

static void *base_rows(void *p) {
  base_job *j = (base_job *)p;
  const int in = j->in, ng = in / 64, m = j->m;
  float w[64];
  float acc[MAXM][16];
  for (int n = j->r0; n < j->r1; ++n) {
    for (int t = 0; t < m; ++t)
      for (int l = 0; l < 16; ++l) acc[t][l] = 0.0f;
    const uint32_t *wrow = j->wq + (size_t)n * (in / 8);
    const uint16_t *srow = j->sb + (size_t)n * 2 * ng;
    for (int g = 0; g < ng; ++g) {
      const float s = q4o_sb_to_f32(srow[g], j->sb_dtype);
      const float b = q4o_sb_to_f32(srow[ng + g], j->sb_dtype);
      for (int wd = 0; wd < 8; ++wd) {
        const uint32_t word = wrow[g * 8 + wd];
        for (int e = 0; e < 8; ++e)
          w[wd * 8 + e] = bf16_rne((float)((word >> (4 * e)) & 0xFu) * s + b);
      }
      for (int t = 0; t < m; ++t) {
        const float *xg = j->x + (size_t)t * in + (size_t)g * 64;
        for (int blk = 0; blk < 4; ++blk)
          for (int l = 0; l < 16; ++l) acc[t][l] += w[blk * 16 + l] * xg[blk * 16 + l];
      }
    }
    for (int t = 0; t < m; ++t) {
      float tot = 0.0f;
      for (int l = 0; l < 16; ++l) tot += acc[t][l];
      j->y[(size_t)t * j->out + n] = tot;
    }
  }
  return NULL;
}

int q4o_cpu_linear(const uint32_t *wq, const uint16_t *sb, int sb_dtype,
                   int out, int in, const float *x, int m, float *y,
                   int nthreads) {
  if (m > MAXM || in % 64 != 0) return -1;
  if (nthreads < 1) nthreads = 1;
  if (nthreads > out) nthreads = out;
  pthread_t th[256];
  base_job jobs[256];
  if (nthreads > 256) nthreads = 256;
  int chunk = (out + nthreads - 1) / nthreads;
  for (int t = 0; t < nthreads; ++t) {
    int b = t * chunk, e = b + chunk < out ? b + chunk : out;
    jobs[t] = (base_job){wq, sb, sb_dtype, out, in, m, x, y, b, e};
  }
  for (int t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, base_rows, &jobs[t]);
  base_rows(&jobs[0]);
  for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
  return nthreads;
}
