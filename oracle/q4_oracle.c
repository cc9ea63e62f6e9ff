/*
 * q4_oracle.c -- CPU restatement of th-engine's Q4 affine matmul path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never part of the
 * product.  See q4_oracle.h for the parity status and conventions; every
 * function cites the reference lines it restates.
 */
#include "q4_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* scalar conversions                                                        */
/* ------------------------------------------------------------------------ */

static inline uint32_t f32_bits(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  return u;
}
static inline float bits_f32(uint32_t u) {
  float v;
  memcpy(&v, &u, 4);
  return v;
}

/* Round to nearest even, the kernels' bfloat conversion.  Same rule as the
 * reference's floatToBf16 (LinearNumerics.hpp:19-23); NaN stays NaN. */
uint16_t q4o_f32_to_bf16(float v) {
  uint32_t u = f32_bits(v);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float q4o_bf16_to_f32(uint16_t v) { return bits_f32((uint32_t)v << 16); }

uint16_t q4o_f32_to_f16(float v) {
  _Float16 h = (_Float16)v;
  uint16_t u;
  memcpy(&u, &h, 2);
  return u;
}
float q4o_f16_to_f32(uint16_t v) {
  _Float16 h;
  memcpy(&h, &v, 2);
  return (float)h;
}
float q4o_sb_to_f32(uint16_t v, int sb_dtype) {
  return sb_dtype == Q4O_SB_F16 ? q4o_f16_to_f32(v) : q4o_bf16_to_f32(v);
}
static uint16_t f32_to_sb(float v, int sb_dtype) {
  return sb_dtype == Q4O_SB_F16 ? q4o_f32_to_f16(v) : q4o_f32_to_bf16(v);
}
void q4o_f32_to_bf16_n(const float *src, uint16_t *dst, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = q4o_f32_to_bf16(src[i]);
}
void q4o_bf16_to_f32_n(const uint16_t *src, float *dst, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = q4o_bf16_to_f32(src[i]);
}
static inline float bf16_round(float v) { return q4o_bf16_to_f32(q4o_f32_to_bf16(v)); }

/* ------------------------------------------------------------------------ */
/* threading helper                                                          */
/* ------------------------------------------------------------------------ */

typedef void (*range_fn)(void *ctx, int begin, int end);
typedef struct {
  range_fn fn;
  void *ctx;
  int begin, end;
} range_job;

static void *range_thread(void *p) {
  range_job *j = (range_job *)p;
  j->fn(j->ctx, j->begin, j->end);
  return NULL;
}

/* Splits [0, n) into nthreads contiguous chunks.  Each chunk writes disjoint
 * outputs, so results do not depend on the thread count. */
static void parallel_for(int n, int nthreads, range_fn fn, void *ctx) {
  if (nthreads < 1) nthreads = 1;
  if (nthreads > n) nthreads = n > 0 ? n : 1;
  if (nthreads == 1) {
    fn(ctx, 0, n);
    return;
  }
  pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nthreads);
  range_job *jobs = (range_job *)malloc(sizeof(range_job) * (size_t)nthreads);
  int chunk = (n + nthreads - 1) / nthreads;
  for (int t = 0; t < nthreads; ++t) {
    int b = t * chunk, e = b + chunk < n ? b + chunk : n;
    jobs[t] = (range_job){fn, ctx, b, e};
    pthread_create(&th[t], NULL, range_thread, &jobs[t]);
  }
  for (int t = 0; t < nthreads; ++t) pthread_join(th[t], NULL);
  free(th);
  free(jobs);
}

/* ------------------------------------------------------------------------ */
/* generators                                                                */
/* ------------------------------------------------------------------------ */

/* qwen35.rs:6889-6892 */
uint64_t q4o_lcg(uint64_t *s) {
  *s = *s * 6364136223846793005ull + 1442695040888963407ull;
  return *s >> 33;
}

/* qwen35.rs:6896-6915: words = lcg ^ (lcg << 16) (two draws per word, in
 * that order); then per row and group a scale 0.002 + (lcg % 1000) * 2e-5 and
 * a bias ((lcg % 2001) - 1000) * 1e-4, both as f32 then bf16. */
void q4o_rand_qlin(int out, int in, uint64_t seed, uint32_t *wq, uint16_t *sb) {
  uint64_t s = seed;
  int ng = in / 64;
  size_t words = (size_t)out * (size_t)in / 8;
  for (size_t i = 0; i < words; ++i) {
    uint32_t a = (uint32_t)q4o_lcg(&s);
    uint32_t b = (uint32_t)q4o_lcg(&s);
    wq[i] = a ^ (b << 16);
  }
  for (int o = 0; o < out; ++o)
    for (int g = 0; g < ng; ++g) {
      float sc = 0.002f + (float)(q4o_lcg(&s) % 1000) * 2e-5f;
      float bi = ((float)(q4o_lcg(&s) % 2001) - 1000.0f) * 1e-4f;
      sb[(size_t)o * 2 * ng + g] = q4o_f32_to_bf16(sc);
      sb[(size_t)o * 2 * ng + ng + g] = q4o_f32_to_bf16(bi);
    }
}

/* qwen35.rs:6917-6923: ((lcg % 4001) - 2000) / 1000 as f32, then bf16. */
void q4o_rand_x(int in, uint64_t seed, uint16_t *x) {
  uint64_t s = seed;
  for (int i = 0; i < in; ++i)
    x[i] = q4o_f32_to_bf16(((float)(q4o_lcg(&s) % 4001) - 2000.0f) / 1000.0f);
}

static inline uint32_t lcg32(uint64_t *s) {
  *s = *s * 6364136223846793005ull + 1442695040888963407ull;
  return (uint32_t)(*s >> 32);
}

void q4o_rand_pf_case(int total_out, int in, int m, uint64_t *state,
                      uint32_t *tw, uint16_t *tsb, uint16_t *x) {
  int ng = in / 64, padded = (total_out + 255) / 256 * 256;
  for (size_t i = 0; i < (size_t)padded * ng * 8; ++i) tw[i] = lcg32(state);
  for (size_t i = 0; i < (size_t)2 * padded * ng; ++i) {
    float u = (float)(lcg32(state) % 1000) / 1000.0f;
    tsb[i] = q4o_f32_to_bf16(i < (size_t)padded * ng ? 0.002f + 0.01f * u : -0.05f + 0.02f * u);
  }
  for (size_t i = 0; i < (size_t)m * in; ++i)
    x[i] = q4o_f32_to_bf16((float)(lcg32(state) % 2000) / 500.0f - 2.0f);
}

/* ------------------------------------------------------------------------ */
/* quantiser                                                                 */
/* ------------------------------------------------------------------------ */

typedef struct {
  const float *w;
  int in, gs, sb_dtype;
  uint32_t *wq;
  uint16_t *sb;
} quant_ctx;

static void quant_rows(void *p, int r0, int r1) {
  quant_ctx *c = (quant_ctx *)p;
  int in = c->in, gs = c->gs, ng = in / gs;
  for (int r = r0; r < r1; ++r) {
    const float *row = c->w + (size_t)r * in;
    uint32_t *wrow = c->wq + (size_t)r * (in / 8);
    memset(wrow, 0, sizeof(uint32_t) * (size_t)(in / 8));
    for (int g = 0; g < ng; ++g) {
      float lo = row[g * gs], hi = row[g * gs];
      for (int k = 1; k < gs; ++k) {
        float v = row[g * gs + k];
        lo = v < lo ? v : lo;
        hi = v > hi ? v : hi;
      }
      uint16_t s16 = f32_to_sb((hi - lo) / 15.0f, c->sb_dtype);
      uint16_t b16 = f32_to_sb(lo, c->sb_dtype);
      double s = q4o_sb_to_f32(s16, c->sb_dtype), b = q4o_sb_to_f32(b16, c->sb_dtype);
      c->sb[(size_t)r * 2 * ng + g] = s16;
      c->sb[(size_t)r * 2 * ng + ng + g] = b16;
      for (int k = 0; k < gs; ++k) {
        int q = 0;
        if (s > 0) {
          double t = nearbyint(((double)row[g * gs + k] - b) / s);
          q = t < 0 ? 0 : t > 15 ? 15 : (int)t;
        }
        int e = g * gs + k;
        wrow[e / 8] |= (uint32_t)q << (4 * (e % 8));
      }
    }
  }
}

void q4o_quantize(const float *w, int out, int in, int gs, int sb_dtype,
                  uint32_t *wq, uint16_t *sb, int nthreads) {
  quant_ctx c = {w, in, gs, sb_dtype, wq, sb};
  parallel_for(out, nthreads, quant_rows, &c);
}

/* ------------------------------------------------------------------------ */
/* layouts                                                                   */
/* ------------------------------------------------------------------------ */

/* QLin::tiled, qwen35.rs:629-697 (addressing q4woff/q4sb,
 * quant_kernel.rs:1085-1101). */
void q4o_mlx_to_tiled(const uint32_t *wq, const uint16_t *sb, int out, int in,
                      uint32_t *tw, uint16_t *tsb) {
  int ng = in / 64, tiles = (out + 255) / 256, padded = tiles * 256;
  memset(tw, 0, sizeof(uint32_t) * (size_t)tiles * ng * 2048);
  memset(tsb, 0, sizeof(uint16_t) * (size_t)2 * padded * ng);
  size_t bias_base = (size_t)padded * ng;
  for (int row = 0; row < out; ++row) {
    int t = row / 256, col = row % 256;
    for (int g = 0; g < ng; ++g) {
      size_t d = (size_t)t * ng * 2048 + (size_t)g * 2048 + (size_t)col * 8;
      memcpy(&tw[d], &wq[(size_t)row * ng * 8 + (size_t)g * 8], 32);
      size_t si = ((size_t)t * ng + g) * 256 + col;
      tsb[si] = sb[(size_t)row * 2 * ng + g];
      tsb[bias_base + si] = sb[(size_t)row * 2 * ng + ng + g];
    }
  }
}

void q4o_tiled_to_mlx(const uint32_t *tw, const uint16_t *tsb, int out, int in,
                      uint32_t *wq, uint16_t *sb) {
  int ng = in / 64, tiles = (out + 255) / 256, padded = tiles * 256;
  size_t bias_base = (size_t)padded * ng;
  for (int row = 0; row < out; ++row) {
    int t = row / 256, col = row % 256;
    for (int g = 0; g < ng; ++g) {
      size_t d = (size_t)t * ng * 2048 + (size_t)g * 2048 + (size_t)col * 8;
      memcpy(&wq[(size_t)row * ng * 8 + (size_t)g * 8], &tw[d], 32);
      size_t si = ((size_t)t * ng + g) * 256 + col;
      sb[(size_t)row * 2 * ng + g] = tsb[si];
      sb[(size_t)row * 2 * ng + ng + g] = tsb[bias_base + si];
    }
  }
}

/* q4PackedBytes, WeightStore.cpp:57-60: elements / 16 * 9. */
size_t q4o_slab_bytes(int out, int in) { return (size_t)out * (size_t)in / 16 * 9; }

/* moe_q4_slab (moe_expert_slab.h:15-28) and packSlab (moe_metal_test.mm:
 * 126-145): nibble (n, k) sits at nibble index parameter(n, k/64)*64 + k%64,
 * low nibble first; parameter(n, g) = ((n/256)*groups + g)*256 + n%256.  The
 * weight bytes are the tiled layout's words byte for byte. */
void q4o_mlx_to_slab(const uint32_t *wq, const uint16_t *sb, int out, int in,
                     uint8_t *slab) {
  size_t elements = (size_t)out * in;
  int ng = in / 64;
  uint8_t *w = slab;
  uint16_t *sc = (uint16_t *)(slab + elements / 2);
  uint16_t *bi = (uint16_t *)(slab + elements / 2 + elements / 32);
  for (int n = 0; n < out; ++n)
    for (int g = 0; g < ng; ++g) {
      size_t prm = ((size_t)(n / 256) * ng + g) * 256 + n % 256;
      memcpy(w + prm * 32, &wq[(size_t)n * ng * 8 + (size_t)g * 8], 32);
      sc[prm] = sb[(size_t)n * 2 * ng + g];
      bi[prm] = sb[(size_t)n * 2 * ng + ng + g];
    }
}

void q4o_slab_to_mlx(const uint8_t *slab, int out, int in, uint32_t *wq,
                     uint16_t *sb) {
  size_t elements = (size_t)out * in;
  int ng = in / 64;
  const uint8_t *w = slab;
  const uint16_t *sc = (const uint16_t *)(slab + elements / 2);
  const uint16_t *bi = (const uint16_t *)(slab + elements / 2 + elements / 32);
  for (int n = 0; n < out; ++n)
    for (int g = 0; g < ng; ++g) {
      size_t prm = ((size_t)(n / 256) * ng + g) * 256 + n % 256;
      memcpy(&wq[(size_t)n * ng * 8 + (size_t)g * 8], w + prm * 32, 32);
      sb[(size_t)n * 2 * ng + g] = sc[prm];
      sb[(size_t)n * 2 * ng + ng + g] = bi[prm];
    }
}

/* The B200 "frag" layout (token-horizon_b200/csrc/thq4_common.cuh): rows pad
 * to slabs of 16*ts rows = ts tiles of 16 (the library uses ts = 8).  Chunk
 * ((slab*ng + g)*ts + t) holds the 512 nibble bytes of tile t of the slab for
 * group g; lane l owns bytes [16l, 16l+16) = words j = 0..3; with r = l/4,
 * c = l%4, the nibble at bits 4i..4i+3 (i = 0..7) of word j holds
 *   row = 16(ts*slab + t) + r + 8((i>>1)&1),
 *   k   = 64g + 32(j>>1) + 8(j&1) + 16(i&1) + 2c + (i>>2).
 * Scales: 64 bytes per chunk, eight quads {s_r, b_r, s_r+8, b_r+8}. */
size_t q4o_frag_qw_bytes(int out, int in, int ts) {
  return (size_t)((out + 16 * ts - 1) / (16 * ts)) * ts * (size_t)(in / 64) * 512;
}
size_t q4o_frag_sb_bytes(int out, int in, int ts) {
  return (size_t)((out + 16 * ts - 1) / (16 * ts)) * ts * (size_t)(in / 64) * 64;
}

/* k of the nibble at bits 4i..4i+3 of word j for lane column c, group g */
static inline int frag_k(int g, int j, int i, int c) {
  return g * 64 + 32 * (j >> 1) + 8 * (j & 1) + 16 * (i & 1) + 2 * c + (i >> 2);
}

static inline uint32_t mlx_nibble(const uint32_t *wq, int in, int row, int k) {
  return (wq[(size_t)row * (in / 8) + k / 8] >> (4 * (k % 8))) & 0xFu;
}

void q4o_mlx_to_frag(const uint32_t *wq, const uint16_t *sb, int out, int in, int ts,
                     uint32_t *fq, uint16_t *fsb) {
  int ng = in / 64, slabs = (out + 16 * ts - 1) / (16 * ts);
  for (int sl = 0; sl < slabs; ++sl)
    for (int g = 0; g < ng; ++g)
      for (int t = 0; t < ts; ++t) {
        size_t chunk = ((size_t)sl * ng + g) * ts + t;
        int row0 = (sl * ts + t) * 16;
        for (int lane = 0; lane < 32; ++lane) {
          int r = lane >> 2, c = lane & 3;
          for (int j = 0; j < 4; ++j) {
            uint32_t word = 0;
            for (int i = 0; i < 8; ++i) {
              int row = row0 + r + 8 * ((i >> 1) & 1);
              int k = frag_k(g, j, i, c);
              uint32_t q = row < out ? mlx_nibble(wq, in, row, k) : 0;
              word |= q << (4 * i);
            }
            fq[(chunk * 32 + lane) * 4 + j] = word;
          }
        }
        for (int r = 0; r < 8; ++r)
          for (int half = 0; half < 2; ++half) {
            int row = row0 + r + 8 * half;
            uint16_t s = 0, bb = 0;
            if (row < out) {
              s = sb[(size_t)row * 2 * ng + g];
              bb = sb[(size_t)row * 2 * ng + ng + g];
            }
            fsb[(chunk * 8 + r) * 4 + 2 * half] = s;
            fsb[(chunk * 8 + r) * 4 + 2 * half + 1] = bb;
          }
      }
}

void q4o_frag_to_mlx(const uint32_t *fq, const uint16_t *fsb, int out, int in, int ts,
                     uint32_t *wq, uint16_t *sb) {
  int ng = in / 64, slabs = (out + 16 * ts - 1) / (16 * ts);
  memset(wq, 0, sizeof(uint32_t) * (size_t)out * (in / 8));
  for (int sl = 0; sl < slabs; ++sl)
    for (int g = 0; g < ng; ++g)
      for (int t = 0; t < ts; ++t) {
        size_t chunk = ((size_t)sl * ng + g) * ts + t;
        int row0 = (sl * ts + t) * 16;
        for (int lane = 0; lane < 32; ++lane) {
          int r = lane >> 2, c = lane & 3;
          for (int j = 0; j < 4; ++j) {
            uint32_t word = fq[(chunk * 32 + lane) * 4 + j];
            for (int i = 0; i < 8; ++i) {
              int row = row0 + r + 8 * ((i >> 1) & 1);
              int k = frag_k(g, j, i, c);
              if (row >= out) continue;
              uint32_t q = (word >> (4 * i)) & 0xFu;
              wq[(size_t)row * (in / 8) + k / 8] |= q << (4 * (k % 8));
            }
          }
        }
        for (int r = 0; r < 8; ++r)
          for (int half = 0; half < 2; ++half) {
            int row = row0 + r + 8 * half;
            if (row >= out) continue;
            sb[(size_t)row * 2 * ng + g] = fsb[(chunk * 8 + r) * 4 + 2 * half];
            sb[(size_t)row * 2 * ng + ng + g] = fsb[(chunk * 8 + r) * 4 + 2 * half + 1];
          }
      }
}

/* ------------------------------------------------------------------------ */
/* products                                                                  */
/* ------------------------------------------------------------------------ */

typedef struct {
  const uint32_t *wq;
  const uint16_t *sb;
  int sb_dtype, out, in, m;
  const float *x;
  double *y;
} lin_ctx;

/* Per-group kernel semantics: acc += s * sum(q*x) + b * sum(x)
 * (quant_kernel.rs:1994-2001, 2887-2890, 4111-4122), in fp64. */
static void lin_group_rows(void *p, int r0, int r1) {
  lin_ctx *c = (lin_ctx *)p;
  int in = c->in, ng = in / 64;
  for (int n = r0; n < r1; ++n) {
    for (int t = 0; t < c->m; ++t) {
      const float *x = c->x + (size_t)t * in;
      double acc = 0;
      for (int g = 0; g < ng; ++g) {
        double s = q4o_sb_to_f32(c->sb[(size_t)n * 2 * ng + g], c->sb_dtype);
        double b = q4o_sb_to_f32(c->sb[(size_t)n * 2 * ng + ng + g], c->sb_dtype);
        double dot = 0, sum = 0;
        for (int k = g * 64; k < g * 64 + 64; ++k) {
          double q = (double)mlx_nibble(c->wq, in, n, k);
          dot += q * (double)x[k];
          sum += (double)x[k];
        }
        acc += s * dot + b * sum;
      }
      c->y[(size_t)t * c->out + n] = acc;
    }
  }
}

void q4o_linear_group(const uint32_t *wq, const uint16_t *sb, int sb_dtype,
                      int out, int in, const float *x, int m, double *y,
                      int nthreads) {
  lin_ctx c = {wq, sb, sb_dtype, out, in, m, x, y};
  parallel_for(out, nthreads, lin_group_rows, &c);
}

/* half::bf16::from_f64: one round-to-nearest-even from f64 to bf16 (8
 * significant bits), returned as the exact f32 value of the bf16. */
static inline float f64_to_bf16_value(double v) {
  if (v == 0.0 || !isfinite(v)) return (float)v;
  int ex;
  (void)frexp(v, &ex); /* |v| in [2^(ex-1), 2^ex) */
  int e = ex - 8;      /* spacing of the bf16 binade holding v */
  if (e < -133) e = -133;
  double r = ldexp(nearbyint(ldexp(v, -e)), e);
  return (float)r;
}

/* dequant_affine (qwen35.rs:110-134): w = bf16(f64(q) * f64(s) + f64(b)). */
static inline float dequant_one(uint32_t q, uint16_t s, uint16_t b, int sb_dtype) {
  double v = (double)q * (double)q4o_sb_to_f32(s, sb_dtype) +
             (double)q4o_sb_to_f32(b, sb_dtype);
  return f64_to_bf16_value(v);
}

void q4o_dequant_bf16(const uint32_t *wq, const uint16_t *sb, int sb_dtype,
                      int out, int in, uint16_t *w) {
  int ng = in / 64;
  for (int n = 0; n < out; ++n)
    for (int k = 0; k < in; ++k) {
      int g = k / 64;
      w[(size_t)n * in + k] = q4o_f32_to_bf16(
          dequant_one(mlx_nibble(wq, in, n, k), sb[(size_t)n * 2 * ng + g],
                      sb[(size_t)n * 2 * ng + ng + g], sb_dtype));
    }
}

static void lin_dequant_rows(void *p, int r0, int r1) {
  lin_ctx *c = (lin_ctx *)p;
  int in = c->in, ng = in / 64;
  double *wrow = (double *)malloc(sizeof(double) * (size_t)in);
  for (int n = r0; n < r1; ++n) {
    for (int k = 0; k < in; ++k) {
      int g = k / 64;
      wrow[k] = dequant_one(mlx_nibble(c->wq, in, n, k), c->sb[(size_t)n * 2 * ng + g],
                            c->sb[(size_t)n * 2 * ng + ng + g], c->sb_dtype);
    }
    for (int t = 0; t < c->m; ++t) {
      const float *x = c->x + (size_t)t * in;
      double acc = 0;
      for (int k = 0; k < in; ++k) acc += wrow[k] * (double)x[k];
      c->y[(size_t)t * c->out + n] = acc;
    }
  }
  free(wrow);
}

void q4o_linear_dequant(const uint32_t *wq, const uint16_t *sb, int sb_dtype,
                        int out, int in, const float *x, int m, double *y,
                        int nthreads) {
  lin_ctx c = {wq, sb, sb_dtype, out, in, m, x, y};
  parallel_for(out, nthreads, lin_dequant_rows, &c);
}

/* quant_kernel.rs:2039-2046: gate = float(bfloat(acc_g)), up = float(bfloat(
 * acc_u)), value = gate / (1 + exp(-gate)) * up, output bfloat(value).  The
 * kernel spells exp(-g) as exp2(-log2(e) g); the reference test computes it
 * with exp (qwen35.rs:7003-7008).  f32 throughout. */
uint16_t q4o_silu_mul_bf16(float gate, float up) {
  float g = bf16_round(gate), u = bf16_round(up);
  float v = g / (1.0f + expf(-g)) * u;
  return q4o_f32_to_bf16(v);
}

void q4o_gate_up(const uint32_t *wq, const uint16_t *sb, int sb_dtype, int out,
                 int in, int up_row, int half, const float *x, int m,
                 uint16_t *out_bf16, int nthreads) {
  double *y = (double *)malloc(sizeof(double) * (size_t)m * out);
  q4o_linear_group(wq, sb, sb_dtype, out, in, x, m, y, nthreads);
  for (int t = 0; t < m; ++t)
    for (int i = 0; i < half; ++i)
      out_bf16[(size_t)t * half + i] = q4o_silu_mul_bf16(
          (float)y[(size_t)t * out + i], (float)y[(size_t)t * out + up_row + i]);
  free(y);
}

/* ------------------------------------------------------------------------ */
/* MoE                                                                       */
/* ------------------------------------------------------------------------ */

/* moe_route_select_q8 (moe.metal:323-360): rank by descending score, ties to
 * the lowest expert id; weight_r = exp(s_r - s_0) / sum_o exp(s_o - s_0) in
 * f32, rounded to bf16. */
void q4o_moe_select(const uint16_t *logits, int T, int E, int k, uint32_t *ids,
                    uint16_t *weights) {
  float *sc = (float *)malloc(sizeof(float) * (size_t)E);
  float *ord = (float *)malloc(sizeof(float) * (size_t)k);
  for (int t = 0; t < T; ++t) {
    for (int e = 0; e < E; ++e) sc[e] = q4o_bf16_to_f32(logits[(size_t)t * E + e]);
    for (int r = 0; r < k; ++r) {
      int best = -1;
      for (int e = 0; e < E; ++e) {
        if (sc[e] == -INFINITY) continue;
        if (best < 0 || sc[e] > sc[best]) best = e; /* strict: lowest id wins ties */
      }
      if (best < 0) best = 0;
      ids[(size_t)t * k + r] = (uint32_t)best;
      ord[r] = sc[best];
      sc[best] = -INFINITY;
    }
    float den = 0.0f;
    for (int o = 0; o < k; ++o) den += expf(ord[o] - ord[0]);
    for (int r = 0; r < k; ++r)
      weights[(size_t)t * k + r] = q4o_f32_to_bf16(expf(ord[r] - ord[0]) / den);
  }
  free(sc);
  free(ord);
}

/* moeMaximumTiles (MoE.hpp:72-77) without the shared expert's tiles. */
uint32_t q4o_moe_max_tiles(int T, int E, int k, int tile_rows) {
  uint32_t routed = (uint32_t)T * (uint32_t)k;
  uint32_t a = routed / (uint32_t)tile_rows + (uint32_t)E;
  return a < routed ? a : routed;
}

/* moe_group_routes (moe.metal:368-449): per-expert counts, tile prefix in
 * expert order, descriptors {expert, min(tile_rows, count - t*tile_rows)},
 * padding rows ~0u; routes scattered in ascending route order (stable). */
int q4o_moe_group(const uint32_t *ids, int T, int k, int E, int tile_rows,
                  int max_tiles, uint32_t *tiles, uint32_t *grouped_routes,
                  uint32_t *route_rows) {
  int routes = T * k;
  uint32_t *count = (uint32_t *)calloc((size_t)E, sizeof(uint32_t));
  uint32_t *offset = (uint32_t *)calloc((size_t)E, sizeof(uint32_t));
  uint32_t *cursor = (uint32_t *)calloc((size_t)E, sizeof(uint32_t));
  for (int r = 0; r < routes; ++r) count[ids[r]]++;
  uint32_t ntiles = 0;
  for (int e = 0; e < E; ++e) {
    offset[e] = ntiles;
    ntiles += (count[e] + (uint32_t)tile_rows - 1) / (uint32_t)tile_rows;
  }
  if ((int)ntiles > max_tiles) {
    free(count);
    free(offset);
    free(cursor);
    return -1;
  }
  for (size_t i = 0; i < (size_t)max_tiles * tile_rows; ++i) grouped_routes[i] = 0xFFFFFFFFu;
  for (size_t i = 0; i < (size_t)max_tiles * 2; ++i) tiles[i] = 0;
  for (int e = 0; e < E; ++e) {
    uint32_t nt = (count[e] + (uint32_t)tile_rows - 1) / (uint32_t)tile_rows;
    for (uint32_t t = 0; t < nt; ++t) {
      uint32_t live = count[e] - t * (uint32_t)tile_rows;
      tiles[(offset[e] + t) * 2] = (uint32_t)e;
      tiles[(offset[e] + t) * 2 + 1] = live < (uint32_t)tile_rows ? live : (uint32_t)tile_rows;
    }
  }
  for (int r = 0; r < routes; ++r) {
    uint32_t e = ids[r];
    uint32_t row = offset[e] * (uint32_t)tile_rows + cursor[e]++;
    grouped_routes[row] = (uint32_t)r;
    route_rows[r] = row;
  }
  free(count);
  free(offset);
  free(cursor);
  return (int)ntiles;
}

typedef struct {
  const uint16_t *x;
  int T, H, I, k; /* k: routes per token (the routed slots plus a shared one) */
  const uint32_t *ids;
  const uint32_t *gu_wq, *dn_wq;
  const uint16_t *gu_sb, *dn_sb;
  int sb_dtype;
  uint16_t *h_out, *d_out;
  uint32_t E; /* expert id E selects the shared expert */
  const uint32_t *sh_gu_wq, *sh_dn_wq;
  const uint16_t *sh_gu_sb, *sh_dn_sb;
} moe_ctx;

/* The CPU `project` of moe_metal_test.mm:147-165 (fp32 group dot and sum,
 * total += dot * s + sum * b, bf16 result) for a single row. */
static void project_row(const uint32_t *wq, const uint16_t *sb, int sb_dtype,
                        int out, int in, const float *x, float *y) {
  int ng = in / 64;
  for (int n = 0; n < out; ++n) {
    float total = 0.0f;
    for (int g = 0; g < ng; ++g) {
      float dot = 0.0f, sum = 0.0f;
      for (int kk = g * 64; kk < g * 64 + 64; ++kk) {
        dot += x[kk] * (float)mlx_nibble(wq, in, n, kk);
        sum += x[kk];
      }
      total += dot * q4o_sb_to_f32(sb[(size_t)n * 2 * ng + g], sb_dtype) +
               sum * q4o_sb_to_f32(sb[(size_t)n * 2 * ng + ng + g], sb_dtype);
    }
    y[n] = total;
  }
}

static void moe_routes(void *p, int r0, int r1) {
  moe_ctx *c = (moe_ctx *)p;
  int H = c->H, I = c->I;
  size_t gu_words = (size_t)2 * I * H / 8, gu_sbn = (size_t)2 * I * 2 * (H / 64);
  size_t dn_words = (size_t)H * I / 8, dn_sbn = (size_t)H * 2 * (I / 64);
  float *x = (float *)malloc(sizeof(float) * (size_t)H);
  float *gu = (float *)malloc(sizeof(float) * (size_t)2 * I);
  float *h = (float *)malloc(sizeof(float) * (size_t)I);
  float *d = (float *)malloc(sizeof(float) * (size_t)H);
  for (int r = r0; r < r1; ++r) {
    int t = r / c->k;
    uint32_t e = c->ids[r];
    int sh = e == c->E;
    const uint32_t *gw = sh ? c->sh_gu_wq : c->gu_wq + e * gu_words;
    const uint16_t *gs = sh ? c->sh_gu_sb : c->gu_sb + e * gu_sbn;
    const uint32_t *dw = sh ? c->sh_dn_wq : c->dn_wq + e * dn_words;
    const uint16_t *ds = sh ? c->sh_dn_sb : c->dn_sb + e * dn_sbn;
    for (int i = 0; i < H; ++i) x[i] = q4o_bf16_to_f32(c->x[(size_t)t * H + i]);
    project_row(gw, gs, c->sb_dtype, 2 * I, H, x, gu);
    for (int i = 0; i < I; ++i) {
      uint16_t hv = q4o_silu_mul_bf16(gu[i], gu[I + i]);
      h[i] = q4o_bf16_to_f32(hv);
      if (c->h_out) c->h_out[(size_t)r * I + i] = hv;
    }
    project_row(dw, ds, c->sb_dtype, H, I, h, d);
    for (int i = 0; i < H; ++i) c->d_out[(size_t)r * H + i] = q4o_f32_to_bf16(d[i]);
  }
  free(x);
  free(gu);
  free(h);
  free(d);
}

void q4o_moe_forward(const uint16_t *x, const uint16_t *residual, int T, int H,
                     int I, int E, int k, const uint32_t *ids,
                     const uint16_t *weights, const uint32_t *gu_wq,
                     const uint16_t *gu_sb, const uint32_t *dn_wq,
                     const uint16_t *dn_sb, int sb_dtype, uint16_t *h_out,
                     uint16_t *d_out, uint16_t *y, int nthreads) {
  q4o_moe_forward_shared(x, residual, T, H, I, E, k, ids, weights, gu_wq, gu_sb, dn_wq, dn_sb, NULL, NULL,
                         NULL, NULL, sb_dtype, h_out, d_out, y, nthreads);
}

void q4o_moe_forward_shared(const uint16_t *x, const uint16_t *residual, int T, int H, int I, int E, int k,
                            const uint32_t *ids, const uint16_t *weights, const uint32_t *gu_wq,
                            const uint16_t *gu_sb, const uint32_t *dn_wq, const uint16_t *dn_sb,
                            const uint32_t *sh_gu_wq, const uint16_t *sh_gu_sb, const uint32_t *sh_dn_wq,
                            const uint16_t *sh_dn_sb, int sb_dtype, uint16_t *h_out, uint16_t *d_out,
                            uint16_t *y, int nthreads) {
  int own_d = d_out == NULL;
  if (own_d) d_out = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)T * k * H);
  moe_ctx c = {x, T, H, I, k, ids, gu_wq, dn_wq, gu_sb, dn_sb, sb_dtype, h_out, d_out,
               sh_gu_wq ? (uint32_t)E : 0xFFFFFFFFu, sh_gu_wq, sh_dn_wq, sh_gu_sb, sh_dn_sb};
  parallel_for(T * k, nthreads, moe_routes, &c);
  /* moe_combine (moe.metal:642-664): value = residual, then += w * d over
   * the slots in order, f32, one bf16 rounding. */
  for (int t = 0; t < T; ++t)
    for (int i = 0; i < H; ++i) {
      float v = residual ? q4o_bf16_to_f32(residual[(size_t)t * H + i]) : 0.0f;
      for (int s = 0; s < k; ++s)
        v += q4o_bf16_to_f32(weights[(size_t)t * k + s]) *
             q4o_bf16_to_f32(d_out[((size_t)t * k + s) * H + i]);
      y[(size_t)t * H + i] = q4o_f32_to_bf16(v);
    }
  if (own_d) free(d_out);
}

/* ---- the Q8 router and the shared expert's gate (moe.metal:1-361) ------ */

/* A Q8 projection in StorageN = 256 order (Linear.hpp:27-33, read by
 * moe.metal:70-121): byte q of output n and input k at ((k/64)*256 + n)*64 +
 * k%64; bf16 scale and bias at (k/64)*256 + n. */
#define Q8_STORAGE_N 256
#define ROUTE_SLICES 8

/* A 64-value group's sum in the router's fixed order: lane l of a warp adds
 * x[l] and x[l + 32] (moe_route_row_sum, moe.metal:22-25), then the lanes
 * combine by xor butterfly, partners 16, 8, 4, 2, 1 (every lane ends with the
 * same value since each step adds a pair in either order). */
static float route_group_sum(const float *x) {
  float v[32], w[32];
  for (int l = 0; l < 32; ++l) v[l] = x[l] + x[l + 32];
  for (int o = 16; o > 0; o >>= 1) {
    for (int l = 0; l < 32; ++l) w[l] = v[l] + v[l ^ o];
    memcpy(v, w, sizeof v);
  }
  return v[0];
}

typedef struct {
  const uint16_t *x;
  int H, ncols;
  const uint8_t *q;
  const uint16_t *scales, *biases;
  uint16_t *scores;
} scores_ctx;

static void scores_rows(void *p, int t0, int t1) {
  scores_ctx *c = (scores_ctx *)p;
  int H = c->H, G = H / 64;
  float *x = (float *)malloc(sizeof(float) * (size_t)H);
  float *sums = (float *)malloc(sizeof(float) * (size_t)G);
  for (int t = t0; t < t1; ++t) {
    for (int i = 0; i < H; ++i) x[i] = q4o_bf16_to_f32(c->x[(size_t)t * H + i]);
    for (int g = 0; g < G; ++g) sums[g] = route_group_sum(x + 64 * g);
    for (int n = 0; n < c->ncols; ++n) {
      float total = 0.0f;
      for (int s = 0; s < ROUTE_SLICES; ++s) {
        /* moe_route_slice (moe.metal:17-20): groups [s*G/8, (s+1)*G/8) */
        int g0 = s * G / ROUTE_SLICES, g1 = (s + 1) * G / ROUTE_SLICES;
        float slice = 0.0f;
        for (int g = g0; g < g1; ++g) {
          const uint8_t *qg = c->q + ((size_t)g * Q8_STORAGE_N + n) * 64;
          float dot = 0.0f;
          for (int j = 0; j < 64; ++j) dot = fmaf(x[64 * g + j], (float)qg[j], dot);
          size_t prm = (size_t)g * Q8_STORAGE_N + n;
          float b = q4o_bf16_to_f32(c->biases[prm]);
          /* moe_route_group_term (moe.metal:29-32): fma(dot, scale, sum*bias) */
          slice = slice + fmaf(dot, q4o_bf16_to_f32(c->scales[prm]), sums[g] * b);
        }
        total = total + slice;
      }
      c->scores[(size_t)t * c->ncols + n] = q4o_f32_to_bf16(total);
    }
  }
  free(x);
  free(sums);
}

/* moe_route_scores_q8_m8 / _m32 (moe.metal:34-262): per row and expert the
 * sum over eight K slices, in slice order, of the slice's groups' terms
 * fma(dot, scale, sum * bias) in group order; a group's dot is the f32 sum of
 * x[k] * q[k] in k order (each product is exact: bf16 x 8-bit integer).  The
 * reference's matmul2d leaves the order inside a group's dot to the
 * hardware; the order above is the one this library's router kernel uses.
 * x bf16 [T][H]; scores bf16 [T][ncols]. */
void q4o_moe_scores_q8(const uint16_t *x, int T, int H, const uint8_t *q, const uint16_t *scales,
                       const uint16_t *biases, int ncols, uint16_t *scores, int nthreads) {
  scores_ctx c = {x, H, ncols, q, scales, biases, scores};
  parallel_for(T, nthreads, scores_rows, &c);
}

/* The shared expert's scalar gate of moe_route_select_q8 (moe.metal:297-322):
 * thread v of 256 accumulates, for d = v, v + 256, ..., x[d] * (q * s + b)
 * with row 0's parameters of group d/64, each step one fma of the dequantised
 * weight (itself fma(q, s, b)); each warp of 32 threads combines by xor
 * butterfly (partners 16 .. 1); the eight warp sums add in warp order.
 * weight = bf16(1 / (1 + exp(-total))).  logit (optional) = total. */
void q4o_moe_shared_gate(const uint16_t *x, int T, int H, const uint8_t *q, const uint16_t *scales,
                         const uint16_t *biases, uint16_t *weights, float *logit) {
  for (int t = 0; t < T; ++t) {
    const uint16_t *row = x + (size_t)t * H;
    float total = 0.0f;
    for (int w = 0; w < Q8_STORAGE_N / 32; ++w) {
      float v[32], u[32];
      for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int d = 32 * w + l; d < H; d += Q8_STORAGE_N) {
          int g = d / 64, j = d % 64;
          size_t prm = (size_t)g * Q8_STORAGE_N;
          float deq = fmaf((float)q[prm * 64 + j], q4o_bf16_to_f32(scales[prm]), q4o_bf16_to_f32(biases[prm]));
          acc = fmaf(q4o_bf16_to_f32(row[d]), deq, acc);
        }
        v[l] = acc;
      }
      for (int o = 16; o > 0; o >>= 1) {
        for (int l = 0; l < 32; ++l) u[l] = v[l] + v[l ^ o];
        memcpy(v, u, sizeof v);
      }
      total = total + v[0];
    }
    if (logit) logit[t] = total;
    weights[t] = q4o_f32_to_bf16(1.0f / (1.0f + expf(-total)));
  }
}

/* moe_group_routes with the shared expert (moe.metal:368-449): every token
 * carries k routed slots and, when rpr == k + 1, a shared slot last.  The
 * routed slots sort as in q4o_moe_group; then ceil(T/tile_rows) tiles of
 * expert E hold the shared routes of tokens 0..T-1 in order.  ids [T][rpr];
 * route_rows [T*rpr].  Returns the tile count or -1. */
int q4o_moe_group_shared(const uint32_t *ids, int T, int k, int rpr, int E, int tile_rows, int max_tiles,
                         uint32_t *tiles, uint32_t *grouped_routes, uint32_t *route_rows) {
  int routes = T * rpr;
  uint32_t *count = (uint32_t *)calloc((size_t)E, sizeof(uint32_t));
  uint32_t *offset = (uint32_t *)calloc((size_t)E, sizeof(uint32_t));
  uint32_t *cursor = (uint32_t *)calloc((size_t)E, sizeof(uint32_t));
  for (int r = 0; r < routes; ++r)
    if (r % rpr < k) count[ids[r]]++;
  uint32_t ntiles = 0;
  for (int e = 0; e < E; ++e) {
    offset[e] = ntiles;
    ntiles += (count[e] + (uint32_t)tile_rows - 1) / (uint32_t)tile_rows;
  }
  uint32_t routed = ntiles;
  uint32_t shared_tiles = rpr > k ? ((uint32_t)T + (uint32_t)tile_rows - 1) / (uint32_t)tile_rows : 0u;
  ntiles += shared_tiles;
  if ((int)ntiles > max_tiles) {
    free(count);
    free(offset);
    free(cursor);
    return -1;
  }
  for (size_t i = 0; i < (size_t)max_tiles * tile_rows; ++i) grouped_routes[i] = 0xFFFFFFFFu;
  for (size_t i = 0; i < (size_t)max_tiles * 2; ++i) tiles[i] = 0;
  for (int e = 0; e < E; ++e) {
    uint32_t nt = (count[e] + (uint32_t)tile_rows - 1) / (uint32_t)tile_rows;
    for (uint32_t t = 0; t < nt; ++t) {
      uint32_t live = count[e] - t * (uint32_t)tile_rows;
      tiles[(offset[e] + t) * 2] = (uint32_t)e;
      tiles[(offset[e] + t) * 2 + 1] = live < (uint32_t)tile_rows ? live : (uint32_t)tile_rows;
    }
  }
  for (int r = 0; r < routes; ++r) {
    if (r % rpr >= k) continue;
    uint32_t e = ids[r];
    uint32_t row = offset[e] * (uint32_t)tile_rows + cursor[e]++;
    grouped_routes[row] = (uint32_t)r;
    route_rows[r] = row;
  }
  for (uint32_t t = 0; t < shared_tiles; ++t) {
    uint32_t live = (uint32_t)T - t * (uint32_t)tile_rows;
    tiles[(routed + t) * 2] = (uint32_t)E;
    tiles[(routed + t) * 2 + 1] = live < (uint32_t)tile_rows ? live : (uint32_t)tile_rows;
  }
  if (rpr > k)
    for (int t = 0; t < T; ++t) {
      uint32_t row = routed * (uint32_t)tile_rows + (uint32_t)t;
      grouped_routes[row] = (uint32_t)(t * rpr + k);
      route_rows[t * rpr + k] = row;
    }
  free(count);
  free(offset);
  free(cursor);
  return (int)ntiles;
}

/* ---- the reference MoE test's fixture (moe_metal_test.mm:46-271) -------- */

static uint32_t splash_next(uint64_t *s) { return (uint32_t)q4o_lcg(s); }
/* Random::unit (moe_metal_test.mm:74) */
static float splash_unit(uint64_t *s) { return (float)(splash_next(s) & 0xFFFFFFu) / 8388608.0f - 1.0f; }

/* randomSlab + packSlab (moe_metal_test.mm:108-145): nibbles n-major, then
 * per parameter index a scale bf16(0.01 + 0.01 (unit + 1)) and a bias
 * bf16(-0.2 + 0.05 unit), drawn in that order; packed into a Splash slab.
 * The multiply-adds are single fmas, as clang contracts them on arm64. */
static void splash_random_slab(uint64_t *s, int out, int in, uint8_t *slab) {
  size_t elements = (size_t)out * in;
  int groups = in / 64;
  uint8_t *nib = (uint8_t *)malloc(elements);
  for (size_t i = 0; i < elements; ++i) nib[i] = (uint8_t)(splash_next(s) & 15u);
  size_t params = elements / 64;
  uint16_t *sc = (uint16_t *)(slab + elements / 2);
  uint16_t *bi = (uint16_t *)(slab + elements / 2 + elements / 32);
  for (size_t i = 0; i < params; ++i) {
    sc[i] = q4o_f32_to_bf16(fmaf(0.01f, splash_unit(s) + 1.0f, 0.01f));
    bi[i] = q4o_f32_to_bf16(fmaf(0.05f, splash_unit(s), -0.2f));
  }
  memset(slab, 0, elements / 2);
  for (int n = 0; n < out; ++n)
    for (int k = 0; k < in; ++k) {
      size_t prm = ((size_t)(n / 256) * groups + (size_t)(k / 64)) * 256 + (size_t)(n % 256);
      size_t idx = prm * 64 + (size_t)(k % 64);
      uint8_t v = nib[(size_t)n * in + k];
      slab[idx / 2] |= (uint8_t)((idx & 1) ? v << 4 : v);
    }
  free(nib);
}

/* makeFixture (moe_metal_test.mm:217-271) with Random(seed): E gate, E up, E
 * down slabs, then the shared gate, up and down slabs (one each), then per
 * row and column an input bf16(sign * (0.55 + 0.45 unit)) (sign -1 on every
 * third row) and a residual bf16(0.1 unit). */
void q4o_splash_moe_fixture(int H, int I, int E, int rows, uint64_t seed, uint8_t *gate, uint8_t *up,
                            uint8_t *down, uint8_t *shared_gate, uint8_t *shared_up, uint8_t *shared_down,
                            uint16_t *x, uint16_t *residual) {
  uint64_t s = seed;
  size_t gs = q4o_slab_bytes(I, H), ds = q4o_slab_bytes(H, I);
  for (int e = 0; e < E; ++e) splash_random_slab(&s, I, H, gate + (size_t)e * gs);
  for (int e = 0; e < E; ++e) splash_random_slab(&s, I, H, up + (size_t)e * gs);
  for (int e = 0; e < E; ++e) splash_random_slab(&s, H, I, down + (size_t)e * ds);
  splash_random_slab(&s, I, H, shared_gate);
  splash_random_slab(&s, I, H, shared_up);
  splash_random_slab(&s, H, I, shared_down);
  for (int r = 0; r < rows; ++r) {
    float sign = r % 3 == 0 ? -1.0f : 1.0f;
    for (int c = 0; c < H; ++c) {
      x[(size_t)r * H + c] = q4o_f32_to_bf16(sign * fmaf(0.45f, splash_unit(&s), 0.55f));
      residual[(size_t)r * H + c] = q4o_f32_to_bf16(0.1f * splash_unit(&s));
    }
  }
}
