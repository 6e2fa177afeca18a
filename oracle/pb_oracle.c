/*
 * pb_oracle.c - CPU restatement of sammcj/purebee's quantized Llama hot path.
 *
 * TEST INFRASTRUCTURE ONLY: parity checker and timed CPU baseline.  Nothing in
 * the product links this file.  Build: oracle/build.py (gcc -O2
 * -ffp-contract=off, so float code keeps the reference's separate multiply
 * and add).  See pb_oracle.h for the arithmetic conventions.
 */
#include "pb_oracle.h"
#include "pb_synth.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* threading: contiguous row split, as thread-pool.js:174-203 does     */
/* ------------------------------------------------------------------ */

static int g_threads = 1;
void orc_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int orc_get_threads(void) { return g_threads; }

typedef void (*orc_range_fn)(void* ctx, int64_t lo, int64_t hi);
typedef struct { orc_range_fn fn; void* ctx; int64_t lo, hi; } orc_job;

static void* orc_job_main(void* p) {
  orc_job* j = (orc_job*)p;
  j->fn(j->ctx, j->lo, j->hi);
  return NULL;
}

static void orc_parallel_rows(int64_t n, orc_range_fn fn, void* ctx) {
  int t = g_threads;
  if (t <= 1 || n < 64) { fn(ctx, 0, n); return; }
  if (t > 256) t = 256;
  pthread_t th[256];
  orc_job jobs[256];
  int64_t per = (n + t - 1) / t;
  int started = 0;
  for (int i = 1; i < t; ++i) {
    int64_t lo = per * i, hi = lo + per > n ? n : lo + per;
    if (lo >= n) break;
    jobs[i].fn = fn; jobs[i].ctx = ctx; jobs[i].lo = lo; jobs[i].hi = hi;
    if (pthread_create(&th[i], NULL, orc_job_main, &jobs[i]) == 0) {
      started = i;
    } else { /* run inline when a thread cannot be created */
      fn(ctx, lo, hi);
      started = i;
      th[i] = 0;
    }
  }
  fn(ctx, 0, per > n ? n : per);
  for (int i = 1; i <= started; ++i)
    if (th[i]) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------------ */
/* f16                                                                  */
/* ------------------------------------------------------------------ */

/* gguf.js:55-70: full IEEE half decode, evaluated in double. */
float orc_f16_exact(uint16_t bits) {
  int sign = (bits >> 15) & 1, e = (bits >> 10) & 0x1f, frac = bits & 0x3ff;
  double s = sign ? -1.0 : 1.0;
  if (e == 0) {
    if (frac == 0) return sign ? -0.0f : 0.0f;
    return (float)(s * pow(2.0, -14.0) * (frac / 1024.0));
  }
  if (e == 0x1f) return frac ? NAN : (sign ? -INFINITY : INFINITY);
  return (float)(s * pow(2.0, (double)(e - 15)) * (1.0 + frac / 1024.0));
}

/* wasm-q4.js:88-109: exponent 0 gives +0; otherwise the bits are rebuilt with
 * no inf/NaN case (exponent 31 becomes an ordinary float exponent). */
float orc_f16_wasm(uint16_t bits) {
  uint32_t e = (bits >> 10) & 0x1f;
  if (e == 0) return 0.0f;
  uint32_t f = ((uint32_t)(bits >> 15) << 31) | ((e + 112u) << 23) | ((uint32_t)(bits & 0x3ff) << 13);
  float r;
  memcpy(&r, &f, 4);
  return r;
}

uint16_t orc_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
  if (ax <= 0x33000000u) return (uint16_t)sign;
  int e = (int)(ax >> 23);
  uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
  if (e < 113) {
    int shift = 126 - e;
    uint32_t h = mant >> shift, rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)(e - 112) << 10) | ((mant >> 13) & 0x3ffu), rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ------------------------------------------------------------------ */
/* GGUF decode (gguf.js:219-315)                                        */
/* ------------------------------------------------------------------ */

void orc_dequant_q4_0(const uint8_t* raw, int64_t n, float* out) {
  int64_t nb = (n + 31) / 32, idx = 0;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = raw + b * 18;
    double scale = orc_f16_exact(rd16(blk));
    int64_t remaining = n - idx < 32 ? n - idx : 32;
    int64_t half = remaining < 16 ? remaining : 16;
    for (int j = 0; j < half; ++j) {
      int byte = blk[2 + j];
      out[idx + j] = (float)(((byte & 0x0F) - 8) * scale);
      if (j + 16 < remaining) out[idx + j + 16] = (float)(((byte >> 4) - 8) * scale);
    }
    idx += remaining;
  }
}

void orc_dequant_q4_1(const uint8_t* raw, int64_t n, float* out) {
  int64_t nb = (n + 31) / 32, idx = 0;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = raw + b * 20;
    double d = orc_f16_exact(rd16(blk)), m = orc_f16_exact(rd16(blk + 2));
    int64_t remaining = n - idx < 32 ? n - idx : 32;
    int64_t half = remaining < 16 ? remaining : 16;
    for (int j = 0; j < half; ++j) {
      int byte = blk[4 + j];
      out[idx + j] = (float)((byte & 0x0F) * d + m);
      if (j + 16 < remaining) out[idx + j + 16] = (float)((byte >> 4) * d + m);
    }
    idx += remaining;
  }
}

void orc_dequant_q8_0(const uint8_t* raw, int64_t n, float* out) {
  int64_t nb = (n + 31) / 32, idx = 0;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = raw + b * 34;
    double scale = orc_f16_exact(rd16(blk));
    int64_t remaining = n - idx < 32 ? n - idx : 32;
    for (int i = 0; i < remaining; ++i) out[idx++] = (float)((int8_t)blk[2 + i] * scale);
  }
}

void orc_dequant_f16(const uint8_t* raw, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = orc_f16_exact(rd16(raw + 2 * i));
}

/* gguf.js:317-355 Q6_K: 210-byte blocks of 256 values, [ql 128][qh 64]
 * [int8 scales 16][f16 d].  Two halves of 128; for l in 0..31 of a half the
 * four values l, l+32, l+64, l+96 take the low nibble of ql[l], the low
 * nibble of ql[l+32], the high nibble of ql[l], the high nibble of ql[l+32],
 * each with two bits of qh[l] (bits 0-1, 2-3, 4-5, 6-7) on top, minus 32,
 * times d times the scale is + 0, 2, 4, 6 (is = 8 half + l / 16).  JS
 * computes d * sc * q in double and stores the f32. */
void orc_dequant_q6_k(const uint8_t* raw, int64_t n, float* out) {
  int64_t nb = (n + 255) / 256, idx = 0;
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = raw + b * 210;
    const uint8_t* ql = blk;
    const uint8_t* qh = blk + 128;
    const int8_t* sc = (const int8_t*)(blk + 192);
    const double d = orc_f16_exact(rd16(blk + 208));
    for (int half = 0; half < 2; ++half) {
      const uint8_t* qlb = ql + half * 64;
      const uint8_t* qhb = qh + half * 32;
      for (int l = 0; l < 32; ++l) {
        const int is = half * 8 + l / 16;
        const int q1 = ((qlb[l] & 0xF) | (((qhb[l] >> 0) & 3) << 4)) - 32;
        const int q2 = ((qlb[l + 32] & 0xF) | (((qhb[l] >> 2) & 3) << 4)) - 32;
        const int q3 = ((qlb[l] >> 4) | (((qhb[l] >> 4) & 3) << 4)) - 32;
        const int q4 = ((qlb[l + 32] >> 4) | (((qhb[l] >> 6) & 3) << 4)) - 32;
        const int64_t base = idx + half * 128;
        if (base + l < n) out[base + l] = (float)(d * sc[is + 0] * q1);
        if (base + l + 32 < n) out[base + l + 32] = (float)(d * sc[is + 2] * q2);
        if (base + l + 64 < n) out[base + l + 64] = (float)(d * sc[is + 4] * q3);
        if (base + l + 96 < n) out[base + l + 96] = (float)(d * sc[is + 6] * q4);
      }
    }
    idx += 256;
  }
}

/* ------------------------------------------------------------------ */
/* GGUF encode: the build's own definition (the reference decodes only). */
/* Q4_0: signed max-magnitude element m, d = m / -8, q = min(15,          */
/* trunc(x/d + 8.5)), low nibbles hold elements 0-15; Q8_0: d = amax/127, */
/* q = round-half-away(x/d); d stored as IEEE half (nearest-even).        */
/* ------------------------------------------------------------------ */

void orc_quantize_gguf_q4_0(const float* x, int64_t n, uint8_t* out) {
  int64_t nb = n / 32;
  for (int64_t b = 0; b < nb; ++b) {
    const float* xb = x + 32 * b;
    float amax = 0.0f, mx = 0.0f;
    for (int j = 0; j < 32; ++j) {
      float a = fabsf(xb[j]);
      if (a > amax) { amax = a; mx = xb[j]; }
    }
    float d = mx / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = orc_f32_to_f16(d);
    uint8_t* o = out + 18 * b;
    o[0] = (uint8_t)(dh & 0xff);
    o[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 16; ++j) {
      float v0 = xb[j] * id + 8.5f, v1 = xb[j + 16] * id + 8.5f;
      int q0 = v0 != v0 ? 0 : (int)fminf(fmaxf(v0, 0.0f), 16.0f);
      int q1 = v1 != v1 ? 0 : (int)fminf(fmaxf(v1, 0.0f), 16.0f);
      if (q0 > 15) q0 = 15;
      if (q1 > 15) q1 = 15;
      o[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
  }
}

void orc_quantize_gguf_q8_0(const float* x, int64_t n, uint8_t* out) {
  int64_t nb = n / 32;
  for (int64_t b = 0; b < nb; ++b) {
    const float* xb = x + 32 * b;
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) {
      float a = fabsf(xb[j]);
      if (a > amax) amax = a;
    }
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = orc_f32_to_f16(d);
    uint8_t* o = out + 34 * b;
    o[0] = (uint8_t)(dh & 0xff);
    o[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 32; ++j) {
      float v = xb[j] * id;
      float r = v != v ? 0.0f : roundf(v);
      if (r > 127.0f) r = 127.0f;
      if (r < -127.0f) r = -127.0f;
      o[2 + j] = (uint8_t)(int8_t)(int)r;
    }
  }
}

/* ------------------------------------------------------------------ */
/* Q4 matvecs                                                           */
/* ------------------------------------------------------------------ */

typedef struct { const float* x; const uint8_t* raw; int N, K; float* y; } mv_args;

/* wasm-q4.js:148-250.  Four f32 lanes; lane L of byte group g uses byte g+L:
 * blockAcc[L] += (lo-8)*x[g+L]; blockAcc[L] += (hi-8)*x[g+16+L] for g=0,4,8,12;
 * acc[L] += blockAcc[L]*d; y = (acc1+acc3) + (acc0+acc2). */
static void q4_0_wasm_rows(void* c, int64_t lo, int64_t hi) {
  mv_args* a = (mv_args*)c;
  int nb = a->K >> 5;
  size_t bpr = (size_t)nb * 18;
  for (int64_t n = lo; n < hi; ++n) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const uint8_t* row = a->raw + (size_t)n * bpr;
    for (int b = 0; b < nb; ++b) {
      const uint8_t* blk = row + (size_t)b * 18;
      float d = orc_f16_wasm(rd16(blk));
      const uint8_t* q = blk + 2;
      const float* xb = a->x + 32 * b;
      float ba[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int g = 0; g < 16; g += 4) {
        for (int L = 0; L < 4; ++L) {
          int byte = q[g + L];
          float plo = (float)((byte & 15) - 8) * xb[g + L];
          ba[L] = ba[L] + plo;
          float phi = (float)((byte >> 4) - 8) * xb[g + 16 + L];
          ba[L] = ba[L] + phi;
        }
      }
      for (int L = 0; L < 4; ++L) {
        float p = ba[L] * d;
        acc[L] = acc[L] + p;
      }
    }
    float t0 = acc[0] + acc[2], t1 = acc[1] + acc[3];
    a->y[n] = t1 + t0;
  }
}
void orc_q4_0_matvec_wasm(const float* x, const uint8_t* raw, int N, int K, float* y) {
  mv_args a = {x, raw, N, K, y};
  orc_parallel_rows(N, q4_0_wasm_rows, &a);
}

/* wasm-q4.js:329-414: nibAcc[L] += nib*x, xAcc[L] += x, per lane lo then hi;
 * acc[L] += nibAcc[L]*delta + xAcc[L]*min. */
static void q4_1_wasm_rows(void* c, int64_t lo, int64_t hi) {
  mv_args* a = (mv_args*)c;
  int nb = a->K >> 5;
  size_t bpr = (size_t)nb * 20;
  for (int64_t n = lo; n < hi; ++n) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const uint8_t* row = a->raw + (size_t)n * bpr;
    for (int b = 0; b < nb; ++b) {
      const uint8_t* blk = row + (size_t)b * 20;
      float delta = orc_f16_wasm(rd16(blk)), mn = orc_f16_wasm(rd16(blk + 2));
      const uint8_t* q = blk + 4;
      const float* xb = a->x + 32 * b;
      float na[4] = {0, 0, 0, 0}, xa[4] = {0, 0, 0, 0};
      for (int g = 0; g < 16; g += 4) {
        for (int L = 0; L < 4; ++L) {
          int byte = q[g + L];
          float xl = xb[g + L], xh = xb[g + 16 + L];
          float pl = (float)(byte & 15) * xl;
          na[L] = na[L] + pl;
          xa[L] = xa[L] + xl;
          float ph = (float)(byte >> 4) * xh;
          na[L] = na[L] + ph;
          xa[L] = xa[L] + xh;
        }
      }
      for (int L = 0; L < 4; ++L) {
        float u = na[L] * delta, v = xa[L] * mn;
        float s = u + v;
        acc[L] = acc[L] + s;
      }
    }
    float t0 = acc[0] + acc[2], t1 = acc[1] + acc[3];
    a->y[n] = t1 + t0;
  }
}
void orc_q4_1_matvec_wasm(const float* x, const uint8_t* raw, int N, int K, float* y) {
  mv_args a = {x, raw, N, K, y};
  orc_parallel_rows(N, q4_1_wasm_rows, &a);
}

/* llama-streaming.js:51-61 (f16 used by the JS fallback kernels). */
static double js_f16(uint16_t bits) {
  int sign = (bits >> 15) & 1, e = (bits >> 10) & 0x1f, frac = bits & 0x3ff;
  if (e == 0) {
    if (frac == 0) return sign ? -0.0 : 0.0;
    return (sign ? -1.0 : 1.0) * pow(2.0, -14.0) * (frac / 1024.0);
  }
  if (e == 0x1f) return frac ? NAN : (sign ? -INFINITY : INFINITY);
  return (sign ? -1.0 : 1.0) * pow(2.0, (double)(e - 15)) * (1.0 + frac / 1024.0);
}

/* llama-streaming.js:72-104, double accumulation. */
void orc_q4_0_matvec_js(const float* x, const uint8_t* raw, int N, int K, float* y) {
  int nb = K >> 5;
  size_t bpr = (size_t)nb * 18;
  for (int n = 0; n < N; ++n) {
    double sum = 0;
    for (int b = 0; b < nb; ++b) {
      const uint8_t* blk = raw + (size_t)n * bpr + (size_t)b * 18;
      double scale = js_f16(rd16(blk));
      double bs = 0;
      for (int j = 0; j < 16; ++j) {
        int byte = blk[2 + j];
        bs += (double)x[32 * b + j] * ((byte & 0x0F) - 8);
        bs += (double)x[32 * b + j + 16] * ((byte >> 4) - 8);
      }
      sum += bs * scale;
    }
    y[n] = (float)sum;
  }
}

/* llama-streaming.js:115-151 */
void orc_q4_1_matvec_js(const float* x, const uint8_t* raw, int N, int K, float* y) {
  int nb = K >> 5;
  size_t bpr = (size_t)nb * 20;
  for (int n = 0; n < N; ++n) {
    double sum = 0;
    for (int b = 0; b < nb; ++b) {
      const uint8_t* blk = raw + (size_t)n * bpr + (size_t)b * 20;
      double delta = js_f16(rd16(blk)), mn = js_f16(rd16(blk + 2));
      double ns = 0, xs = 0;
      for (int j = 0; j < 16; ++j) {
        int byte = blk[4 + j];
        ns += (double)x[32 * b + j] * (byte & 0x0F);
        ns += (double)x[32 * b + j + 16] * (byte >> 4);
        xs += (double)x[32 * b + j] + (double)x[32 * b + j + 16];
      }
      sum += delta * ns + mn * xs;
    }
    y[n] = (float)sum;
  }
}

/* ------------------------------------------------------------------ */
/* f32 kernels                                                          */
/* ------------------------------------------------------------------ */

typedef struct { const float* x; const float* W; int N, K; float* out; } bd_args;

/* wasm-q4.js:467-549: acc[k%4] += x[k]*W[n,k] for k < K&~3, horizontal sum
 * (acc1+acc3)+(acc0+acc2), then a scalar tail. */
static void batch_dot_rows(void* c, int64_t lo, int64_t hi) {
  bd_args* a = (bd_args*)c;
  int K = a->K, K4 = K & ~3;
  for (int64_t n = lo; n < hi; ++n) {
    const float* w = a->W + (size_t)n * K;
    float acc[4] = {0, 0, 0, 0};
    for (int k = 0; k < K4; k += 4)
      for (int L = 0; L < 4; ++L) {
        float p = a->x[k + L] * w[k + L];
        acc[L] = acc[L] + p;
      }
    float t0 = acc[0] + acc[2], t1 = acc[1] + acc[3];
    float sum = t1 + t0;
    for (int k = K4; k < K; ++k) {
      float p = a->x[k] * w[k];
      sum = sum + p;
    }
    a->out[n] = sum;
  }
}
void orc_batch_dot(const float* x, const float* W, int N, int K, float* out) {
  bd_args a = {x, W, N, K, out};
  orc_parallel_rows(N, batch_dot_rows, &a);
}

typedef struct { const float* A; int M, K; const float* B; int N; float* C; } mm_args;

/* wasm-simd.js:71-91: for m, for k: C[m,n] = C[m,n] + a*B[k,n]. Rows of C
 * are independent, so the split is over output columns here. */
static void matmul_cols(void* c, int64_t lo, int64_t hi) {
  mm_args* a = (mm_args*)c;
  for (int m = 0; m < a->M; ++m) {
    float* crow = a->C + (size_t)m * a->N;
    for (int k = 0; k < a->K; ++k) {
      float av = a->A[(size_t)m * a->K + k];
      const float* brow = a->B + (size_t)k * a->N;
      for (int64_t n = lo; n < hi; ++n) {
        float p = av * brow[n];
        crow[n] = crow[n] + p;
      }
    }
  }
}
void orc_matmul_wasm(const float* A, int M, int K, const float* B, int N, const float* bias, float* C) {
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) C[(size_t)m * N + n] = bias ? bias[n] : 0.0f; /* wasm-simd.js:492-499 */
  mm_args a = {A, M, K, B, N, C};
  orc_parallel_rows(N, matmul_cols, &a);
}

/* ------------------------------------------------------------------ */
/* quantize.js format (a)                                               */
/* ------------------------------------------------------------------ */

/* Math.round: the nearest integer, ties toward +infinity. */
static double js_round(double v) {
  if (v != v || isinf(v)) return v;
  double f = floor(v);
  return (v - f >= 0.5) ? f + 1.0 : f;
}

/* ToInt8 of a Number (Int8Array store). */
static int8_t js_to_int8(double v) {
  if (v != v || isinf(v)) return 0;
  double t = trunc(v);
  double m = fmod(t, 256.0);
  if (m < 0) m += 256.0;
  int iv = (int)m;
  return (int8_t)(iv >= 128 ? iv - 256 : iv);
}

/* ToInt32(v) & 0x0F for the Q4 nibble store. */
static int js_low_nibble(double v) {
  if (v != v || isinf(v)) return 0;
  double t = trunc(v);
  double m = fmod(t, 16.0);
  if (m < 0) m += 16.0;
  return (int)m;
}

void orc_quantize_q8a(const float* data, int64_t size, float* scales, int8_t* q) {
  int64_t nblocks = (size + 31) / 32;
  memset(q, 0, (size_t)nblocks * 32);
  for (int64_t b = 0; b < nblocks; ++b) {
    int64_t off = b * 32, end = off + 32 < size ? off + 32 : size;
    double maxAbs = 0;
    for (int64_t i = off; i < end; ++i) {
      double a = fabs((double)data[i]);
      if (a > maxAbs) maxAbs = a;
    }
    double scale = maxAbs / 127;
    scales[b] = (float)scale;
    if (scale > 0) {
      double inv = 127 / maxAbs;
      for (int64_t i = off; i < end; ++i) q[i] = js_to_int8(js_round((double)data[i] * inv));
    }
  }
}

void orc_quantize_q4a(const float* data, int64_t size, float* scales, uint8_t* q) {
  int64_t nblocks = (size + 31) / 32;
  memset(q, 0, (size_t)(nblocks * 32 + 1) / 2);
  for (int64_t b = 0; b < nblocks; ++b) {
    int64_t off = b * 32, end = off + 32 < size ? off + 32 : size;
    double maxAbs = 0;
    for (int64_t i = off; i < end; ++i) {
      double a = fabs((double)data[i]);
      if (a > maxAbs) maxAbs = a;
    }
    double scale = maxAbs / 7;
    scales[b] = (float)scale;
    if (scale > 0) {
      double inv = 7 / maxAbs;
      for (int64_t i = off; i < end; ++i) {
        double v = js_round((double)data[i] * inv);
        /* Math.max(-8, Math.min(7, v)); NaN propagates */
        if (v == v) { if (v > 7) v = 7; if (v < -8) v = -8; }
        int u = js_low_nibble(v + 8);
        int64_t bi = i / 2;
        if (i % 2 == 0) q[bi] = (uint8_t)((q[bi] & 0xF0) | (u & 0x0F));
        else q[bi] = (uint8_t)((q[bi] & 0x0F) | ((u & 0x0F) << 4));
      }
    }
  }
}

void orc_dequantize_q8a(const float* scales, const int8_t* q, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = (float)((double)q[i] * (double)scales[i / 32]);
}

void orc_dequantize_q4a(const float* scales, const uint8_t* q, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    int nib = (i % 2 == 0) ? (q[i / 2] & 0x0F) : ((q[i / 2] >> 4) & 0x0F);
    out[i] = (float)((double)(nib - 8) * (double)scales[i / 32]);
  }
}

typedef struct {
  const float* a; int M, K; const float* scales; const int8_t* q; int N; float* out;
} mq_args;

/* quantize.js:242-265: for m, for k (skip a == 0), for each 32-column chunk:
 * aScaled = a*scale[floor((k*N + nStart)/32)]; out += aScaled*q (double, f32 store). */
static void matmul_q8_cols(void* c, int64_t lo, int64_t hi) {
  mq_args* a = (mq_args*)c;
  int N = a->N;
  for (int m = 0; m < a->M; ++m) {
    float* orow = a->out + (size_t)m * N;
    for (int k = 0; k < a->K; ++k) {
      double av = a->a[(size_t)m * a->K + k];
      if (av == 0) continue;
      int64_t rowOff = (int64_t)k * N;
      for (int64_t n = lo; n < hi; ++n) {
        int64_t nStart = (n / 32) * 32;
        double sc = a->scales[(rowOff + nStart) / 32];
        double as = av * sc;
        orow[n] = (float)((double)orow[n] + as * (double)a->q[rowOff + n]);
      }
    }
  }
}
void orc_matmul_q8(const float* a, int M, int K, const float* scales, const int8_t* q, int N,
                   const float* bias, float* out) {
  for (int m = 0; m < M; ++m)
    for (int n = 0; n < N; ++n) out[(size_t)m * N + n] = bias ? bias[n] : 0.0f;
  mq_args ar = {a, M, K, scales, q, N, out};
  orc_parallel_rows(N, matmul_q8_cols, &ar);
}

/* ------------------------------------------------------------------ */
/* engine.js ops                                                        */
/* ------------------------------------------------------------------ */

void orc_rmsnorm(const float* x, int seq, int dim, const float* w, double eps, float* out) {
  for (int s = 0; s < seq; ++s) {
    const float* xr = x + (size_t)s * dim;
    double ss = 0;
    for (int d = 0; d < dim; ++d) ss += (double)xr[d] * (double)xr[d];
    double rms = sqrt(ss / dim + eps);
    for (int d = 0; d < dim; ++d) out[(size_t)s * dim + d] = (float)(((double)xr[d] / rms) * (double)w[d]);
  }
}

static double js_max(double a, double b) {
  if (a != a || b != b) return NAN;
  return a > b ? a : b;
}

void orc_softmax(const float* in, int rows, int cols, float* out) {
  for (int r = 0; r < rows; ++r) {
    const float* ir = in + (size_t)r * cols;
    float* orow = out + (size_t)r * cols;
    double mx = -INFINITY;
    for (int c = 0; c < cols; ++c) mx = js_max(mx, ir[c]);
    double sum = 0;
    for (int c = 0; c < cols; ++c) {
      orow[c] = (float)exp((double)ir[c] - mx);
      sum += orow[c];
    }
    for (int c = 0; c < cols; ++c) orow[c] = (float)((double)orow[c] / sum);
  }
}

void orc_layernorm(const float* x, int seq, int dim, const float* w, const float* b, double eps, float* out) {
  for (int s = 0; s < seq; ++s) {
    const float* xr = x + (size_t)s * dim;
    double mean = 0;
    for (int d = 0; d < dim; ++d) mean += xr[d];
    mean /= dim;
    double var = 0;
    for (int d = 0; d < dim; ++d) {
      double diff = xr[d] - mean;
      var += diff * diff;
    }
    var /= dim;
    double sd = sqrt(var + eps);
    for (int d = 0; d < dim; ++d)
      out[(size_t)s * dim + d] = (float)(((xr[d] - mean) / sd) * (double)w[d] + (b ? (double)b[d] : 0.0));
  }
}

void orc_gelu(const float* x, int64_t n, float* out) {
  double c = sqrt(2.0 / M_PI);
  for (int64_t i = 0; i < n; ++i) {
    double v = x[i];
    double inner = c * (v + 0.044715 * v * v * v);
    out[i] = (float)(0.5 * v * (1 + tanh(inner)));
  }
}

void orc_silu(const float* x, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    double v = x[i];
    out[i] = (float)(v / (1 + exp(-v)));
  }
}

void orc_elementmul(const float* a, const float* b, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = (float)((double)a[i] * (double)b[i]);
}

void orc_tensoradd(const float* a, const float* b, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = (float)((double)a[i] + (double)b[i]);
}

void orc_attention(const float* Q, const float* K, const float* V, int seqQ, int seqK, int dK, int dV,
                   int causal, float* out) {
  double scale = 1.0 / sqrt((double)dK);
  float* scores = (float*)calloc((size_t)seqQ * seqK + 1, sizeof(float));
  float* wts = (float*)calloc((size_t)seqQ * seqK + 1, sizeof(float));
  for (int i = 0; i < seqQ; ++i)
    for (int j = 0; j < seqK; ++j) {
      if (causal && j > i) { scores[(size_t)i * seqK + j] = (float)-1e9; continue; }
      double dot = 0;
      for (int k = 0; k < dK; ++k) dot += (double)Q[(size_t)i * dK + k] * (double)K[(size_t)j * dK + k];
      scores[(size_t)i * seqK + j] = (float)(dot * scale);
    }
  orc_softmax(scores, seqQ, seqK, wts);
  for (int i = 0; i < seqQ; ++i)
    for (int d = 0; d < dV; ++d) {
      double s = 0;
      for (int j = 0; j < seqK; ++j) s += (double)wts[(size_t)i * seqK + j] * (double)V[(size_t)j * dV + d];
      out[(size_t)i * dV + d] = (float)s;
    }
  free(scores);
  free(wts);
}

/* ------------------------------------------------------------------ */
/* llama pieces                                                         */
/* ------------------------------------------------------------------ */

void orc_rope(float* q, float* k, int seq, int start_pos, int dim, int n_heads, int n_kv, int head_dim,
              double theta) {
  int kv_dim = n_kv * head_dim;
  for (int t = 0; t < seq; ++t) {
    int pos = start_pos + t;
    for (int i = 0; i < head_dim; i += 2) {
      double freq = 1.0 / pow(theta, (double)i / head_dim);
      double angle = pos * freq;
      double c = cos(angle), s = sin(angle);
      for (int h = 0; h < n_heads; ++h) {
        size_t idx = (size_t)t * dim + (size_t)h * head_dim + i;
        double q0 = q[idx], q1 = q[idx + 1];
        q[idx] = (float)(q0 * c - q1 * s);
        q[idx + 1] = (float)(q0 * s + q1 * c);
      }
      for (int h = 0; h < n_kv; ++h) {
        size_t idx = (size_t)t * kv_dim + (size_t)h * head_dim + i;
        double k0 = k[idx], k1 = k[idx + 1];
        k[idx] = (float)(k0 * c - k1 * s);
        k[idx + 1] = (float)(k0 * s + k1 * c);
      }
    }
  }
}

void orc_attn_cached(const float* q, const float* kc, const float* vc, int seq, int start_pos, int dim,
                     int n_heads, int n_kv, int head_dim, float* out) {
  int kv_dim = n_kv * head_dim, cache_len = start_pos + seq;
  int per = n_heads / n_kv;
  double scale = 1.0 / sqrt((double)head_dim);
  float* sc = (float*)malloc(sizeof(float) * (size_t)cache_len);
  for (int t = 0; t < seq; ++t)
    for (int h = 0; h < n_heads; ++h) {
      int kh = h / per;
      const float* qh = q + (size_t)t * dim + (size_t)h * head_dim;
      for (int j = 0; j < cache_len; ++j) {
        if (j > start_pos + t) { sc[j] = -INFINITY; continue; }
        double dot = 0;
        const float* kr = kc + (size_t)j * kv_dim + (size_t)kh * head_dim;
        for (int d = 0; d < head_dim; ++d) dot += (double)qh[d] * (double)kr[d];
        sc[j] = (float)(dot * scale);
      }
      double mx = -INFINITY;
      for (int j = 0; j < cache_len; ++j) if (sc[j] > mx) mx = sc[j];
      double sum = 0;
      for (int j = 0; j < cache_len; ++j) { sc[j] = (float)exp((double)sc[j] - mx); sum += sc[j]; }
      for (int j = 0; j < cache_len; ++j) sc[j] = (float)((double)sc[j] / sum);
      for (int d = 0; d < head_dim; ++d) {
        double v = 0;
        for (int j = 0; j < cache_len; ++j)
          v += (double)sc[j] * (double)vc[(size_t)j * kv_dim + (size_t)kh * head_dim + d];
        out[(size_t)t * dim + (size_t)h * head_dim + d] = (float)v;
      }
    }
  free(sc);
}

void orc_swiglu_fused(const float* g, const float* u, int n, float* out) {
  for (int i = 0; i < n; ++i) {
    double gv = g[i];
    double silu = gv / (1 + exp(-gv));
    out[i] = (float)(silu * (double)u[i]);
  }
}

int orc_argmax(const float* logits, int n) {
  double mv = -INFINITY;
  int mi = 0;
  for (int i = 0; i < n; ++i)
    if (logits[i] > mv) { mv = logits[i]; mi = i; }
  return mi;
}

/* ------------------------------------------------------------------ */
/* synthetic inputs                                                     */
/* ------------------------------------------------------------------ */

typedef struct { float* out; uint64_t seed, tid; double sd; int act; } syn_args;
static void synth_rows(void* c, int64_t lo, int64_t hi) {
  syn_args* a = (syn_args*)c;
  uint64_t key = pb_stream_key(a->seed, a->tid);
  for (int64_t i = lo; i < hi; ++i)
    a->out[i] = a->act ? (float)pb_normal(key, (uint64_t)i) : (float)PB_DMUL(a->sd, pb_normal(key, (uint64_t)i));
}
void orc_synth_weights(float* out, int64_t n, uint64_t seed, uint64_t tensor_id, double stdev) {
  syn_args a = {out, seed, tensor_id, stdev, 0};
  orc_parallel_rows(n, synth_rows, &a);
}
void orc_synth_activation(float* out, int64_t n, uint64_t seed, uint64_t stream) {
  syn_args a = {out, seed, stream, 1.0, 1};
  orc_parallel_rows(n, synth_rows, &a);
}
void orc_synth_tokens(int* out, int n, uint64_t seed, int lo, int hi) {
  for (int i = 0; i < n; ++i) out[i] = pb_synth_token(seed, (uint64_t)i, lo, hi);
}

/* ------------------------------------------------------------------ */
/* whole model                                                          */
/* ------------------------------------------------------------------ */

/* Matrix shapes.  Streaming (GGUF) tensors are [out rows][in cols]; llama.js
 * (PureBee convention, already transposed) tensors are [in][out]. */
static void mat_shape(const orc_config* c, int which, int* rows_out, int* cols_in) {
  int kv = c->n_kv_heads * c->head_dim;
  switch (which) {
    case 1: *rows_out = c->dim; *cols_in = c->dim; break;        /* wq */
    case 2: *rows_out = kv; *cols_in = c->dim; break;            /* wk */
    case 3: *rows_out = kv; *cols_in = c->dim; break;            /* wv */
    case 4: *rows_out = c->dim; *cols_in = c->dim; break;        /* wo */
    case 5: *rows_out = c->hidden_dim; *cols_in = c->dim; break; /* w1 gate */
    case 6: *rows_out = c->dim; *cols_in = c->hidden_dim; break; /* w2 down */
    case 7: *rows_out = c->hidden_dim; *cols_in = c->dim; break; /* w3 up */
    default: *rows_out = c->vocab; *cols_in = c->dim; break;     /* embedding [V][dim] */
  }
}

struct orc_model {
  orc_config c;
  uint8_t* raw[1 + 7 * 512]; /* [0] embedding, then 7 per layer */
  int64_t raw_bytes[1 + 7 * 512];
  float* q8a_scales[1 + 7 * 512];
  int64_t q8a_count[1 + 7 * 512];
  float* emb_f32;            /* dequantized embedding [V][dim] */
  float* head_f32;           /* dequantized untied LM head [V][dim], NULL when tied */
  float* rms_att;            /* [L][dim] */
  float* rms_ffn;
  float* rms_final;
  float* kc;                 /* [L][seq_len][kv_dim] */
  float* vc;
};

static int tidx(int layer, int which) { return which == 0 ? 0 : 1 + 7 * layer + (which - 1); }

orc_model* orc_model_create(const orc_config* cfg) {
  if (cfg->n_layers > 512) return NULL;
  orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
  m->c = *cfg;
  const orc_config* c = &m->c;
  int kv = c->n_kv_heads * c->head_dim;
  for (int l = 0; l < c->n_layers; ++l)
    for (int w = 1; w <= 7; ++w) {
      int r, k;
      mat_shape(c, w, &r, &k);
      int64_t n = (int64_t)r * k;
      int t = tidx(l, w);
      if (c->kind == ORC_KIND_STREAMING_Q4) {
        m->raw_bytes[t] = n / 32 * 18;
      } else {
        m->raw_bytes[t] = (n + 31) / 32 * 32;
        m->q8a_count[t] = (n + 31) / 32;
        m->q8a_scales[t] = (float*)calloc((size_t)m->q8a_count[t], sizeof(float));
      }
      m->raw[t] = (uint8_t*)calloc((size_t)m->raw_bytes[t], 1);
    }
  int64_t ne = (int64_t)c->vocab * c->dim;
  if (c->emb_type == ORC_EMB_Q4_0) m->raw_bytes[0] = ne / 32 * 18;
  else if (c->emb_type == ORC_EMB_Q8_0) m->raw_bytes[0] = ne / 32 * 34;
  else m->raw_bytes[0] = ne * 4;
  m->raw[0] = (uint8_t*)calloc((size_t)m->raw_bytes[0], 1);
  m->emb_f32 = c->emb_type == ORC_EMB_F32 ? (float*)m->raw[0] : (float*)calloc((size_t)ne, sizeof(float));
  m->rms_att = (float*)malloc(sizeof(float) * (size_t)c->n_layers * c->dim);
  m->rms_ffn = (float*)malloc(sizeof(float) * (size_t)c->n_layers * c->dim);
  m->rms_final = (float*)malloc(sizeof(float) * (size_t)c->dim);
  for (int64_t i = 0; i < (int64_t)c->n_layers * c->dim; ++i) m->rms_att[i] = m->rms_ffn[i] = 1.0f;
  for (int i = 0; i < c->dim; ++i) m->rms_final[i] = 1.0f;
  m->kc = (float*)calloc((size_t)c->n_layers * c->seq_len * kv, sizeof(float));
  m->vc = (float*)calloc((size_t)c->n_layers * c->seq_len * kv, sizeof(float));
  return m;
}

void orc_model_free(orc_model* m) {
  if (!m) return;
  for (int i = 0; i < 1 + 7 * m->c.n_layers; ++i) { free(m->raw[i]); free(m->q8a_scales[i]); }
  if (m->c.emb_type != ORC_EMB_F32) free(m->emb_f32);
  free(m->head_f32);
  free(m->rms_att); free(m->rms_ffn); free(m->rms_final); free(m->kc); free(m->vc);
  free(m);
}

uint8_t* orc_model_tensor(orc_model* m, int layer, int which, int64_t* nbytes) {
  int t = tidx(layer, which);
  if (nbytes) *nbytes = m->raw_bytes[t];
  return m->raw[t];
}
float* orc_model_q8a_scales(orc_model* m, int layer, int which, int64_t* count) {
  int t = tidx(layer, which);
  if (count) *count = m->q8a_count[t];
  return m->q8a_scales[t];
}
float* orc_kv(orc_model* m, int layer, int which_v) {
  int kv = m->c.n_kv_heads * m->c.head_dim;
  return (which_v ? m->vc : m->kc) + (size_t)layer * m->c.seq_len * kv;
}

void orc_model_refresh(orc_model* m) {
  int64_t ne = (int64_t)m->c.vocab * m->c.dim;
  /* streaming-loader.js:324-335 -> gguf.js loadTensorData: f32 embedding table */
  if (m->c.emb_type == ORC_EMB_Q4_0) orc_dequant_q4_0(m->raw[0], ne, m->emb_f32);
  else if (m->c.emb_type == ORC_EMB_Q8_0) orc_dequant_q8_0(m->raw[0], ne, m->emb_f32);
}

void orc_model_init_synthetic(orc_model* m, uint64_t seed, double stdev) {
  const orc_config* c = &m->c;
  int64_t ne = (int64_t)c->vocab * c->dim;
  float* tmp = (float*)malloc(sizeof(float) * (size_t)ne);
  orc_synth_weights(tmp, ne, seed, 0, stdev);
  if (c->emb_type == ORC_EMB_Q4_0) orc_quantize_gguf_q4_0(tmp, ne, m->raw[0]);
  else if (c->emb_type == ORC_EMB_Q8_0) orc_quantize_gguf_q8_0(tmp, ne, m->raw[0]);
  else memcpy(m->raw[0], tmp, sizeof(float) * (size_t)ne);
  for (int l = 0; l < c->n_layers; ++l)
    for (int w = 1; w <= 7; ++w) {
      int r, k;
      mat_shape(c, w, &r, &k);
      int64_t n = (int64_t)r * k;
      int t = tidx(l, w);
      float* buf = n <= ne ? tmp : (float*)malloc(sizeof(float) * (size_t)n);
      orc_synth_weights(buf, n, seed, (uint64_t)t, stdev);
      if (c->kind == ORC_KIND_STREAMING_Q4) orc_quantize_gguf_q4_0(buf, n, m->raw[t]);
      else orc_quantize_q8a(buf, n, m->q8a_scales[t], (int8_t*)m->raw[t]);
      if (buf != tmp) free(buf);
    }
  free(tmp);
  orc_model_refresh(m);
}

void orc_reset_cache(orc_model* m) {
  int kv = m->c.n_kv_heads * m->c.head_dim;
  size_t n = (size_t)m->c.n_layers * m->c.seq_len * kv;
  memset(m->kc, 0, n * sizeof(float));
  memset(m->vc, 0, n * sizeof(float));
}

void orc_rollback_cache(orc_model* m, int pos) {
  int kv = m->c.n_kv_heads * m->c.head_dim;
  if (pos < 0) pos = 0;
  for (int l = 0; l < m->c.n_layers; ++l)
    for (int p = pos; p < m->c.seq_len; ++p) {
      memset(orc_kv(m, l, 0) + (size_t)p * kv, 0, sizeof(float) * kv);
      memset(orc_kv(m, l, 1) + (size_t)p * kv, 0, sizeof(float) * kv);
    }
}

/* Streaming prefill LINEAR: dequantize the GGUF rows (gguf.js:259-286),
 * transpose to [in][out] (streaming-loader.js:196-200) and run the WASM
 * matmul (llama-streaming.js:398 -> engine.js:190 -> wasm-simd.js:469). */
static void prefill_linear(const uint8_t* raw, int rows_out, int cols_in, const float* x, int M, float* out) {
  int64_t n = (int64_t)rows_out * cols_in;
  float* w = (float*)malloc(sizeof(float) * (size_t)n);
  float* wt = (float*)malloc(sizeof(float) * (size_t)n);
  orc_dequant_q4_0(raw, n, w);
  for (int r = 0; r < rows_out; ++r)
    for (int k = 0; k < cols_in; ++k) wt[(size_t)k * rows_out + r] = w[(size_t)r * cols_in + k];
  orc_matmul_wasm(x, M, cols_in, wt, rows_out, NULL, out);
  free(w);
  free(wt);
}

/* llama-streaming.js:350-493 (seq > 1) */
static void run_layer_prefill(orc_model* m, int l, float* x, int seq, int start_pos) {
  const orc_config* c = &m->c;
  int dim = c->dim, F = c->hidden_dim, kv = c->n_kv_heads * c->head_dim;
  float* xn = (float*)malloc(sizeof(float) * (size_t)seq * dim);
  float* q = (float*)malloc(sizeof(float) * (size_t)seq * dim);
  float* k = (float*)malloc(sizeof(float) * (size_t)seq * kv);
  float* v = (float*)malloc(sizeof(float) * (size_t)seq * kv);
  float* att = (float*)malloc(sizeof(float) * (size_t)seq * dim);
  float* proj = (float*)malloc(sizeof(float) * (size_t)seq * dim);
  float* g = (float*)malloc(sizeof(float) * (size_t)seq * F);
  float* ga = (float*)malloc(sizeof(float) * (size_t)seq * F);
  float* u = (float*)malloc(sizeof(float) * (size_t)seq * F);
  float* h = (float*)malloc(sizeof(float) * (size_t)seq * F);

  orc_rmsnorm(x, seq, dim, m->rms_att + (size_t)l * dim, c->eps, xn);
  prefill_linear(m->raw[tidx(l, 1)], dim, dim, xn, seq, q);
  prefill_linear(m->raw[tidx(l, 2)], kv, dim, xn, seq, k);
  prefill_linear(m->raw[tidx(l, 3)], kv, dim, xn, seq, v);
  orc_rope(q, k, seq, start_pos, dim, c->n_heads, c->n_kv_heads, c->head_dim, c->rope_theta);
  float *kc = orc_kv(m, l, 0), *vc = orc_kv(m, l, 1);
  for (int t = 0; t < seq; ++t) {
    memcpy(kc + (size_t)(start_pos + t) * kv, k + (size_t)t * kv, sizeof(float) * kv);
    memcpy(vc + (size_t)(start_pos + t) * kv, v + (size_t)t * kv, sizeof(float) * kv);
  }
  orc_attn_cached(q, kc, vc, seq, start_pos, dim, c->n_heads, c->n_kv_heads, c->head_dim, att);
  prefill_linear(m->raw[tidx(l, 4)], dim, dim, att, seq, proj);
  orc_tensoradd(x, proj, (int64_t)seq * dim, x);
  orc_rmsnorm(x, seq, dim, m->rms_ffn + (size_t)l * dim, c->eps, xn);
  prefill_linear(m->raw[tidx(l, 5)], F, dim, xn, seq, g);
  orc_silu(g, (int64_t)seq * F, ga);
  prefill_linear(m->raw[tidx(l, 7)], F, dim, xn, seq, u);
  orc_elementmul(ga, u, (int64_t)seq * F, h);
  prefill_linear(m->raw[tidx(l, 6)], dim, F, h, seq, proj);
  orc_tensoradd(x, proj, (int64_t)seq * dim, x);
  free(xn); free(q); free(k); free(v); free(att); free(proj); free(g); free(ga); free(u); free(h);
}

/* llama-streaming.js:505-606 (seq == 1): raw Q4_0 matvecs in WASM order. */
static void run_layer_q4(orc_model* m, int l, float* x, int start_pos) {
  const orc_config* c = &m->c;
  int dim = c->dim, F = c->hidden_dim, kv = c->n_kv_heads * c->head_dim;
  float* xn = (float*)malloc(sizeof(float) * dim);
  float* q = (float*)malloc(sizeof(float) * dim);
  float* k = (float*)malloc(sizeof(float) * kv);
  float* v = (float*)malloc(sizeof(float) * kv);
  float* att = (float*)malloc(sizeof(float) * dim);
  float* proj = (float*)malloc(sizeof(float) * dim);
  float* g = (float*)malloc(sizeof(float) * F);
  float* u = (float*)malloc(sizeof(float) * F);
  float* h = (float*)malloc(sizeof(float) * F);

  orc_rmsnorm(x, 1, dim, m->rms_att + (size_t)l * dim, c->eps, xn);
  orc_q4_0_matvec_wasm(xn, m->raw[tidx(l, 1)], dim, dim, q);
  orc_q4_0_matvec_wasm(xn, m->raw[tidx(l, 2)], kv, dim, k);
  orc_q4_0_matvec_wasm(xn, m->raw[tidx(l, 3)], kv, dim, v);
  orc_rope(q, k, 1, start_pos, dim, c->n_heads, c->n_kv_heads, c->head_dim, c->rope_theta);
  float *kc = orc_kv(m, l, 0), *vc = orc_kv(m, l, 1);
  memcpy(kc + (size_t)start_pos * kv, k, sizeof(float) * kv);
  memcpy(vc + (size_t)start_pos * kv, v, sizeof(float) * kv);
  orc_attn_cached(q, kc, vc, 1, start_pos, dim, c->n_heads, c->n_kv_heads, c->head_dim, att);
  orc_q4_0_matvec_wasm(att, m->raw[tidx(l, 4)], dim, dim, proj);
  for (int d = 0; d < dim; ++d) x[d] = (float)((double)x[d] + (double)proj[d]);
  orc_rmsnorm(x, 1, dim, m->rms_ffn + (size_t)l * dim, c->eps, xn);
  orc_q4_0_matvec_wasm(xn, m->raw[tidx(l, 5)], F, dim, g);
  orc_q4_0_matvec_wasm(xn, m->raw[tidx(l, 7)], F, dim, u);
  orc_swiglu_fused(g, u, F, h);
  orc_q4_0_matvec_wasm(h, m->raw[tidx(l, 6)], dim, F, proj);
  for (int d = 0; d < dim; ++d) x[d] = (float)((double)x[d] + (double)proj[d]);
  free(xn); free(q); free(k); free(v); free(att); free(proj); free(g); free(u); free(h);
}

/* llama.js:228-337: every LINEAR goes to matmul_q8 (purebee.js:81-82); the
 * SwiGLU is SILU then ELEMENT_MUL for prefill and decode alike. */
static void run_layer_q8a(orc_model* m, int l, float* x, int seq, int start_pos) {
  const orc_config* c = &m->c;
  int dim = c->dim, F = c->hidden_dim, kv = c->n_kv_heads * c->head_dim;
  float* xn = (float*)malloc(sizeof(float) * (size_t)seq * dim);
  float* q = (float*)malloc(sizeof(float) * (size_t)seq * dim);
  float* k = (float*)malloc(sizeof(float) * (size_t)seq * kv);
  float* v = (float*)malloc(sizeof(float) * (size_t)seq * kv);
  float* att = (float*)malloc(sizeof(float) * (size_t)seq * dim);
  float* proj = (float*)malloc(sizeof(float) * (size_t)seq * dim);
  float* g = (float*)malloc(sizeof(float) * (size_t)seq * F);
  float* ga = (float*)malloc(sizeof(float) * (size_t)seq * F);
  float* u = (float*)malloc(sizeof(float) * (size_t)seq * F);
  float* h = (float*)malloc(sizeof(float) * (size_t)seq * F);
#define Q8(w, xin, K_, N_, out) \
  orc_matmul_q8(xin, seq, K_, m->q8a_scales[tidx(l, w)], (const int8_t*)m->raw[tidx(l, w)], N_, NULL, out)
  orc_rmsnorm(x, seq, dim, m->rms_att + (size_t)l * dim, c->eps, xn);
  Q8(1, xn, dim, dim, q);
  Q8(2, xn, dim, kv, k);
  Q8(3, xn, dim, kv, v);
  orc_rope(q, k, seq, start_pos, dim, c->n_heads, c->n_kv_heads, c->head_dim, c->rope_theta);
  float *kc = orc_kv(m, l, 0), *vc = orc_kv(m, l, 1);
  for (int t = 0; t < seq; ++t) {
    memcpy(kc + (size_t)(start_pos + t) * kv, k + (size_t)t * kv, sizeof(float) * kv);
    memcpy(vc + (size_t)(start_pos + t) * kv, v + (size_t)t * kv, sizeof(float) * kv);
  }
  orc_attn_cached(q, kc, vc, seq, start_pos, dim, c->n_heads, c->n_kv_heads, c->head_dim, att);
  Q8(4, att, dim, dim, proj);
  orc_tensoradd(x, proj, (int64_t)seq * dim, x);
  orc_rmsnorm(x, seq, dim, m->rms_ffn + (size_t)l * dim, c->eps, xn);
  Q8(5, xn, dim, F, g);
  orc_silu(g, (int64_t)seq * F, ga);
  Q8(7, xn, dim, F, u);
  orc_elementmul(ga, u, (int64_t)seq * F, h);
  Q8(6, h, F, dim, proj);
  orc_tensoradd(x, proj, (int64_t)seq * dim, x);
#undef Q8
  free(xn); free(q); free(k); free(v); free(att); free(proj); free(g); free(ga); free(u); free(h);
}

typedef struct { const float* h; const float* E; int dim; float* out; } hd_args;
/* llama.js:359-367: logit = f32(sum_d h[d]*E[v,d]) in double. */
static void head_double_rows(void* c, int64_t lo, int64_t hi) {
  hd_args* a = (hd_args*)c;
  for (int64_t v = lo; v < hi; ++v) {
    const float* e = a->E + (size_t)v * a->dim;
    double dot = 0;
    for (int d = 0; d < a->dim; ++d) dot += (double)a->h[d] * (double)e[d];
    a->out[v] = (float)dot;
  }
}

/* An untied LM head (GGUF output.weight, streaming-loader.js:77-86 and
 * :330-334): dequantized to f32 like the embedding, then used by the head in
 * place of the tied table. */
int orc_model_set_head(orc_model* m, int emb_type, const uint8_t* raw) {
  const int64_t ne = (int64_t)m->c.vocab * m->c.dim;
  if (!m->head_f32) m->head_f32 = (float*)malloc(sizeof(float) * (size_t)ne);
  if (emb_type == ORC_EMB_Q4_0) orc_dequant_q4_0(raw, ne, m->head_f32);
  else if (emb_type == ORC_EMB_Q8_0) orc_dequant_q8_0(raw, ne, m->head_f32);
  else if (emb_type == ORC_EMB_F32) memcpy(m->head_f32, raw, sizeof(float) * (size_t)ne);
  else return -1;
  return 0;
}

typedef struct { double v; int i; } orc_vi;
static int orc_vi_cmp(const void* a, const void* b) {
  const orc_vi* x = (const orc_vi*)a;
  const orc_vi* y = (const orc_vi*)b;
  if (x->v != y->v) return x->v > y->v ? -1 : 1; /* value descending */
  return x->i - y->i;                            /* stable: lower index first */
}

/* final RMSNorm and LM head of one hidden state (llama-streaming.js:616-679). */
static void orc_head(orc_model* m, const float* x, float* logits) {
  const orc_config* c = &m->c;
  float* hn = (float*)malloc(sizeof(float) * c->dim);
  orc_rmsnorm(x, 1, c->dim, m->rms_final, c->eps, hn);
  if (c->kind == ORC_KIND_LLAMA_Q8A) {
    hd_args a = {hn, m->emb_f32, c->dim, logits};
    orc_parallel_rows(c->vocab, head_double_rows, &a);
  } else {
    /* llama-streaming.js:640-642 -> wasm-q4.js:798-839 (batch_dot) */
    orc_batch_dot(hn, m->head_f32 ? m->head_f32 : m->emb_f32, c->vocab, c->dim, logits);
  }
  free(hn);
}

/* _checkEarlyExit's confidence (llama-streaming.js:695-725), with the tail
 * count the code means (logits.length - topK; the reference reads an
 * undefined `candidates` there and throws). */
double orc_exit_prob(const float* logits, int V) {
  orc_vi* a = (orc_vi*)malloc(sizeof(orc_vi) * (size_t)(V > 0 ? V : 1));
  int n = 0;
  for (int i = 0; i < V; ++i)
    if (logits[i] == logits[i]) { a[n].v = (double)logits[i]; a[n].i = i; ++n; }
  qsort(a, (size_t)n, sizeof(orc_vi), orc_vi_cmp);
  const int top = n < 8 ? n : 8;
  double s = 0;
  for (int i = 0; i < top; ++i) s += exp(a[i].v - a[0].v);
  const int tail = V - 8 > 0 ? V - 8 : 0;
  s += (double)tail * exp(-20.0);
  free(a);
  return exp(0.0) / s;
}

/* forward(tokenIds, startPos, {maxLayers}) with the early exit of
 * llama-streaming.js:746-803 (single tokens, every `interval` layers, not
 * after the last layer). */
int orc_forward_ex(orc_model* m, const int* tokens, int n, int start_pos, int max_layers, double exit_threshold,
                   int exit_interval, float* logits, int* layers_used) {
  const orc_config* c = &m->c;
  int dim = c->dim;
  if (n <= 0 || start_pos < 0 || start_pos + n > c->seq_len) return -1;
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= c->vocab) return -2;
  const int L = max_layers <= 0 || max_layers > c->n_layers ? c->n_layers : max_layers;
  const int interval = exit_interval > 0 ? exit_interval : 4;
  const int early = exit_threshold > 0 && n == 1;
  float* x = (float*)malloc(sizeof(float) * (size_t)n * dim);
  for (int i = 0; i < n; ++i) memcpy(x + (size_t)i * dim, m->emb_f32 + (size_t)tokens[i] * dim, sizeof(float) * dim);
  int used = 0, exited = 0;
  for (int l = 0; l < L && !exited; ++l) {
    if (c->kind == ORC_KIND_LLAMA_Q8A) run_layer_q8a(m, l, x, n, start_pos);
    else if (n == 1) run_layer_q4(m, l, x, start_pos);
    else run_layer_prefill(m, l, x, n, start_pos);
    ++used;
    if (early && l < c->n_layers - 1 && (l + 1) % interval == 0) {
      orc_head(m, x, logits);
      if (orc_exit_prob(logits, c->vocab) >= exit_threshold) exited = 1;
    }
  }
  if (!exited) orc_head(m, x + (size_t)(n - 1) * dim, logits);
  if (layers_used) *layers_used = used;
  free(x);
  return 0;
}

int orc_forward(orc_model* m, const int* tokens, int n, int start_pos, float* logits) {
  return orc_forward_ex(m, tokens, n, start_pos, 0, 0.0, 0, logits, NULL);
}

int orc_generate(orc_model* m, const int* prompt, int n_prompt, int max_tokens, int eos_id, int* out, int cap) {
  float* logits = (float*)malloc(sizeof(float) * (size_t)m->c.vocab);
  orc_reset_cache(m);
  int cnt = 0;
  for (int i = 0; i < n_prompt && cnt < cap; ++i) out[cnt++] = prompt[i];
  if (orc_forward(m, prompt, n_prompt, 0, logits) != 0) { free(logits); return -1; }
  int pos = n_prompt;
  int next = orc_argmax(logits, m->c.vocab);
  if (cnt < cap) out[cnt++] = next;
  for (int i = 1; i < max_tokens; ++i) {
    if (next == eos_id) break;
    if (orc_forward(m, &next, 1, pos, logits) != 0) break;
    pos++;
    next = orc_argmax(logits, m->c.vocab);
    if (cnt < cap) out[cnt++] = next;
    if (next == eos_id) break;
  }
  free(logits);
  return cnt;
}

/* ---- sampling (llama-streaming.js:868-894) ---------------------------- */

/* sample(logits, topK, temperature) with the uniform draw r given (the
 * reference's Math.random()).  NaN logits are left out of the ranking. */
int orc_sample(const float* logits, int V, int topK, double temperature, double r) {
  orc_vi* a = (orc_vi*)malloc(sizeof(orc_vi) * (size_t)(V > 0 ? V : 1));
  int n = 0;
  for (int i = 0; i < V; ++i)
    if (logits[i] == logits[i]) { a[n].v = (double)logits[i] / temperature; a[n].i = i; ++n; }
  qsort(a, (size_t)n, sizeof(orc_vi), orc_vi_cmp);
  const int k = topK < n ? topK : n;
  int tok = k > 0 ? a[0].i : 0;
  if (k > 0) {
    double* e = (double*)malloc(sizeof(double) * (size_t)k);
    const double maxv = a[0].v;
    double sum = 0;
    for (int i = 0; i < k; ++i) { e[i] = exp(a[i].v - maxv); sum += e[i]; }
    double cum = 0;
    for (int i = 0; i < k; ++i) {
      cum += e[i] / sum;
      if (r <= cum) { tok = a[i].i; break; }
    }
    free(e);
  }
  free(a);
  return tok;
}

/* splitmix64 (Steele, Lea, Flood 2014) of seed + (counter + 1) * golden
 * gamma, top 53 bits as a double in [0, 1): the draw the device uses. */
double orc_sample_uniform(uint64_t seed, uint64_t counter) {
  uint64_t z = seed + (counter + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (double)(z >> 11) * (1.0 / 9007199254740992.0);
}
