/*
 * pb_synth.h - seeded synthetic inputs, bit-identical on host and device.
 *
 * The benchmark configurations use random-init weights N(0, std) and random
 * token ids from a fixed seed.  The same values must come out of the CUDA
 * library (which fills device memory directly) and out of the CPU oracle
 * (which fills host memory), so this generator uses only integer mixing and
 * IEEE basic operations (+ - * / sqrt), each correctly rounded on both sides:
 *
 *   - counter-based SplitMix64 (Steele, Lea, Flood 2014): value i of tensor t
 *     depends only on (seed, t, i), so any thread can produce any element;
 *   - Box-Muller (1958) normal from two uniforms in (0,1);
 *   - ln(u) by exponent split plus the atanh series
 *     ln(m) = 2*(s + s^3/3 + s^5/5 + ...), s = (m-1)/(m+1), m in [sqrt(1/2), sqrt(2));
 *   - cos(2*pi*u) by quadrant reduction on u itself and Taylor series in
 *     Horner form for |r| <= pi/4.
 *
 * On the device every double operation goes through a *_rn intrinsic so the
 * compiler cannot contract a multiply and an add into one FMA; on the host the
 * translation units that include this header are built with
 * -ffp-contract=off.  No libm call is made anywhere in this file.
 */
#ifndef PB_SYNTH_H
#define PB_SYNTH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define PB_HD __host__ __device__ __forceinline__
#else
#define PB_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define PB_DADD(a, b) __dadd_rn((a), (b))
#define PB_DSUB(a, b) __dsub_rn((a), (b))
#define PB_DMUL(a, b) __dmul_rn((a), (b))
#define PB_DDIV(a, b) __ddiv_rn((a), (b))
#define PB_DSQRT(a) __dsqrt_rn(a)
#else
#define PB_DADD(a, b) ((a) + (b))
#define PB_DSUB(a, b) ((a) - (b))
#define PB_DMUL(a, b) ((a) * (b))
#define PB_DDIV(a, b) ((a) / (b))
PB_HD double pb__host_sqrt(double v) {
  /* correctly rounded square root without libm: SSE2 sqrtsd */
#if defined(__x86_64__)
  double r;
  __asm__("sqrtsd %1, %0" : "=x"(r) : "x"(v));
  return r;
#else
  return __builtin_sqrt(v);
#endif
}
#define PB_DSQRT(a) pb__host_sqrt(a)
#endif

#define PB_GOLDEN 0x9E3779B97F4A7C15ULL

/* Tensor ids used by the synthetic models: embedding 0, then per layer
 * [wq, wk, wv, wo, w1, w2, w3] at 1 + 7*l + j, an untied head at 1 + 7*L,
 * and the prompt token stream at PB_SYNTH_TOKEN_STREAM. */
#define PB_SYNTH_TOKEN_STREAM 0x70C3E5ULL

PB_HD uint64_t pb_mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

/* Key of one tensor's stream. */
PB_HD uint64_t pb_stream_key(uint64_t seed, uint64_t tensor_id) {
  return pb_mix64(seed ^ pb_mix64(tensor_id * PB_GOLDEN + 0x1234567ULL));
}

/* The j-th 64-bit word of a stream. */
PB_HD uint64_t pb_stream_word(uint64_t key, uint64_t j) {
  return pb_mix64(key + (j + 1) * PB_GOLDEN);
}

/* Uniform double strictly inside (0, 1): 53 random bits plus one half ulp. */
PB_HD double pb_u01(uint64_t bits) {
  return ((double)(bits >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

PB_HD double pb_bits_to_double(uint64_t b) {
  union { uint64_t u; double d; } c;
  c.u = b;
  return c.d;
}
PB_HD uint64_t pb_double_to_bits(double d) {
  union { uint64_t u; double d; } c;
  c.d = d;
  return c.u;
}

/* Natural log of u in (0, 1) (normal numbers only, which pb_u01 guarantees). */
PB_HD double pb_ln(double u) {
  uint64_t b = pb_double_to_bits(u);
  int e = (int)((b >> 52) & 0x7FF) - 1023;
  double m = pb_bits_to_double((b & 0x000FFFFFFFFFFFFFULL) | 0x3FF0000000000000ULL);
  if (m > 1.4142135623730951) { /* keep m in [sqrt(1/2), sqrt(2)) */
    m = PB_DMUL(m, 0.5);
    e += 1;
  }
  double s = PB_DDIV(PB_DSUB(m, 1.0), PB_DADD(m, 1.0));
  double s2 = PB_DMUL(s, s);
  /* 2*atanh(s) = 2*s*(1 + s2/3 + s2^2/5 + ...), Horner from the top term */
  double t = PB_DDIV(1.0, 27.0);
  for (int k = 12; k >= 0; --k) t = PB_DADD(PB_DDIV(1.0, (double)(2 * k + 1)), PB_DMUL(s2, t));
  double lnm = PB_DMUL(PB_DMUL(2.0, s), t);
  const double ln2 = 0.69314718055994530942;
  return PB_DADD(PB_DMUL((double)e, ln2), lnm);
}

/* sin and cos of r for |r| <= pi/4 by Taylor series in Horner form. */
PB_HD double pb_cos_small(double r) {
  double r2 = PB_DMUL(r, r);
  double t = 1.0;
  for (int k = 9; k >= 1; --k) /* 1 - r2/((2k-1)(2k)) * t */
    t = PB_DSUB(1.0, PB_DMUL(PB_DDIV(r2, (double)((2 * k - 1) * (2 * k))), t));
  return t;
}
PB_HD double pb_sin_small(double r) {
  double r2 = PB_DMUL(r, r);
  double t = 1.0;
  for (int k = 9; k >= 1; --k) /* 1 - r2/((2k)(2k+1)) * t */
    t = PB_DSUB(1.0, PB_DMUL(PB_DDIV(r2, (double)((2 * k) * (2 * k + 1))), t));
  return PB_DMUL(r, t);
}

/* cos(2*pi*u) for u in (0, 1). */
PB_HD double pb_cos2pi(double u) {
  double u4 = PB_DMUL(u, 4.0);            /* exact */
  double qf = (double)(int64_t)PB_DADD(u4, 0.5); /* floor for positive values */
  double t = PB_DSUB(u4, qf);             /* in [-0.5, 0.5], exact */
  const double half_pi = 1.5707963267948966;
  double r = PB_DMUL(t, half_pi);
  int q = ((int)qf) & 3;
  if (q == 0) return pb_cos_small(r);
  if (q == 1) return -pb_sin_small(r);
  if (q == 2) return -pb_cos_small(r);
  return pb_sin_small(r);
}

/* Standard normal sample number i of a stream (Box-Muller, cosine branch). */
PB_HD double pb_normal(uint64_t key, uint64_t i) {
  double u1 = pb_u01(pb_stream_word(key, 2 * i));
  double u2 = pb_u01(pb_stream_word(key, 2 * i + 1));
  double rad = PB_DSQRT(PB_DMUL(-2.0, pb_ln(u1)));
  return PB_DMUL(rad, pb_cos2pi(u2));
}

/* Weight value i of tensor `tensor_id`: float(std * N(0,1)). */
PB_HD float pb_synth_weight(uint64_t seed, uint64_t tensor_id, uint64_t i, double stdev) {
  return (float)PB_DMUL(stdev, pb_normal(pb_stream_key(seed, tensor_id), i));
}

/* Prompt token i: uniform integer in [lo, hi). */
PB_HD int pb_synth_token(uint64_t seed, uint64_t i, int lo, int hi) {
  uint64_t w = pb_stream_word(pb_stream_key(seed, PB_SYNTH_TOKEN_STREAM), i);
  return lo + (int)(w % (uint64_t)(hi - lo));
}

/* Activation vector value i: float(N(0,1)) (the matvec sweep's input). */
PB_HD float pb_synth_activation(uint64_t seed, uint64_t stream, uint64_t i) {
  return (float)pb_normal(pb_stream_key(seed, stream), i);
}

#endif /* PB_SYNTH_H */
