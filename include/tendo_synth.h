/*
 * tendo_synth.h — deterministic, counter-based synthetic workload generator.
 *
 * The benchmark workloads are defined by distribution and seed only: weights
 * N(0, 0.02) fp32, microbench activations N(0, 1), prompt tokens uniform over
 * [0, vocab).  Any element can be produced on its own from (seed, stream,
 * index), so a 70B weight matrix can be streamed row by row on the GPU and
 * any row re-derived on the host for a check, bit for bit.
 *
 * Bit-identity between gcc (host) and nvcc (device) is the whole point:
 *  - integer mixing is splitmix64 (Steele, Lea, Flood 2014);
 *  - normals are Box–Muller in fp64, built only from +, -, *, / and sqrt
 *    (IEEE correctly rounded everywhere) with no fused multiply-add: on the
 *    device every operation goes through an explicit _rn intrinsic; host code
 *    that includes this header must be compiled with -ffp-contract=off;
 *  - ln(u) uses the atanh series ln m = 2*(s + s^3/3 + s^5/5 + ...),
 *    s = (m-1)/(m+1), after splitting u = m * 2^e with m in [sqrt(1/2), sqrt(2));
 *  - sin/cos of 2*pi*u use the quadrant split of u and the Taylor series on
 *    [0, pi/2) evaluated by Horner's rule.
 * None of this calls a libm or CUDA math routine.
 */
#ifndef TENDO_SYNTH_H
#define TENDO_SYNTH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define TS_HD __host__ __device__ __forceinline__
#else
#define TS_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define TS_MUL(a, b) __dmul_rn((a), (b))
#define TS_ADD(a, b) __dadd_rn((a), (b))
#define TS_SUB(a, b) __dsub_rn((a), (b))
#define TS_DIV(a, b) __ddiv_rn((a), (b))
#define TS_SQRT(a) __dsqrt_rn(a)
#else
#include <math.h>
#include <string.h>
#define TS_MUL(a, b) ((a) * (b))
#define TS_ADD(a, b) ((a) + (b))
#define TS_SUB(a, b) ((a) - (b))
#define TS_DIV(a, b) ((a) / (b))
#define TS_SQRT(a) sqrt(a)
#endif

/* Stream ids of the synthetic model (stream = layer * TS_MATS + matrix). */
enum {
  TS_MAT_Q = 0, TS_MAT_K = 1, TS_MAT_V = 2, TS_MAT_O = 3,
  TS_MAT_GATE = 4, TS_MAT_UP = 5, TS_MAT_DOWN = 6,
  TS_MATS = 8
};
/* Streams outside the per-layer range. */
#define TS_STREAM_EMBED 0x7fff0001ull
#define TS_STREAM_LMHEAD 0x7fff0002ull
#define TS_STREAM_PROMPT 0x7fff0003ull
#define TS_STREAM_X 0x7fff0004ull
#define TS_STREAM_W 0x7fff0005ull

TS_HD uint64_t ts_mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* Key of one (seed, stream) pair. */
TS_HD uint64_t ts_key(uint64_t seed, uint64_t stream) {
  return ts_mix64(ts_mix64(seed) ^ (stream * 0xD1B54A32D192ED03ull));
}

TS_HD uint64_t ts_bits(uint64_t key, uint64_t counter) {
  return ts_mix64(key + counter * 0x9E3779B97F4A7C15ull);
}

TS_HD double ts_d_from_bits(uint64_t b) {
#if defined(__CUDA_ARCH__)
  return __longlong_as_double((long long)b);
#else
  double d;
  memcpy(&d, &b, sizeof d);
  return d;
#endif
}

TS_HD uint64_t ts_bits_from_d(double d) {
#if defined(__CUDA_ARCH__)
  return (uint64_t)__double_as_longlong(d);
#else
  uint64_t b;
  memcpy(&b, &d, sizeof b);
  return b;
#endif
}

/* Natural log of u in (0, 1] (u is a normal number here: u >= 2^-53). */
TS_HD double ts_ln(double u) {
  uint64_t b = ts_bits_from_d(u);
  int e = (int)((b >> 52) & 0x7ff) - 1023;
  double m = ts_d_from_bits((b & 0x000FFFFFFFFFFFFFull) | 0x3FF0000000000000ull); /* [1,2) */
  if (m > 1.4142135623730951) { /* sqrt(2) */
    m = TS_MUL(m, 0.5);
    e += 1;
  }
  double s = TS_DIV(TS_SUB(m, 1.0), TS_ADD(m, 1.0));
  double s2 = TS_MUL(s, s);
  /* Horner over 1/(2k+1), k = 13..0 */
  double p = 1.0 / 27.0;
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 25.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 23.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 21.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 19.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 17.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 15.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 13.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 11.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 9.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 7.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 5.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0 / 3.0);
  p = TS_ADD(TS_MUL(p, s2), 1.0);
  double lnm = TS_MUL(TS_MUL(2.0, s), p);
  return TS_ADD(TS_MUL((double)e, 0.69314718055994530942), lnm);
}

/* sin and cos of a in [0, pi/2), Taylor series to a^23 / a^22. */
TS_HD void ts_sincos_q(double a, double* sn, double* cs) {
  double a2 = TS_MUL(a, a);
  /* Alternating Horner chains in a^2 with inverse-factorial constants, which
     the compilers fold identically: sin a = a*(1 - a^2/3! + a^4/5! - ...). */
  double ps = 1.0 / 25852016738884976640000.0;               /* 1/23! */
  ps = TS_SUB(1.0 / 51090942171709440000.0, TS_MUL(ps, a2)); /* 1/21! - a2/23! */
  ps = TS_SUB(1.0 / 121645100408832000.0, TS_MUL(ps, a2));   /* 1/19! */
  ps = TS_SUB(1.0 / 355687428096000.0, TS_MUL(ps, a2));      /* 1/17! */
  ps = TS_SUB(1.0 / 1307674368000.0, TS_MUL(ps, a2));        /* 1/15! */
  ps = TS_SUB(1.0 / 6227020800.0, TS_MUL(ps, a2));           /* 1/13! */
  ps = TS_SUB(1.0 / 39916800.0, TS_MUL(ps, a2));             /* 1/11! */
  ps = TS_SUB(1.0 / 362880.0, TS_MUL(ps, a2));               /* 1/9! */
  ps = TS_SUB(1.0 / 5040.0, TS_MUL(ps, a2));                 /* 1/7! */
  ps = TS_SUB(1.0 / 120.0, TS_MUL(ps, a2));                  /* 1/5! */
  ps = TS_SUB(1.0 / 6.0, TS_MUL(ps, a2));                    /* 1/3! */
  ps = TS_SUB(1.0, TS_MUL(ps, a2));
  *sn = TS_MUL(a, ps);
  double pc = 1.0 / 1124000727777607680000.0;                /* 1/22! */
  pc = TS_SUB(1.0 / 2432902008176640000.0, TS_MUL(pc, a2));  /* 1/20! */
  pc = TS_SUB(1.0 / 6402373705728000.0, TS_MUL(pc, a2));     /* 1/18! */
  pc = TS_SUB(1.0 / 20922789888000.0, TS_MUL(pc, a2));       /* 1/16! */
  pc = TS_SUB(1.0 / 87178291200.0, TS_MUL(pc, a2));          /* 1/14! */
  pc = TS_SUB(1.0 / 479001600.0, TS_MUL(pc, a2));            /* 1/12! */
  pc = TS_SUB(1.0 / 3628800.0, TS_MUL(pc, a2));              /* 1/10! */
  pc = TS_SUB(1.0 / 40320.0, TS_MUL(pc, a2));                /* 1/8! */
  pc = TS_SUB(1.0 / 720.0, TS_MUL(pc, a2));                  /* 1/6! */
  pc = TS_SUB(1.0 / 24.0, TS_MUL(pc, a2));                   /* 1/4! */
  pc = TS_SUB(1.0 / 2.0, TS_MUL(pc, a2));                    /* 1/2! */
  pc = TS_SUB(1.0, TS_MUL(pc, a2));
  *cs = pc;
}

/* Standard normal draw number `index` of the (seed, stream) sequence.
 * Draws come in Box–Muller pairs: pair p = index / 2 uses two 53-bit
 * uniforms; even indices take r*cos(t), odd ones r*sin(t). */
TS_HD double ts_normal(uint64_t key, uint64_t index) {
  uint64_t p = index >> 1;
  uint64_t b1 = ts_bits(key, 2 * p);
  uint64_t b2 = ts_bits(key, 2 * p + 1);
  double u1 = TS_MUL((double)((b1 >> 11) + 1), 1.1102230246251565e-16); /* (0, 1] */
  double u2 = TS_MUL((double)(b2 >> 11), 1.1102230246251565e-16);       /* [0, 1) */
  double r = TS_SQRT(TS_MUL(-2.0, ts_ln(u1)));
  double t4 = TS_MUL(u2, 4.0); /* quadrant coordinate in [0, 4) */
  int q = (int)t4;
  double f = TS_SUB(t4, (double)q);
  double a = TS_MUL(f, 1.5707963267948966); /* pi / 2 */
  double sn, cs;
  ts_sincos_q(a, &sn, &cs);
  double c, s;
  switch (q & 3) {
    case 0: c = cs; s = sn; break;
    case 1: c = -sn; s = cs; break;
    case 2: c = -cs; s = -sn; break;
    default: c = sn; s = -cs; break;
  }
  return TS_MUL(r, (index & 1) ? s : c);
}

/* fp32 draw of N(0, std): the fp64 product rounded once to fp32. */
TS_HD float ts_normal_f32(uint64_t key, uint64_t index, double std_) {
  return (float)TS_MUL(ts_normal(key, index), std_);
}

/* Uniform integer in [0, n) (multiply-shift on the top 32 bits). */
TS_HD uint32_t ts_uniform_int(uint64_t key, uint64_t index, uint32_t n) {
  uint64_t b = ts_bits(key, index) >> 32;
  return (uint32_t)((b * (uint64_t)n) >> 32);
}

/* Uniform float in [0, 1): the top 24 bits of the draw times 2^-24 (exact in
 * fp32, identical on host and device). */
TS_HD float ts_uniform_f32(uint64_t key, uint64_t index) {
  return (float)(uint32_t)(ts_bits(key, index) >> 40) * (1.0f / 16777216.0f);
}

#define TS_STREAM_SAMPLE 0x7fff0006ull /* the sampler's uniforms: index = step * B + row */

#endif /* TENDO_SYNTH_H */
