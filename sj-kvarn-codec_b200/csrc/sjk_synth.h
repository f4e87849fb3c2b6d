/*
 * sjk_synth.h - seeded synthetic K/V/Q rows of the benchmark configurations, bit-identical on the host (C) and
 * on the device (CUDA). Input generation only: nothing here is part of the codec.
 *
 * Distributions (the configurations' documented generator):
 *   K[pos][h][d] = X * s[layer][h][d]    X ~ N(0, 1), or Student-t(4) = N / sqrt(chi2_4 / 4) with
 *                                         chi2_4 = ((n0^2 + n1^2) + n2^2) + n3^2 when `heavy`
 *   s[layer][h][d] = exp(N(0, 1))        LogNormal(0, 1) channel scales; 4 distinct outlier channels per
 *                                         (layer, head), drawn from their own stream, have their scale x 8
 *   V[pos][h][d] ~ N(0, 1)
 *   Q[row][d] ~ N(0, 1) rounded to fp16 (round to nearest even), returned as float
 *
 * Randomness: SplitMix64 (G. Steele, D. Lea, C. Flood, "Fast splittable pseudorandom number generators",
 * OOPSLA 2014) used as a counter-based generator: draw i of a stream with key k is mix64(k + (i + 1) * gamma),
 * so every value is a pure function of (seed, layer, stream, index) and any range of positions can be produced
 * independently, in any order, on either side. Stream keys: key(seed, layer, kind) =
 * splitmix(splitmix(seed, layer), kind). Element j = (pos * H + h) * D + d of a K or V stream is a Box-Muller
 * normal (Box & Muller 1958): pair m = j / 2 takes draws 2m and 2m + 1 as uniforms u1, u2 in (0, 1]
 * (53-bit: ((x >> 11) + 1) * 2^-53), r = sqrt(-2 ln u1), and element 2m is r cos(2 pi u2), element 2m + 1 is
 * r sin(2 pi u2). The Student-t chi-square normals of element j are normals 4j .. 4j + 3 of the layer's
 * chi-square stream.
 *
 * Portability: every floating-point step is a correctly rounded IEEE-754 double operation (+, -, *, /, sqrt),
 * an exact one (floor, scaling by a power of two, splitting off the exponent) or a final rounding to float, with
 * no contraction into fused multiply-adds (the device uses the _rn intrinsics; the host is compiled with
 * -ffp-contract=off). ln, exp, cos and sin are therefore computed here rather than taken from a math library:
 *   ln u:  u = m 2^e with m in [sqrt(1/2), sqrt(2)), ln m = 2 atanh(s), s = (m - 1) / (m + 1), summed as the odd
 *          power series of atanh to s^25 (|s| < 0.1716), plus e ln 2 with ln 2 split into a 32-bit head and a tail;
 *   exp x: x = k ln 2 + r with k = floor(x / ln 2 + 1/2), e^r by its Taylor series to r^16 / 16!, times 2^k;
 *   cos / sin (2 pi v): v in turns, reduced exactly to a quarter turn q and a remainder f in [-1/2, 1/2) of a
 *          quarter, x = f pi / 2, Taylor series of sin x to x^19 and cos x to x^20, then the quadrant symmetry.
 * All constants are written as hexadecimal floats (each the correctly rounded value of the quantity named).
 * The series are accurate to about one unit in the last place, which is more than a data generator needs; the
 * point is that both sides evaluate the same operations in the same order.
 */
#ifndef SJK_SYNTH_H
#define SJK_SYNTH_H

#include <stdint.h>

#if defined(__CUDACC__)
#define SJK_SYN_FN static __host__ __device__ __forceinline__
#else
#define SJK_SYN_FN static inline
#include <math.h>
#include <string.h>
#endif

#if defined(__CUDA_ARCH__)
#define SJK_SYN_ADD(a, b) __dadd_rn((a), (b))
#define SJK_SYN_SUB(a, b) __dsub_rn((a), (b))
#define SJK_SYN_MUL(a, b) __dmul_rn((a), (b))
#define SJK_SYN_DIV(a, b) __ddiv_rn((a), (b))
#define SJK_SYN_SQRT(a) __dsqrt_rn(a)
#define SJK_SYN_FLOOR(a) floor(a)
#else
#define SJK_SYN_ADD(a, b) ((a) + (b))
#define SJK_SYN_SUB(a, b) ((a) - (b))
#define SJK_SYN_MUL(a, b) ((a) * (b))
#define SJK_SYN_DIV(a, b) ((a) / (b))
#define SJK_SYN_SQRT(a) sqrt(a)
#define SJK_SYN_FLOOR(a) floor(a)
#endif

#define SJK_SYN_GAMMA 0x9E3779B97F4A7C15ULL

enum { SJK_SYN_K = 0, SJK_SYN_V = 1, SJK_SYN_CHI = 2, SJK_SYN_SCALE = 3, SJK_SYN_OUTLIER = 4, SJK_SYN_Q = 5 };

SJK_SYN_FN uint64_t sjk_syn_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* draw i (i >= 0) of the SplitMix64 sequence whose state starts at `key` */
SJK_SYN_FN uint64_t sjk_syn_draw(uint64_t key, uint64_t i) { return sjk_syn_mix(key + (i + 1) * SJK_SYN_GAMMA); }

SJK_SYN_FN uint64_t sjk_syn_key(uint64_t seed, uint32_t layer, uint32_t kind) {
    return sjk_syn_draw(sjk_syn_draw(seed, layer), kind);
}

SJK_SYN_FN uint64_t sjk_syn_bits(double x) {
#if defined(__CUDA_ARCH__)
    return (uint64_t) __double_as_longlong(x);
#else
    uint64_t b;
    memcpy(&b, &x, 8);
    return b;
#endif
}

SJK_SYN_FN double sjk_syn_from_bits(uint64_t b) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long) b);
#else
    double x;
    memcpy(&x, &b, 8);
    return x;
#endif
}

/* uniform in (0, 1]: 53 random bits, never zero (exact) */
SJK_SYN_FN double sjk_syn_unif(uint64_t x) { return (double) ((x >> 11) + 1) * 0x1.0p-53; }

/* natural log of a positive normal double */
SJK_SYN_FN double sjk_syn_ln(double u) {
    const uint64_t b = sjk_syn_bits(u);
    int e = (int) ((b >> 52) & 0x7FF) - 1023;
    double m = sjk_syn_from_bits((b & 0x000FFFFFFFFFFFFFULL) | 0x3FF0000000000000ULL);     /* [1, 2) */
    if (m > 0x1.6a09e667f3bcdp+0) {                                                         /* > sqrt(2) */
        m = SJK_SYN_MUL(m, 0.5);
        e += 1;
    }
    const double s = SJK_SYN_DIV(SJK_SYN_SUB(m, 1.0), SJK_SYN_ADD(m, 1.0));
    const double s2 = SJK_SYN_MUL(s, s);
    /* 1 + s^2/3 + s^4/5 + ... + s^24/25, Horner from the highest term */
    double p = 0x1.47ae147ae147bp-5;                        /* 1/25 */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 0x1.642c8590b2164p-5);   /* 1/23 */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 0x1.8618618618618p-5);   /* 1/21 */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 0x1.af286bca1af28p-5);   /* 1/19 */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 0x1.e1e1e1e1e1e1ep-5);   /* 1/17 */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 0x1.1111111111111p-4);   /* 1/15 */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 0x1.3b13b13b13b14p-4);   /* 1/13 */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 0x1.745d1745d1746p-4);   /* 1/11 */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 0x1.c71c71c71c71cp-4);   /* 1/9 */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 0x1.2492492492492p-3);   /* 1/7 */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 0x1.999999999999ap-3);   /* 1/5 */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 0x1.5555555555555p-2);   /* 1/3 */
    const double lnm = SJK_SYN_MUL(SJK_SYN_MUL(2.0, s), SJK_SYN_ADD(SJK_SYN_MUL(p, s2), 1.0));
    const double de = (double) e;
    /* ln 2 = 0x1.62e42fee00000p-1 (32-bit head, e * head is exact) + 0x1.a39ef35793c76p-33 */
    return SJK_SYN_ADD(SJK_SYN_MUL(de, 0x1.62e42fee00000p-1), SJK_SYN_ADD(SJK_SYN_MUL(de, 0x1.a39ef35793c76p-33), lnm));
}

/* e^x for |x| < 700 */
SJK_SYN_FN double sjk_syn_exp(double x) {
    const double k = SJK_SYN_FLOOR(SJK_SYN_ADD(SJK_SYN_MUL(x, 0x1.71547652b82fep+0), 0.5));   /* x / ln 2 */
    const double r = SJK_SYN_SUB(SJK_SYN_SUB(x, SJK_SYN_MUL(k, 0x1.62e42fee00000p-1)), SJK_SYN_MUL(k, 0x1.a39ef35793c76p-33));
    double p = 0x1.ae7f3e733b81fp-45;                       /* 1/16! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.ae7f3e733b81fp-41);   /* 1/15! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.93974a8c07c9dp-37);   /* 1/14! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.6124613a86d09p-33);   /* 1/13! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.1eed8eff8d898p-29);   /* 1/12! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.ae64567f544e4p-26);   /* 1/11! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.27e4fb7789f5cp-22);   /* 1/10! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.71de3a556c734p-19);   /* 1/9! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.a01a01a01a01ap-16);   /* 1/8! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.a01a01a01a01ap-13);   /* 1/7! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.6c16c16c16c17p-10);   /* 1/6! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.1111111111111p-7);    /* 1/5! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.5555555555555p-5);    /* 1/4! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0x1.5555555555555p-3);    /* 1/3! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 0.5);                     /* 1/2! */
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 1.0);
    p = SJK_SYN_ADD(SJK_SYN_MUL(p, r), 1.0);
    /* times 2^k (exact: k is small and the result stays normal) */
    return SJK_SYN_MUL(p, sjk_syn_from_bits((uint64_t) (1023 + (int) k) << 52));
}

/* c = cos(2 pi v), s = sin(2 pi v) for v in [0, 1] */
SJK_SYN_FN void sjk_syn_cossin_turns(double v, double * c, double * s) {
    const double v4 = SJK_SYN_MUL(v, 4.0);                           /* exact */
    double q = SJK_SYN_FLOOR(SJK_SYN_ADD(v4, 0.5));                   /* nearest quarter turn */
    const double f = SJK_SYN_SUB(v4, q);                              /* exact, in [-1/2, 1/2) */
    const double x = SJK_SYN_MUL(f, 0x1.921fb54442d18p+0);           /* f pi / 2, |x| <= pi / 4 */
    const double x2 = SJK_SYN_MUL(x, x);
    double ps = -0x1.2f49b46814157p-57;                               /* -1/19! */
    ps = SJK_SYN_ADD(SJK_SYN_MUL(ps, x2), 0x1.952c77030ad4ap-49);    /* 1/17! */
    ps = SJK_SYN_ADD(SJK_SYN_MUL(ps, x2), -0x1.ae7f3e733b81fp-41);   /* -1/15! */
    ps = SJK_SYN_ADD(SJK_SYN_MUL(ps, x2), 0x1.6124613a86d09p-33);    /* 1/13! */
    ps = SJK_SYN_ADD(SJK_SYN_MUL(ps, x2), -0x1.ae64567f544e4p-26);   /* -1/11! */
    ps = SJK_SYN_ADD(SJK_SYN_MUL(ps, x2), 0x1.71de3a556c734p-19);    /* 1/9! */
    ps = SJK_SYN_ADD(SJK_SYN_MUL(ps, x2), -0x1.a01a01a01a01ap-13);   /* -1/7! */
    ps = SJK_SYN_ADD(SJK_SYN_MUL(ps, x2), 0x1.1111111111111p-7);     /* 1/5! */
    ps = SJK_SYN_ADD(SJK_SYN_MUL(ps, x2), -0x1.5555555555555p-3);    /* -1/3! */
    const double sx = SJK_SYN_ADD(SJK_SYN_MUL(SJK_SYN_MUL(ps, x2), x), x);
    double pc = 0x1.e542ba4020225p-62;                                /* 1/20! */
    pc = SJK_SYN_ADD(SJK_SYN_MUL(pc, x2), -0x1.6827863b97d97p-53);   /* -1/18! */
    pc = SJK_SYN_ADD(SJK_SYN_MUL(pc, x2), 0x1.ae7f3e733b81fp-45);    /* 1/16! */
    pc = SJK_SYN_ADD(SJK_SYN_MUL(pc, x2), -0x1.93974a8c07c9dp-37);   /* -1/14! */
    pc = SJK_SYN_ADD(SJK_SYN_MUL(pc, x2), 0x1.1eed8eff8d898p-29);    /* 1/12! */
    pc = SJK_SYN_ADD(SJK_SYN_MUL(pc, x2), -0x1.27e4fb7789f5cp-22);   /* -1/10! */
    pc = SJK_SYN_ADD(SJK_SYN_MUL(pc, x2), 0x1.a01a01a01a01ap-16);    /* 1/8! */
    pc = SJK_SYN_ADD(SJK_SYN_MUL(pc, x2), -0x1.6c16c16c16c17p-10);   /* -1/6! */
    pc = SJK_SYN_ADD(SJK_SYN_MUL(pc, x2), 0x1.5555555555555p-5);     /* 1/4! */
    pc = SJK_SYN_ADD(SJK_SYN_MUL(pc, x2), -0.5);                     /* -1/2! */
    const double cx = SJK_SYN_ADD(SJK_SYN_MUL(pc, x2), 1.0);
    const int quad = ((int) q) & 3;
    *c = quad == 0 ? cx : quad == 1 ? -sx : quad == 2 ? -cx : sx;
    *s = quad == 0 ? sx : quad == 1 ? cx : quad == 2 ? -sx : -cx;
}

/* Box-Muller pair m of the stream `key`: normals 2m (cosine) and 2m + 1 (sine) */
SJK_SYN_FN void sjk_syn_normal_pair(uint64_t key, uint64_t m, double * n0, double * n1) {
    const double u1 = sjk_syn_unif(sjk_syn_draw(key, 2 * m));
    const double u2 = sjk_syn_unif(sjk_syn_draw(key, 2 * m + 1));
    const double r = SJK_SYN_SQRT(SJK_SYN_MUL(-2.0, sjk_syn_ln(u1)));
    double c, s;
    sjk_syn_cossin_turns(u2, &c, &s);
    *n0 = SJK_SYN_MUL(r, c);
    *n1 = SJK_SYN_MUL(r, s);
}

/* Student-t(4) from the normal x and normals 4j .. 4j + 3 of the chi-square stream */
SJK_SYN_FN double sjk_syn_student4(double x, uint64_t chi_key, uint64_t j) {
    double a, b, c, d;
    sjk_syn_normal_pair(chi_key, 2 * j, &a, &b);
    sjk_syn_normal_pair(chi_key, 2 * j + 1, &c, &d);
    const double chi = SJK_SYN_ADD(SJK_SYN_ADD(SJK_SYN_ADD(SJK_SYN_MUL(a, a), SJK_SYN_MUL(b, b)), SJK_SYN_MUL(c, c)),
                                   SJK_SYN_MUL(d, d));
    return SJK_SYN_DIV(x, SJK_SYN_SQRT(SJK_SYN_MUL(chi, 0.25)));
}

/* One layer's channel scales s[h][d], h < H, d < D (D <= 1024): LogNormal(0, 1) from the scale stream (normal
 * h * D + d), then x 8 for 4 distinct outlier channels per head: draws h * 64 + i, i = 0, 1, ... of the outlier
 * stream, channel = draw % D, repeats skipped. Sequential per head; one call per (layer, head). */
SJK_SYN_FN void sjk_syn_scales_head(uint64_t seed, uint32_t layer, int h, int D, float * s) {
    const uint64_t ks = sjk_syn_key(seed, layer, SJK_SYN_SCALE), ko = sjk_syn_key(seed, layer, SJK_SYN_OUTLIER);
    int d, picked[4], n = 0;
    uint64_t i = 0;
    for (d = 0; d < D; d += 2) {
        const uint64_t j = (uint64_t) h * (uint64_t) D + (uint64_t) d;
        double n0, n1;
        sjk_syn_normal_pair(ks, j >> 1, &n0, &n1);
        s[d] = (float) sjk_syn_exp(n0);
        s[d + 1] = (float) sjk_syn_exp(n1);
    }
    while (n < 4 && i < 4096) {
        const int c = (int) (sjk_syn_draw(ko, (uint64_t) h * 64 + i) % (uint64_t) D);
        int k, dup = 0;
        ++i;
        for (k = 0; k < n; ++k) dup |= picked[k] == c;
        if (!dup) picked[n++] = c;
    }
    for (d = 0; d < n; ++d) s[picked[d]] = s[picked[d]] * 8.0f;
}

/* Elements 2m and 2m + 1 of a layer's K and V streams (element j = (pos * H + h) * D + d), given the scales of
 * their channels (s0 for element 2m, s1 for element 2m + 1). */
SJK_SYN_FN void sjk_syn_kv_pair(uint64_t kkey, uint64_t vkey, uint64_t chikey, int heavy, uint64_t m, float s0, float s1,
                                float * k0, float * k1, float * v0, float * v1) {
    double a, b;
    sjk_syn_normal_pair(kkey, m, &a, &b);
    if (heavy) {
        a = sjk_syn_student4(a, chikey, 2 * m);
        b = sjk_syn_student4(b, chikey, 2 * m + 1);
    }
    *k0 = (float) SJK_SYN_MUL(a, (double) s0);
    *k1 = (float) SJK_SYN_MUL(b, (double) s1);
    sjk_syn_normal_pair(vkey, m, &a, &b);
    *v0 = (float) a;
    *v1 = (float) b;
}

/* float -> fp16 bits, round to nearest even, by integer operations (finite inputs below 65520 in magnitude) */
SJK_SYN_FN uint16_t sjk_syn_f16(float f) {
    uint32_t x;
#if defined(__CUDA_ARCH__)
    x = __float_as_uint(f);
#else
    memcpy(&x, &f, 4);
#endif
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int e = (int) ((x >> 23) & 0xFF) - 127;
    uint32_t mant = x & 0x7FFFFFu;
    if (e > 15) return (uint16_t) (sign | 0x7C00u);
    if (e >= -14) {                                   /* normal half */
        uint32_t h = ((uint32_t) (e + 15) << 10) | (mant >> 13);
        const uint32_t rem = mant & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;   /* a carry into the exponent is correct */
        return (uint16_t) (sign | h);
    }
    if (e < -25) return (uint16_t) sign;
    mant |= 0x800000u;                               /* subnormal half: value = mant * 2^(e - 23) */
    {
        const int shift = -e - 1;                    /* value * 2^24 = mant * 2^(e + 1): bits dropped */
        const uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
        return (uint16_t) (sign | (h + ((rem > half || (rem == half && (h & 1u))) ? 1u : 0u)));
    }
}

SJK_SYN_FN float sjk_syn_h2f(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t x;
    float f;
    if (e == 0) {
        f = (float) m * 0x1.0p-24f;                  /* exact */
#if defined(__CUDA_ARCH__)
        return __uint_as_float(__float_as_uint(f) | sign);
#else
        memcpy(&x, &f, 4);
        x |= sign;
        memcpy(&f, &x, 4);
        return f;
#endif
    }
    x = sign | ((e == 31 ? 0xFFu : e + 112u) << 23) | (m << 13);
#if defined(__CUDA_ARCH__)
    return __uint_as_float(x);
#else
    memcpy(&f, &x, 4);
    return f;
#endif
}

/* Elements 2m and 2m + 1 of a layer's query stream (element row * D + d), rounded to fp16 */
SJK_SYN_FN void sjk_syn_q_pair(uint64_t qkey, uint64_t m, float * q0, float * q1) {
    double a, b;
    sjk_syn_normal_pair(qkey, m, &a, &b);
    *q0 = sjk_syn_h2f(sjk_syn_f16((float) a));
    *q1 = sjk_syn_h2f(sjk_syn_f16((float) b));
}

#endif /* SJK_SYNTH_H */
