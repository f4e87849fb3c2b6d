/*
 * sjk_oracle.c - CPU oracle for the SJ-KVaRN hot path. TEST INFRASTRUCTURE ONLY: it is the
 * checker that tests/, smoke() and bench.py's CPU-baseline leg compare the B200 kernels
 * against; the product library never links it. See sjk_oracle.h for the parity pins.
 *
 * Restates the algorithm of sj_kvarn.h (reference file:line cited per function) in plain
 * C. Built with -ffp-contract=off and no fast-math so each float operation rounds once,
 * which is the numeric contract of sj_kvarn.h:37-42.
 */
#define _GNU_SOURCE
#include "sjk_oracle.h"
#include "../sj-kvarn-codec_b200/csrc/sjk_tables.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static const uint16_t CB3K[512] = SJK_CB3_K_INIT;
static const uint16_t CB3V[512] = SJK_CB3_V_INIT;
static const uint16_t CB2K[256] = SJK_CB2_K_INIT;
static const uint16_t CB2V[256] = SJK_CB2_V_INIT;
static const float TQ6C[64] = SJK_TQ6_CENT_INIT;
static const float TQ6M[63] = SJK_TQ6_MID_INIT;

static const uint16_t * codebook(int bits, int is_v) {
    if (bits == 3) return is_v ? CB3V : CB3K;
    return is_v ? CB2V : CB2K;
}

static uint32_t fbits(float f) { uint32_t w; memcpy(&w, &f, 4); return w; }
static float bitsf(uint32_t w) { float f; memcpy(&f, &w, 4); return f; }

uint64_t ora_fnv(const void * p, size_t n, uint64_t h) {
    const uint8_t * b = (const uint8_t *) p;
    size_t i;
    for (i = 0; i < n; ++i) { h ^= b[i]; h *= 1099511628211ULL; }
    return h;
}

/* ---- fp16 (sj_kvarn.h:693-731): round to nearest even, NaN -> quiet 0x7E00 with sign ---- */
uint16_t ora_f2h(float f) {
    const uint32_t w = fbits(f), sign = (w >> 16) & 0x8000u, a = w & 0x7FFFFFFFu;
    uint32_t q, rem, half;
    if (a > 0x7F800000u) return (uint16_t) (sign | 0x7E00u);
    if (a >= 0x477FF000u) return (uint16_t) (sign | 0x7C00u);      /* >= 65520 rounds to inf */
    if (a < 0x38800000u) {                                          /* below 2^-14: subnormal half */
        int sh;
        uint32_t m;
        if (a < 0x33000000u) return (uint16_t) sign;                /* < 2^-25 (2^-25 itself ties to 0) */
        sh = 126 - (int) (a >> 23);
        m = (a & 0x7FFFFFu) | 0x800000u;
        q = m >> sh; rem = m & ((1u << sh) - 1u); half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t) (sign | q);
    }
    q = (a - 0x38000000u) >> 13;                                    /* rebias exponent 127 -> 15 */
    rem = a & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t) (sign | q);
}

float ora_h2f(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 31u;
    uint32_t m = h & 0x3FFu;
    if (e == 31u) return bitsf(sign | 0x7F800000u | (m << 13));
    if (e) return bitsf(sign | ((e + 112u) << 23) | (m << 13));
    if (!m) return bitsf(sign);
    {
        uint32_t ex = 113u;
        while (!(m & 0x400u)) { m <<= 1; ex--; }
        return bitsf(sign | (ex << 23) | ((m & 0x3FFu) << 13));
    }
}

/* ---- rotation (sj_kvarn.h:735-752): butterfly stages h = 1, 2, 4, ..., then x 1/sqrt(n) ---- */
void ora_fwht(float * x, int n) {
    int h, b, j;
    float s;
    for (h = 1; h < n; h *= 2)
        for (b = 0; b < n; b += 2 * h)
            for (j = b; j < b + h; ++j) {
                const float u = x[j], w = x[j + h];
                x[j] = u + w;
                x[j + h] = u - w;
            }
    s = 1.0f / sqrtf((float) n);
    for (j = 0; j < n; ++j) x[j] = x[j] * s;
}

/* ---- layout (sj_kvarn.h:771-790, 803-849) ---- */
int ora_layout_init(ora_layout * l, int D, int G, int bits_k, int bits_v, int trellis) {
    if (D < 32 || (D & (D - 1)) || G <= 0 || G % 16) return -1;
    if (bits_k < 2 || bits_k > 4 || bits_v < 2 || bits_v > 4) return -2;
    if (trellis && (bits_k == 4 || bits_v == 4 || bits_v > bits_k || G != 128 || D % 128)) return -4;
    l->D = D; l->G = G; l->bits_k = bits_k; l->bits_v = bits_v; l->trellis = trellis ? 1 : 0;
    l->kp = 0;
    l->vp = (uint32_t) (G * D * bits_k / 8);
    l->ks = l->vp + (uint32_t) (G * D * bits_v / 8);
    l->kz = l->ks + 2u * (uint32_t) D;
    l->kt = l->kz + 2u * (uint32_t) D;
    l->vc = l->kt + 2u * (uint32_t) G;
    l->vs = l->vc + 2u * (uint32_t) D;
    l->vz = l->vs + 2u * (uint32_t) G;
    l->bytes = l->vz + 2u * (uint32_t) G;
    return 0;
}

/* 4-bit scalar payloads are in 16x16 tensor-core fragment order (sj_kvarn.h:800-805) */
static int frag_side(const ora_layout * l, int bits) {
    return !l->trellis && bits == 4 && l->D % 16 == 0 && l->G % 16 == 0;
}

uint32_t ora_code_bit(const ora_layout * l, int t, int d, int is_v) {
    const int bits = is_v ? l->bits_v : l->bits_k;
    int tile, lane, reg, hi;
    if (l->trellis) return ((uint32_t) d * (uint32_t) l->G + (uint32_t) t) * (uint32_t) bits;   /* channel-major */
    if (!frag_side(l, bits)) return ((uint32_t) t * (uint32_t) l->D + (uint32_t) d) * (uint32_t) bits; /* token-major */
    tile = (t >> 4) * (l->D >> 4) + (d >> 4);
    {
        /* inside a 16x16 tile: the "row" index walks the 16 rows of the MMA operand,
         * the "col" index its 16 k-values; K has rows = tokens, V has rows = channels */
        const int row = is_v ? (d & 15) : (t & 15);
        const int col = is_v ? (t & 15) : (d & 15);
        lane = 4 * (row & 7) + ((col >> 1) & 3);
        reg = (row >> 3) + 2 * (col >> 3);
        hi = col & 1;
    }
    return ((uint32_t) tile * 32u + (uint32_t) lane) * 32u + (uint32_t) (reg + 4 * hi) * 4u;
}

int ora_k_ch(const ora_layout * l, int d) {
    int dd, pair;
    if (!frag_side(l, l->bits_k)) return d;
    dd = d & 15; pair = dd >> 1;
    return (pair & 3) * (l->D / 4) + (d >> 4) * 4 + (pair >> 2) * 2 + (dd & 1);
}

int ora_v_ch(const ora_layout * l, int d) {
    const int dd = d & 15;
    if (!frag_side(l, l->bits_v)) return d;
    return (dd & 7) * (l->D / 8) + (d >> 4) * 2 + (dd >> 3);
}

static void put_code(uint8_t * p, uint32_t bit, int bits, uint32_t v) {
    const uint32_t w = (v & ((1u << bits) - 1u)) << (bit & 7u);
    p[bit >> 3] |= (uint8_t) w;
    if ((bit & 7u) + (uint32_t) bits > 8u) p[(bit >> 3) + 1] |= (uint8_t) (w >> 8);
}

static uint32_t get_code(const uint8_t * p, uint32_t bit, int bits) {
    uint32_t w = p[bit >> 3];
    if ((bit & 7u) + (uint32_t) bits > 8u) w |= (uint32_t) p[(bit >> 3) + 1] << 8;
    return (w >> (bit & 7u)) & ((1u << bits) - 1u);
}

/* trellis window of code i of channel seq (sj_kvarn.h:879-900): current code in bits
 * [6, 6+bits), the previous codes below it (newest highest), zero before t = 0 */
static uint32_t window(const uint8_t * payload, int bits, int seq, int i, int seq_len) {
    const int hist = (6 + bits - 1) / bits;
    const uint32_t base = (uint32_t) seq * (uint32_t) seq_len * (uint32_t) bits;
    uint32_t w = 0;
    int k;
    for (k = 0; k <= hist && k <= i; ++k) {
        const int shift = 6 - k * bits;
        const uint32_t c = get_code(payload, base + (uint32_t) (i - k) * (uint32_t) bits, bits);
        w |= shift >= 0 ? c << shift : c >> (-shift);
    }
    return w & ((1u << (6 + bits)) - 1u);
}

/* ---- tq6_0 staging (sj_kvarn.h:1211-1284) ---- */
#define TQ6_BLOCK 98

/* code = number of decision midpoints not above v (binary search, sj_kvarn.h:1211-1219);
 * NaN compares false everywhere and lands on 63, as the reference's search does */
static int tq6_code(float v) {
    int lo = 0, hi = 63;
    while (lo < hi) {
        const int m = (lo + hi) >> 1;
        if (v < TQ6M[m]) hi = m; else lo = m + 1;
    }
    return lo;
}

void ora_tq6_encode(const float * x, uint8_t * blocks, int n) {
    int b, i;
    for (b = 0; b < n / 128; ++b) {
        const float * v = x + (size_t) b * 128;
        uint8_t * blk = blocks + (size_t) b * TQ6_BLOCK;
        uint8_t code[128];
        float ss = 0.0f, nrm, inv = 0.0f, cs = 0.0f, cn;
        uint16_t h;
        for (i = 0; i < 128; ++i) ss = ss + v[i] * v[i];          /* sequential, one rounding per op */
        nrm = sqrtf(ss);
        if (nrm > 1e-10f) inv = 1.0f / nrm;
        for (i = 0; i < 128; ++i) code[i] = (uint8_t) tq6_code(nrm > 1e-10f ? v[i] * inv : 0.0f);
        for (i = 0; i < 128; ++i) cs = cs + TQ6C[code[i]] * TQ6C[code[i]];
        cn = sqrtf(cs);
        h = ora_f2h(cn > 1e-10f ? nrm / cn : nrm);
        memset(blk, 0, TQ6_BLOCK);
        blk[0] = (uint8_t) h; blk[1] = (uint8_t) (h >> 8);
        for (i = 0; i < 128; ++i) {
            blk[2 + i / 2]  |= (uint8_t) ((code[i] & 15u) << (4 * (i & 1)));
            blk[66 + i / 4] |= (uint8_t) (((code[i] >> 4) & 3u) << (2 * (i & 3)));
        }
    }
}

void ora_tq6_decode(const uint8_t * blocks, float * x, int n) {
    int b, i;
    for (b = 0; b < n / 128; ++b) {
        const uint8_t * blk = blocks + (size_t) b * TQ6_BLOCK;
        const float nrm = ora_h2f((uint16_t) (blk[0] | (blk[1] << 8)));
        for (i = 0; i < 128; ++i) {
            const int c = ((blk[2 + i / 2] >> (4 * (i & 1))) & 15) | (((blk[66 + i / 4] >> (2 * (i & 3))) & 3) << 4);
            x[(size_t) b * 128 + i] = TQ6C[c] * nrm;
        }
    }
}

size_t ora_stage_bytes(int staging, int D) { return staging ? (size_t) D * 2 : (size_t) (D / 128) * TQ6_BLOCK; }

void ora_stage_row(int staging, const float * x, uint8_t * dst, int D) {
    int i;
    if (!staging) { ora_tq6_encode(x, dst, D); return; }
    for (i = 0; i < D; ++i) { const uint16_t h = ora_f2h(x[i]); dst[2 * i] = (uint8_t) h; dst[2 * i + 1] = (uint8_t) (h >> 8); }
}

void ora_unstage_row(int staging, const uint8_t * src, float * x, int D) {
    int i;
    if (!staging) { ora_tq6_decode(src, x, D); return; }
    for (i = 0; i < D; ++i) x[i] = ora_h2f((uint16_t) (src[2 * i] | (src[2 * i + 1] << 8)));
}

/* ---- seal (sj_kvarn.h:939-1174) ---- */

/* comparisons written exactly as the reference helpers (sj_kvarn.h:679-682), which
 * matters for NaN and signed zeros */
static float lesser_f(float a, float b) { return b < a ? b : a; }
static float greater_f(float a, float b) { return a < b ? b : a; }
static double lesser_d(double a, double b) { return b < a ? b : a; }
static double greater_d(double a, double b) { return a < b ? b : a; }

/* reduction contract (sj_kvarn.h:939-978): 8 contiguous chunks, each summed in order in
 * double, partials combined pairwise ((0+1)+(2+3))+((4+5)+(6+7)); second pass with fma */
static double tree8(const double * p) {
    return ((p[0] + p[1]) + (p[2] + p[3])) + ((p[4] + p[5]) + (p[6] + p[7]));
}

static float chunked_std(const float * x, int n, size_t stride) {
    const int len = n / 8;
    double part[8], mean;
    int c, i;
    for (c = 0; c < 8; ++c) {
        double s = 0.0;
        for (i = 0; i < len; ++i) s = s + (double) x[(size_t) (c * len + i) * stride];
        part[c] = s;
    }
    mean = tree8(part) / (double) n;
    for (c = 0; c < 8; ++c) {
        double s = 0.0;
        for (i = 0; i < len; ++i) {
            const double dv = (double) x[(size_t) (c * len + i) * stride] - mean;
            s = fma(dv, dv, s);
        }
        part[c] = s;
    }
    return (float) sqrt(tree8(part) / (double) (n > 1 ? n - 1 : 1));
}

static void rescale(const float * M, int R, int C, const float * srow, const float * scol, float * cur) {
    int r, c;
    for (r = 0; r < R; ++r)
        for (c = 0; c < C; ++c) cur[(size_t) r * C + c] = (M[(size_t) r * C + c] / scol[c]) / srow[r];
}

/* Optional trace of every argument the balancing passes to log() and exp() (for the check of the device's double
 * log/exp against this host's libm): slots are claimed atomically, so tracing works under the threaded seals. */
static double * g_trace_log, * g_trace_prev, * g_trace_exp;
static size_t g_trace_cap, g_trace_n_log, g_trace_n_exp;

void ora_trace_balance(double * log_args, double * log_prev, double * exp_args, size_t cap) {
    g_trace_log = log_args; g_trace_prev = log_prev; g_trace_exp = exp_args; g_trace_cap = cap;
    __atomic_store_n(&g_trace_n_log, 0, __ATOMIC_SEQ_CST);
    __atomic_store_n(&g_trace_n_exp, 0, __ATOMIC_SEQ_CST);
}

void ora_trace_counts(size_t * n_log, size_t * n_exp) {
    *n_log = __atomic_load_n(&g_trace_n_log, __ATOMIC_SEQ_CST);
    *n_exp = __atomic_load_n(&g_trace_n_exp, __ATOMIC_SEQ_CST);
}

/* log(x) of a scale update whose running log-scale before the update is `prev` (both traced) */
static double traced_log(double prev, double x) {
    if (g_trace_log) {
        const size_t i = __atomic_fetch_add(&g_trace_n_log, 1, __ATOMIC_RELAXED);
        if (i < g_trace_cap) { g_trace_log[i] = x; g_trace_prev[i] = prev; }
    }
    return log(x);
}

static double traced_exp(double x) {
    if (g_trace_exp) {
        const size_t i = __atomic_fetch_add(&g_trace_n_exp, 1, __ATOMIC_RELAXED);
        if (i < g_trace_cap) g_trace_exp[i] = x;
    }
    return exp(x);
}

/* this host's libm log and exp of n doubles (the functions the reference's balancing calls) */
/* next running log-scale of a scale update, as the balancing forms it (sj_kvarn.h:1001-1008) */
void ora_balance_step(const double * prev, const double * lg, size_t n, double * out) {
    size_t i;
    for (i = 0; i < n; ++i) out[i] = lesser_d(greater_d(prev[i] + lg[i], -0.3), 10.0);
}

void ora_libm_log_exp(const double * x, size_t n, double * lg, double * ex) {
    size_t i;
    for (i = 0; i < n; ++i) { lg[i] = log(x[i]); ex[i] = exp(x[i]); }
}

/* log-domain variance balancing, exactly `iters` column-then-row passes (sj_kvarn.h:989-1012) */
static void balance(const float * M, int R, int C, int iters, float * srow, float * scol, float * cur,
                    double * lrow, double * lcol) {
    int it, r, c;
    for (c = 0; c < C; ++c) { scol[c] = 1.0f; lcol[c] = 0.0; }
    for (r = 0; r < R; ++r) { srow[r] = 1.0f; lrow[r] = 0.0; }
    rescale(M, R, C, srow, scol, cur);
    for (it = 0; it < iters; ++it) {
        for (c = 0; c < C; ++c) {
            const float sd = lesser_f(greater_f(chunked_std(cur + c, R, (size_t) C), 1e-3f), 1e3f);
            lcol[c] = lesser_d(greater_d(lcol[c] + traced_log(lcol[c], (double) sd), -0.3), 10.0);
            scol[c] = (float) traced_exp(lcol[c]);
        }
        rescale(M, R, C, srow, scol, cur);
        for (r = 0; r < R; ++r) {
            const float sd = lesser_f(greater_f(chunked_std(cur + (size_t) r * C, C, 1), 1e-3f), 1e3f);
            lrow[r] = lesser_d(greater_d(lrow[r] + traced_log(lrow[r], (double) sd), -0.3), 10.0);
            srow[r] = (float) traced_exp(lrow[r]);
        }
        rescale(M, R, C, srow, scol, cur);
    }
}

/* Viterbi over one channel's token sequence (sj_kvarn.h:1021-1053): backward recursion over
 * 64 history states, branch j selects window s + 64 j, strict < over ascending j, start
 * state 0, no termination cost */
static void viterbi(const float * y, int n, int bits, const float * cbf, uint8_t * codes, uint8_t * back) {
    float m[64], mn[64];
    int i, s, j;
    for (s = 0; s < 64; ++s) m[s] = 0.0f;
    for (i = n - 1; i >= 0; --i) {
        for (s = 0; s < 64; ++s) {
            float best = INFINITY;
            int bj = 0;
            for (j = 0; j < (1 << bits); ++j) {
                const int w = s + 64 * j;
                const float dlt = y[i] - cbf[w];
                const float cost = dlt * dlt + m[w >> bits];
                if (cost < best) { best = cost; bj = j; }
            }
            mn[s] = best;
            back[i * 64 + s] = (uint8_t) bj;
        }
        memcpy(m, mn, sizeof m);
    }
    s = 0;
    for (i = 0; i < n; ++i) {
        j = back[i * 64 + s];
        codes[i] = (uint8_t) j;
        s = (s + 64 * j) >> bits;
    }
}

typedef struct seal_scratch {
    float * M, * cur, * srow, * scol, * lo, * step, * cbf, * y;
    double * lrow, * lcol;
    uint8_t * codes, * back;
} seal_scratch;

static int scratch_alloc(seal_scratch * w, const ora_layout * l) {
    const size_t DG = (size_t) l->D * l->G, R = (size_t) (l->D > l->G ? l->D : l->G);
    w->M = (float *) malloc(DG * 4); w->cur = (float *) malloc(DG * 4);
    w->srow = (float *) malloc(R * 4); w->scol = (float *) malloc(R * 4);
    w->lo = (float *) malloc(R * 4); w->step = (float *) malloc(R * 4);
    w->lrow = (double *) malloc(R * 8); w->lcol = (double *) malloc(R * 8);
    w->cbf = (float *) malloc(512 * 4); w->y = (float *) malloc(128 * 4);
    w->codes = (uint8_t *) malloc(128); w->back = (uint8_t *) malloc(128 * 64);
    return w->M && w->cur && w->srow && w->scol && w->lo && w->step && w->lrow && w->lcol && w->cbf && w->y && w->codes && w->back ? 0 : -1;
}

static void scratch_free(seal_scratch * w) {
    free(w->M); free(w->cur); free(w->srow); free(w->scol); free(w->lo); free(w->step);
    free(w->lrow); free(w->lcol); free(w->cbf); free(w->y); free(w->codes); free(w->back);
}

static void put_half(uint8_t * rec, uint32_t off, float v) {
    const uint16_t h = ora_f2h(v);
    rec[off] = (uint8_t) h; rec[off + 1] = (uint8_t) (h >> 8);
}
static float get_half(const uint8_t * rec, uint32_t off) { return ora_h2f((uint16_t) (rec[off] | (rec[off + 1] << 8))); }

/* quantize one balanced side (sj_kvarn.h:1111-1147). K: cur is [D][G] (rows = channels);
 * V: [G][D] (rows = tokens). Trellis sides are coded per channel and refitted afterwards. */
static void quantize_side(const ora_layout * l, int is_v, uint8_t * rec, seal_scratch * w) {
    const int D = l->D, G = l->G, R = is_v ? G : D, C = is_v ? D : G;
    const int bits = is_v ? l->bits_v : l->bits_k;
    const uint32_t qmax = (1u << bits) - 1u;
    const uint32_t off_scale = is_v ? l->vs : l->ks, off_zero = is_v ? l->vz : l->kz;
    uint8_t * payload = rec + (is_v ? l->vp : l->kp);
    int r, c;
    for (r = 0; r < R; ++r) {
        const float * row = w->cur + (size_t) r * C;
        float lo = row[0], hi = row[0], step;
        uint32_t ri;
        for (c = 1; c < C; ++c) { lo = lesser_f(lo, row[c]); hi = greater_f(hi, row[c]); }
        step = greater_f((hi - lo) / (float) qmax, 1e-10f);
        ri = (uint32_t) (is_v ? r : ora_k_ch(l, r));
        put_half(rec, off_scale + 2u * ri, w->srow[r] * step);
        put_half(rec, off_zero + 2u * ri, w->srow[r] * lo);
        w->lo[r] = lo; w->step[r] = step;
        if (l->trellis) continue;
        for (c = 0; c < C; ++c) {
            float q = rintf((row[c] - lo) / step);                  /* ties to even */
            if (q < 0.0f) q = 0.0f;
            if (q > (float) qmax) q = (float) qmax;
            put_code(payload, ora_code_bit(l, is_v ? r : c, is_v ? c : r, is_v), bits, (uint32_t) q);
        }
    }
    if (l->trellis) {
        /* one Viterbi sequence per channel along the G tokens (sj_kvarn.h:1055-1073) */
        const uint16_t * cb = codebook(bits, is_v);
        const int nwin = 1 << (6 + bits);
        int d, t;
        for (d = 0; d < nwin; ++d) w->cbf[d] = ora_h2f(cb[d]);
        for (d = 0; d < D; ++d) {
            for (t = 0; t < G; ++t) {
                const int rr = is_v ? t : d, cc = is_v ? d : t;
                w->y[t] = (w->cur[(size_t) rr * C + cc] - w->lo[rr]) / w->step[rr];
            }
            viterbi(w->y, G, bits, w->cbf, w->codes, w->back);
            for (t = 0; t < G; ++t) put_code(payload, ((uint32_t) d * (uint32_t) G + (uint32_t) t) * (uint32_t) bits, bits, w->codes[t]);
        }
        /* moment-matching refit of each row's affine (sj_kvarn.h:1075-1109) */
        for (r = 0; r < R; ++r) {
            double sx = 0.0, sy = 0.0, sxx = 0.0, syy = 0.0, vx, vy, a, b;
            const double n = (double) C;
            for (c = 0; c < C; ++c) {
                const int tt = is_v ? r : c, dd = is_v ? c : r;
                const double x = (double) w->cur[(size_t) r * C + c];
                const double yh = (double) ora_h2f(cb[window(payload, bits, dd, tt, G)]);
                sx = sx + x; sy = sy + yh;
                sxx = sxx + x * x; syy = syy + yh * yh;
            }
            vy = n * syy - sy * sy;
            if (!(vy > 0.0)) continue;
            vx = n * sxx - sx * sx;
            if (!(vx > 0.0)) continue;
            a = sqrt(vx / vy);
            b = (sx - a * sy) / n;
            if (!(a > 0.0) || !(b == b) || a > 1e30 || fabs(b) > 1e30) continue;
            {
                const uint32_t ri = (uint32_t) (is_v ? r : ora_k_ch(l, r));
                put_half(rec, off_scale + 2u * ri, w->srow[r] * (float) a);
                put_half(rec, off_zero + 2u * ri, w->srow[r] * (float) b);
            }
        }
    }
    /* column scales: Ktok[t] for K (columns = tokens), Vch[v_ch(d)] for V (columns = channels) */
    for (c = 0; c < C; ++c) put_half(rec, is_v ? l->vc + 2u * (uint32_t) ora_v_ch(l, c) : l->kt + 2u * (uint32_t) c, w->scol[c]);
}

static void seal_one(const ora_layout * l, const uint16_t * K, const uint16_t * V, size_t row_stride, int iters,
                     uint8_t * rec, seal_scratch * w) {
    const int D = l->D, G = l->G;
    int t, d;
    memset(rec, 0, l->bytes);
    for (t = 0; t < G; ++t)
        for (d = 0; d < D; ++d) w->M[(size_t) d * G + t] = ora_h2f(K[(size_t) t * row_stride + d]);
    balance(w->M, D, G, iters, w->srow, w->scol, w->cur, w->lrow, w->lcol);
    quantize_side(l, 0, rec, w);
    for (t = 0; t < G; ++t)
        for (d = 0; d < D; ++d) w->M[(size_t) t * D + d] = ora_h2f(V[(size_t) t * row_stride + d]);
    balance(w->M, G, D, iters, w->srow, w->scol, w->cur, w->lrow, w->lcol);
    quantize_side(l, 1, rec, w);
}

void ora_seal(const ora_layout * l, const uint16_t * K, const uint16_t * V, size_t row_stride, int iters, uint8_t * rec) {
    seal_scratch w;
    if (scratch_alloc(&w, l) == 0) seal_one(l, K, V, row_stride, iters, rec, &w);
    scratch_free(&w);
}

/* ---- threaded batch seal (CPU baseline harness; one scratch per thread) ---- */
typedef struct seal_job {
    const ora_layout * l;
    const uint16_t * k, * v;
    size_t row_stride;
    int H, n_rec, iters, n_threads, tid;
    uint8_t * body;
} seal_job;

static void * seal_worker(void * arg) {
    seal_job * j = (seal_job *) arg;
    seal_scratch w;
    int r;
    if (scratch_alloc(&w, j->l) == 0) {
        for (r = j->tid; r < j->n_rec; r += j->n_threads) {
            const int g = r / j->H, h = r % j->H;
            const size_t off = (size_t) g * j->l->G * j->row_stride + (size_t) h * j->l->D;
            seal_one(j->l, j->k + off, j->v + off, j->row_stride, j->iters, j->body + (size_t) r * j->l->bytes, &w);
        }
    }
    scratch_free(&w);
    return NULL;
}

static int resolve_threads(int n) {
    if (n > 0) return n;
    n = (int) sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? n : 1;
}

void ora_seal_batch(const ora_layout * l, const uint16_t * k, const uint16_t * v, size_t row_stride, int H,
                    int n_rec, int iters, uint8_t * body, int n_threads) {
    pthread_t th[256];
    seal_job jobs[256];
    int i, nt = resolve_threads(n_threads);
    if (nt > 256) nt = 256;
    if (nt > n_rec) nt = n_rec > 0 ? n_rec : 1;
    for (i = 0; i < nt; ++i) {
        jobs[i].l = l; jobs[i].k = k; jobs[i].v = v; jobs[i].row_stride = row_stride; jobs[i].H = H;
        jobs[i].n_rec = n_rec; jobs[i].iters = iters; jobs[i].n_threads = nt; jobs[i].tid = i; jobs[i].body = body;
    }
    if (nt == 1) { seal_worker(&jobs[0]); return; }
    for (i = 0; i < nt; ++i) pthread_create(&th[i], NULL, seal_worker, &jobs[i]);
    for (i = 0; i < nt; ++i) pthread_join(th[i], NULL);
}

/* ---- decode (sj_kvarn.h:1176-1207): no FMA, three single-rounded ops per value ---- */
static float code_value(const ora_layout * l, const uint8_t * rec, int t, int d, int is_v) {
    const int bits = is_v ? l->bits_v : l->bits_k;
    const uint8_t * payload = rec + (is_v ? l->vp : l->kp);
    if (l->trellis) return ora_h2f(codebook(bits, is_v)[window(payload, bits, d, t, l->G)]);
    return (float) get_code(payload, ora_code_bit(l, t, d, is_v), bits);
}

void ora_decode_k(const ora_layout * l, const uint8_t * rec, int t, float * out) {
    const float tok = get_half(rec, l->kt + 2u * (uint32_t) t);
    int d;
    for (d = 0; d < l->D; ++d) {
        const uint32_t di = (uint32_t) ora_k_ch(l, d);
        out[d] = (code_value(l, rec, t, d, 0) * get_half(rec, l->ks + 2u * di) + get_half(rec, l->kz + 2u * di)) * tok;
    }
}

void ora_decode_v(const ora_layout * l, const uint8_t * rec, int t, float * out) {
    const float sc = get_half(rec, l->vs + 2u * (uint32_t) t), zp = get_half(rec, l->vz + 2u * (uint32_t) t);
    int d;
    for (d = 0; d < l->D; ++d)
        out[d] = (code_value(l, rec, t, d, 1) * sc + zp) * get_half(rec, l->vc + 2u * (uint32_t) ora_v_ch(l, d));
}

/* ---- adaptive-tail policy (sj_kvarn.h:1315-1407) ---- */
void ora_policy_init(ora_policy * p, uint32_t sink, uint32_t tail, uint32_t tail_max, uint32_t group, uint32_t flush_chunk) {
    p->sink = sink; p->tail = tail; p->tail_max = tail_max; p->group = group; p->flush_chunk = flush_chunk;
    p->B = p->B_prev = p->B_pending = sink;
    p->draining = 0;
}

uint32_t ora_group_floor(uint32_t sink, uint32_t group, uint32_t pos) {
    return pos <= sink ? pos : sink + group * ((pos - sink) / group);
}

uint32_t ora_policy_begin(ora_policy * p, uint32_t pos0, uint32_t n_tokens) {
    int due = p->tail_max == 0 || p->draining || (pos0 > p->B && pos0 - p->B >= p->tail_max);
    p->B_pending = p->B;
    p->draining = 0;
    if (due && pos0 > p->sink + p->tail) {
        uint32_t target = ora_group_floor(p->sink, p->group, pos0 - p->tail);
        if (target < p->B) target = p->B;
        if (p->tail_max && p->flush_chunk && n_tokens < p->group && target > p->B + p->group * p->flush_chunk) {
            target = p->B + p->group * p->flush_chunk;
            p->draining = 1;
        }
        p->B_pending = target;
    }
    return p->B_pending;
}

void ora_policy_commit(ora_policy * p) { p->B_prev = p->B; p->B = p->B_pending; }

uint32_t ora_policy_idle(ora_policy * p, uint32_t end, uint32_t keep_recent) {
    uint32_t target;
    int clamped = 0;
    p->B_pending = p->B;
    if (p->tail_max == 0 || end <= p->sink + p->tail) return p->B;
    target = ora_group_floor(p->sink, p->group, end - p->tail);
    if (keep_recent > p->tail) {
        const uint32_t from = end > keep_recent ? end - keep_recent : 0;
        const uint32_t lim = from <= p->sink ? p->sink : ora_group_floor(p->sink, p->group, from);
        if (lim < target) { target = lim; clamped = 1; }
    }
    if (!clamped) p->draining = 0;
    if (target <= p->B) return p->B;
    p->B_pending = target;
    return target;
}

uint32_t ora_policy_truncate(ora_policy * p, uint32_t pos, uint32_t * n_dropped) {
    uint32_t r;
    if (n_dropped) *n_dropped = 0;
    if (p->B_pending != p->B) return UINT32_MAX;
    r = (pos >= p->B || pos <= p->sink) ? pos : ora_group_floor(p->sink, p->group, pos);
    if (r < p->B) {
        const uint32_t nb = r > p->sink ? r : p->sink;
        if (n_dropped) *n_dropped = (p->B - nb) / p->group;
        p->B = p->B_prev = p->B_pending = nb;
        p->draining = 0;
    }
    return r;
}

uint32_t ora_ring_capacity(uint32_t tail, uint32_t tail_max, uint32_t group, uint32_t n_ubatch) {
    const uint32_t need = (tail > tail_max ? tail : tail_max) + group + 2u * n_ubatch;
    return (need + 127u) / 128u * 128u;
}

/* ---- host per-layer cache (sj_kvarn.h:1436-1564) ---- */
int ora_cache_init(ora_cache * c, int D, int H, int bits_k, int bits_v, int trellis, int iters, int staging,
                   int sink_f16, uint32_t S, uint32_t tail, uint32_t tail_max, uint32_t n_ubatch, uint32_t n_ctx) {
    memset(c, 0, sizeof(*c));
    if (ora_layout_init(&c->lay, D, 128, bits_k, bits_v, trellis)) return -1;
    c->H = H; c->staging = staging; c->sink_f16 = sink_f16; c->iters = iters; c->S = S;
    c->cap = ora_ring_capacity(tail, tail_max, 128, n_ubatch);
    c->n_groups = n_ctx > S ? (n_ctx - S + 127u) / 128u : 1u;
    c->stage_bytes = ora_stage_bytes(staging, D);
    c->ring = (uint8_t *) calloc((size_t) c->cap * H, 2 * c->stage_bytes);
    c->sink = (uint8_t *) calloc((size_t) S * H, sink_f16 ? (size_t) D * 4 : 2 * c->stage_bytes);
    c->body = (uint8_t *) calloc((size_t) c->n_groups * H, c->lay.bytes);
    if (!c->ring || !c->sink || !c->body) { ora_cache_free(c); return -1; }
    return 0;
}

void ora_cache_free(ora_cache * c) {
    free(c->ring); free(c->sink); free(c->body);
    c->ring = c->sink = c->body = NULL;
}

static size_t sink_entry(const ora_cache * c) { return c->sink_f16 ? (size_t) c->lay.D * 4 : 2 * c->stage_bytes; }
static uint8_t * sink_row(const ora_cache * c, uint32_t pos, int h) { return c->sink + ((size_t) pos * c->H + h) * sink_entry(c); }
static uint8_t * ring_row(const ora_cache * c, uint32_t pos, int h) {
    return c->ring + ((size_t) ((pos - c->S) % c->cap) * c->H + h) * 2 * c->stage_bytes;
}

uint8_t * ora_record(const ora_cache * c, uint32_t g, int h) {
    const uint32_t blk = c->blocks ? c->blocks[g] : g;
    return c->body + ((size_t) blk * c->H + h) * c->lay.bytes;
}

void ora_store(ora_cache * c, uint32_t pos, const float * k_rot, const float * v_rot) {
    const int D = c->lay.D;
    int h, i;
    for (h = 0; h < c->H; ++h) {
        const float * kr = k_rot + (size_t) h * D, * vr = v_rot + (size_t) h * D;
        if (pos < c->S && c->sink_f16) {
            uint8_t * dst = sink_row(c, pos, h);
            for (i = 0; i < D; ++i) {
                const uint16_t a = ora_f2h(kr[i]), b = ora_f2h(vr[i]);
                dst[2 * i] = (uint8_t) a; dst[2 * i + 1] = (uint8_t) (a >> 8);
                dst[2 * D + 2 * i] = (uint8_t) b; dst[2 * D + 2 * i + 1] = (uint8_t) (b >> 8);
            }
        } else {
            uint8_t * dst = pos < c->S ? sink_row(c, pos, h) : ring_row(c, pos, h);
            ora_stage_row(c->staging, kr, dst, D);
            ora_stage_row(c->staging, vr, dst + c->stage_bytes, D);
        }
    }
}

/* seal [B_from, B_to): seal input = staged ring row widened to float, rounded to fp16
 * (sj_kvarn.h:1494-1514) */
void ora_seal_range(ora_cache * c, uint32_t B_from, uint32_t B_to, int n_threads) {
    const int D = c->lay.D, G = 128, H = c->H;
    uint32_t ng, gi, p0;
    uint16_t * k, * v;
    uint8_t * tmp;
    float * row;
    int h, t, i;
    if (B_to <= B_from) return;
    ng = (B_to - B_from) / (uint32_t) G;
    if (!ng) return;
    /* gather all groups' seal inputs as [ng*G][H][D] fp16 rows, then seal in a batch */
    k = (uint16_t *) malloc((size_t) ng * G * H * D * 2);
    v = (uint16_t *) malloc((size_t) ng * G * H * D * 2);
    tmp = (uint8_t *) malloc((size_t) ng * H * c->lay.bytes);
    row = (float *) malloc((size_t) D * 4);
    if (!k || !v || !tmp || !row) { free(k); free(v); free(tmp); free(row); return; }
    for (gi = 0; gi < ng; ++gi)
        for (t = 0; t < G; ++t)
            for (h = 0; h < H; ++h) {
                const uint8_t * src = ring_row(c, B_from + gi * (uint32_t) G + (uint32_t) t, h);
                const size_t o = (((size_t) gi * G + t) * H + h) * D;
                ora_unstage_row(c->staging, src, row, D);
                for (i = 0; i < D; ++i) k[o + i] = ora_f2h(row[i]);
                ora_unstage_row(c->staging, src + c->stage_bytes, row, D);
                for (i = 0; i < D; ++i) v[o + i] = ora_f2h(row[i]);
            }
    ora_seal_batch(&c->lay, k, v, (size_t) H * D, H, (int) (ng * H), c->iters, tmp, n_threads);
    for (gi = 0, p0 = B_from; gi < ng; ++gi, p0 += (uint32_t) G)
        for (h = 0; h < H; ++h)
            memcpy(ora_record(c, (p0 - c->S) / (uint32_t) G, h), tmp + ((size_t) gi * H + h) * c->lay.bytes, c->lay.bytes);
    free(k); free(v); free(tmp); free(row);
}

void ora_kv_row(const ora_cache * c, uint32_t B, uint32_t pos, int h, float * k, float * v) {
    const int D = c->lay.D;
    int i;
    if (pos >= c->S && pos < B) {
        const uint32_t g = (pos - c->S) / 128u, t = (pos - c->S) % 128u;
        const uint8_t * rec = ora_record(c, g, h);
        ora_decode_k(&c->lay, rec, (int) t, k);
        ora_decode_v(&c->lay, rec, (int) t, v);
    } else if (pos < c->S && c->sink_f16) {
        const uint8_t * src = sink_row(c, pos, h);
        for (i = 0; i < D; ++i) {
            k[i] = ora_h2f((uint16_t) (src[2 * i] | (src[2 * i + 1] << 8)));
            v[i] = ora_h2f((uint16_t) (src[2 * D + 2 * i] | (src[2 * D + 2 * i + 1] << 8)));
        }
    } else {
        const uint8_t * src = pos < c->S ? sink_row(c, pos, h) : ring_row(c, pos, h);
        ora_unstage_row(c->staging, src, k, D);
        ora_unstage_row(c->staging, src + c->stage_bytes, v, D);
    }
}

/* single-pass online softmax in position order, causal over [0, min(N, qpos+1))
 * (sj_kvarn.h:1535-1564); the dot product is a sequential fp32 sum */
void ora_attend_row(const ora_cache * c, uint32_t B, uint32_t N, const float * q, int h, uint32_t qpos, float scale, float * out) {
    const int D = c->lay.D;
    const uint32_t end = N < qpos + 1 ? N : qpos + 1;
    float * kr = (float *) malloc((size_t) D * 12), * vr = kr + D, * acc = vr + D;
    float mx = -INFINITY, den = 0.0f, inv;
    uint32_t p;
    int d;
    for (d = 0; d < D; ++d) acc[d] = 0.0f;
    for (p = 0; p < end; ++p) {
        float s = 0.0f, ms = 1.0f, vs = 1.0f;
        ora_kv_row(c, B, p, h, kr, vr);
        for (d = 0; d < D; ++d) s = s + q[d] * kr[d];
        s = s * scale;
        if (s > mx) {
            const float old = mx;
            mx = s;
            ms = expf(old - mx);
            for (d = 0; d < D; ++d) acc[d] = acc[d] * ms;
        } else {
            vs = expf(s - mx);
        }
        for (d = 0; d < D; ++d) acc[d] = acc[d] + vr[d] * vs;
        den = den * ms + vs;
    }
    inv = den == 0.0f ? 0.0f : 1.0f / den;
    for (d = 0; d < D; ++d) out[d] = acc[d] * inv;
    free(kr);
}

typedef struct attend_job {
    const ora_cache * c;
    uint32_t B, N, qpos0;
    int n_q, n_head, n_threads, tid;
    const float * q;
    float scale;
    float * out;
} attend_job;

static void * attend_worker(void * arg) {
    attend_job * j = (attend_job *) arg;
    const int D = j->c->lay.D, grp = j->n_head / j->c->H;
    int i;
    for (i = j->tid; i < j->n_q * j->n_head; i += j->n_threads) {
        const int iq = i / j->n_head, hq = i % j->n_head;
        ora_attend_row(j->c, j->B, j->N, j->q + (size_t) i * D, hq / grp, j->qpos0 + (uint32_t) iq, j->scale, j->out + (size_t) i * D);
    }
    return NULL;
}

void ora_attend(const ora_cache * c, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, const float * q,
                float scale, float * out, int n_threads) {
    pthread_t th[256];
    attend_job jobs[256];
    int i, nt = resolve_threads(n_threads);
    if (nt > 256) nt = 256;
    if (nt > n_q * n_head) nt = n_q * n_head > 0 ? n_q * n_head : 1;
    for (i = 0; i < nt; ++i) {
        jobs[i].c = c; jobs[i].B = B; jobs[i].N = N; jobs[i].qpos0 = qpos0; jobs[i].n_q = n_q; jobs[i].n_head = n_head;
        jobs[i].n_threads = nt; jobs[i].tid = i; jobs[i].q = q; jobs[i].scale = scale; jobs[i].out = out;
    }
    if (nt == 1) { attend_worker(&jobs[0]); return; }
    for (i = 0; i < nt; ++i) pthread_create(&th[i], NULL, attend_worker, &jobs[i]);
    for (i = 0; i < nt; ++i) pthread_join(th[i], NULL);
}

/* ---- sequence-state stream (sj_kvarn.h:417-431, 1813-1929) ---- */
static void le32(uint8_t * p, uint32_t v) { p[0] = (uint8_t) v; p[1] = (uint8_t) (v >> 8); p[2] = (uint8_t) (v >> 16); p[3] = (uint8_t) (v >> 24); }
static void le64(uint8_t * p, uint64_t v) { le32(p, (uint32_t) v); le32(p + 4, (uint32_t) (v >> 32)); }

size_t ora_state_write(const ora_cache * layers, int nl, const ora_policy * p, uint32_t n, int bits_k, int bits_v,
                       int trellis, int iters, int staging, int sink_f16, uint32_t tail, uint32_t tail_max,
                       uint32_t flush_chunk, uint8_t * dst) {
    const ora_cache * c0 = &layers[0];
    const uint32_t S = c0->S, B = p->B;
    const int H = c0->H, D = c0->lay.D;
    const size_t srb = sink_entry(c0), rrb = 2 * c0->stage_bytes;
    const uint32_t n_sink = n < S ? n : S, n_rec = (B - S) / 128u, n_tail = n > B ? n - B : 0;
    const size_t payload = (size_t) nl * ((size_t) n_sink * H * srb + (size_t) n_rec * H * c0->lay.bytes + (size_t) n_tail * H * rrb);
    const size_t total = 128 + payload + 8;
    uint8_t * w;
    uint32_t pos, g;
    int il, h;
    uint64_t cbid = 0;
    if (!dst) return total;
    if (trellis) {
        cbid = ora_fnv(codebook(bits_k, 0), (size_t) (bits_k == 3 ? 512 : 256) * 2, ORA_FNV0);
        cbid = ora_fnv(codebook(bits_v, 1), (size_t) (bits_v == 3 ? 512 : 256) * 2, cbid);
    }
    memset(dst, 0, 128);
    memcpy(dst, "SJKVSEQ", 8);
    le32(dst + 8, 1); le32(dst + 12, 1); le32(dst + 16, 128);
    le32(dst + 20, (uint32_t) D); le32(dst + 24, (uint32_t) H); le32(dst + 28, 128); le32(dst + 32, S);
    le32(dst + 36, sink_f16 ? 0u : 1u); le32(dst + 40, (uint32_t) bits_k); le32(dst + 44, (uint32_t) bits_v);
    le32(dst + 48, trellis ? 1u : 0u); le32(dst + 52, (uint32_t) iters); le32(dst + 56, (uint32_t) staging);
    le32(dst + 60, tail); le32(dst + 64, tail_max); le32(dst + 68, flush_chunk);
    le32(dst + 72, 1); le32(dst + 76, (uint32_t) D); le64(dst + 80, cbid);
    le32(dst + 88, (uint32_t) nl); le32(dst + 92, n); le32(dst + 96, B); le32(dst + 100, p->B_prev);
    le32(dst + 104, (uint32_t) p->draining); le64(dst + 108, (uint64_t) payload);
    w = dst + 128;
    for (il = 0; il < nl; ++il) {
        const ora_cache * c = &layers[il];
        for (pos = 0; pos < n_sink; ++pos) for (h = 0; h < H; ++h) { memcpy(w, sink_row(c, pos, h), srb); w += srb; }
        for (g = 0; g < n_rec; ++g) for (h = 0; h < H; ++h) { memcpy(w, ora_record(c, g, h), c->lay.bytes); w += c->lay.bytes; }
        for (pos = B; pos < n; ++pos) for (h = 0; h < H; ++h) { memcpy(w, ring_row(c, pos, h), rrb); w += rrb; }
    }
    le64(w, ora_fnv(dst, (size_t) (w - dst), ORA_FNV0));
    return total;
}
