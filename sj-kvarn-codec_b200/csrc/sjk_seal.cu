// sjk_seal.cu - the sealer (encode) of SJ-KVaRN records (sj_kvarn.h:902-1174) on B200.
//
// Grid: one CTA per (record, side). The K side and the V side of a record are independent problems
// (each balances its own tile and writes disjoint byte ranges of the record), so they run on different
// SMs. A CTA keeps its whole tile on chip for all balancing iterations:
//   cur   [R][C+1] fp32   the balanced tile M / s_col / s_row (padded: row and column walks are both
//                         bank-conflict free)
//   M     [R][C]   fp16   the seal input (the reference rounds it to fp16 before sealing)
//   part  [8][max(R,C)] f64  chunk partials of the reduction contract
// with K: R = D channels x C = G tokens; V: R = G tokens x C = D channels. After balancing, M's space
// holds the Viterbi back-pointers and `part`'s space the trellis payload.
//
// Bit-exactness: every rounding follows the reference's order - the 8-chunk double reduction with the
// fixed pairwise combine and an fma second pass (sj_kvarn.h:939-978), two correctly rounded divides per
// rescaled element (980-987; each from the scale's reciprocal and one residual correction, which yields
// the IEEE quotient), the clamp/compare forms of 679-682 and 1000-1008, ties-to-even rint (1014-1019),
// strict-< ascending-branch Viterbi from state 0 (1021-1053), sequential double sums in column order for
// the refit (1078-1109). Only the order of independent work differs.
#include <cuda_fp16.h>

#include "sjk_common.cuh"
#include "sjk_desc.cuh"

namespace {

constexpr int G = 128;
constexpr int NT = 1024;                // threads per CTA (64 registers each: the whole register file)
constexpr int VNW = 16;                 // warps running the Viterbi (its per-warp tables fill M's and part's space)
constexpr unsigned FULL = 0xFFFFFFFFu;

enum SealSource { SRC_F16_ROWS = 0, SRC_RING = 1 };

struct SealParams {
    sj_kvarn_layout lay;
    int H, iters;
    // fp16 rows (sjk_seal)
    const uint16_t * k;
    const uint16_t * v;
    size_t row_stride;
    // staging ring (sjk_seal_ring)
    int source, staging;
    const uint8_t * ring;
    uint32_t S, cap, B_from, stage_bytes;
    const uint32_t * blocks;
    // output
    uint8_t * body;
    // descriptor-driven ring seal (sjk_seal_dyn): B_from and the group count come from desc when the kernel runs
    const int32_t * desc;
    sjk_desc_ref dref;
    uint32_t n_groups_max;
};

// Shared-memory carve for one side. All offsets are multiples of 16 bytes.
template <int D, bool IS_V>
struct Carve {
    static constexpr int R = IS_V ? G : D;
    static constexpr int C = IS_V ? D : G;
    static constexpr int LD = C + 1;                                 // padded row stride of cur
    static constexpr int LM = C + 2;                                 // padded row stride of M (fp16): rows 1 bank apart
    static constexpr int MX = R > C ? R : C;
    static constexpr size_t cur = 0;
    static constexpr size_t cur_bytes = ((size_t) R * LD * 4 + 15) / 16 * 16;
    static constexpr size_t regA = cur + cur_bytes;                  // M fp16 / Viterbi back-pointers
    static constexpr size_t regA_bytes = ((size_t) R * LM * 2 > 65536 ? (size_t) R * LM * 2 : 65536) + 15 & ~(size_t) 15;
    static constexpr size_t regB = regA + regA_bytes;                // partials / trellis payload + M rows
    static constexpr size_t regB_bytes = 16384;
    static constexpr size_t srow = regB + regB_bytes;                // float[R]
    static constexpr size_t scol = srow + (size_t) MX * 4;           // float[C]
    static constexpr size_t lo = scol + (size_t) MX * 4;             // float[R]
    static constexpr size_t step = lo + (size_t) MX * 4;             // float[R]
    static constexpr size_t lrow = step + (size_t) MX * 4;           // double[R]
    static constexpr size_t lcol = lrow + (size_t) MX * 8;           // double[C]
    static constexpr size_t mean = lcol + (size_t) MX * 8;           // double[max]
    static constexpr size_t fit = mean + (size_t) MX * 8;            // uint32[R] refit scale|zero halves
    static constexpr size_t total = fit + (size_t) MX * 4 * 2;
};

template <int D>
constexpr size_t seal_smem_bytes() {
    return Carve<D, false>::total > Carve<D, true>::total ? Carve<D, false>::total : Carve<D, true>::total;
}

SJK_DEV float lesser_f(float a, float b) { return b < a ? b : a; }
SJK_DEV float greater_f(float a, float b) { return a < b ? b : a; }
SJK_DEV double lesser_d(double a, double b) { return b < a ? b : a; }
SJK_DEV double greater_d(double a, double b) { return a < b ? b : a; }

SJK_DEV double tree8(const double * p, int stride) {
    return __dadd_rn(__dadd_rn(__dadd_rn(p[0], p[stride]), __dadd_rn(p[2 * stride], p[3 * stride])),
                     __dadd_rn(__dadd_rn(p[4 * stride], p[5 * stride]), __dadd_rn(p[6 * stride], p[7 * stride])));
}

// ---- phase 0: the seal input -> M (fp16 bits); returns whether this thread stored an Inf or NaN ------------
template <int D, bool IS_V>
SJK_DEV bool load_input(const SealParams & p, int rec_local, uint16_t * M, const float * cent, const size_t * rowoff) {
    using CV = Carve<D, IS_V>;
    const int g = rec_local / p.H, h = rec_local % p.H;
    bool nonfinite = false;
    for (int e = threadIdx.x; e < G * D; e += NT) {
        const int t = e / D, d = e % D;                               // token-major walk: coalesced reads
        uint16_t hv;
        if (p.source == SRC_F16_ROWS) {
            const uint16_t * src = (IS_V ? p.v : p.k) + ((size_t) g * G + t) * p.row_stride + (size_t) h * D;
            hv = src[d];
        } else {
            const uint8_t * row = p.ring + rowoff[t];
            if (p.staging == SJKVARN_STAGING_F16) {
                hv = sjk_ld_u16(row + 2 * d);
                hv = sjk_f2h(sjk_h2f(hv));                              // widen + round back, as the reference
            } else {
                const uint8_t * b = row + (d >> 7) * SJKVARN_TQ6_BLOCK_BYTES;
                const int j = d & 127;
                const int code = ((b[2 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((b[66 + (j >> 2)] >> (2 * (j & 3))) & 3) << 4);
                // hardware conversions (exact, and round-to-nearest-even like the reference's) except for Inf / NaN
                const uint16_t nb = sjk_ld_u16(b);
                const float nf = (nb & 0x7C00u) == 0x7C00u ? sjk_h2f(nb) : __half2float(__ushort_as_half(nb));
                const float xv = __fmul_rn(cent[code], nf);
                hv = xv != xv ? sjk_f2h(xv) : __half_as_ushort(__float2half_rn(xv));
            }
        }
        const int r = IS_V ? t : d, c = IS_V ? d : t;
        M[r * CV::LM + c] = hv;
        nonfinite |= (hv & 0x7C00u) == 0x7C00u;
    }
    return nonfinite;
}

// RN(a / b) given y = RN(1 / b). q = RN(a y) lies within one ulp of a / b, so the residual b q - a is exact in one
// fma, and one correction step RN(q - (b q - a) y) is the correctly rounded quotient (Markstein's theorem; the
// residual is formed as b q - a so that a = -0 keeps its sign). It holds while the quotient and the residual stay
// in the normal range, which the balancing guarantees for finite inputs: a is 0 or at least 2^-24 / s in magnitude
// with every scale s = exp(clamp(., -0.3, 10)) in [0.74, 22027], so every quotient is 0 or between 1e-16 and 1.2e5.
SJK_DEV float div_by_rcp(float a, float b, float y) {
    const float q = __fmul_rn(a, y);
    const float t = __fmaf_rn(q, b, -a);
    return __fmaf_rn(t, -y, q);
}

// cur = (M / s_col) / s_row, two IEEE divides per element (sj_kvarn.h:980-987). Finite inputs divide through
// rrow / rcol = RN(1 / s) of every scale (div_by_rcp; the row pairs also sit interleaved in sr2); a tile holding
// an Inf or NaN uses the IEEE divides themselves. A thread keeps one column (C divides the CTA size), so its
// column scale stays in registers.
template <int D, bool IS_V>
SJK_DEV void rescale(float * cur, const uint16_t * M, const float * srow, const float * scol, const float * rrow,
                     const float * rcol, const float2 * sr2, bool finite) {
    using CV = Carve<D, IS_V>;
    constexpr int R = CV::R, C = CV::C, RSTEP = NT / C;
    static_assert(NT % C == 0, "a thread keeps one column");
    const int c = threadIdx.x % C;
    if (finite) {
        const float sc = scol[c], rc = rcol[c];
#pragma unroll 4
        for (int r = threadIdx.x / C; r < R; r += RSTEP) {
            const float m = __half2float(__ushort_as_half(M[r * CV::LM + c]));
            const float2 rs = sr2[r];                                 // (s_row, 1 / s_row): one broadcast load
            cur[r * CV::LD + c] = div_by_rcp(div_by_rcp(m, sc, rc), rs.x, rs.y);
        }
    } else {
        for (int r = threadIdx.x / C; r < R; r += RSTEP)
            cur[r * CV::LD + c] = __fdiv_rn(__fdiv_rn(sjk_h2f(M[r * CV::LM + c]), scol[c]), srow[r]);
    }
}

// One balancing half-step over columns (COLS = true: std of each column over the R rows) or rows.
// Chunked double sums (8 contiguous chunks), fixed pairwise combine, fma second pass (sj_kvarn.h:939-978).
// The half-step with the rescale fused into its first pass: each thread forms the balanced values of its
// chunk(s), cur = (M / s_col) / s_row with the current scales (the rescale's own divides, in its order), sums them as
// it stores them, and its second pass reads back only the values it stored itself (no barrier between the two). The
// next half-step forms its values from M again with the updated scales, so the separate rescale sweeps, their reads
// of the tile and their barriers disappear. Same arithmetic, same order, same results.
template <int D, bool IS_V, bool COLS, bool FIN>
SJK_DEV void balance_half_m(float * cur, const uint16_t * M, const float * srow, const float * scol, const float * rcol,
                            const float2 * srr, double * part, double * mean, double * lacc, float * sacc, float * racc,
                            float2 * sr2) {
    using CV = Carve<D, IS_V>;
    constexpr int N = COLS ? CV::C : CV::R;        // number of vectors
    constexpr int L = COLS ? CV::R : CV::C;        // length of each vector
    constexpr int CH = L / 8;                      // chunk length
    constexpr int TPT = N * 8 / NT;                // chunks per thread
    static_assert(N * 8 % NT == 0 && TPT * CH * NT == CV::R * CV::C, "every thread takes its share of the tile");
#pragma unroll
    for (int k = 0; k < TPT; ++k) {
        const int task = threadIdx.x + k * NT, v = task % N, ch = task / N;
        double s = 0.0;
        if (COLS) {
            const int c = v;
            const float sc = scol[c], rc = rcol[c];
#pragma unroll 8
            for (int i = 0; i < CH; ++i) {
                const int r = ch * CH + i;
                const float m = __half2float(__ushort_as_half(M[r * CV::LM + c]));
                const float2 rs = srr[r];
                const float x = FIN ? div_by_rcp(div_by_rcp(m, sc, rc), rs.x, rs.y) : __fdiv_rn(__fdiv_rn(m, sc), rs.x);
                cur[r * CV::LD + c] = x;
                s = __dadd_rn(s, (double) x);
            }
        } else {
            const int r = v;
            const float2 rs = srr[r];
            const uint32_t * mrow = reinterpret_cast<const uint32_t *>(M + r * CV::LM + ch * CH);   // 4-byte aligned
#pragma unroll 4
            for (int i = 0; i < CH; i += 2) {
                const uint32_t w = mrow[i / 2];
                const float m0 = __half2float(__ushort_as_half((unsigned short) (w & 0xFFFFu)));
                const float m1 = __half2float(__ushort_as_half((unsigned short) (w >> 16)));
                const int c0 = ch * CH + i, c1 = c0 + 1;
                const float x0 = FIN ? div_by_rcp(div_by_rcp(m0, scol[c0], rcol[c0]), rs.x, rs.y)
                                     : __fdiv_rn(__fdiv_rn(m0, scol[c0]), rs.x);
                const float x1 = FIN ? div_by_rcp(div_by_rcp(m1, scol[c1], rcol[c1]), rs.x, rs.y)
                                     : __fdiv_rn(__fdiv_rn(m1, scol[c1]), rs.x);
                cur[r * CV::LD + c0] = x0;
                cur[r * CV::LD + c1] = x1;
                s = __dadd_rn(s, (double) x0);
                s = __dadd_rn(s, (double) x1);
            }
        }
        part[ch * N + v] = s;
    }
    __syncthreads();
    for (int v = threadIdx.x; v < N; v += NT) mean[v] = __ddiv_rn(tree8(part + v, N), (double) L);
    __syncthreads();
    constexpr int STR = COLS ? CV::LD : 1;         // element stride inside a vector
    constexpr int VSTR = COLS ? 1 : CV::LD;        // stride between vectors
#pragma unroll
    for (int k = 0; k < TPT; ++k) {
        const int task = threadIdx.x + k * NT, v = task % N, ch = task / N;
        const float * x = cur + v * VSTR + ch * CH * STR;
        const double mu = mean[v];
        double s = 0.0;
#pragma unroll 8
        for (int i = 0; i < CH; ++i) {
            const double dv = __dsub_rn((double) x[i * STR], mu);
            s = fma(dv, dv, s);
        }
        part[ch * N + v] = s;
    }
    __syncthreads();
    for (int v = threadIdx.x; v < N; v += NT) {
        const float sdv = (float) sqrt(__ddiv_rn(tree8(part + v, N), (double) (L > 1 ? L - 1 : 1)));
        const float sd = lesser_f(greater_f(sdv, 1e-3f), 1e3f);
        const double lg = lesser_d(greater_d(__dadd_rn(lacc[v], log((double) sd)), -0.3), 10.0);
        lacc[v] = lg;
        const float sv = (float) exp(lg);
        const float rv = __frcp_rn(sv);
        sacc[v] = sv;
        racc[v] = rv;
        if (!COLS) sr2[v] = make_float2(sv, rv);
    }
    __syncthreads();
}

// ---- scalar payload words ---------------------------------------------------------------------------------
SJK_DEV uint32_t rtn_code(float x, float lo, float step, uint32_t qmax) {
    float r = rintf(__fdiv_rn(__fsub_rn(x, lo), step));                // ties to even (sj_kvarn.h:1014-1019)
    if (r < 0.0f) r = 0.0f;
    if (r > (float) qmax) r = (float) qmax;
    return (uint32_t) r;
}

template <int D, bool IS_V>
SJK_DEV uint32_t code_at(const sj_kvarn_layout & l, const float * cur, const float * lo, const float * step, int t, int d,
                         uint32_t qmax) {
    using CV = Carve<D, IS_V>;
    const int r = IS_V ? t : d, c = IS_V ? d : t;
    return rtn_code(cur[r * CV::LD + c], lo[r], step[r], qmax);
}

// Emit the scalar payload one 32-bit word per thread step, straight to the record in global memory.
template <int D, bool IS_V>
SJK_DEV void scalar_payload(const sj_kvarn_layout & l, const float * cur, const float * lo, const float * step,
                            uint8_t * payload) {
    const int bits = IS_V ? l.bits_v : l.bits_k;
    const uint32_t qmax = (1u << bits) - 1u;
    const int words = D * G * bits / 32;
    uint32_t * out = reinterpret_cast<uint32_t *>(payload);
    if (sjk_frag(l, bits)) {
        for (int w = threadIdx.x; w < words; w += NT) {
            uint32_t acc = 0;
#pragma unroll
            for (int nib = 0; nib < 8; ++nib) {
                int t, d;
                sjk_frag_pos(l, (uint32_t) w, nib, IS_V, &t, &d);
                acc |= code_at<D, IS_V>(l, cur, lo, step, t, d, qmax) << (4 * nib);
            }
            out[w] = acc;
        }
        return;
    }
    // token-major stream: code k = t*D + d at bit k*bits
    for (int w = threadIdx.x; w < words; w += NT) {
        const uint32_t b0 = 32u * (uint32_t) w;
        uint32_t acc = 0;
        for (uint32_t k = b0 / (uint32_t) bits; k * (uint32_t) bits < b0 + 32u; ++k) {
            const int t = (int) (k / (uint32_t) D), d = (int) (k % (uint32_t) D);
            const uint32_t c = code_at<D, IS_V>(l, cur, lo, step, t, d, qmax);
            const int sh = (int) (k * (uint32_t) bits) - (int) b0;
            acc |= sh >= 0 ? c << sh : c >> (-sh);
        }
        out[w] = acc;
    }
}

// ---- trellis: Viterbi per channel, one warp per sequence (sj_kvarn.h:1021-1073) ---------------------------
// Lane L owns states 2L and 2L+1. Both states read the same previous-metric entries M[a + (64/NB) j]
// (a = state >> bits), so M lives in a per-warp transposed table where those NB entries are contiguous.
// Back-pointers: one byte per (step, lane), branch of state 2L in the low nibble, 2L+1 in the high one.
template <int D, bool IS_V, int BITS>
SJK_DEV void viterbi_side(const float * cur, const float * lo, const float * step, const uint16_t * cb16,
                          uint8_t * bp_all, float * mt_all, uint8_t * payload) {
    using CV = Carve<D, IS_V>;
    constexpr int NB = 1 << BITS;
    constexpr int NA = 64 / NB;                 // distinct history groups
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (warp >= VNW) return;
    uint8_t * bp = bp_all + warp * (G * 32);
    float * mt = mt_all + warp * 64;
    const int s0 = 2 * lane, s1 = 2 * lane + 1;
    const int a = s0 >> BITS;                   // == s1 >> BITS
    // transposed position of metric index k: (k % NA) * NB + k / NA
    const int p0 = (s0 % NA) * NB + s0 / NA, p1 = (s1 % NA) * NB + s1 / NA;
    float cA[NB], cB[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) { cA[j] = sjk_h2f(cb16[s0 + 64 * j]); cB[j] = sjk_h2f(cb16[s1 + 64 * j]); }
    for (int d = warp; d < D; d += VNW) {
        // targets y[t] = (bal - lo) / step of this channel, lane holds t = lane + 32 k
        float y[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int t = lane + 32 * k;
            const int r = IS_V ? t : d, c = IS_V ? d : t;
            y[k] = __fdiv_rn(__fsub_rn(cur[r * CV::LD + c], lo[r]), step[r]);
        }
        mt[2 * lane] = 0.0f; mt[2 * lane + 1] = 0.0f;
        __syncwarp();
#pragma unroll
        for (int k = 3; k >= 0; --k) {
            const float yk = y[k];
            for (int ii = 31; ii >= 0; --ii) {
                const int i = 32 * k + ii;
                const float yi = __shfl_sync(FULL, yk, ii);
                float mv[NB];
#pragma unroll
                for (int j = 0; j < NB; ++j) mv[j] = mt[a * NB + j];
                float best0 = __int_as_float(0x7F800000), best1 = __int_as_float(0x7F800000);
                int bj0 = 0, bj1 = 0;
#pragma unroll
                for (int j = 0; j < NB; ++j) {
                    const float d0 = __fsub_rn(yi, cA[j]), d1 = __fsub_rn(yi, cB[j]);
                    const float c0 = __fadd_rn(__fmul_rn(d0, d0), mv[j]);
                    const float c1 = __fadd_rn(__fmul_rn(d1, d1), mv[j]);
                    if (c0 < best0) { best0 = c0; bj0 = j; }
                    if (c1 < best1) { best1 = c1; bj1 = j; }
                }
                __syncwarp();
                mt[p0] = best0; mt[p1] = best1;
                bp[i * 32 + lane] = (uint8_t) (bj0 | (bj1 << 4));
                __syncwarp();
            }
        }
        // traceback from state 0 (no termination cost); lane L keeps the codes of tokens 4L..4L+3
        uint32_t mine = 0;
        int s = 0;
        for (int i = 0; i < G; ++i) {
            const int j = (bp[i * 32 + (s >> 1)] >> (4 * (s & 1))) & 15;
            if ((i >> 2) == lane) mine |= (uint32_t) j << (BITS * (i & 3));
            s = (s + 64 * j) >> BITS;
        }
        // channel-major stream: channel d's codes occupy bits [d*G*BITS, (d+1)*G*BITS)
        uint8_t * cp = payload + (size_t) d * G * BITS / 8;
        if (BITS == 2) {
            cp[lane] = (uint8_t) mine;                              // 4 codes x 2 bits = one byte per lane
        } else {
            const uint32_t other = __shfl_down_sync(FULL, mine, 1);   // lanes 2m, 2m+1: 24 bits = 3 bytes
            if ((lane & 1) == 0) {
                const uint32_t v = mine | (other << 12);
                cp[3 * (lane >> 1)] = (uint8_t) v;
                cp[3 * (lane >> 1) + 1] = (uint8_t) (v >> 8);
                cp[3 * (lane >> 1) + 2] = (uint8_t) (v >> 16);
            }
        }
        __syncwarp();
    }
}

// Moment-matching refit of each row's affine from the trellis reconstruction (sj_kvarn.h:1075-1109).
// One thread per row, sequential double sums in column order. Returns 1 and the (a, b) pair when valid.
template <int D, bool IS_V>
SJK_DEV int refit_row(const sj_kvarn_layout & l, const float * cur, int r, const uint8_t * payload, const float * cbf,
                      int bits, double * ad_out, double * bd_out) {
    using CV = Carve<D, IS_V>;
    double sx = 0.0, sy = 0.0, sxx = 0.0, syy = 0.0;
    const double n = (double) CV::C;
    for (int c = 0; c < CV::C; ++c) {
        const int t = IS_V ? r : c, d = IS_V ? c : r;
        const double x = (double) cur[r * CV::LD + c];
        const double yh = (double) cbf[sjk_window(payload, bits, d, t, G)];
        sx = __dadd_rn(sx, x);
        sy = __dadd_rn(sy, yh);
        sxx = __dadd_rn(sxx, __dmul_rn(x, x));
        syy = __dadd_rn(syy, __dmul_rn(yh, yh));
    }
    const double vy = __dsub_rn(__dmul_rn(n, syy), __dmul_rn(sy, sy));
    if (!(vy > 0.0)) return 0;
    const double vx = __dsub_rn(__dmul_rn(n, sxx), __dmul_rn(sx, sx));
    if (!(vx > 0.0)) return 0;
    const double ad = sqrt(__ddiv_rn(vx, vy));
    const double bd = __ddiv_rn(__dsub_rn(sx, __dmul_rn(ad, sy)), n);
    if (!(ad > 0.0) || !(bd == bd) || ad > 1e30 || fabs(bd) > 1e30) return 0;
    *ad_out = ad; *bd_out = bd;
    return 1;
}

SJK_DEV void put_half_g(uint8_t * rec, uint32_t off, float v) {
    const uint16_t h = sjk_f2h(v);
    rec[off] = (uint8_t) h;
    rec[off + 1] = (uint8_t) (h >> 8);
}

// ---- one side of one record ------------------------------------------------------------------------------------
template <int D, bool IS_V>
SJK_DEV void seal_side(const SealParams & p, uint8_t * smem) {
    using CV = Carve<D, IS_V>;
    constexpr int R = CV::R, C = CV::C;
    const sj_kvarn_layout & l = p.lay;
    float * cur = reinterpret_cast<float *>(smem + CV::cur);
    uint16_t * M = reinterpret_cast<uint16_t *>(smem + CV::regA);
    double * part = reinterpret_cast<double *>(smem + CV::regB);
    float * srow = reinterpret_cast<float *>(smem + CV::srow);
    float * scol = reinterpret_cast<float *>(smem + CV::scol);
    float * lo = reinterpret_cast<float *>(smem + CV::lo);
    float * step = reinterpret_cast<float *>(smem + CV::step);
    double * lrow = reinterpret_cast<double *>(smem + CV::lrow);
    double * lcol = reinterpret_cast<double *>(smem + CV::lcol);
    double * mean = reinterpret_cast<double *>(smem + CV::mean);
    uint32_t * fit = reinterpret_cast<uint32_t *>(smem + CV::fit);
    float * cent = reinterpret_cast<float *>(smem + CV::regB);   // tq6 centroids, only during the load

    const int rec_local = blockIdx.x;
    const int g_local = rec_local / p.H, h = rec_local % p.H;
    uint32_t g_abs = (uint32_t) g_local;
    if (p.source == SRC_RING) g_abs += (p.B_from - p.S) / (uint32_t) G;
    const uint32_t blk = p.blocks ? p.blocks[g_abs] : g_abs;
    uint8_t * rec = p.body + ((size_t) blk * p.H + h) * l.bytes;

    if (threadIdx.x < 64) cent[threadIdx.x] = sjk_tq6_cent[threadIdx.x];
    // byte offset of each token's K or V row in the ring, one ring-slot division per token (only during the load)
    size_t * rowoff = reinterpret_cast<size_t *>(smem + CV::regB + 256);
    if (p.source == SRC_RING && threadIdx.x < G) {
        const uint32_t pos = p.B_from + (uint32_t) (g_local * G + threadIdx.x);
        rowoff[threadIdx.x] = ((size_t) sjk_ring_slot(p.S, p.cap, pos) * p.H + h) * 2 * p.stage_bytes + (IS_V ? p.stage_bytes : 0);
    }
    float * rrow = lo, * rcol = step;                            // reciprocals of the scales while balancing
    float2 * sr2 = reinterpret_cast<float2 *>(fit);              // (srow, rrow) pairs while balancing
    for (int c = threadIdx.x; c < C; c += NT) { scol[c] = 1.0f; rcol[c] = 1.0f; lcol[c] = 0.0; }
    for (int r = threadIdx.x; r < R; r += NT) { srow[r] = 1.0f; rrow[r] = 1.0f; sr2[r] = make_float2(1.0f, 1.0f); lrow[r] = 0.0; }
    __syncthreads();
    const bool finite = !__syncthreads_or(load_input<D, IS_V>(p, rec_local, M, cent, rowoff));

    // ---- log-domain variance balancing, exactly `iters` column-then-row passes (sj_kvarn.h:989-1012); every
    // half-step forms the balanced tile from M with the current scales (the reference's rescale after each
    // half-step), and the tile itself is stored once, after the last one ----
    for (int it = 0; it < p.iters; ++it) {
        if (finite) {
            balance_half_m<D, IS_V, true, true>(cur, M, srow, scol, rcol, sr2, part, mean, lcol, scol, rcol, sr2);
            balance_half_m<D, IS_V, false, true>(cur, M, srow, scol, rcol, sr2, part, mean, lrow, srow, rrow, sr2);
        } else {
            balance_half_m<D, IS_V, true, false>(cur, M, srow, scol, rcol, sr2, part, mean, lcol, scol, rcol, sr2);
            balance_half_m<D, IS_V, false, false>(cur, M, srow, scol, rcol, sr2, part, mean, lrow, srow, rrow, sr2);
        }
    }
    rescale<D, IS_V>(cur, M, srow, scol, rrow, rcol, sr2, finite);
    __syncthreads();

    // ---- per-row asymmetric range (sj_kvarn.h:1120-1128) ----
    const int bits = IS_V ? l.bits_v : l.bits_k;
    const uint32_t qmax = (1u << bits) - 1u;
    for (int r = threadIdx.x; r < R; r += NT) {
        const float * row = cur + r * CV::LD;
        float a = row[0], b = row[0];
        for (int c = 1; c < C; ++c) { a = lesser_f(a, row[c]); b = greater_f(b, row[c]); }
        lo[r] = a;
        step[r] = greater_f(__fdiv_rn(__fsub_rn(b, a), (float) qmax), 1e-10f);
    }
    __syncthreads();

    const uint32_t pay_off = IS_V ? l.v_payload : l.k_payload;
    const uint32_t sc_off = IS_V ? l.v_scale : l.k_scale, zp_off = IS_V ? l.v_zero : l.k_zero;
    if (l.body != SJKVARN_BODY_TRELLIS) {
        scalar_payload<D, IS_V>(l, cur, lo, step, rec + pay_off);
        for (int r = threadIdx.x; r < R; r += NT) {
            const uint32_t ri = (uint32_t) (IS_V ? r : sjk_k_ch(l, r));
            put_half_g(rec, sc_off + 2u * ri, __fmul_rn(srow[r], step[r]));
            put_half_g(rec, zp_off + 2u * ri, __fmul_rn(srow[r], lo[r]));
        }
    } else {
        // trellis: M's space -> back-pointers, part's space -> payload + per-warp metric tables
        uint8_t * bp = smem + CV::regA;
        uint8_t * payload = smem + CV::regB;
        const int pay_bytes = D * G * bits / 8;
        float * mt = reinterpret_cast<float *>(smem + CV::regB + 12288);
        const uint16_t * cb16 = sjk_codebook(bits, IS_V);
        if (bits == 3) viterbi_side<D, IS_V, 3>(cur, lo, step, cb16, bp, mt, payload);
        else viterbi_side<D, IS_V, 2>(cur, lo, step, cb16, bp, mt, payload);
        __syncthreads();
        // codebook as float for the refit (back-pointer space is free now)
        float * cbf = reinterpret_cast<float *>(smem + CV::regA);
        for (int i = threadIdx.x; i < (1 << (6 + bits)); i += NT) cbf[i] = sjk_h2f(cb16[i]);
        __syncthreads();
        for (int r = threadIdx.x; r < R; r += NT) {
            double ad, bd;
            float sv = __fmul_rn(srow[r], step[r]), zv = __fmul_rn(srow[r], lo[r]);
            if (refit_row<D, IS_V>(l, cur, r, payload, cbf, bits, &ad, &bd)) {
                sv = __fmul_rn(srow[r], (float) ad);
                zv = __fmul_rn(srow[r], (float) bd);
            }
            fit[2 * r] = sjk_f2h(sv);
            fit[2 * r + 1] = sjk_f2h(zv);
        }
        __syncthreads();
        for (int r = threadIdx.x; r < R; r += NT) {
            const uint32_t ri = (uint32_t) (IS_V ? r : sjk_k_ch(l, r));
            rec[sc_off + 2u * ri] = (uint8_t) fit[2 * r];
            rec[sc_off + 2u * ri + 1] = (uint8_t) (fit[2 * r] >> 8);
            rec[zp_off + 2u * ri] = (uint8_t) fit[2 * r + 1];
            rec[zp_off + 2u * ri + 1] = (uint8_t) (fit[2 * r + 1] >> 8);
        }
        const uint32_t * ps = reinterpret_cast<const uint32_t *>(payload);
        uint32_t * pd = reinterpret_cast<uint32_t *>(rec + pay_off);
        for (int w = threadIdx.x; w < pay_bytes / 4; w += NT) pd[w] = ps[w];
    }
    // column scales: Ktok[t] (K columns are tokens), Vch[v_ch(d)] (V columns are channels)
    for (int c = threadIdx.x; c < C; c += NT) {
        const uint32_t off = IS_V ? l.v_ch + 2u * (uint32_t) sjk_v_ch(l, c) : l.k_tok + 2u * (uint32_t) c;
        put_half_g(rec, off, scol[c]);
    }
}

template <int D>
__global__ void __launch_bounds__(NT, 1) seal_kernel(SealParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    if (p.desc) {
        // groups [(B_OLD - S) / G, (B - S) / G) of the descriptor; the launch covers n_groups_max of them
        sjk_desc_vals dv;
        const bool ok = sjk_desc_read(p.desc, p.dref, &dv) && (dv.B - dv.B_old) / (uint32_t) G <= p.n_groups_max;
        if (!ok) {
            if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) sjk_desc_fault();
            return;
        }
        if ((uint32_t) blockIdx.x >= (dv.B - dv.B_old) / (uint32_t) G * (uint32_t) p.H) return;
        p.B_from = dv.B_old;
    }
    if (blockIdx.y == 0) seal_side<D, false>(p, smem);
    else seal_side<D, true>(p, smem);
}

template <int D>
int launch_seal(const SealParams & p, int n_rec, sjk_stream st) {
    const size_t smem = seal_smem_bytes<D>();
    cudaError_t e = cudaFuncSetAttribute(seal_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e != cudaSuccess) return sjk_check(e);
    seal_kernel<D><<<dim3((unsigned) n_rec, 2), NT, smem, st>>>(p);
    return sjk_check_launch();
}

int seal_dispatch(const SealParams & p, int n_rec, sjk_stream st) {
    const sj_kvarn_layout & l = p.lay;
    if (l.G != G) return SJK_ERR_UNSUPPORTED;
    if (l.body == SJKVARN_BODY_TRELLIS && (l.bits_k > 3 || l.bits_v > 3)) return SJKVARN_ERR_ARG;
    switch (l.D) {
        case 128: return launch_seal<128>(p, n_rec, st);
        case 256: return launch_seal<256>(p, n_rec, st);
        default: return SJK_ERR_UNSUPPORTED;
    }
}

}  // namespace

extern "C" int sjk_seal(const sj_kvarn_layout * lay, const uint16_t * k, const uint16_t * v, size_t row_stride,
                        int n_head_kv, int n_groups, int iters, uint8_t * body, void * work, sjk_stream st) {
    (void) work;
    if (!lay || !k || !v || !body || n_head_kv <= 0 || n_groups < 0 || iters < 0) return SJKVARN_ERR_ARG;
    if (n_groups == 0) return 0;
    SealParams p = {};
    p.lay = *lay; p.H = n_head_kv; p.iters = iters;
    p.k = k; p.v = v; p.row_stride = row_stride; p.source = SRC_F16_ROWS;
    p.body = body;
    return seal_dispatch(p, n_groups * n_head_kv, st);
}

extern "C" int sjk_seal_ring(const sjk_view * v, uint8_t * body, uint32_t B_from, uint32_t B_to, int iters, sjk_stream st) {
    if (!v || !body || !v->ring || iters < 0 || B_to < B_from || B_from < v->S) return SJKVARN_ERR_ARG;
    const uint32_t G_ = (uint32_t) v->lay.G;
    if ((B_from - v->S) % G_ || (B_to - v->S) % G_) return SJKVARN_ERR_ARG;
    const uint32_t ng = (B_to - B_from) / G_;
    if (ng == 0) return 0;
    SealParams p = {};
    p.lay = v->lay; p.H = v->n_head_kv; p.iters = iters;
    p.source = SRC_RING; p.staging = v->staging; p.ring = v->ring; p.S = v->S; p.cap = v->cap; p.B_from = B_from;
    p.stage_bytes = (uint32_t) v->stage_bytes; p.blocks = v->blocks; p.body = body;
    return seal_dispatch(p, (int) (ng * (uint32_t) v->n_head_kv), st);
}

// Descriptor-driven ring seal (the reference's seal_dyn op, INTEGRATION_LLAMACPP.md:49): a fixed launch over
// n_groups_max groups x n_head_kv heads whose CTAs read [B_OLD, B) from the descriptor; CTAs past the descriptor's
// groups return at once.
extern "C" int sjk_seal_dyn(const sjk_view * v, const int32_t * desc, uint32_t n_groups_max, int iters, sjk_stream st) {
    if (!v || !desc || !v->body || !v->ring || iters < 0 || v->n_head_kv <= 0) return SJKVARN_ERR_ARG;
    if (n_groups_max == 0) return 0;
    if ((uint64_t) n_groups_max * (uint32_t) v->n_head_kv > 0x7FFFFFFFu) return SJKVARN_ERR_ARG;
    SealParams p = {};
    p.lay = v->lay; p.H = v->n_head_kv; p.iters = iters;
    p.source = SRC_RING; p.staging = v->staging; p.ring = v->ring; p.S = v->S; p.cap = v->cap; p.B_from = v->S;
    p.stage_bytes = (uint32_t) v->stage_bytes; p.blocks = v->blocks; p.body = const_cast<uint8_t *>(v->body);
    p.desc = desc; p.dref = sjk_desc_ref_of(*v); p.n_groups_max = n_groups_max;
    return seal_dispatch(p, (int) (n_groups_max * (uint32_t) v->n_head_kv), st);
}

SJK_DESC_STATUS_READER(sjk_seal_desc_status_take)

namespace {
// the double log and exp of the balancing (the calls of seal_kernel's scale updates), on a list of arguments
__global__ void libm_probe_kernel(const double * x, size_t n, double * lg, double * ex) {
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t) gridDim.x * blockDim.x) {
        const double a = x[i];
        lg[i] = log(a);
        ex[i] = exp(a);
    }
}
}  // namespace

extern "C" int sjk_seal_libm_probe(const double * x, size_t n, double * lg, double * ex, sjk_stream st) {
    if (n == 0) return 0;
    if (!x || !lg || !ex) return SJKVARN_ERR_ARG;
    const size_t blocks = (n + 255) / 256;
    libm_probe_kernel<<<(unsigned) (blocks < 4096 ? blocks : 4096), 256, 0, st>>>(x, n, lg, ex);
    return sjk_check_launch();
}
