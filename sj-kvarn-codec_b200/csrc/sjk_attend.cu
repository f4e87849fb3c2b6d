// sjk_attend.cu - causal decode attention over the three regions of an SJ-KVaRN layer cache
// (fp16 sink [0, S), sealed body [S, B), staging ring [B, N)), flash-decoding style:
//
//   split kernel  grid (splits, KV heads). Each CTA walks a contiguous range of 128-position chunks
//                 (a chunk never straddles two regions; a body chunk is one record), decodes the K/V rows
//                 of 32 positions at a time into shared memory exactly as the reference decoders do, and
//                 keeps a running (max, sum, output) per query row of its KV head (all GQA heads x rows).
//   merge kernel  one CTA per (query row, query head) combines the splits' partials.
//
// Scores use the reference's sequential fp32 dot (sj_kvarn.h:1288-1293) on identically decoded rows, so
// they are bit-equal to the reference's; only the softmax accumulation order differs (chunk-wise online
// softmax + merge instead of one position-ordered pass), which the 1e-3 relative contract covers.
#include <mutex>

#include "sjk_common.cuh"
#include "sjk_internal.h"

namespace {

constexpr int NT = 256;
constexpr int SUB = 32;             // positions decoded per step
constexpr int MAXROWS = 16;         // query rows per KV head handled by one CTA (n_q * GQA group)

struct AttnParams {
    sjk_view v;
    int kv0;                        // first KV head of the call (grid.y walks kv0 .. kv0 + n_kv - 1)
    uint32_t B, N, qpos0;
    int n_q, n_head, grp, rows;     // rows = n_q * grp
    const float * q;
    float scale;
    float * part;                   // [splits][n_q*n_head][D + 2]: m, l, o[D]
    int split0;                     // partial slot of this kernel's first split
    int chunks_per_split, n_chunks;
    uint32_t n_sink_chunks, n_body_chunks;
    uint32_t body_skip;             // leading body records handled by the tensor-core kernel
};

struct Chunk { int region; uint32_t p0, len, g; };   // region 0 sink, 1 body, 2 ring

SJK_DEV Chunk chunk_of(const AttnParams & p, uint32_t ci) {
    Chunk c;
    const uint32_t S = p.v.S;
    const uint32_t s_end = S < p.N ? S : p.N;
    if (ci < p.n_sink_chunks) {
        c.region = 0; c.p0 = ci * 128u; c.len = min(128u, s_end - c.p0); c.g = 0;
    } else if (ci < p.n_sink_chunks + p.n_body_chunks) {
        const uint32_t b_end = p.B < p.N ? p.B : p.N;      // a query over a prefix may end inside a record
        c.region = 1; c.g = p.body_skip + ci - p.n_sink_chunks; c.p0 = S + c.g * 128u; c.len = min(128u, b_end - c.p0);
    } else {
        const uint32_t k = ci - p.n_sink_chunks - p.n_body_chunks;
        const uint32_t b0 = p.B > S ? p.B : S;
        c.region = 2; c.p0 = b0 + k * 128u; c.len = min(128u, p.N - c.p0); c.g = 0;
    }
    return c;
}

// Decode rows [t0, t0+n) of a chunk into K/V shared tiles [SUB][D+1] (sj_kvarn.h:1516-1533).
template <int D>
SJK_DEV void load_rows(const AttnParams & p, const Chunk & c, uint32_t t0, uint32_t n, int h, float * Ks, float * Vs,
                       const float * sc, const float * cbk, const float * cbv) {
    const sjk_view & v = p.v;
    const sj_kvarn_layout & l = v.lay;
    const int H = v.n_head_kv;
    for (int e = threadIdx.x; e < (int) n * D; e += NT) {
        const int t = e / D, d = e % D;
        const uint32_t pos = c.p0 + t0 + (uint32_t) t;
        float kv, vv;
        if (c.region == 1) {
            const uint32_t blk = v.blocks ? v.blocks[c.g] : c.g;
            const uint8_t * rec = v.body + ((size_t) blk * H + h) * l.bytes;
            const int tt = (int) (t0 + (uint32_t) t);
            float qk, qv;
            if (l.body == SJKVARN_BODY_TRELLIS) {
                qk = cbk[sjk_window(rec + l.k_payload, l.bits_k, d, tt, 128)];
                qv = cbv[sjk_window(rec + l.v_payload, l.bits_v, d, tt, 128)];
            } else {
                qk = (float) sjk_get_bits(rec + l.k_payload, sjk_code_bit(l, tt, d, 0), l.bits_k);
                qv = (float) sjk_get_bits(rec + l.v_payload, sjk_code_bit(l, tt, d, 1), l.bits_v);
            }
            // sc: ks[D], kz[D], vc[D], kt[128], vs[128], vz[128] of this record, natural order
            kv = __fmul_rn(__fadd_rn(__fmul_rn(qk, sc[d]), sc[D + d]), sc[3 * D + tt]);
            vv = __fmul_rn(__fadd_rn(__fmul_rn(qv, sc[3 * D + 128 + tt]), sc[3 * D + 256 + tt]), sc[2 * D + d]);
        } else if (c.region == 0 && v.sink_type == SJKVARN_SINK_F16) {
            const uint8_t * row = v.sink + ((size_t) pos * H + h) * 4 * D;
            kv = sjk_h2f(sjk_ld_u16(row + 2 * d));
            vv = sjk_h2f(sjk_ld_u16(row + 2 * D + 2 * d));
        } else {
            const uint8_t * row = c.region == 0 ? v.sink + ((size_t) pos * H + h) * 2 * v.stage_bytes
                                                : v.ring + ((size_t) sjk_ring_slot(v.S, v.cap, pos) * H + h) * 2 * v.stage_bytes;
            if (v.staging == SJKVARN_STAGING_F16) {
                kv = sjk_h2f(sjk_ld_u16(row + 2 * d));
                vv = sjk_h2f(sjk_ld_u16(row + v.stage_bytes + 2 * d));
            } else {
                const int j = d & 127;
                const uint8_t * bk = row + (d >> 7) * SJKVARN_TQ6_BLOCK_BYTES;
                const uint8_t * bv = bk + v.stage_bytes;
                const int ck = ((bk[2 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((bk[66 + (j >> 2)] >> (2 * (j & 3))) & 3) << 4);
                const int cv = ((bv[2 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((bv[66 + (j >> 2)] >> (2 * (j & 3))) & 3) << 4);
                kv = __fmul_rn(sjk_tq6_cent[ck], sjk_h2f(sjk_ld_u16(bk)));
                vv = __fmul_rn(sjk_tq6_cent[cv], sjk_h2f(sjk_ld_u16(bv)));
            }
        }
        Ks[t * (D + 1) + d] = kv;
        Vs[t * (D + 1) + d] = vv;
    }
}

template <int D>
__global__ void __launch_bounds__(NT) attend_split_kernel(AttnParams p) {
    extern __shared__ __align__(16) float sm[];
    float * Ks = sm;                                  // [SUB][D+1]
    float * Vs = Ks + SUB * (D + 1);                  // [SUB][D+1]
    float * Qs = Vs + SUB * (D + 1);                  // [MAXROWS][D]
    float * Ss = Qs + MAXROWS * D;                    // [MAXROWS][SUB] scores -> weights
    float * sc = Ss + MAXROWS * SUB;                  // record scales: 3D + 384
    float * cbk = sc + 3 * D + 384;                   // 512
    float * cbv = cbk + 512;                          // 512
    float * rowm = cbv + 512;                         // [MAXROWS] running max
    float * rowl = rowm + MAXROWS;                    // [MAXROWS] running sum
    float * rowa = rowl + MAXROWS;                    // [MAXROWS] rescale factor of the current step
    const int hl = blockIdx.y, h = p.kv0 + hl, split = blockIdx.x;   // hl: head index inside q / out
    const sj_kvarn_layout & l = p.v.lay;
    const int R = p.rows;

    // query rows of this KV head: row r = iq * grp + j  <->  query head h*grp + j, row iq
    for (int e = threadIdx.x; e < R * D; e += NT) {
        const int r = e / D, d = e % D;
        const int iq = r / p.grp, hq = hl * p.grp + r % p.grp;
        Qs[e] = p.q[((size_t) iq * p.n_head + hq) * D + d];
    }
    if (l.body == SJKVARN_BODY_TRELLIS) {
        const uint16_t * ck = sjk_codebook(l.bits_k, 0), * cv = sjk_codebook(l.bits_v, 1);
        for (int i = threadIdx.x; i < (1 << (6 + l.bits_k)); i += NT) cbk[i] = sjk_h2f(ck[i]);
        for (int i = threadIdx.x; i < (1 << (6 + l.bits_v)); i += NT) cbv[i] = sjk_h2f(cv[i]);
    }
    if (threadIdx.x < MAXROWS) { rowm[threadIdx.x] = -__int_as_float(0x7F800000); rowl[threadIdx.x] = 0.0f; }
    // accumulator: thread owns row r_own for channels d = g + 16 i (i < D/16)
    const int r_own = threadIdx.x / 16, g_own = threadIdx.x % 16;
    float acc[D / 16];
#pragma unroll
    for (int i = 0; i < D / 16; ++i) acc[i] = 0.0f;
    __syncthreads();

    const int c_begin = split * p.chunks_per_split;
    const int c_end = min(p.n_chunks, c_begin + p.chunks_per_split);
    for (int ci = c_begin; ci < c_end; ++ci) {
        const Chunk c = chunk_of(p, (uint32_t) ci);
        if (c.region == 1) {
            const uint32_t blk = p.v.blocks ? p.v.blocks[c.g] : c.g;
            const uint8_t * rec = p.v.body + ((size_t) blk * p.v.n_head_kv + h) * l.bytes;
            __syncthreads();
            for (int d = threadIdx.x; d < D; d += NT) {
                const int kc = sjk_k_ch(l, d), vc = sjk_v_ch(l, d);
                sc[d] = sjk_h2f(sjk_ld_u16(rec + l.k_scale + 2 * kc));
                sc[D + d] = sjk_h2f(sjk_ld_u16(rec + l.k_zero + 2 * kc));
                sc[2 * D + d] = sjk_h2f(sjk_ld_u16(rec + l.v_ch + 2 * vc));
            }
            for (int t = threadIdx.x; t < 128; t += NT) {
                sc[3 * D + t] = sjk_h2f(sjk_ld_u16(rec + l.k_tok + 2 * t));
                sc[3 * D + 128 + t] = sjk_h2f(sjk_ld_u16(rec + l.v_scale + 2 * t));
                sc[3 * D + 256 + t] = sjk_h2f(sjk_ld_u16(rec + l.v_zero + 2 * t));
            }
        }
        for (uint32_t t0 = 0; t0 < c.len; t0 += SUB) {
            const uint32_t n = min((uint32_t) SUB, c.len - t0);
            __syncthreads();
            load_rows<D>(p, c, t0, n, h, Ks, Vs, sc, cbk, cbv);
            __syncthreads();
            // scores: the reference's sequential dot, then x scale; masked beyond each row's causal end
            for (int e = threadIdx.x; e < R * SUB; e += NT) {
                const int r = e / SUB, t = e % SUB;
                const uint32_t pos = c.p0 + t0 + (uint32_t) t;
                const uint32_t qpos = p.qpos0 + (uint32_t) (r / p.grp);
                float s = -__int_as_float(0x7F800000);
                if ((uint32_t) t < n && pos <= qpos) {
                    const float * qr = Qs + r * D;
                    const float * kr = Ks + t * (D + 1);
                    float dot = 0.0f;
                    for (int d = 0; d < D; ++d) dot = __fadd_rn(dot, __fmul_rn(qr[d], kr[d]));
                    s = __fmul_rn(dot, p.scale);
                }
                Ss[r * SUB + t] = s;
            }
            __syncthreads();
            // online softmax per row over this step's positions
            if (threadIdx.x < R) {
                const int r = threadIdx.x;
                float mx = rowm[r];
                for (int t = 0; t < SUB; ++t) mx = fmaxf(mx, Ss[r * SUB + t]);
                float alpha = 1.0f, sum = 0.0f;
                if (mx == -__int_as_float(0x7F800000)) {
                    for (int t = 0; t < SUB; ++t) Ss[r * SUB + t] = 0.0f;
                } else {
                    alpha = expf(rowm[r] - mx);
                    for (int t = 0; t < SUB; ++t) {
                        const float w = expf(Ss[r * SUB + t] - mx);
                        Ss[r * SUB + t] = w;
                        sum += w;
                    }
                    rowm[r] = mx;
                }
                rowl[r] = rowl[r] * alpha + sum;
                rowa[r] = alpha;
            }
            __syncthreads();
            if (r_own < R) {
                const float alpha = rowa[r_own];
#pragma unroll
                for (int i = 0; i < D / 16; ++i) acc[i] *= alpha;
                for (int t = 0; t < (int) n; ++t) {
                    const float w = Ss[r_own * SUB + t];
                    const float * vr = Vs + t * (D + 1) + g_own;
#pragma unroll
                    for (int i = 0; i < D / 16; ++i) acc[i] = fmaf(w, vr[16 * i], acc[i]);
                }
            }
        }
    }
    // partials: (m, l, o[D]) per (row, query head)
    __syncthreads();
    if (r_own < R) {
        const int iq = r_own / p.grp, hq = hl * p.grp + r_own % p.grp;
        float * dst = p.part + ((size_t) (p.split0 + split) * p.n_q * p.n_head + (size_t) iq * p.n_head + hq) * (D + 2);
        if (g_own == 0) { dst[0] = rowm[r_own]; dst[1] = rowl[r_own]; }
#pragma unroll
        for (int i = 0; i < D / 16; ++i) dst[2 + g_own + 16 * i] = acc[i];
    }
}

// out[row, head] = sum_i o_i e^(m_i - m) / sum_i l_i e^(m_i - m). Grid (query row x head, channel tiles of
// 64); each CTA recomputes the split weights (cheap) into shared memory and sums its 64 channels.
constexpr int MERGE_SPLITS = 768;                     // >= the most splits a call can make (148 + 296 + 296)
constexpr int MERGE_PRE = 24;                         // outputs per thread loaded ahead of the weights

// part_out (optional): instead of out, write the combined partial (m, l, o[D]) of each row (o not normalized), the
// form sjk_attend_partial returns
__global__ void __launch_bounds__(256) attend_merge_kernel(const float * part, int splits, int n_rows, int D, float * out,
                                                           float * part_out) {
    extern __shared__ float wts[];                     // [splits] weights, then [4][64] partial sums
    __shared__ float s_red[16];
    const int row = blockIdx.x, d0 = blockIdx.y * 64;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // launched as a programmatic dependent of the kernels that write the partials: wait until they completed
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the outputs of the first MERGE_PRE splits of this thread's group go in flight with the (m, l) loads
    const int dl = tid & 63, grp4 = tid >> 6;
    const bool live = d0 + dl < D;
    const float * src = part + (size_t) row * (D + 2) + 2 + d0 + (live ? dl : 0);
    const size_t step = (size_t) n_rows * (D + 2);
    float xo[MERGE_PRE];
#pragma unroll
    for (int k = 0; k < MERGE_PRE; ++k) {
        const int i = grp4 + 4 * k;
        xo[k] = i < splits ? src[(size_t) i * step] : 0.0f;
    }
    // one pass over (m, l) of the splits this thread owns (at most MERGE_SPLITS / 256)
    float mi[MERGE_SPLITS / 256], li[MERGE_SPLITS / 256];
#pragma unroll
    for (int k = 0; k < MERGE_SPLITS / 256; ++k) {
        const int i = tid + 256 * k;
        mi[k] = -INFINITY; li[k] = 0.0f;
        if (i < splits) {
            const float2 ml = *reinterpret_cast<const float2 *>(part + ((size_t) i * n_rows + row) * (D + 2));
            mi[k] = ml.x; li[k] = ml.y;
        }
    }
    float m = fmaxf(fmaxf(mi[0], mi[1]), mi[2]);
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (lane == 0) s_red[warp] = m;
    __syncthreads();
    m = s_red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, s_red[w]);
    float den = 0.0f;
#pragma unroll
    for (int k = 0; k < MERGE_SPLITS / 256; ++k) {
        const int i = tid + 256 * k;
        if (i < splits) {
            const float w = mi[k] == -INFINITY ? 0.0f : expf(mi[k] - m);
            wts[i] = w;
            den += li[k] * w;
        }
    }
    for (int o = 16; o; o >>= 1) den += __shfl_xor_sync(0xFFFFFFFFu, den, o);
    if (lane == 0) s_red[8 + warp] = den;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += s_red[8 + w];
    const float s_inv = t == 0.0f ? 0.0f : 1.0f / t;
    // 4 groups of 64 threads walk the splits in strides of 4; failed or empty splits carry weight 0 and zero
    // outputs. The first MERGE_PRE splits of each group were loaded together with (m, l), before the barriers.
    float o = 0.0f;
#pragma unroll
    for (int k = 0; k < MERGE_PRE; ++k) {
        const int i = grp4 + 4 * k;
        if (i < splits) o = fmaf(xo[k], wts[i], o);
    }
    for (int i = grp4 + 4 * MERGE_PRE; i < splits; i += 4) o = fmaf(src[(size_t) i * step], wts[i], o);
    float * acc = wts + splits;
    acc[grp4 * 64 + dl] = o;
    __syncthreads();
    if (part_out) {
        if (tid < 64 && d0 + tid < D) part_out[(size_t) row * (D + 2) + 2 + d0 + tid] = (acc[tid] + acc[64 + tid]) + (acc[128 + tid] + acc[192 + tid]);
        if (blockIdx.y == 0 && tid == 0) { part_out[(size_t) row * (D + 2)] = m; part_out[(size_t) row * (D + 2) + 1] = t; }
    } else if (tid < 64 && d0 + tid < D) {
        out[(size_t) row * D + d0 + tid] = ((acc[tid] + acc[64 + tid]) + (acc[128 + tid] + acc[192 + tid])) * s_inv;
    }
}

struct Plan { int splits, chunks_per_split, n_chunks; uint32_t n_sink, n_body; };

// upper bound of the split count: about two CTAs per SM over the call's KV heads
int split_target(int n_kv) {
    const int H = n_kv > 0 ? n_kv : 1;
    const int t = (2 * 148 + H - 1) / H;
    return t < 1 ? 1 : t;
}

// chunks left to the CUDA-core kernel: the body after the first body_skip records, plus the sink and the
// staging ring unless the dense tensor-core kernel takes them (no_staged)
Plan make_plan(const sjk_view * v, uint32_t B, uint32_t N, int n_kv, uint32_t body_skip, bool no_staged, unsigned regions) {
    Plan pl;
    const uint32_t S = v->S;
    const uint32_t s_end = S < N ? S : N;
    pl.n_sink = (no_staged || !(regions & SJK_REGION_SINK)) ? 0u : (s_end + 127u) / 128u;
    const uint32_t b_end = B < N ? B : N;
    pl.n_body = (b_end > S && (regions & SJK_REGION_BODY)) ? (b_end - S + 127u) / 128u : 0u;
    pl.n_body = pl.n_body > body_skip ? pl.n_body - body_skip : 0u;
    const uint32_t t0 = B > S ? B : S;
    const uint32_t n_tail = (N > t0 && !no_staged && (regions & SJK_REGION_RING)) ? (N - t0 + 127u) / 128u : 0u;
    pl.n_chunks = (int) (pl.n_sink + pl.n_body + n_tail);
    const int target = split_target(n_kv);
    pl.chunks_per_split = (pl.n_chunks + target - 1) / target;
    if (pl.chunks_per_split < 1) pl.chunks_per_split = 1;
    pl.splits = pl.n_chunks > 0 ? (pl.n_chunks + pl.chunks_per_split - 1) / pl.chunks_per_split : 1;
    return pl;
}

template <int D>
size_t split_smem() {
    return (size_t) (2 * SUB * (D + 1) + MAXROWS * D + MAXROWS * SUB + 3 * D + 384 + 1024 + 3 * MAXROWS) * sizeof(float);
}

}  // namespace

size_t sjk_attend_heads_scratch_bytes(const sjk_view * v, int n_q, int n_head, int n_kv) {
    if (!v || n_q <= 0 || n_head <= 0) return 0;
    // CUDA-core, tensor-core body and tensor-core staged-row splits, each bounded by the per-call target
    return (size_t) 3 * split_target(n_kv) * n_q * n_head * (v->lay.D + 2) * sizeof(float);
}

extern "C" size_t sjk_attend_scratch_bytes(const sjk_view * v, uint32_t N, int n_q, int n_head) {
    (void) N;
    if (!v) return 0;
    return sjk_attend_heads_scratch_bytes(v, n_q, n_head, v->n_head_kv);
}

int sjk_attend_heads(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, int kv_head0, int n_kv,
                     const float * q, float scale, float * out, void * scratch, size_t scratch_bytes, sjk_stream st,
                     unsigned regions, float * part_out) {
    if (!v || !q || !(out || part_out) || n_q <= 0 || n_head <= 0 || n_kv <= 0 || kv_head0 < 0 || kv_head0 + n_kv > v->n_head_kv ||
        n_head % n_kv)
        return SJKVARN_ERR_ARG;
    if (B < v->S) return SJKVARN_ERR_ARG;
    const int grp = n_head / n_kv;
    if (n_q * grp > MAXROWS) return SJK_ERR_UNSUPPORTED;
    // sealed records [0, n_tc) go to the tensor-core kernel when it supports the body format; when it also supports
    // the staged-row formats, the same kernel takes the sink and the staging ring, else the dense kernel does
    const uint32_t b_end = B < N ? B : N;
    const bool tc_body = sjk_tc_body_supported(v, n_q, grp) != 0;
    const bool tc_trellis = !tc_body && sjk_tc_trellis_supported(v, n_q, grp) != 0;
    const bool dense = sjk_tc_dense_supported(v, n_q, grp) != 0;
    const bool fused = tc_body && dense;
    const bool body_on = (regions & SJK_REGION_BODY) != 0;
    const uint32_t n_tc = ((tc_body || tc_trellis) && body_on && b_end > v->S) ? (b_end - v->S) / 128u : 0u;
    const unsigned staged = regions & (SJK_REGION_SINK | SJK_REGION_RING);
    uint32_t n_sink_d = 0, n_dense = 0;
    if (dense && !fused) {
        const uint32_t s_end = v->S < N ? v->S : N, t0 = B > v->S ? B : v->S;
        n_sink_d = (regions & SJK_REGION_SINK) ? (s_end + 127u) / 128u : 0u;
        n_dense = n_sink_d + ((regions & SJK_REGION_RING) && N > t0 ? (N - t0 + 127u) / 128u : 0u);
    }
    int cps_d = 1;
    const int splits_d = (dense && !fused) ? sjk_tc_dense_splits(n_dense, n_kv, &cps_d) : 0;
    const Plan pl = make_plan(v, B, N, n_kv, n_tc, dense, regions);
    const int splits_v1 = pl.n_chunks > 0 ? pl.splits : 0;
    // the tensor-core kernel's split count is known after its launch plan; bound it for the scratch check
    const int splits_tc_max = (tc_body && (n_tc > 0 || (fused && staged))) ? sjk_tc_body_max_splits(n_kv)
                              : (tc_trellis && n_tc > 0)      ? sjk_tc_trellis_max_splits(n_kv)
                                                              : 0;
    const size_t need = (size_t) (splits_tc_max + splits_d + splits_v1) * n_q * n_head * (v->lay.D + 2) * sizeof(float);
    if (!scratch || scratch_bytes < need) return SJKVARN_ERR_ARG;
    if (splits_tc_max + splits_d + splits_v1 > MERGE_SPLITS) return SJK_ERR_UNSUPPORTED;
    int splits_tc = 0;
    if (splits_tc_max) {
        const unsigned dense_regions = fused ? ((regions & SJK_REGION_SINK) ? 1u : 0u) | ((regions & SJK_REGION_RING) ? 2u : 0u) : 0u;
        const int rc = tc_body ? sjk_tc_body_launch(v, B, N, n_tc, (int) dense_regions, qpos0, n_q, n_head, kv_head0, n_kv, q, scale,
                                                    (float *) scratch, 0, &splits_tc, st)
                               : sjk_tc_trellis_launch(v, B, N, n_tc, qpos0, n_q, n_head, kv_head0, n_kv, q, scale,
                                                       (float *) scratch, 0, &splits_tc, st);
        if (rc) return rc;
    }
    const int splits = splits_tc + splits_d + splits_v1;
    // nothing to attend to: a zero output; an empty partial (m = -inf, l = 0, o = 0) comes from the merge kernel
    if (splits == 0 && !part_out) return sjk_check(cudaMemsetAsync(out, 0, (size_t) n_q * n_head * v->lay.D * sizeof(float), st));
    if (splits_d) {
        const int rc = sjk_tc_dense_launch(v, B, N, qpos0, n_q, n_head, kv_head0, n_kv, q, scale, (float *) scratch,
                                           splits_tc, splits_d, n_sink_d, n_dense, cps_d, st);
        if (rc) return rc;
    }
    AttnParams p;
    p.v = *v; p.kv0 = kv_head0; p.B = B; p.N = N; p.qpos0 = qpos0; p.n_q = n_q; p.n_head = n_head; p.grp = grp;
    p.rows = n_q * grp; p.q = q; p.scale = scale; p.part = (float *) scratch; p.split0 = splits_tc + splits_d;
    p.chunks_per_split = pl.chunks_per_split; p.n_chunks = pl.n_chunks; p.n_sink_chunks = pl.n_sink; p.n_body_chunks = pl.n_body;
    p.body_skip = n_tc;
    if (splits_v1) {
        const dim3 grid((unsigned) splits_v1, (unsigned) n_kv);
        cudaError_t e = cudaSuccess;
        switch (v->lay.D) {
            case 128: {
                const size_t sm = split_smem<128>();
                e = cudaFuncSetAttribute(attend_split_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) sm);
                if (e == cudaSuccess) attend_split_kernel<128><<<grid, NT, sm, st>>>(p);
                break;
            }
            case 256: {
                const size_t sm = split_smem<256>();
                e = cudaFuncSetAttribute(attend_split_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) sm);
                if (e == cudaSuccess) attend_split_kernel<256><<<grid, NT, sm, st>>>(p);
                break;
            }
            default: return SJK_ERR_UNSUPPORTED;
        }
        if (sjk_check(e)) return SJK_ERR_DEVICE;
        if (sjk_check_launch()) return SJK_ERR_DEVICE;
    }
    // programmatic dependent launch: the merge grid is set up while the partial kernels run and waits for them
    // on the device (griddepcontrol.wait), so the launch gap between the two kernels disappears
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) (n_q * n_head), (unsigned) ((v->lay.D + 63) / 64));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = (size_t) (splits + 256) * sizeof(float);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (sjk_check(cudaLaunchKernelEx(&cfg, attend_merge_kernel, (const float *) p.part, splits, n_q * n_head, v->lay.D, out, part_out)))
        return SJK_ERR_DEVICE;
    return sjk_check_launch();
}

// Attention over a subset of the regions, as one partial (m, l, o[D]) per (query row, query head). The
// partials of disjoint region sets, or of context slices held by different GPUs, combine with sjk_attend_merge.
extern "C" int sjk_attend_partial(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                                  unsigned regions, const float * q, float scale, float * part_out, void * scratch,
                                  size_t scratch_bytes, sjk_stream st) {
    if (!v || !part_out || (regions & ~(unsigned) SJK_REGION_ALL)) return SJKVARN_ERR_ARG;
    return sjk_attend_heads(v, B, N, qpos0, n_q, n_head, 0, v->n_head_kv, q, scale, nullptr, scratch, scratch_bytes, st,
                            regions, part_out);
}

// out[n_rows][D] from n_parts partial sets parts[n_parts][n_rows][D + 2], combined in index order
extern "C" int sjk_attend_merge(const float * parts, int n_parts, int n_rows, int D, float * out, sjk_stream st) {
    if (!parts || !out || n_parts <= 0 || n_rows <= 0 || D <= 0 || n_parts > MERGE_SPLITS) return SJKVARN_ERR_ARG;
    attend_merge_kernel<<<dim3((unsigned) n_rows, (unsigned) ((D + 63) / 64)), 256, (size_t) (n_parts + 256) * sizeof(float), st>>>(
        parts, n_parts, n_rows, D, out, nullptr);
    return sjk_check_launch();
}

// status words of every kernel with bounded waits: 1 if any wait ran out since the last call
extern "C" int sjk_device_status(void) {
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    const int a = sjk_tc_body_status_take(), b = sjk_tc_dense_status_take(), c = sjk_tc_trellis_status_take();
    if (a < 0 || b < 0 || c < 0) return -1;
    return a | b | c;
}

extern "C" int sjk_attend(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, const float * q,
                          float scale, float * out, void * scratch, size_t scratch_bytes, sjk_stream st) {
    if (!v) return SJKVARN_ERR_ARG;
    return sjk_attend_heads(v, B, N, qpos0, n_q, n_head, 0, v->n_head_kv, q, scale, out, scratch, scratch_bytes, st,
                            SJK_REGION_ALL, nullptr);
}

// ---- attention for callers that cannot allocate ------------------------------------------------------------
// sjk_attend_static: sjk_attend with its split-partial scratch in a fixed device array instead of a caller
// buffer. Capacity SJK_STATIC_SCRATCH_BYTES (16 MiB): every GPU that loads this library holds the array until
// the process exits. The array's host-side name is only a stand-in for its device address, so the address is
// looked up once per device (cudaGetSymbolAddress, with that device current) on the first call there and
// cached; that first call should therefore come before any stream capture. Shapes whose scratch bound
// (sjk_attend_scratch_bytes) exceeds the capacity are rejected with SJK_ERR_SCRATCH_LIMIT. Every call
// writes all the partials it later reads, so nothing needs clearing between calls; calls that overlap on
// the GPU (other streams, other host threads) share the array and race.
#define SJK_STATIC_SCRATCH_BYTES ((size_t) 16 << 20)
static __device__ __align__(256) unsigned char sjk_static_scratch[SJK_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_static_mu;
void * g_static_ptr[256];                    // device address of sjk_static_scratch, per device ordinal
}

extern "C" int sjk_attend_static(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                                 const float * q, float scale, float * out, sjk_stream st) {
    if (!v || n_q <= 0 || n_head <= 0) return SJKVARN_ERR_ARG;
    const size_t need = sjk_attend_scratch_bytes(v, N, n_q, n_head);
    if (need > SJK_STATIC_SCRATCH_BYTES) return SJK_ERR_SCRATCH_LIMIT;
    int dev = 0;
    if (sjk_check(cudaGetDevice(&dev))) return SJK_ERR_DEVICE;
    if (dev < 0 || dev >= 256) return SJK_ERR_UNSUPPORTED;
    void * ptr = NULL;
    {
        std::lock_guard<std::mutex> lk(g_static_mu);
        ptr = g_static_ptr[dev];
        if (!ptr) {
            if (sjk_check(cudaGetSymbolAddress(&ptr, sjk_static_scratch))) return SJK_ERR_DEVICE;
            g_static_ptr[dev] = ptr;
        }
    }
    return sjk_attend_heads(v, B, N, qpos0, n_q, n_head, 0, v->n_head_kv, q, scale, out, ptr, SJK_STATIC_SCRATCH_BYTES, st,
                            SJK_REGION_ALL, nullptr);
}
