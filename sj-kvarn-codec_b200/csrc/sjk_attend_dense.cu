// sjk_attend_dense.cu - tensor-core (tcgen05, kind::f16) attention over the staged rows of a layer: the
// staging ring [B, N) and the sink [0, S), in tq6_0 or fp16 form (sj_kvarn.h:1249-1284, 1516-1533).
//
// One CTA = one KV head x a contiguous range of 128-position chunks, 256 threads (8 warps, 2 CTAs per SM).
// A tq6_0 value is centroid[code] * norm, with one norm per (token, 128-channel block). The block structure
// puts the norm outside the MMA:
//
//   K side, block b   S_b^T[t, r] = sum_{d in b} cent[code_K(t, d)] * q[r, d];   dot = sum_b normK(t, b) S_b
//   V side, tile b    O_b^T[d, r] = sum_t cent[code_V(t, d)] * P'_b[r, t],       P'_b = p * normV(t, b)
//
// The centroids enter as exact fp16 hi + lo halves (a 64-entry table), q and P' as fp16 hi + lo halves
// (q with an exact power-of-two row rescale), and the products hi*hi + hi*lo + lo*hi accumulate in fp32
// (the dropped lo*lo term is below 2^-22 relative). fp16 rows (fp16 sink, fp16 staging) enter exactly
// with lo = 0. Rows of a chunk are staged in shared memory with coalesced loads; softmax is online per
// chunk; partials go to the same split buffer as the other attention kernels. Waits are bounded.
#include <cuda_fp16.h>

#include "sjk_common.cuh"
#include "sjk_internal.h"
#include "sjk_tc.cuh"

namespace {

using namespace tc::num;

constexpr int NT = 256;
constexpr int NR = 16;
constexpr int D = 256;
constexpr int CH = 128;
constexpr uint32_t TM_COLS = 256;
constexpr uint32_t COL_AH = 0, COL_AL = 64, COL_S = 128, COL_O = 160;   // A hi | A lo | S0 S1 | O0 O1

struct DenseParams {
    sjk_view v;
    int kv0;
    uint32_t B, N, qpos0;
    int n_q, n_head, grp, rows;
    const float * q;
    float scale;
    float * part;
    int split0;
    uint32_t n_sink_chunks, n_chunks;   // chunk list: sink chunks first, then ring chunks from B
    int chunks_per_split;
};

constexpr uint32_t STG_F16 = 528;       // staged fp16 row stride (512 B + 16: 16-byte rows, conflict-free LDS.128)
constexpr uint32_t STG_TQ6 = 2 * SJKVARN_TQ6_BLOCK_BYTES;      // 196 B = 49 words: conflict-free row walks
constexpr uint32_t OFF_BQ = 0;                                  // q hi [16][256] fp16, then lo
constexpr uint32_t OFF_BV = OFF_BQ + 2 * 8192;                  // P' tile0 hi, tile0 lo, tile1 hi, tile1 lo
constexpr uint32_t OFF_STG = OFF_BV + 4 * 4096;                 // 128 staged rows of one side
constexpr uint32_t OFF_CENT = OFF_STG + CH * STG_F16;           // u32[64]: fp16 hi | lo << 16 of each centroid
constexpr uint32_t OFF_RED = OFF_CENT + 64 * 4;                 // [2 quantities][64] floats
constexpr uint32_t OFF_ROW = OFF_RED + 2 * 64 * 4;              // per-row arrays
constexpr uint32_t OFF_NRM = OFF_ROW + 6 * 16 * 4;              // normK[2][128], normV[2][128]
constexpr uint32_t OFF_ROWP = OFF_NRM + 4 * CH * 4;             // global address of each token's K row
constexpr uint32_t OFF_BAR = OFF_ROWP + CH * 8;
constexpr uint32_t OFF_TMEM = OFF_BAR + 16;
constexpr uint32_t SMEM_TOTAL = OFF_TMEM + 16;
enum { ROW_QINV = 0, ROW_M2 = 16, ROW_MNEW = 32, ROW_ALPHA = 48, ROW_L = 64 };
enum { RED_MAX = 0, RED_L = 64 };

// fp16 K-major no-swizzle operand with 16 rows: element (row n, k) at (k/8)*256 + n*16 + (k%8)*2 bytes;
// an MMA's 16-element K step is 512 bytes (LBO 256, SBO 128)
__device__ __forceinline__ uint32_t h_off(int n, int k) { return (uint32_t) ((k >> 3) * 256 + n * 16 + (k & 7) * 2); }

__device__ __forceinline__ uint32_t f2h_bits(float v) { return (uint32_t) __half_as_ushort(__float2half_rn(v)); }

__global__ void __launch_bounds__(NT, 2) attend_dense_tc_kernel(DenseParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int quarter = warp & 3, half = warp >> 2, tl = quarter * 32 + lane;
    const int hl = blockIdx.y, h = p.kv0 + hl, split = blockIdx.x;
    const sjk_view & v = p.v;
    const int H = v.n_head_kv;
    uint8_t * bq = sm + OFF_BQ;
    uint8_t * bvp = sm + OFF_BV;
    uint8_t * stg = sm + OFF_STG;
    uint32_t * cent2 = reinterpret_cast<uint32_t *>(sm + OFF_CENT);
    float * red = reinterpret_cast<float *>(sm + OFF_RED);
    float * row = reinterpret_cast<float *>(sm + OFF_ROW);
    float * nrm = reinterpret_cast<float *>(sm + OFF_NRM);           // [0,256): normK b*128+t; [256,512): normV
    const uint8_t ** rowp = reinterpret_cast<const uint8_t **>(sm + OFF_ROWP);
    uint64_t * bar = reinterpret_cast<uint64_t *>(sm + OFF_BAR);
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(sm + OFF_TMEM);

    const uint32_t c_begin = (uint32_t) split * (uint32_t) p.chunks_per_split;
    const uint32_t c_end = min(c_begin + (uint32_t) p.chunks_per_split, p.n_chunks);

    if (warp == 0) { tc::tmem_alloc(tmem_slot, TM_COLS); tc::tmem_relinquish(); }
    if (tid == 0) { tc::mbar_init(bar, 1); tc::mbar_fence_init(); }
    if (tid < 64) {
        const float c = sjk_tq6_cent[tid];
        const uint32_t hi = f2h_bits(c);
        const uint32_t lo = f2h_bits(c - __half2float(__ushort_as_half((unsigned short) hi)));
        cent2[tid] = hi | (lo << 16);
    }
    if (tid < NR) { row[ROW_M2 + tid] = -INFINITY; row[ROW_L + tid] = 0.0f; }
    // ---- B_Q: q rows (rotated) as fp16 hi + lo, each row rescaled by a power of two to max |q| < 2^13 ----
    {
        const int d = tid;                               // one channel per thread, all 16 rows
        float qv[NR];
        float qm = 0.0f;
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            float x = 0.0f;
            if (r < p.rows) {
                const int iq = r / p.grp, hq = hl * p.grp + r % p.grp;
                x = p.q[((size_t) iq * p.n_head + hq) * D + d];
            }
            qv[r] = x;
        }
        // row maxima across the 256 threads
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            float m = fabsf(qv[r]);
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
            if (lane == 0) red[warp * NR + r] = m;      // 8 warps x 16 rows = 128 floats (both red areas)
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            qm = 0.0f;
            for (int w = 0; w < 8; ++w) qm = fmaxf(qm, red[w * NR + r]);
            const int e = (qm > 0.0f && qm < INFINITY) ? 13 - pow2_exp(qm) : 0;
            const float x = qv[r] * pow2f(e);
            const uint32_t hi = f2h_bits(x);
            const uint32_t lo = f2h_bits(x - __half2float(__ushort_as_half((unsigned short) hi)));
            const uint32_t off = h_off(r, d);
            *reinterpret_cast<uint16_t *>(bq + off) = (uint16_t) hi;
            *reinterpret_cast<uint16_t *>(bq + 8192 + off) = (uint16_t) lo;
            if (d == 0) row[ROW_QINV + r] = pow2f(-e);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t) (quarter * 32) << 16;
    const uint32_t idesc = tc::idesc_f16(128, NR);
    const float sl2 = p.scale * LOG2E;
    uint32_t qlim[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = 8 * half + i;
        qlim[i] = r < p.rows ? p.qpos0 + (uint32_t) (r / p.grp) + 1u : 0u;
    }
    float acc[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
    bool ok = true;
    uint32_t mma_phase = 0;
    bool mma_pending = false;
    const uint32_t S_eff = v.S < p.N ? v.S : p.N;
    const uint32_t t0_ring = p.B > v.S ? p.B : v.S;

    for (uint32_t ci = c_begin; ci < c_end && ok; ++ci) {
        // ---- chunk geometry and row kind ----
        const bool in_sink = ci < p.n_sink_chunks;
        const uint32_t p0 = in_sink ? ci * (uint32_t) CH : t0_ring + (ci - p.n_sink_chunks) * (uint32_t) CH;
        const uint32_t len = min((uint32_t) CH, (in_sink ? S_eff : p.N) - p0);
        // f16 rows: the fp16 sink, or an fp16 staging ring / inherited sink; otherwise tq6_0 rows
        const bool f16 = (in_sink && v.sink_type == SJKVARN_SINK_F16) || v.staging == SJKVARN_STAGING_F16;
        const uint32_t side_off = (in_sink && v.sink_type == SJKVARN_SINK_F16) ? 2u * D : (uint32_t) v.stage_bytes;
        const uint32_t sstride = f16 ? STG_F16 : STG_TQ6;
        // global K row of each token (the V row follows at side_off); one ring-slot division per token
        if (tid < CH) {
            const uint32_t pos = p0 + (uint32_t) min(tid, (int) len - 1);
            const uint8_t * r;
            if (in_sink && v.sink_type == SJKVARN_SINK_F16) r = v.sink + ((size_t) pos * H + h) * 4 * D;
            else if (in_sink) r = v.sink + ((size_t) pos * H + h) * 2 * v.stage_bytes;
            else r = v.ring + ((size_t) sjk_ring_slot(v.S, v.cap, pos) * H + h) * 2 * v.stage_bytes;
            rowp[tid] = r;
        }
        __syncthreads();
        // stage the chunk's rows of one side (asynchronous copies; zeros past len)
        auto stage = [&](int side) {
            const uint32_t so = side ? side_off : 0u;
            if (f16) {
#pragma unroll 4
                for (int i = tid; i < CH * 32; i += NT) {
                    const int t = i >> 5, u = i & 31;
                    tc::cp_async16(stg + t * STG_F16 + 16 * u, rowp[t] + so + 16 * u, (uint32_t) t < len ? 16u : 0u);
                }
            } else {
#pragma unroll 4
                for (int i = tid; i < CH * 49; i += NT) {
                    const int t = i / 49, u = i - 49 * t;
                    tc::cp_async4(stg + t * STG_TQ6 + 4 * u, rowp[t] + so + 4 * u, (uint32_t) t < len ? 4u : 0u);
                }
            }
        };
        stage(0);
        tc::cp_async_wait_all();
        __syncthreads();
        if (tid < CH) {
            const uint8_t * r0 = stg + tid * sstride;
            nrm[tid] = f16 ? 1.0f : h2f(*reinterpret_cast<const uint16_t *>(r0));
            nrm[CH + tid] = f16 ? 1.0f : h2f(*reinterpret_cast<const uint16_t *>(r0 + SJKVARN_TQ6_BLOCK_BYTES));
        }
        // ---- K side: block by block, A (token tl, 64 channels of this half) -> TMEM, then 24 MMAs ----
        for (int b = 0; b < 2; ++b) {
            {
                uint32_t ch[32], cl[32];
                const uint8_t * r0 = stg + tl * sstride;
                if (f16) {
                    const uint4 * src = reinterpret_cast<const uint4 *>(r0 + 2 * (128 * b + 64 * half));
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const uint4 x = src[c];
                        ch[4 * c] = x.x; ch[4 * c + 1] = x.y; ch[4 * c + 2] = x.z; ch[4 * c + 3] = x.w;
                    }
#pragma unroll
                    for (int c = 0; c < 32; ++c) cl[c] = 0u;
                } else {
                    const uint8_t * blk = r0 + SJKVARN_TQ6_BLOCK_BYTES * b;
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        const int j0 = 64 * half + 8 * g;
                        const uint32_t qs = (uint32_t) *reinterpret_cast<const uint16_t *>(blk + 2 + j0 / 2) |
                                            ((uint32_t) *reinterpret_cast<const uint16_t *>(blk + 4 + j0 / 2) << 16);
                        const uint32_t qh = *reinterpret_cast<const uint16_t *>(blk + 66 + j0 / 4);
#pragma unroll
                        for (int pp = 0; pp < 4; ++pp) {
                            const int i0 = 2 * pp, i1 = 2 * pp + 1;
                            const uint32_t e0 = cent2[((qs >> (4 * i0)) & 15u) | (((qh >> (2 * i0)) & 3u) << 4)];
                            const uint32_t e1 = cent2[((qs >> (4 * i1)) & 15u) | (((qh >> (2 * i1)) & 3u) << 4)];
                            ch[4 * g + pp] = prmt(e0, e1, 0x5410u);
                            cl[4 * g + pp] = prmt(e0, e1, 0x7632u);
                        }
                    }
                }
                tc::st_x16(tmem + lane_base + COL_AH + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(ch));
                tc::st_x16(tmem + lane_base + COL_AH + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(ch + 16));
                tc::st_x16(tmem + lane_base + COL_AL + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(cl));
                tc::st_x16(tmem + lane_base + COL_AL + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(cl + 16));
            }
            tc::wait_st();
            tc::fence_proxy_async();
            tc::fence_before_sync();
            __syncthreads();
            tc::fence_after_sync();
            if (tid == 0) {
#pragma unroll 1
                for (int k = 0; k < 8; ++k) {
                    const int kq = 8 * b + k;
                    const uint32_t a_hi = tmem + COL_AH + 8 * k, a_lo = tmem + COL_AL + 8 * k;
                    tc::mma_ts(tmem + COL_S + 16 * b, a_hi, tc::smem_desc(bq + 512 * kq, 256, 128), idesc, k ? 1u : 0u);
                    tc::mma_ts(tmem + COL_S + 16 * b, a_hi, tc::smem_desc(bq + 8192 + 512 * kq, 256, 128), idesc, 1u);
                    if (!f16) tc::mma_ts(tmem + COL_S + 16 * b, a_lo, tc::smem_desc(bq + 512 * kq, 256, 128), idesc, 1u);
                }
                tc::mma_commit(bar);
            }
            mma_pending = true;
            if (b == 1) stage(1);                         // V rows replace K rows in the staging buffer meanwhile
            const bool got = tc::mbar_wait(bar, mma_phase);
            if (b == 1) tc::cp_async_wait_all();
            ok = __syncthreads_and(got);
            if (!ok) break;
            mma_phase ^= 1u;
            mma_pending = false;
            tc::fence_after_sync();
        }
        if (!ok) break;
        if (tid < CH) {
            const uint8_t * r0 = stg + tid * sstride;
            nrm[2 * CH + tid] = f16 ? 1.0f : h2f(*reinterpret_cast<const uint16_t *>(r0));
            nrm[3 * CH + tid] = f16 ? 1.0f : h2f(*reinterpret_cast<const uint16_t *>(r0 + SJKVARN_TQ6_BLOCK_BYTES));
        }
        // ---- scores of token tl, rows 8 half .. 8 half + 7 (log2 domain), row maxima ----
        float s2[8];
        {
            float a0[8], a1[8];
            uint32_t u0[8], u1[8];
            tc::ld_x8_u(tmem + lane_base + COL_S + 8 * half, u0);
            tc::ld_x8_u(tmem + lane_base + COL_S + 16 + 8 * half, u1);
            tc::wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i) { a0[i] = __uint_as_float(u0[i]); a1[i] = __uint_as_float(u1[i]); }
            const float nk0 = nrm[tl], nk1 = nrm[CH + tl];
            const uint32_t pos = p0 + (uint32_t) tl;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = 8 * half + i;
                const float dot = (nk0 * a0[i] + nk1 * a1[i]) * row[ROW_QINV + r];
                s2[i] = ((uint32_t) tl < len && pos < qlim[i]) ? dot * sl2 : -INFINITY;
            }
            const float mw = warp_rows8<true>(s2, lane);
            if ((lane & 3) == 0) red[RED_MAX + half * 32 + quarter * 8 + (lane >> 2)] = mw;
        }
        __syncthreads();
        if (tid < NR) {
            const int hh = tid >> 3, rr = tid & 7;
            const float * mr = red + RED_MAX + hh * 32 + rr;
            const float mrec = fmaxf(fmaxf(mr[0], mr[8]), fmaxf(mr[16], mr[24]));
            const float mold = row[ROW_M2 + tid], mnew = fmaxf(mold, mrec);
            row[ROW_MNEW + tid] = mnew;
            row[ROW_ALPHA + tid] = mnew == -INFINITY ? 1.0f : ex2(mold - mnew);
            row[ROW_M2 + tid] = mnew;
        }
        __syncthreads();
        // ---- P'_b = p * normV(t, b) as fp16 hi + lo (B of the V MMAs), row sums ----
        {
            const float nv0 = nrm[2 * CH + tl], nv1 = nrm[3 * CH + tl];
            float ls[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = 8 * half + i;
                const float mnew = row[ROW_MNEW + r];
                const float pw = mnew == -INFINITY ? 0.0f : ex2(s2[i] - mnew);
                ls[i] = pw;
                const uint32_t off = h_off(r, tl);
                const float x0 = pw * nv0, x1 = pw * nv1;
                const uint32_t h0 = f2h_bits(x0), h1 = f2h_bits(x1);
                *reinterpret_cast<uint16_t *>(bvp + off) = (uint16_t) h0;
                *reinterpret_cast<uint16_t *>(bvp + 4096 + off) = (uint16_t) f2h_bits(x0 - __half2float(__ushort_as_half((unsigned short) h0)));
                *reinterpret_cast<uint16_t *>(bvp + 8192 + off) = (uint16_t) h1;
                *reinterpret_cast<uint16_t *>(bvp + 12288 + off) = (uint16_t) f2h_bits(x1 - __half2float(__ushort_as_half((unsigned short) h1)));
            }
            const float lw = warp_rows8<false>(ls, lane);
            if ((lane & 3) == 0) red[RED_L + half * 32 + quarter * 8 + (lane >> 2)] = lw;
        }
        // ---- V side: tile by tile, A (channel 128 b + tl, 64 tokens of this half) -> TMEM, then 24 MMAs ----
        for (int b = 0; b < 2; ++b) {
            {
                uint32_t ch[32], cl[32];
                const int d = 128 * b + tl;
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const int t0 = 64 * half + 2 * c;
                    const uint8_t * ra = stg + t0 * sstride, * rb = ra + sstride;
                    if (f16) {
                        const uint32_t x0 = *reinterpret_cast<const uint16_t *>(ra + 2 * d);
                        const uint32_t x1 = *reinterpret_cast<const uint16_t *>(rb + 2 * d);
                        ch[c] = x0 | (x1 << 16);
                        cl[c] = 0u;
                    } else {
                        const int j = d & 127;
                        const uint8_t * ba = ra + SJKVARN_TQ6_BLOCK_BYTES * b, * bb = rb + SJKVARN_TQ6_BLOCK_BYTES * b;
                        const uint32_t c0 = ((ba[2 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((ba[66 + (j >> 2)] >> (2 * (j & 3))) & 3) << 4);
                        const uint32_t c1 = ((bb[2 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((bb[66 + (j >> 2)] >> (2 * (j & 3))) & 3) << 4);
                        const uint32_t e0 = cent2[c0], e1 = cent2[c1];
                        ch[c] = prmt(e0, e1, 0x5410u);
                        cl[c] = prmt(e0, e1, 0x7632u);
                    }
                }
                tc::st_x16(tmem + lane_base + COL_AH + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(ch));
                tc::st_x16(tmem + lane_base + COL_AH + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(ch + 16));
                tc::st_x16(tmem + lane_base + COL_AL + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(cl));
                tc::st_x16(tmem + lane_base + COL_AL + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(cl + 16));
            }
            tc::wait_st();
            tc::fence_proxy_async();
            tc::fence_before_sync();
            __syncthreads();
            tc::fence_after_sync();
            if (tid == 0) {
                const uint8_t * bhi = bvp + 8192 * b, * blo = bhi + 4096;
#pragma unroll 1
                for (int k = 0; k < 8; ++k) {
                    const uint32_t a_hi = tmem + COL_AH + 8 * k, a_lo = tmem + COL_AL + 8 * k;
                    tc::mma_ts(tmem + COL_O + 16 * b, a_hi, tc::smem_desc(bhi + 512 * k, 256, 128), idesc, k ? 1u : 0u);
                    tc::mma_ts(tmem + COL_O + 16 * b, a_hi, tc::smem_desc(blo + 512 * k, 256, 128), idesc, 1u);
                    if (!f16) tc::mma_ts(tmem + COL_O + 16 * b, a_lo, tc::smem_desc(bhi + 512 * k, 256, 128), idesc, 1u);
                }
                tc::mma_commit(bar);
            }
            mma_pending = true;
            if (b == 0 && tid < NR) {
                const int hh = tid >> 3, rr = tid & 7;
                const float * lr = red + RED_L + hh * 32 + rr;
                row[ROW_L + tid] = row[ROW_L + tid] * row[ROW_ALPHA + tid] + ((lr[0] + lr[8]) + (lr[16] + lr[24]));
            }
            ok = __syncthreads_and(tc::mbar_wait(bar, mma_phase));
            if (!ok) break;
            mma_phase ^= 1u;
            mma_pending = false;
            tc::fence_after_sync();
        }
        if (!ok) break;
        // ---- epilogue: channel 128 half + tl ----
        {
            float o[16];
            tc::ld_x16(tmem + lane_base + COL_O + 16 * half, o);
            tc::wait_ld();
#pragma unroll
            for (int r = 0; r < NR; ++r) acc[r] = fmaf(acc[r], row[ROW_ALPHA + r], o[r]);
        }
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
    }
    if (!ok && mma_pending) tc::mbar_wait(bar, mma_phase);
    __syncthreads();
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        if (r < p.rows) {
            const int iq = r / p.grp, hq = hl * p.grp + r % p.grp;
            float * dst = p.part + ((size_t) (p.split0 + split) * p.n_q * p.n_head + (size_t) iq * p.n_head + hq) * (D + 2);
            if (tid == 0) {
                const float m2 = row[ROW_M2 + r];
                dst[0] = ok ? (m2 == -INFINITY ? m2 : m2 * LN2) : -INFINITY;
                dst[1] = ok ? row[ROW_L + r] : 0.0f;
            }
            dst[2 + 128 * half + tl] = ok ? acc[r] : 0.0f;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace

// Whether the dense tensor-core path applies to the staged regions: D = 256, <= 16 query rows per KV head.
int sjk_tc_dense_supported(const sjk_view * v, int n_q, int grp) {
    return v->lay.D == D && n_q * grp <= NR && v->stage_bytes == (v->staging == SJKVARN_STAGING_F16 ? 512u : 196u);
}

int sjk_tc_dense_splits(uint32_t n_chunks, int n_kv, int * chunks_per_split) {
    if (n_chunks == 0) { *chunks_per_split = 1; return 0; }
    const int target = (2 * 148 + n_kv - 1) / n_kv;
    int cps = (int) ((n_chunks + (uint32_t) target - 1) / (uint32_t) target);
    if (cps < 1) cps = 1;
    *chunks_per_split = cps;
    return (int) ((n_chunks + (uint32_t) cps - 1) / (uint32_t) cps);
}

int sjk_tc_dense_launch(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, int kv0, int n_kv,
                        const float * q, float scale, float * part, int split0, int splits, uint32_t n_sink_chunks,
                        uint32_t n_chunks, int chunks_per_split, sjk_stream st) {
    DenseParams p;
    p.v = *v; p.kv0 = kv0; p.B = B; p.N = N; p.qpos0 = qpos0; p.n_q = n_q; p.n_head = n_head; p.grp = n_head / n_kv;
    p.rows = n_q * p.grp; p.q = q; p.scale = scale; p.part = part; p.split0 = split0;
    p.n_sink_chunks = n_sink_chunks; p.n_chunks = n_chunks; p.chunks_per_split = chunks_per_split;
    cudaError_t e = cudaFuncSetAttribute(attend_dense_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_TOTAL);
    if (e != cudaSuccess) return sjk_check(e);
    attend_dense_tc_kernel<<<dim3((unsigned) splits, (unsigned) n_kv), NT, SMEM_TOTAL, st>>>(p);
    return sjk_check_launch();
}

SJK_STATUS_READER(sjk_tc_dense_status_take)
