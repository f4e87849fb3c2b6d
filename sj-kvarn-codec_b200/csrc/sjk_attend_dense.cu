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
// The centroids enter as fp16 hi + lo halves (a 64-entry table), q and P' as fp16 hi + lo halves side by
// side in the MMA's N dimension (B = [hi | lo], N = 32). Two MMAs per k step, A_hi x [hi | lo] and
// A_lo x hi, accumulate hi*hi + lo*hi in columns 0..15 and hi*lo in columns 16..31 (the dropped lo*lo
// term is below 2^-22 relative); the result is the sum of the two column groups. fp16 rows (fp16 sink,
// fp16 staging) enter exactly with lo = 0 and skip the second MMA. Rows of a chunk are staged in shared
// memory with asynchronous copies (tq6_0: K and V rows at once); softmax is online per chunk; partials go to
// the same split buffer as the other attention kernels. Waits are bounded.
#include <cuda_fp16.h>

#include "sjk_common.cuh"
#include "sjk_internal.h"
#include "sjk_plan.cuh"
#include "sjk_tc.cuh"

namespace {

using namespace tc::num;

constexpr int NT = 256;
constexpr int NR = 16;
constexpr int NB = 2 * NR;              // B operands: hi rows 0..15, lo rows 16..31
constexpr int D = 256;
constexpr int CH = 128;
constexpr uint32_t TM_COLS = 256;
constexpr uint32_t COL_AH = 0, COL_AL = 64, COL_S = 128, COL_O = 192;   // A hi | A lo | S0 S1 (2 x 32) | O0 O1

constexpr int MAX_SEQS = 128;
constexpr int MAX_ITEMS = 768;

struct DenseSeq {                       // one sequence of the call
    const uint8_t * sink;
    const uint8_t * ring;
    const float * q;                    // [n_q][n_head][D] rotated queries
    uint32_t B, N, qpos0;
    uint32_t n_sink_chunks;             // chunk list: sink chunks first, then ring chunks from max(B, S)
};
struct DenseItem {                      // chunks [c0, c1) of KV head h of sequence seq, partial slot `slot`
    uint32_t seq_hl;                    // seq | hl << 16 (hl: head index inside q and the partial rows)
    uint32_t h_slot;                    // h | slot << 16
    uint32_t c0, c1;
};
struct DenseParams {
    sjk_view v;                         // layout, staging formats, S, cap (the per-sequence pointers are in seq[])
    int n_q, n_head, grp, rows;
    float scale;
    float * part;                       // [slots][n_q n_head][D + 2]
    int n_items;                        // CTAs with an item (the descriptor-driven grid may be larger)
    DenseSeq seq[MAX_SEQS];
    DenseItem item[MAX_ITEMS];          // one per CTA
};

// B operand (K-major, no swizzle, 32 rows): element (n, k) at (k / 8) * HCH + n * 16 + (k % 8) * 2 with an 8-element
// K chunk every HCH = 528 bytes (512 + 16: consecutive chunks start 4 banks apart, so the builders' stores are
// conflict-free); one MMA k step (16 elements) is two chunks (LBO = HCH, SBO 128 between 8-row groups)
constexpr uint32_t HCH = 528;
__device__ __forceinline__ uint32_t h_off(int n, int k) { return (uint32_t) (k >> 3) * HCH + (uint32_t) (n * 16 + (k & 7) * 2); }

constexpr uint32_t STG_F16 = 528;       // staged fp16 row stride (512 B + 16: 16-byte rows, conflict-free LDS.128)
constexpr uint32_t TQ6_ROW = 2 * SJKVARN_TQ6_BLOCK_BYTES;      // 196 B: one K or V row of tq6_0 blocks
constexpr uint32_t STG_TQ6 = 2 * TQ6_ROW;                       // staged K row + V row of a token (392 B = 49 x 8)
constexpr uint32_t TILE_B = 16 * HCH;                          // one B operand over 128 k (8 k steps)
constexpr uint32_t OFF_BQ = 0;                                  // [q hi | q lo] for 256 channels: 2 x TILE_B
constexpr uint32_t OFF_BV = OFF_BQ + 2 * TILE_B;                // [P' hi | P' lo] per tile: 2 x TILE_B
constexpr uint32_t OFF_STG = OFF_BV + 2 * TILE_B;               // staged rows: fp16 one side, tq6_0 both sides
constexpr uint32_t OFF_CENT = OFF_STG + CH * STG_F16;           // u32[64]: fp16 hi | lo << 16 of each centroid
constexpr uint32_t OFF_RED = OFF_CENT + 64 * 4;                 // [2 quantities][64] floats
constexpr uint32_t OFF_ROW = OFF_RED + 2 * 64 * 4;              // per-row arrays
constexpr uint32_t OFF_NRM = OFF_ROW + 6 * 16 * 4;              // normK[2][128], normV[2][128]
constexpr uint32_t OFF_ROWP = OFF_NRM + 4 * CH * 4;             // global address of each token's K row
constexpr uint32_t OFF_BAR = OFF_ROWP + CH * 8;
constexpr uint32_t OFF_TMEM = OFF_BAR + 16;
constexpr uint32_t SMEM_TOTAL = OFF_TMEM + 16;
static_assert(CH * STG_TQ6 <= CH * STG_F16, "staging area holds both tq6_0 sides");
enum { ROW_M2 = 16, ROW_MNEW = 32, ROW_ALPHA = 48, ROW_L = 64 };
enum { RED_MAX = 0, RED_L = 64 };

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {    // fp16 pair, a in the low half
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ float2 unpack_h2(uint32_t w) {
    const __half2 h = *reinterpret_cast<const __half2 *>(&w);
    return __half22float2(h);
}

SJK_DEV void dense_body(const DenseParams & p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int quarter = warp & 3, half = warp >> 2, tl = quarter * 32 + lane;
    const DenseItem & item = p.item[blockIdx.x];
    const DenseSeq & sq = p.seq[item.seq_hl & 0xFFFFu];
    const int hl = (int) (item.seq_hl >> 16), h = (int) (item.h_slot & 0xFFFFu), slot = (int) (item.h_slot >> 16);
    const sjk_view & v = p.v;
    const int H = v.n_head_kv;
    uint8_t * bq = sm + OFF_BQ;
    uint8_t * bvp = sm + OFF_BV;
    uint8_t * stg = sm + OFF_STG;
    uint32_t * cent2 = reinterpret_cast<uint32_t *>(sm + OFF_CENT);
    float * red = reinterpret_cast<float *>(sm + OFF_RED);
    float * row = reinterpret_cast<float *>(sm + OFF_ROW);
    float * nrm = reinterpret_cast<float *>(sm + OFF_NRM);           // normK b*128+t, then normV at 256 + b*128+t
    const uint8_t ** rowp = reinterpret_cast<const uint8_t **>(sm + OFF_ROWP);
    uint64_t * bar = reinterpret_cast<uint64_t *>(sm + OFF_BAR);
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(sm + OFF_TMEM);

    const uint32_t c_begin = item.c0, c_end = item.c1;

    if (warp == 0) { tc::tmem_alloc(tmem_slot, TM_COLS); tc::tmem_relinquish(); }
    if (tid == 0) { tc::mbar_init(bar, 1); tc::mbar_fence_init(); }
    if (tid < 64) {
        const float c = sjk_tq6_cent[tid];
        const __half hi = __float2half_rn(c);
        cent2[tid] = pack_h2(__half2float(hi), c - __half2float(hi));
    }
    if (tid < NR) { row[ROW_M2 + tid] = -INFINITY; row[ROW_L + tid] = 0.0f; }
    const uint32_t S_eff = v.S < sq.N ? v.S : sq.N;
    const uint32_t t0_ring = sq.B > v.S ? sq.B : v.S;
    const uint32_t idesc32 = tc::idesc_f16(128, NB), idesc16 = tc::idesc_f16(128, NR);
    const float sl2 = p.scale * LOG2E;
    uint32_t qlim[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = 8 * half + i;
        qlim[i] = r < p.rows ? sq.qpos0 + (uint32_t) (r / p.grp) + 1u : 0u;
    }
    float acc[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
    bool ok = true;
    uint32_t mma_phase = 0;
    bool mma_pending = false, bq_done = false;
    uint32_t tmem = 0;
    const uint32_t lane_base = (uint32_t) (quarter * 32) << 16;
    // issue the MMAs of one side (thread 0): D (32 columns) += A_hi x B[hi | lo] (+ A_lo x B_hi), 8 k steps
    auto mma_side = [&](uint32_t d_col, const uint8_t * b_base, bool f16) {
        const uint64_t db = tc::smem_desc(b_base, HCH, 128);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            tc::mma_ts(tmem + d_col, tmem + COL_AH + 8 * k, db + (uint64_t) ((2 * HCH * k) >> 4), idesc32, k ? 1u : 0u);
            if (!f16) tc::mma_ts(tmem + d_col, tmem + COL_AL + 8 * k, db + (uint64_t) ((2 * HCH * k) >> 4), idesc16, 1u);
        }
        tc::mma_commit(bar);
    };
    // all threads: A stores visible to the MMA, thread 0 issues, everyone waits for the commit (bounded)
    auto run_mma = [&](uint32_t d_col, const uint8_t * b_base, bool f16) -> bool {
        tc::wait_st();
        tc::fence_proxy_async();
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        if (tid == 0) mma_side(d_col, b_base, f16);
        mma_pending = true;
        const bool got = __syncthreads_and(tc::mbar_wait(bar, mma_phase));
        if (got) { mma_phase ^= 1u; mma_pending = false; }
        tc::fence_after_sync();
        return got;
    };

    for (uint32_t ci = c_begin; ci < c_end && ok; ++ci) {
        // ---- chunk geometry and row kind ----
        const bool in_sink = ci < sq.n_sink_chunks;
        const uint32_t p0 = in_sink ? ci * (uint32_t) CH : t0_ring + (ci - sq.n_sink_chunks) * (uint32_t) CH;
        const uint32_t len = min((uint32_t) CH, (in_sink ? S_eff : sq.N) - p0);
        // f16 rows: the fp16 sink, or an fp16 staging ring / inherited sink; otherwise tq6_0 rows
        const bool f16 = (in_sink && v.sink_type == SJKVARN_SINK_F16) || v.staging == SJKVARN_STAGING_F16;
        const uint32_t side_off = (in_sink && v.sink_type == SJKVARN_SINK_F16) ? 2u * D : (uint32_t) v.stage_bytes;
        const uint32_t sstride = f16 ? STG_F16 : STG_TQ6;
        // global K row of each token (the V row follows at side_off); one ring-slot division per token
        if (tid < CH) {
            const uint32_t pos = p0 + (uint32_t) min(tid, (int) len - 1);
            const uint8_t * r;
            if (in_sink && v.sink_type == SJKVARN_SINK_F16) r = sq.sink + ((size_t) pos * H + h) * 4 * D;
            else if (in_sink) r = sq.sink + ((size_t) pos * H + h) * 2 * v.stage_bytes;
            else r = sq.ring + ((size_t) sjk_ring_slot(v.S, v.cap, pos) * H + h) * 2 * v.stage_bytes;
            rowp[tid] = r;
        }
        __syncthreads();
        // stage the chunk's rows (asynchronous copies, zeros past len), one warp per token: tq6_0 K and V rows
        // together (392 contiguous bytes, 49 x 8 bytes); fp16 rows one side at a time (512 bytes, 32 x 16)
        auto stage = [&](int side) {
            if (f16) {
                const uint32_t so = side ? side_off : 0u;
#pragma unroll 4
                for (int t = warp; t < CH; t += NT / 32)
                    tc::cp_async16(stg + t * STG_F16 + 16 * lane, rowp[t] + so + 16 * lane, (uint32_t) t < len ? 16u : 0u);
            } else {
#pragma unroll 4
                for (int t = warp; t < CH; t += NT / 32) {
                    const uint8_t * src = rowp[t];
                    const uint32_t n = (uint32_t) t < len ? 8u : 0u;
                    tc::cp_async8(stg + t * STG_TQ6 + 8 * lane, src + 8 * lane, n);
                    if (lane < 17) tc::cp_async8(stg + t * STG_TQ6 + 256 + 8 * lane, src + 256 + 8 * lane, n);
                }
            }
        };
        stage(0);
        if (!bq_done) {
            // ---- B_Q = [q hi | q lo] (rotated rows), built while the first chunk's rows stream in ----
            const int d = tid;
            const float * __restrict__ qg = sq.q;
            float x[NR];                                         // all loads first: the stores below are shared
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const int rr = r < p.rows ? r : 0;
                const int iq = rr / p.grp, hq = hl * p.grp + rr % p.grp;
                x[r] = __ldg(qg + ((size_t) iq * p.n_head + hq) * D + d);
            }
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const float xr = r < p.rows ? x[r] : 0.0f;
                const __half hi = __float2half_rn(xr);
                *reinterpret_cast<__half *>(bq + h_off(r, d)) = hi;
                *reinterpret_cast<__half *>(bq + h_off(NR + r, d)) = __float2half_rn(xr - __half2float(hi));
            }
            bq_done = true;
        }
        tc::cp_async_wait_all();
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        tmem = *tmem_slot;
        if (tid < CH) {
            const uint8_t * r0 = stg + tid * sstride;
            nrm[tid] = f16 ? 1.0f : h2f(*reinterpret_cast<const uint16_t *>(r0));
            nrm[CH + tid] = f16 ? 1.0f : h2f(*reinterpret_cast<const uint16_t *>(r0 + SJKVARN_TQ6_BLOCK_BYTES));
            if (!f16) {
                const uint8_t * v0 = stg + tid * STG_TQ6 + TQ6_ROW;
                nrm[2 * CH + tid] = h2f(*reinterpret_cast<const uint16_t *>(v0));
                nrm[3 * CH + tid] = h2f(*reinterpret_cast<const uint16_t *>(v0 + SJKVARN_TQ6_BLOCK_BYTES));
            }
        }
        // ---- K side, block by block: A (token tl, channels 128 b + 64 half ..) -> TMEM, then the MMAs ----
        for (int b = 0; b < 2 && ok; ++b) {
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
                } else {
                    const uint8_t * blk = r0 + SJKVARN_TQ6_BLOCK_BYTES * b;
#pragma unroll
                    for (int g = 0; g < 8; ++g) {
                        const int j0 = 64 * half + 8 * g;                  // elements j0 .. j0 + 7 of the block
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
                    tc::st_x16(tmem + lane_base + COL_AL + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(cl));
                    tc::st_x16(tmem + lane_base + COL_AL + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(cl + 16));
                }
                tc::st_x16(tmem + lane_base + COL_AH + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(ch));
                tc::st_x16(tmem + lane_base + COL_AH + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(ch + 16));
            }
            ok = run_mma(COL_S + 32 * b, bq + TILE_B * b, f16);
        }
        if (!ok) break;
        // ---- scores of token tl, rows 8 half .. 8 half + 7 (log2 domain), row maxima ----
        float s2[8];
        {
            uint32_t a0[8], a0l[8], a1[8], a1l[8];
            tc::ld_x8_u(tmem + lane_base + COL_S + 8 * half, a0);
            tc::ld_x8_u(tmem + lane_base + COL_S + 16 + 8 * half, a0l);
            tc::ld_x8_u(tmem + lane_base + COL_S + 32 + 8 * half, a1);
            tc::ld_x8_u(tmem + lane_base + COL_S + 48 + 8 * half, a1l);
            tc::wait_ld();
            const float nk0 = nrm[tl] * sl2, nk1 = nrm[CH + tl] * sl2;
            const uint32_t pos = p0 + (uint32_t) tl;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float dot = nk0 * (__uint_as_float(a0[i]) + __uint_as_float(a0l[i])) +
                                  nk1 * (__uint_as_float(a1[i]) + __uint_as_float(a1l[i]));
                s2[i] = ((uint32_t) tl < len && pos < qlim[i]) ? dot : -INFINITY;
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
        // fp16 rows: the V rows replace the K rows in the staging area now (the K side is done with them)
        if (f16) stage(1);
        __syncthreads();
        // ---- P'_b = p * normV(t, b) as [hi | lo] (B of the V MMAs), row sums ----
        {
            float ls[8];
            if (f16) {
                tc::cp_async_wait_all();
            }
            const float nv0 = f16 ? 1.0f : nrm[2 * CH + tl], nv1 = f16 ? 1.0f : nrm[3 * CH + tl];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = 8 * half + i;
                const float mnew = row[ROW_MNEW + r];
                const float pw = mnew == -INFINITY ? 0.0f : ex2(s2[i] - mnew);
                ls[i] = pw;
                const float x0 = pw * nv0, x1 = pw * nv1;
                const uint32_t hh = pack_h2(x0, x1);
                const float2 hf = unpack_h2(hh);
                const uint32_t ll = pack_h2(x0 - hf.x, x1 - hf.y);
                const uint32_t o = h_off(r, tl);
                *reinterpret_cast<uint16_t *>(bvp + o) = (uint16_t) hh;                   // tile 0 hi
                *reinterpret_cast<uint16_t *>(bvp + o + 256) = (uint16_t) ll;             // tile 0 lo (row 16 + r)
                *reinterpret_cast<uint16_t *>(bvp + TILE_B + o) = (uint16_t) (hh >> 16);  // tile 1 hi
                *reinterpret_cast<uint16_t *>(bvp + TILE_B + o + 256) = (uint16_t) (ll >> 16);
            }
            const float lw = warp_rows8<false>(ls, lane);
            if ((lane & 3) == 0) red[RED_L + half * 32 + quarter * 8 + (lane >> 2)] = lw;
        }
        __syncthreads();                                  // staged V rows and P' complete
        if (tid < NR) {
            const int hh = tid >> 3, rr = tid & 7;
            const float * lr = red + RED_L + hh * 32 + rr;
            row[ROW_L + tid] = row[ROW_L + tid] * row[ROW_ALPHA + tid] + ((lr[0] + lr[8]) + (lr[16] + lr[24]));
        }
        // ---- V side, tile by tile: A (channel 128 b + tl, tokens 64 half ..) -> TMEM, then the MMAs ----
        const uint8_t * vbase = f16 ? stg : stg + TQ6_ROW;      // tq6_0: the V row follows the K row
        for (int b = 0; b < 2 && ok; ++b) {
            {
                uint32_t ch[32], cl[32];
                const int d = 128 * b + tl;
                if (f16) {
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        const uint8_t * ra = vbase + (64 * half + 2 * c) * STG_F16;
                        const uint32_t x0 = *reinterpret_cast<const uint16_t *>(ra + 2 * d);
                        const uint32_t x1 = *reinterpret_cast<const uint16_t *>(ra + STG_F16 + 2 * d);
                        ch[c] = x0 | (x1 << 16);
                    }
                } else {
                    // the thread's channel: qs byte j/2 (nibble j%2), qh byte j/4 (2 bits at 2 (j%4)) of block b
                    const int j = d & 127;
                    const uint8_t * base = vbase + SJKVARN_TQ6_BLOCK_BYTES * b;
                    const int oqs = 2 + (j >> 1), sqs = 4 * (j & 1), oqh = 66 + (j >> 2), sqh = 2 * (j & 3);
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        const uint8_t * ra = base + (64 * half + 2 * c) * STG_TQ6, * rb = ra + STG_TQ6;
                        const uint32_t c0 = ((ra[oqs] >> sqs) & 15) | (((ra[oqh] >> sqh) & 3) << 4);
                        const uint32_t c1 = ((rb[oqs] >> sqs) & 15) | (((rb[oqh] >> sqh) & 3) << 4);
                        const uint32_t e0 = cent2[c0], e1 = cent2[c1];
                        ch[c] = prmt(e0, e1, 0x5410u);
                        cl[c] = prmt(e0, e1, 0x7632u);
                    }
                    tc::st_x16(tmem + lane_base + COL_AL + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(cl));
                    tc::st_x16(tmem + lane_base + COL_AL + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(cl + 16));
                }
                tc::st_x16(tmem + lane_base + COL_AH + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(ch));
                tc::st_x16(tmem + lane_base + COL_AH + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(ch + 16));
            }
            ok = run_mma(COL_O + 32 * b, bvp + TILE_B * b, f16);
        }
        if (!ok) break;
        // ---- epilogue: channel 128 half + tl, all rows (column groups hi*hi + lo*hi and hi*lo) ----
        {
            float o[16], ol[16];
            tc::ld_x16(tmem + lane_base + COL_O + 32 * half, o);
            tc::ld_x16(tmem + lane_base + COL_O + 32 * half + 16, ol);
            tc::wait_ld();
#pragma unroll
            for (int r = 0; r < NR; ++r) acc[r] = fmaf(acc[r], row[ROW_ALPHA + r], o[r] + ol[r]);
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
            float * dst = p.part + ((size_t) slot * p.n_q * p.n_head + (size_t) iq * p.n_head + hq) * (D + 2);
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
    if (warp == 0) tc::tmem_dealloc(*tmem_slot, TM_COLS);
}

__global__ void __launch_bounds__(NT, 2) attend_dense_tc_kernel(const __grid_constant__ DenseParams p) { dense_body(p); }

// the descriptor-driven form: items planned on the device (dense_dyn_plan_kernel); CTAs past them return at once
__global__ void __launch_bounds__(NT, 2) attend_dense_tc_dyn_kernel(const DenseParams * __restrict__ pp) {
    if ((int) blockIdx.x >= pp->n_items) return;
    dense_body(*pp);
}

// One sequence: chunk list [0, n_chunks) (sink chunks first) of KV heads kv0 .. kv0 + n_kv - 1, `splits` items of
// chunks_per_split chunks per head; item (head hl, split s) writes partial slot split0 + s. Runs on the host and in
// the planner kernel of the descriptor-driven call.
SJK_HD void fill_single(DenseParams & p, const sjk_view & v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                        int kv0, int n_kv, const float * q, float scale, float * part, int split0, int splits,
                        uint32_t n_sink_chunks, uint32_t n_chunks, int chunks_per_split) {
    p.v = v; p.n_q = n_q; p.n_head = n_head; p.grp = n_head / n_kv; p.rows = n_q * p.grp; p.scale = scale; p.part = part;
    p.seq[0].sink = v.sink; p.seq[0].ring = v.ring; p.seq[0].q = q; p.seq[0].B = B; p.seq[0].N = N; p.seq[0].qpos0 = qpos0;
    p.seq[0].n_sink_chunks = n_sink_chunks;
    int k = 0;
    for (int hl = 0; hl < n_kv; ++hl)
        for (int s = 0; s < splits; ++s, ++k) {
            DenseItem & it = p.item[k];
            it.seq_hl = (uint32_t) hl << 16;
            it.h_slot = (uint32_t) (kv0 + hl) | ((uint32_t) (split0 + s) << 16);
            it.c0 = (uint32_t) s * (uint32_t) chunks_per_split;
            it.c1 = it.c0 + (uint32_t) chunks_per_split < n_chunks ? it.c0 + (uint32_t) chunks_per_split : n_chunks;
        }
    p.n_items = k;
}

// planner of the descriptor-driven call: the plan of sjk_tc_dense_launch for the counts in *ds
__global__ void dense_dyn_plan_kernel(const sjk_dyn_state * __restrict__ ds, sjk_view v, int n_q, int n_head, int kv0, int n_kv,
                                      const float * q, float scale, float * part, DenseParams * out) {
    if (threadIdx.x != 0) return;
    const sjk_dyn_state d = *ds;
    fill_single(*out, v, d.B, d.N, d.qpos0, n_q, n_head, kv0, n_kv, q, scale, part, d.splits_tc, d.ok ? d.splits_d : 0,
                d.n_sink_d, d.n_dense, d.cps_d);
}

}  // namespace

// Whether the dense tensor-core path applies to the staged regions: D = 256, <= 16 query rows per KV head.
int sjk_tc_dense_supported(const sjk_view * v, int n_q, int grp) {
    return v->lay.D == D && n_q * grp <= NR && v->stage_bytes == (v->staging == SJKVARN_STAGING_F16 ? 512u : 196u);
}

int sjk_tc_dense_splits(uint32_t n_chunks, int n_kv, int * chunks_per_split) {
    return sjk_dense_split_count(n_chunks, n_kv, chunks_per_split);
}

size_t sjk_tc_dense_params_bytes(void) { return sizeof(DenseParams); }

namespace {
int dense_launch_params(const DenseParams & p, int n_items, sjk_stream st) {
    cudaError_t e = cudaFuncSetAttribute(attend_dense_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_TOTAL);
    if (e != cudaSuccess) return sjk_check(e);
    attend_dense_tc_kernel<<<(unsigned) n_items, NT, SMEM_TOTAL, st>>>(p);
    return sjk_check_launch();
}
}  // namespace

// One sequence: chunk list [0, n_chunks) (sink chunks first) of KV heads kv0 .. kv0 + n_kv - 1, `splits` items of
// chunks_per_split chunks per head; item (head hl, split s) writes partial slot split0 + s.
int sjk_tc_dense_launch(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, int kv0, int n_kv,
                        const float * q, float scale, float * part, int split0, int splits, uint32_t n_sink_chunks,
                        uint32_t n_chunks, int chunks_per_split, sjk_stream st) {
    if (splits <= 0) return 0;
    if (splits * n_kv > MAX_ITEMS || split0 + splits > 0xFFFF) return SJK_ERR_UNSUPPORTED;
    static thread_local DenseParams p;
    fill_single(p, *v, B, N, qpos0, n_q, n_head, kv0, n_kv, q, scale, part, split0, splits, n_sink_chunks, n_chunks,
                chunks_per_split);
    return dense_launch_params(p, p.n_items, st);
}

// Descriptor-driven form: the counts come from *ds (written on the device by the call's planner), this function's
// planner kernel writes the plan into `params` (sjk_tc_dense_params_bytes() bytes of device memory) and the kernel
// reads it there. The grid covers max_items CTAs, the most items a plan of this cache can have.
int sjk_tc_dense_dyn_launch(const sjk_view * v, int n_q, int n_head, int kv0, int n_kv, const float * q, float scale,
                            float * part, const sjk_dyn_state * ds, void * params, int max_items, sjk_stream st) {
    if (max_items <= 0) return 0;
    if (max_items > MAX_ITEMS) return SJK_ERR_UNSUPPORTED;
    DenseParams * dp = static_cast<DenseParams *>(params);
    dense_dyn_plan_kernel<<<1, 32, 0, st>>>(ds, *v, n_q, n_head, kv0, n_kv, q, scale, part, dp);
    if (sjk_check_launch()) return SJK_ERR_DEVICE;
    cudaError_t e = cudaFuncSetAttribute(attend_dense_tc_dyn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_TOTAL);
    if (e != cudaSuccess) return sjk_check(e);
    attend_dense_tc_dyn_kernel<<<(unsigned) max_items, NT, SMEM_TOTAL, st>>>(dp);
    return sjk_check_launch();
}

// Many sequences of one layer (same layout and formats as *v): sequence s has sink / ring pointers views[s], query
// rows q + s n_q n_head D and positions [0, N[s]) with B[s] sealed; its staged chunks (sink, then ring) are cut into
// items of at most cps chunks per KV head. Items get partial slots slot0, slot0 + 1, ...; for pair (s, h) the items
// are slots first[s H + h] .. first[s H + h + 1] - 1. Returns the item count in *n_items.
int sjk_tc_dense_batch_launch(const sjk_view * views, const uint32_t * B, const uint32_t * N, const uint32_t * qpos0,
                              int n_seq, int n_q, int n_head, const float * q, float scale, float * part, int slot0,
                              uint16_t * first, int * n_items, sjk_stream st) {
    const sjk_view & v0 = views[0];
    const int H = v0.n_head_kv;
    if (n_seq > MAX_SEQS) return SJK_ERR_UNSUPPORTED;
    static thread_local DenseParams p;
    p.v = v0; p.n_q = n_q; p.n_head = n_head; p.grp = n_head / H; p.rows = n_q * p.grp; p.scale = scale; p.part = part;
    uint64_t total = 0;
    for (int s = 0; s < n_seq; ++s) {
        const uint32_t S = v0.S, s_end = S < N[s] ? S : N[s], t0 = B[s] > S ? B[s] : S;
        DenseSeq & d = p.seq[s];
        d.sink = views[s].sink; d.ring = views[s].ring; d.q = q + (size_t) s * n_q * n_head * D;
        d.B = B[s]; d.N = N[s]; d.qpos0 = qpos0[s];
        d.n_sink_chunks = (s_end + 127u) / 128u;
        total += (uint64_t) (d.n_sink_chunks + (N[s] > t0 ? (N[s] - t0 + 127u) / 128u : 0u)) * (uint32_t) H;
    }
    const int pairs = n_seq * H;
    if (pairs >= MAX_ITEMS) return SJK_ERR_UNSUPPORTED;
    // sum over pairs of ceil(c / cps) <= total / cps + pairs <= MAX_ITEMS; also at least ~2 CTAs per SM of work items
    uint64_t cps = (total + (uint64_t) (MAX_ITEMS - pairs) - 1) / (uint64_t) (MAX_ITEMS - pairs);
    const uint64_t cps_fill = (total + 2 * 148 - 1) / (2 * 148);
    if (cps < cps_fill) cps = cps_fill;
    if (cps < 1) cps = 1;
    int k = 0;
    for (int s = 0; s < n_seq; ++s) {
        const uint32_t S = v0.S, t0 = B[s] > S ? B[s] : S;
        const uint32_t nc = p.seq[s].n_sink_chunks + (N[s] > t0 ? (N[s] - t0 + 127u) / 128u : 0u);
        for (int h = 0; h < H; ++h) {
            first[s * H + h] = (uint16_t) (slot0 + k);
            for (uint32_t c = 0; c < nc; c += (uint32_t) cps, ++k) {
                if (k >= MAX_ITEMS || slot0 + k > 0xFFFF) return SJK_ERR_UNSUPPORTED;
                DenseItem & it = p.item[k];
                it.seq_hl = (uint32_t) s | ((uint32_t) h << 16);
                it.h_slot = (uint32_t) h | ((uint32_t) (slot0 + k) << 16);
                it.c0 = c;
                it.c1 = c + (uint32_t) cps < nc ? c + (uint32_t) cps : nc;
            }
        }
    }
    first[pairs] = (uint16_t) (slot0 + k);
    *n_items = k;
    p.n_items = k;
    if (k == 0) return 0;
    return dense_launch_params(p, k, st);
}

SJK_STATUS_READER(sjk_tc_dense_status_take)
