// sjk_attend_dense.cu - tensor-core (tcgen05, kind::f16) attention over the staged rows of a layer: the
// staging ring [B, N) and the sink [0, S), in tq6_0 or fp16 form (sj_kvarn.h:1249-1284, 1516-1533).
//
// One CTA per SM walks a list of items, each a contiguous range of 128-position chunks of one (sequence, KV head),
// with one online-softmax state and one partial per item. A tq6_0 value is
// centroid[code] * norm, with one norm per (token, 128-channel block). The block structure puts the norm outside
// the MMA:
//
//   K side, block b   S_b^T[t, r] = sum_{d in b} cent[code_K(t, d)] * q[r, d];   dot = sum_b normK(t, b) S_b
//   V side, tile b    O_b^T[d, r] = sum_t cent[code_V(t, d)] * P'_b[r, t],       P'_b = p * normV(t, b)
//
// The centroids enter as fp16 hi + lo halves (A operands in TMEM, from a 64-entry table with one copy per bank),
// q and P' as fp16 hi + lo halves side by side in the MMA's N dimension (B = [hi | lo], N = 32). Two MMAs per k
// step, A_hi x [hi | lo] and A_lo x hi, accumulate hi*hi + lo*hi in columns 0..15 and hi*lo in columns 16..31 (the
// dropped lo*lo term is below 2^-22 relative); the result is the sum of the two column groups. fp16 rows (fp16
// sink, fp16 staging) enter exactly with lo = 0 and skip the second MMA.
//
// 16 worker warps split each chunk: quarter w % 4 is the warp's TMEM lane quarter (tokens or channels), group w / 4
// picks the block / tile and the half of the k range; both K blocks and both V tiles are built at once, so a chunk
// takes two MMA round trips. The rows of the CTA's next chunk (possibly the next item's first) stream into the second
// staging buffer (asynchronous copies, tq6_0 K and V rows together) while a chunk is processed; the V codes of a chunk are unpacked to bytes while its
// K MMAs run. Softmax is online over the chunks; thread 0 issues the MMAs. 16 warps (4 per SM sub-partition) leave
// 128 registers per thread. Partials go to the same split buffer as the other attention kernels. Waits are bounded.
#include <cuda_fp16.h>

#include "sjk_common.cuh"
#include "sjk_internal.h"
#include "sjk_plan.cuh"
#include "sjk_tc.cuh"

namespace {

using namespace tc::num;

constexpr int NW = 16;                  // warps (thread 0 also issues the MMAs)
constexpr int NT = NW * 32;
constexpr int NR = 16;
constexpr int D = 256;
constexpr int CH = 128;
constexpr uint32_t TM_COLS = 512;
constexpr uint32_t DCOL_A = 0, DCOL_S = 256, DCOL_O = 320;   // A (2 x [hi 64 | lo 64]) | S (2 x 32) | O (2 x 32)

constexpr int MAX_SEQS = 128;
constexpr int MAX_ITEMS = 768;
constexpr int MAX_CTAS = 148;

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
    // query row r (r < rows) of a KV head's group: position r / grp, query head hl grp + r % grp; the divisions are
    // done once on the host
    uint32_t row_iq[NR];                // r / grp
    int row_q[NR];                      // (r / grp) n_head + r % grp: q row and partial row of r, less hl grp
    float scale;
    float * part;                       // [slots][n_q n_head][D + 2]
    int n_items;
    int n_cta;                          // CTAs with work (the descriptor-driven grid may be larger)
    uint16_t cta_item[MAX_ITEMS + 1];   // items of CTA c: [cta_item[c], cta_item[c + 1]), in order
    DenseSeq seq[MAX_SEQS];
    DenseItem item[MAX_ITEMS];
};

// B operand (K-major, no swizzle, 32 rows): element (n, k) at (k / 8) * HCH + n * 16 + (k % 8) * 2 with an 8-element
// K chunk every HCH = 528 bytes (512 + 16: consecutive chunks start 4 banks apart, so the builders' stores are
// conflict-free); one MMA k step (16 elements) is two chunks (LBO = HCH, SBO 128 between 8-row groups)
constexpr uint32_t HCH = 528;
__device__ __forceinline__ uint32_t h_off(int n, int k) { return (uint32_t) (k >> 3) * HCH + (uint32_t) (n * 16 + (k & 7) * 2); }

constexpr uint32_t STG_F16 = 528;       // staged fp16 row stride (512 B + 16: 16-byte rows, conflict-free LDS.128)
constexpr uint32_t TQ6_ROW = 2 * SJKVARN_TQ6_BLOCK_BYTES;      // 196 B: one K or V row of tq6_0 blocks
constexpr uint32_t STG_TQ6 = 2 * TQ6_ROW;                       // staged K row + V row of a token (392 B = 49 x 8)
constexpr uint32_t STG_BYTES = CH * STG_F16;                    // one staging buffer
constexpr uint32_t TILE_B = 16 * HCH;                           // one B operand over 128 k (8 k steps)
constexpr uint32_t OFF_STG = 0;                                 // 2 staging buffers (chunk i % 2)
constexpr uint32_t OFF_BQ = OFF_STG + 2 * STG_BYTES;            // [q hi | q lo] for 256 channels: 2 x TILE_B
constexpr uint32_t OFF_BV = OFF_BQ + 2 * TILE_B;                // [P' hi | P' lo] per tile: 2 x TILE_B
constexpr uint32_t OFF_VC = OFF_BV + 2 * TILE_B;                // V codes of the chunk, [token][channel] bytes
constexpr uint32_t OFF_CENT = OFF_VC + CH * D;                  // u32 [64][32]: fp16 hi | lo << 16 per centroid, per bank
constexpr uint32_t OFF_QH = OFF_CENT + 64 * 32 * 4;             // u32 [256]: 2-bit fields of a byte spread to bits 4-5
constexpr uint32_t OFF_NRM = OFF_QH + 256 * 4;                  // normK[2][128], normV[2][128]
constexpr uint32_t OFF_RED = OFF_NRM + 4 * CH * 4;              // row maxima, then row sums: [4 groups][4 quarters][4]
constexpr uint32_t OFF_ROW = OFF_RED + 2 * 64 * 4;              // per-row state, floats below
constexpr uint32_t OFF_BAR = OFF_ROW + 4 * NR * 4;
constexpr uint32_t OFF_TMEM = OFF_BAR + 16;
constexpr uint32_t SMEM_TOTAL = OFF_TMEM + 16;
static_assert(CH * STG_TQ6 <= STG_BYTES, "a staging buffer holds both tq6_0 sides");
static_assert(SMEM_TOTAL <= 227 * 1024, "shared memory");
static_assert(OFF_BQ % 16 == 0 && OFF_BV % 16 == 0 && OFF_VC % 16 == 0 && OFF_CENT % 16 == 0 && OFF_BAR % 8 == 0, "alignment");
enum { ROW_M2 = 0, ROW_L = 16, ROW_MNEW = 32, ROW_ALPHA = 48 };
enum { RED_MAX = 0, RED_L = 64 };

SJK_DEV void dense_body(const DenseParams & p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int quarter = warp & 3, grp = warp >> 2, tl = quarter * 32 + lane;
    const sjk_view & v = p.v;
    const int H = v.n_head_kv;
    uint8_t * bq = sm + OFF_BQ;
    uint8_t * bvp = sm + OFF_BV;
    uint8_t * vcodes = sm + OFF_VC;
    uint32_t * centr = reinterpret_cast<uint32_t *>(sm + OFF_CENT);
    uint32_t * qh_lut = reinterpret_cast<uint32_t *>(sm + OFF_QH);
    float * nrm = reinterpret_cast<float *>(sm + OFF_NRM);           // normK b*128+t, then normV at 256 + b*128+t
    float * red = reinterpret_cast<float *>(sm + OFF_RED);
    float * row = reinterpret_cast<float *>(sm + OFF_ROW);
    uint64_t * bar = reinterpret_cast<uint64_t *>(sm + OFF_BAR);
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(sm + OFF_TMEM);
    const int i_begin = p.cta_item[blockIdx.x], i_end = p.cta_item[blockIdx.x + 1];

    // chunk ci of item it: first position, length, row format, first ring slot, row bases
    struct Chunk { const uint8_t * sink, * ring; uint32_t p0, len, side_off, slot0; int h; bool f16, in_sink, f16_sink; };
    auto chunk_of = [&](int it, uint32_t ci) -> Chunk {
        const DenseItem & im = p.item[it];
        const DenseSeq & sq = p.seq[im.seq_hl & 0xFFFFu];
        const uint32_t S_eff = v.S < sq.N ? v.S : sq.N, t0_ring = sq.B > v.S ? sq.B : v.S;
        Chunk c;
        c.sink = sq.sink; c.ring = sq.ring; c.h = (int) (im.h_slot & 0xFFFFu);
        c.in_sink = ci < sq.n_sink_chunks;
        c.p0 = c.in_sink ? ci * (uint32_t) CH : t0_ring + (ci - sq.n_sink_chunks) * (uint32_t) CH;
        c.len = min((uint32_t) CH, (c.in_sink ? S_eff : sq.N) - c.p0);
        c.f16_sink = c.in_sink && v.sink_type == SJKVARN_SINK_F16;
        // f16 rows: the fp16 sink, or an fp16 staging ring / inherited sink; otherwise tq6_0 rows
        c.f16 = c.f16_sink || v.staging == SJKVARN_STAGING_F16;
        c.side_off = c.f16_sink ? 2u * D : (uint32_t) v.stage_bytes;
        c.slot0 = c.in_sink ? 0u : sjk_ring_slot(v.S, v.cap, c.p0);
        return c;
    };
    // global K row of token t (clamped to the chunk; the V row follows at side_off); ring slots are consecutive mod cap
    auto row_of = [&](const Chunk & c, uint32_t t) -> const uint8_t * {
        t = min(t, c.len - 1u);
        if (c.f16_sink) return c.sink + ((size_t) (c.p0 + t) * H + c.h) * 4 * D;
        if (c.in_sink) return c.sink + ((size_t) (c.p0 + t) * H + c.h) * 2 * v.stage_bytes;
        const uint32_t s = c.slot0 + t >= v.cap ? c.slot0 + t - v.cap : c.slot0 + t;
        return c.ring + ((size_t) s * H + c.h) * 2 * v.stage_bytes;
    };
    // the rows of chunk c into staging buffer dst (asynchronous copies, zeros past len), one warp per token: tq6_0 K
    // and V rows together (392 contiguous bytes, 49 x 8); fp16 rows one side at a time (512 bytes, 32 x 16)
    auto stage = [&](const Chunk & c, int side, uint8_t * dst) {
        if (c.f16) {
            const uint32_t so = side ? c.side_off : 0u;
            for (int t = warp; t < CH; t += NW)
                tc::cp_async16(dst + t * STG_F16 + 16 * lane, row_of(c, (uint32_t) t) + so + 16 * lane, (uint32_t) t < c.len ? 16u : 0u);
        } else {
            for (int t = warp; t < CH; t += NW) {
                const uint8_t * src = row_of(c, (uint32_t) t);
                const uint32_t nb = (uint32_t) t < c.len ? 8u : 0u;
                tc::cp_async8(dst + t * STG_TQ6 + 8 * lane, src + 8 * lane, nb);
                if (lane < 17) tc::cp_async8(dst + t * STG_TQ6 + 256 + 8 * lane, src + 256 + 8 * lane, nb);
            }
        }
    };
    // the first (item, chunk) at or after item it with a chunk (it = i_end: none)
    auto first_unit = [&](int it) -> int {
        while (it < i_end && p.item[it].c0 >= p.item[it].c1) ++it;
        return it;
    };
    // this thread's q values of item it: channel tid % 256, rows 8 (tid / 256) ..
    auto load_q = [&](int it, float (&x)[8]) {
        const DenseItem & im = p.item[it];
        const DenseSeq & sq = p.seq[im.seq_hl & 0xFFFFu];
        const int hl = (int) (im.seq_hl >> 16), d = tid & 255, r0 = (tid >> 8) * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = r0 + i, rr = r < p.rows ? r : 0;
            x[i] = __ldg(sq.q + (size_t) (p.row_q[rr] + hl * p.grp) * D + d);
        }
    };
    // [q hi | q lo] of the item (B of the K MMAs)
    auto store_bq = [&](const float (&x)[8]) {
        const int d = tid & 255, r0 = (tid >> 8) * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = r0 + i;
            const float xr = r < p.rows ? x[i] : 0.0f;
            const __half hi = __float2half_rn(xr);
            *reinterpret_cast<__half *>(bq + h_off(r, d)) = hi;
            *reinterpret_cast<__half *>(bq + h_off(NR + r, d)) = __float2half_rn(xr - __half2float(hi));
        }
    };

    // ---- setup: the query and table loads go out first, then the first chunk's rows, which stream in while the
    // tables, [q hi | q lo], TMEM and the barrier are made ----
    const int u_first = first_unit(i_begin);
    float x[8];
    load_q(i_begin < i_end ? i_begin : 0, x);
    float cent[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) cent[k] = sjk_tq6_cent[(tid + NT * k) >> 5];
    if (u_first < i_end) stage(chunk_of(u_first, p.item[u_first].c0), 0, sm + OFF_STG);
    tc::cp_async_commit();
    if (warp == 0) { tc::tmem_alloc(tmem_slot, TM_COLS); tc::tmem_relinquish(); }
    if (tid == 32) { tc::mbar_init(bar, 1); tc::mbar_fence_init(); }
    if (tid < 256) {
        const uint32_t y = (uint32_t) tid;
        qh_lut[tid] = ((y & 3u) << 4) | (((y >> 2) & 3u) << 12) | (((y >> 4) & 3u) << 20) | (((y >> 6) & 3u) << 28);
    }
    static_assert(64 * 32 == 4 * NT, "four table words per thread");
#pragma unroll
    for (int k = 0; k < 4; ++k) {                               // entry c of lane L at word 32 c + L
        const float c = cent[k];
        const __half hi = __float2half_rn(c);
        const __half2 hl2 = __floats2half2_rn(__half2float(hi), c - __half2float(hi));
        centr[tid + NT * k] = *reinterpret_cast<const uint32_t *>(&hl2);
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t) (quarter * 32) << 16;
    const float sl2 = p.scale * LOG2E;
    bool ok = true;
    uint32_t mma_phase = 0, n_done = 0;                         // n_done: chunks processed (staging buffer parity)
    bool mma_pending = false;
    // all threads: operand stores visible to the MMA, thread 0 issues both blocks / tiles, nobody waits
    auto mma_issue = [&](const uint8_t * b_base, uint32_t d_col, bool f16) {
        tc::wait_st();
        tc::fence_proxy_async();
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        if (tid == 0) {
            const uint32_t idesc32 = tc::idesc_f16(128, 2 * NR), idesc16 = tc::idesc_f16(128, NR);
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                const uint64_t db = tc::smem_desc(b_base + TILE_B * b, HCH, 128);
                const uint32_t ah = tmem + DCOL_A + 128 * b, dc = tmem + d_col + 32 * b;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    tc::mma_ts(dc, ah + 8 * k, db + (uint64_t) ((2 * HCH * k) >> 4), idesc32, k ? 1u : 0u);
                    if (!f16) tc::mma_ts(dc, ah + 64 + 8 * k, db + (uint64_t) ((2 * HCH * k) >> 4), idesc16, 1u);
                }
            }
            tc::mma_commit(bar);
        }
        mma_pending = true;
    };
    auto mma_wait = [&]() -> bool {
        const bool got = __syncthreads_and(tc::mbar_wait(bar, mma_phase));
        if (got) { mma_phase ^= 1u; mma_pending = false; }
        tc::fence_after_sync();
        return got;
    };
    // the partial of item it (after the barrier that ended its last chunk); then the row state starts over
    float acc[NR];                                              // warps 0..7: running output of channel 128 (w / 4) + tl
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
    auto finish_item = [&](int it, bool good) {
        const DenseItem & im = p.item[it];
        const int hl = (int) (im.seq_hl >> 16), slot = (int) (im.h_slot >> 16);
        if (tid < NR) {
            const int r = tid;
            if (r < p.rows) {
                float * dst = p.part + ((size_t) slot * p.n_q * p.n_head + (size_t) (p.row_q[r] + hl * p.grp)) * (D + 2);
                const float m2 = row[ROW_M2 + r];
                dst[0] = good ? (m2 == -INFINITY ? m2 : m2 * LN2) : -INFINITY;
                dst[1] = good ? row[ROW_L + r] : 0.0f;
            }
            row[ROW_M2 + r] = -INFINITY;
            row[ROW_L + r] = 0.0f;
        }
        if (warp < 8) {
            const int half = warp >> 2;
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                if (r < p.rows)
                    p.part[((size_t) slot * p.n_q * p.n_head + (size_t) (p.row_q[r] + hl * p.grp)) * (D + 2) + 2 + 128 * half + tl] =
                        good ? acc[r] : 0.0f;
                acc[r] = 0.0f;
            }
        }
    };
    if (tid < NR) { row[ROW_M2 + tid] = -INFINITY; row[ROW_L + tid] = 0.0f; }

    int it = i_begin;
    for (; it < i_end && ok; ++it) {
        const DenseItem & im = p.item[it];
        const DenseSeq & sq = p.seq[im.seq_hl & 0xFFFFu];
        if (it != i_begin) load_q(it, x);
        store_bq(x);                                            // read by the item's K MMAs, after the barriers below
        uint32_t qlim4[4];                                      // rows 4 grp + i: positions < qlim4[i] are visible
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = 4 * grp + i;
            qlim4[i] = r < p.rows ? sq.qpos0 + p.row_iq[r] + 1u : 0u;
        }
        for (uint32_t ci = im.c0; ci < im.c1 && ok; ++ci, ++n_done) {
            const Chunk ck = chunk_of(it, ci);
            const bool f16 = ck.f16;
            const uint32_t sstride = f16 ? STG_F16 : STG_TQ6;
            uint8_t * stg = sm + OFF_STG + (n_done & 1u) * STG_BYTES;
            // the CTA's next chunk goes to the other buffer (free: its last chunk ended at a barrier)
            {
                const int nit = ci + 1 < im.c1 ? it : first_unit(it + 1);
                if (nit < i_end)
                    stage(chunk_of(nit, nit == it ? ci + 1 : p.item[nit].c0), 0, sm + OFF_STG + ((n_done + 1) & 1u) * STG_BYTES);
            }
            tc::cp_async_commit();
            tc::cp_async_wait_group<1>();                       // this chunk's rows are in
            tc::fence_before_sync();
            __syncthreads();
            tc::fence_after_sync();
            if (tid < CH) {
                const uint8_t * r0 = stg + tid * sstride;
                nrm[tid] = f16 ? 1.0f : h2f_at(r0);
                nrm[CH + tid] = f16 ? 1.0f : h2f_at(r0 + SJKVARN_TQ6_BLOCK_BYTES);
                nrm[2 * CH + tid] = f16 ? 1.0f : h2f_at(r0 + TQ6_ROW);
                nrm[3 * CH + tid] = f16 ? 1.0f : h2f_at(r0 + TQ6_ROW + SJKVARN_TQ6_BLOCK_BYTES);
            }
            // ---- K side: block grp / 2, channels 64 (grp % 2) .. of token tl -> A (hi | lo) ----
            {
                const int b = grp >> 1, half = grp & 1;
                const uint8_t * r0 = stg + tl * sstride;
                const uint32_t ta = tmem + lane_base + DCOL_A + 128 * b + 32 * half;
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {                    // 16 columns (32 channels) at a time
                    uint32_t ch[16], cl[16];
                    if (f16) {
                        const uint4 * src = reinterpret_cast<const uint4 *>(r0 + 2 * (128 * b + 64 * half + 32 * hh));
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const uint4 x = src[c];
                            ch[4 * c] = x.x; ch[4 * c + 1] = x.y; ch[4 * c + 2] = x.z; ch[4 * c + 3] = x.w;
                        }
                    } else {
                        const uint8_t * blk = r0 + SJKVARN_TQ6_BLOCK_BYTES * b;
#pragma unroll
                        for (int g = 0; g < 4; ++g) {
                            const uint2 cw = tq6_codes8(blk, 64 * half + 32 * hh + 8 * g, qh_lut);
#pragma unroll
                            for (int pp = 0; pp < 4; ++pp) {
                                const uint32_t w = pp < 2 ? cw.x : cw.y, sh = 16 * (pp & 1);
                                const uint32_t e0 = centr[32 * ((w >> sh) & 0xFFu) + lane];
                                const uint32_t e1 = centr[32 * ((w >> (sh + 8)) & 0xFFu) + lane];
                                ch[4 * g + pp] = prmt(e0, e1, 0x5410u);
                                cl[4 * g + pp] = prmt(e0, e1, 0x7632u);
                            }
                        }
                        tc::st_x16(ta + 64 + 16 * hh, cl);
                    }
                    tc::st_x16(ta + 16 * hh, ch);
                }
            }
            mma_issue(bq, DCOL_S, f16);
            // tq6_0, while the K MMAs run: the chunk's V codes in natural order (token, 8 channels per item)
            if (!f16) {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int it = tid + NW * 32 * k, t = it >> 5, gch = it & 31;        // channels 8 gch ..
                    const uint8_t * vblk = stg + t * STG_TQ6 + TQ6_ROW + SJKVARN_TQ6_BLOCK_BYTES * (gch >> 4);
                    *reinterpret_cast<uint2 *>(vcodes + t * D + 8 * gch) = tq6_codes8(vblk, 8 * (gch & 15), qh_lut);
                }
            }
            ok = mma_wait();
            if (!ok) break;
            // ---- scores of token tl for rows 4 grp .. 4 grp + 3 (log2 domain), row maxima ----
            float s2[4];
            {
                uint32_t a0[4], a0l[4], a1[4], a1l[4];
                tc::ld_x4_u(tmem + lane_base + DCOL_S + 4 * grp, a0);
                tc::ld_x4_u(tmem + lane_base + DCOL_S + 16 + 4 * grp, a0l);
                tc::ld_x4_u(tmem + lane_base + DCOL_S + 32 + 4 * grp, a1);
                tc::ld_x4_u(tmem + lane_base + DCOL_S + 48 + 4 * grp, a1l);
                tc::wait_ld();
                const float nk0 = nrm[tl] * sl2, nk1 = nrm[CH + tl] * sl2;
                const uint32_t pos = ck.p0 + (uint32_t) tl;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float dot = nk0 * (__uint_as_float(a0[i]) + __uint_as_float(a0l[i])) +
                                      nk1 * (__uint_as_float(a1[i]) + __uint_as_float(a1l[i]));
                    s2[i] = ((uint32_t) tl < ck.len && pos < qlim4[i]) ? dot : -INFINITY;
                }
                const float mw = warp_rows4<true>(s2, lane);
                if ((lane & 7) == 0) red[RED_MAX + (grp * 4 + quarter) * 4 + (lane >> 3)] = mw;
            }
            tc::fence_before_sync();
            __syncthreads();
            if (tid < NR) {
                const int r = tid, gq = (r >> 2) * 16 + (r & 3);
                const float * mr = red + RED_MAX + gq;
                const float mrec = fmaxf(fmaxf(mr[0], mr[4]), fmaxf(mr[8], mr[12]));
                const float mold = row[ROW_M2 + r], mnew = fmaxf(mold, mrec);
                row[ROW_MNEW + r] = mnew;
                row[ROW_ALPHA + r] = mnew == -INFINITY ? 1.0f : ex2(mold - mnew);
                row[ROW_M2 + r] = mnew;
            }
            // fp16 rows: the V rows replace the K rows in this chunk's buffer (the K side is done with them)
            if (f16) {
                stage(ck, 1, stg);
                tc::cp_async_commit();
            }
            __syncthreads();
            // ---- P'_b = p normV(t, b) as [hi | lo] per tile (B of the V MMAs), row sums ----
            {
                if (f16) tc::cp_async_wait_group<0>();
                const float nv0 = nrm[2 * CH + tl], nv1 = nrm[3 * CH + tl];
                float ls[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = 4 * grp + i;
                    const float mnew = row[ROW_MNEW + r];
                    const float pw = mnew == -INFINITY ? 0.0f : ex2(s2[i] - mnew);
                    ls[i] = pw;
                    const float x0 = pw * nv0, x1 = pw * nv1;
                    const __half2 hh = __floats2half2_rn(x0, x1);
                    const float2 hf = __half22float2(hh);
                    const __half2 ll = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
                    const uint32_t o = h_off(r, tl);
                    *reinterpret_cast<__half *>(bvp + o) = __low2half(hh);                 // tile 0 hi
                    *reinterpret_cast<__half *>(bvp + o + 256) = __low2half(ll);           // tile 0 lo (row 16 + r)
                    *reinterpret_cast<__half *>(bvp + TILE_B + o) = __high2half(hh);       // tile 1 hi
                    *reinterpret_cast<__half *>(bvp + TILE_B + o + 256) = __high2half(ll);
                }
                const float lw = warp_rows4<false>(ls, lane);
                if ((lane & 7) == 0) red[RED_L + (grp * 4 + quarter) * 4 + (lane >> 3)] = lw;
            }
            __syncthreads();                                        // staged V rows, P' and the row sums complete
            if (tid < NR) {
                const int r = tid, gq = (r >> 2) * 16 + (r & 3);
                const float * lr = red + RED_L + gq;
                row[ROW_L + r] = row[ROW_L + r] * row[ROW_ALPHA + r] + ((lr[0] + lr[4]) + (lr[8] + lr[12]));
            }
            // ---- V side: tile grp / 2, channel 128 (grp / 2) + tl, tokens 64 (grp % 2) .. -> A (hi | lo) ----
            {
                const int t = grp >> 1, half = grp & 1, d = 128 * t + tl;
                const uint32_t ta = tmem + lane_base + DCOL_A + 128 * t + 32 * half;
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {                    // 16 columns (32 tokens) at a time
                    uint32_t ch[16], cl[16];
                    const int tk0 = 64 * half + 32 * hh;
                    if (f16) {
#pragma unroll
                        for (int c = 0; c < 16; ++c) {
                            const uint8_t * ra = stg + (tk0 + 2 * c) * STG_F16;
                            const uint32_t x0 = *reinterpret_cast<const uint16_t *>(ra + 2 * d);
                            const uint32_t x1 = *reinterpret_cast<const uint16_t *>(ra + STG_F16 + 2 * d);
                            ch[c] = x0 | (x1 << 16);
                        }
                    } else {
                        const uint8_t * col = vcodes + tk0 * D + d;
#pragma unroll
                        for (int c = 0; c < 16; ++c) {
                            const uint32_t e0 = centr[32 * col[(2 * c) * D] + lane], e1 = centr[32 * col[(2 * c + 1) * D] + lane];
                            ch[c] = prmt(e0, e1, 0x5410u);
                            cl[c] = prmt(e0, e1, 0x7632u);
                        }
                        tc::st_x16(ta + 64 + 16 * hh, cl);
                    }
                    tc::st_x16(ta + 16 * hh, ch);
                }
            }
            mma_issue(bvp, DCOL_O, f16);
            ok = mma_wait();
            if (!ok) break;
            // ---- epilogue (warps 0..7): channel 128 (w / 4) + tl, all rows (column groups hi*hi + lo*hi and hi*lo) ----
            if (warp < 8) {
                const int half = warp >> 2;
                float o[16], ol[16];
                tc::ld_x16(tmem + lane_base + DCOL_O + 32 * half, o);
                tc::ld_x16(tmem + lane_base + DCOL_O + 32 * half + 16, ol);
                tc::wait_ld();
#pragma unroll
                for (int r = 0; r < NR; ++r) acc[r] = fmaf(acc[r], row[ROW_ALPHA + r], o[r] + ol[r]);
            }
            tc::fence_before_sync();
            __syncthreads();
            tc::fence_after_sync();
        }
        if (ok) finish_item(it, true);
    }
    if (!ok && mma_pending) tc::mbar_wait(bar, mma_phase);      // a chunk that gave up: its MMAs first (bounded)
    tc::cp_async_wait_group<0>();                               // no copy outlives the CTA
    __syncthreads();
    if (!ok)                                                    // the item that gave up and the ones after it: empty
        for (int j = it > i_begin ? it - 1 : i_begin; j < i_end; ++j) finish_item(j, false);
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, TM_COLS);
    // launched as the trellis kernel's programmatic dependent, this grid completes only after that one did, so what
    // runs after it in the stream sees both kernels' partials (otherwise a no-op)
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__global__ void __launch_bounds__(NT, 1) attend_dense_tc_kernel(const __grid_constant__ DenseParams p) { dense_body(p); }

// the descriptor-driven form: items planned on the device (dense_dyn_plan_kernel); CTAs past them return at once
__global__ void __launch_bounds__(NT, 1) attend_dense_tc_dyn_kernel(const DenseParams * __restrict__ pp) {
    if ((int) blockIdx.x >= pp->n_cta) return;
    dense_body(*pp);
}

SJK_HD void fill_rows(DenseParams & p, int n_q, int n_head, int n_kv) {
    p.grp = n_head / n_kv;
    p.rows = n_q * p.grp;
    for (int r = 0; r < NR; ++r) {
        const int iq = r < p.rows ? r / p.grp : 0, g = r < p.rows ? r % p.grp : 0;
        p.row_iq[r] = (uint32_t) iq;
        p.row_q[r] = iq * n_head + g;
    }
}

// One sequence: chunk list [0, n_chunks) (sink chunks first) of KV heads kv0 .. kv0 + n_kv - 1, `splits` items of
// chunks_per_split chunks per head; item (head hl, split s) writes partial slot split0 + s. Runs on the host and in
// the planner kernel of the descriptor-driven call.
SJK_HD void fill_single(DenseParams & p, const sjk_view & v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                        int kv0, int n_kv, const float * q, float scale, float * part, int split0, int splits,
                        uint32_t n_sink_chunks, uint32_t n_chunks, int chunks_per_split) {
    p.v = v; p.n_q = n_q; p.n_head = n_head; p.scale = scale; p.part = part;
    fill_rows(p, n_q, n_head, n_kv);
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
            p.cta_item[k] = (uint16_t) k;                      // one item per CTA
        }
    p.cta_item[k] = (uint16_t) k;
    p.n_items = k;
    p.n_cta = k;
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
int dense_launch_params(const DenseParams & p, int n_cta, sjk_stream st, bool dependent = false) {
    cudaError_t e = cudaFuncSetAttribute(attend_dense_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_TOTAL);
    if (e != cudaSuccess) return sjk_check(e);
    if (!dependent) {
        attend_dense_tc_kernel<<<(unsigned) n_cta, NT, SMEM_TOTAL, st>>>(p);
        return sjk_check_launch();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) n_cta);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = SMEM_TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (sjk_check(cudaLaunchKernelEx(&cfg, attend_dense_tc_kernel, p))) return SJK_ERR_DEVICE;
    return sjk_check_launch();
}
}  // namespace

// One sequence: chunk list [0, n_chunks) (sink chunks first) of KV heads kv0 .. kv0 + n_kv - 1, `splits` items of
// chunks_per_split chunks per head; item (head hl, split s) writes partial slot split0 + s.
int sjk_tc_dense_launch(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, int kv0, int n_kv,
                        const float * q, float scale, float * part, int split0, int splits, uint32_t n_sink_chunks,
                        uint32_t n_chunks, int chunks_per_split, bool beside_tc, sjk_stream st) {
    if (splits <= 0) return 0;
    if (splits * n_kv > MAX_ITEMS || split0 + splits > 0xFFFF) return SJK_ERR_UNSUPPORTED;
    static thread_local DenseParams p;
    fill_single(p, *v, B, N, qpos0, n_q, n_head, kv0, n_kv, q, scale, part, split0, splits, n_sink_chunks, n_chunks,
                chunks_per_split);
    return dense_launch_params(p, p.n_cta, st, beside_tc);
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
// rows q + s n_q n_head D and positions [0, N[s]) with B[s] sealed; its staged chunks (sink, then ring) per KV head
// form one list over all (sequence, KV head) pairs, cut into at most one contiguous range per SM, each range into
// items that stay inside one pair. Items get partial slots slot0, slot0 + 1, ...; for pair (s, h) the items are
// slots first[s H + h] .. first[s H + h + 1] - 1. Returns the item count in *n_items.
int sjk_tc_dense_batch_launch(const sjk_view * views, const uint32_t * B, const uint32_t * N, const uint32_t * qpos0,
                              int n_seq, int n_q, int n_head, const float * q, float scale, float * part, int slot0,
                              uint16_t * first, int * n_items, sjk_stream st) {
    const sjk_view & v0 = views[0];
    const int H = v0.n_head_kv;
    if (n_seq > MAX_SEQS) return SJK_ERR_UNSUPPORTED;
    static thread_local DenseParams p;
    static thread_local uint32_t n_chunks[MAX_SEQS];
    p.v = v0; p.n_q = n_q; p.n_head = n_head; p.scale = scale; p.part = part;
    fill_rows(p, n_q, n_head, H);
    uint64_t total = 0;
    for (int s = 0; s < n_seq; ++s) {
        const uint32_t S = v0.S, s_end = S < N[s] ? S : N[s], t0 = B[s] > S ? B[s] : S;
        DenseSeq & d = p.seq[s];
        d.sink = views[s].sink; d.ring = views[s].ring; d.q = q + (size_t) s * n_q * n_head * D;
        d.B = B[s]; d.N = N[s]; d.qpos0 = qpos0[s];
        d.n_sink_chunks = (s_end + 127u) / 128u;
        n_chunks[s] = d.n_sink_chunks + (N[s] > t0 ? (N[s] - t0 + 127u) / 128u : 0u);
        total += (uint64_t) n_chunks[s] * (uint32_t) H;
    }
    const int n_cta = total < (uint64_t) MAX_CTAS ? (int) total : MAX_CTAS;
    int k = 0, cta = 0;
    if (n_cta > 0) {
        const uint64_t per = (total + (uint64_t) n_cta - 1) / (uint64_t) n_cta;
        uint64_t filled = 0;
        p.cta_item[0] = 0;
        for (int s = 0; s < n_seq; ++s)
            for (int h = 0; h < H; ++h) {
                first[s * H + h] = (uint16_t) (slot0 + k);
                uint32_t c = 0;
                while (c < n_chunks[s]) {
                    const uint32_t take = (uint32_t) (per - filled < (uint64_t) (n_chunks[s] - c) ? per - filled : (uint64_t) (n_chunks[s] - c));
                    if (k >= MAX_ITEMS || slot0 + k > 0xFFFF) return SJK_ERR_UNSUPPORTED;
                    DenseItem & it = p.item[k++];
                    it.seq_hl = (uint32_t) s | ((uint32_t) h << 16);
                    it.h_slot = (uint32_t) h | ((uint32_t) (slot0 + k - 1) << 16);
                    it.c0 = c;
                    it.c1 = c + take;
                    c += take;
                    filled += take;
                    if (filled == per) { p.cta_item[++cta] = (uint16_t) k; filled = 0; }
                }
            }
        if (filled > 0) p.cta_item[++cta] = (uint16_t) k;
    } else {
        for (int i = 0; i < n_seq * H; ++i) first[i] = (uint16_t) slot0;
    }
    first[n_seq * H] = (uint16_t) (slot0 + k);
    *n_items = k;
    p.n_items = k;
    p.n_cta = cta;
    if (cta == 0) return 0;
    return dense_launch_params(p, cta, st);
}

SJK_STATUS_READER(sjk_tc_dense_status_take)
