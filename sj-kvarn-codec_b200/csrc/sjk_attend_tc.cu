// sjk_attend_tc.cu - tensor-core (tcgen05, kind::i8) attention over the sealed body of a 4-bit scalar layer.
//
// One CTA = one KV head x a contiguous range of records, 256 threads (8 warps); warp w owns TMEM lane
// quarter w % 4, and the two warps of a quarter split the columns (half = w / 4). The query rows of the
// KV head (decode width x GQA group, padded to N = 16) are the MMA's N dimension, the 128 tokens (K side)
// or 128 channels (V side, two tiles) its M dimension:
//
//   K side  S^T[t, r] = sum_d code_K[t, d] * Q'[r, d],   Q'[r, d] = q[r, d] * Kscale[d]
//           dot[t, r] = Ktok[t] * (S^T[t, r] + sum_d q[r, d] * Kzero[d])
//   V side  O^T[d, r] = sum_t code_V[d, t] * P'[r, t],   P'[r, t] = p[r, t] * Vscale[t]
//           out[d, r] = Vch[d] * (O^T[d, r] + sum_t p[r, t] * Vzero[t])
//
// i.e. the reference reconstruction K = (q*Ks + Kz)*Kt, V = (q*Vs + Vz)*Vc (sj_kvarn.h:1187-1207) regrouped
// so the 4-bit codes enter the tensor core as exact signed 8-bit integers (A operand in TMEM, unpacked from
// the fragment-ordered payload with LOP3/PRMT). Q' and P' are each rounded to a 21-bit integer after an
// exact power-of-two rescale (per query row; P' by the row's largest weight in the record) and split into
// three signed 8-bit digits (B operands in shared memory); each digit is its own exact s32 accumulation
// and the digits recombine in fp32. Integer <-> float conversions use the 1.5 * 2^23 magic constant, so the XU pipe is left to exp2.
//
// Records stream in through a double-buffered 1-D bulk copy (cp.async.bulk, no multicast). All waits are
// bounded (sjk_tc.cuh); the kernel always waits for its own copies and MMAs and releases its TMEM.
#include "sjk_common.cuh"
#include "sjk_internal.h"
#include "sjk_tc.cuh"

namespace {

using namespace tc::num;

constexpr int NT = 256;
constexpr int NR = 16;                  // MMA N: query rows per KV head, padded
constexpr int D = 256;
constexpr int G = 128;
constexpr uint32_t TM_COLS = 256;
constexpr uint32_t COL_AK = 0;          // A for K: 128 lanes x 256 s8 = 64 columns (dead once the K MMAs end)
constexpr uint32_t COL_O = 0;           // O^T: 2 tiles x 3 digits x 16 columns, written after A_K is dead
constexpr uint32_t COL_AV = 96;         // A for V: 2 tiles x 128 lanes x 128 s8 = 2 x 32 columns
constexpr uint32_t COL_S = 160;         // S^T digits: 3 x 16 columns

struct TcParams {
    sj_kvarn_layout lay;
    const uint8_t * body;
    const uint32_t * blocks;
    int H, kv0;
    uint32_t S;                 // sink length: record g covers positions S + 128 g ..
    uint32_t n_rec;             // sealed records per head in [S, B)
    uint32_t qpos0;
    int n_q, n_head, grp, rows;
    const float * q;
    float scale;
    float * part;               // [splits][n_q*n_head][D + 2]
    int split0;                 // partial slot of this kernel's first split
    int recs_per_split;
};

// shared memory (bytes)
constexpr uint32_t REC_MAX = 35072;
constexpr uint32_t OFF_REC0 = 0;
constexpr uint32_t OFF_REC1 = REC_MAX;
constexpr uint32_t OFF_BK = 2 * REC_MAX;            // B_K: 16 K chunks (256 channels) x 48 rows
constexpr uint32_t OFF_BV = OFF_BK + 16 * 784;      // B_V: 8 K chunks (128 tokens) x 48 rows
constexpr uint32_t OFF_RED = OFF_BV + 8 * 784;      // 4 reduction areas x 128 floats
constexpr uint32_t OFF_ROW = OFF_RED + 4 * 128 * 4;
constexpr uint32_t OFF_BAR = OFF_ROW + 12 * 16 * 4;
constexpr uint32_t OFF_TMEM = OFF_BAR + 32;
constexpr uint32_t SMEM_TOTAL = OFF_TMEM + 16;
// per-row broadcast arrays (16 floats each) inside OFF_ROW
enum { ROW_C = 0, ROW_KINV = 16, ROW_M2 = 32, ROW_MNEW = 48, ROW_ALPHA = 64, ROW_L = 80, ROW_Z = 96, ROW_MAXK = 112,
       ROW_MAXV = 128, ROW_VSCL = 144, ROW_VINV = 160 };
enum { RED_C = 0, RED_MAX = 128, RED_L = 256, RED_Z = 384 };

// element (n, k) of a K-major, no-swizzle s8 B operand with N = 48 rows, n = 16 digit + query row: 8-row x
// 16-byte core matrices (SBO 128), one 16-element K chunk every BCH = 784 bytes (768 + 16: consecutive chunks
// start 4 banks apart, so the builders' stores are conflict-free); an MMA's 32-element K step spans two
// chunks (LBO = BCH). The three digit planes side by side in N let one MMA produce all three digit sums.
constexpr int NB = 3 * NR;
constexpr uint32_t BCH = 784;
__device__ __forceinline__ uint32_t b_off(int n, int k) { return (uint32_t) (k >> 4) * BCH + (uint32_t) (n * 16 + (k & 15)); }

// 16 consecutive K elements of one 16x16 tile from its 4 fragment-order words (the thread's row is in the
// nibbles selected by `shift`): word j holds elements {2j, 2j+8, 2j+1, 2j+9} -> 4 columns of 4 bytes
__device__ __forceinline__ void unpack16(uint4 w, int shift, uint32_t * col) {
    const uint32_t b0 = (w.x >> shift) & 0x0F0F0F0Fu, b1 = (w.y >> shift) & 0x0F0F0F0Fu;
    const uint32_t b2 = (w.z >> shift) & 0x0F0F0F0Fu, b3 = (w.w >> shift) & 0x0F0F0F0Fu;
    col[0] = prmt(b0, b1, 0x6420u);      // elements 0..3
    col[1] = prmt(b2, b3, 0x6420u);      // 4..7
    col[2] = prmt(b0, b1, 0x7531u);      // 8..11
    col[3] = prmt(b2, b3, 0x7531u);      // 12..15
}

__global__ void __launch_bounds__(NT, 2) attend_body_tc_kernel(TcParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int quarter = warp & 3, half = warp >> 2, tl = quarter * 32 + lane;   // tl: this thread's TMEM lane
    const int hl = blockIdx.y, h = p.kv0 + hl, split = blockIdx.x;
    const sj_kvarn_layout & l = p.lay;
    auto rec_buf = [&](uint32_t b) -> uint8_t * { return sm + OFF_REC0 + b * REC_MAX; };
    uint8_t * bk = sm + OFF_BK;
    uint8_t * bv = sm + OFF_BV;
    float * red = reinterpret_cast<float *>(sm + OFF_RED);
    float * row = reinterpret_cast<float *>(sm + OFF_ROW);
    uint64_t * bars = reinterpret_cast<uint64_t *>(sm + OFF_BAR);    // [0],[1] record loads, [2] MMAs
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(sm + OFF_TMEM);

    const uint32_t r_begin = (uint32_t) split * (uint32_t) p.recs_per_split;
    const uint32_t r_end = min(r_begin + (uint32_t) p.recs_per_split, p.n_rec);

    if (warp == 0) { tc::tmem_alloc(tmem_slot, TM_COLS); tc::tmem_relinquish(); }
    if (tid == 0) {
        tc::mbar_init(&bars[0], 1); tc::mbar_init(&bars[1], 1); tc::mbar_init(&bars[2], 1);
        tc::mbar_fence_init();
    }
    if (tid < NR) { row[ROW_M2 + tid] = -INFINITY; row[ROW_L + tid] = 0.0f; }

    // B_K builder role: channels 4bg..4bg+3 x rows 4brg..4brg+3 per thread, query values kept in registers
    const int bg = tid & 63, brg = tid >> 6;
    float qv[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = 4 * brg + i;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float v = 0.0f;
            if (r < p.rows) {
                const int iq = r / p.grp, hq = hl * p.grp + r % p.grp;
                v = p.q[((size_t) iq * p.n_head + hq) * D + 4 * bg + j];
            }
            qv[i][j] = v;
        }
    }
    int kcol[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) kcol[j] = sjk_k_ch(l, 4 * bg + j);
    const int vcol = sjk_v_ch(l, 128 * half + tl);
    // per-row max |q| over the 256 channels (rows 4brg.. live in warps 2brg and 2brg + 1)
    float qmax[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float m = fmaxf(fmaxf(fabsf(qv[i][0]), fabsf(qv[i][1])), fmaxf(fabsf(qv[i][2]), fabsf(qv[i][3])));
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        qmax[i] = m;
    }
    if (lane == 0) for (int i = 0; i < 4; ++i) red[RED_C + warp * 4 + i] = qmax[i];
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
#pragma unroll
    for (int i = 0; i < 4; ++i) qmax[i] = fmaxf(red[RED_C + (2 * brg) * 4 + i], red[RED_C + (2 * brg + 1) * 4 + i]);
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t) (quarter * 32) << 16;
    const uint32_t idesc = tc::idesc_s8(128, NB);
    const float sl2 = p.scale * LOG2E;
    // causal bound of this thread's 8 score rows (8 half + i); rows past p.rows are padding (never valid)
    uint32_t qlim[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = 8 * half + i;
        qlim[i] = r < p.rows ? p.qpos0 + (uint32_t) (r / p.grp) + 1u : 0u;     // positions < qlim are visible
    }

    float acc[NR];                                    // running output of channel 128 half + tl, all rows
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
    bool ok = true;
    uint32_t mma_phase = 0;
    int load_pending = -1;
    bool mma_pending = false;

    auto rec_ptr = [&](uint32_t g) -> const uint8_t * {
        const uint32_t blk = p.blocks ? p.blocks[g] : g;
        return p.body + ((size_t) blk * p.H + h) * l.bytes;
    };
    __syncthreads();                                  // red[] reused below
    if (r_begin < r_end) {
        if (tid == 0) { tc::mbar_expect_tx(&bars[0], l.bytes); tc::bulk_g2s(rec_buf(0), rec_ptr(r_begin), l.bytes, &bars[0]); }
        load_pending = 0;
    }

    for (uint32_t g = r_begin; g < r_end; ++g) {
        const uint32_t it = g - r_begin, buf = it & 1u;
        const uint8_t * rec = rec_buf(buf);
        ok = __syncthreads_and(tc::mbar_wait(&bars[buf], (it >> 1) & 1u));
        if (!ok) break;
        load_pending = -1;
        if (g + 1 < r_end) {
            if (tid == 0) {
                tc::mbar_expect_tx(&bars[buf ^ 1u], l.bytes);
                tc::bulk_g2s(rec_buf(buf ^ 1u), rec_ptr(g + 1), l.bytes, &bars[buf ^ 1u]);
            }
            load_pending = (int) it + 1;
        }
        // ---- A: scales, record-wide maxima, A_K (token tl, channel tiles 8 half .. 8 half + 7) ----
        float ks[4], kz[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) { ks[j] = h2f_at(rec + l.k_scale + 2 * kcol[j]); kz[j] = h2f_at(rec + l.k_zero + 2 * kcol[j]); }
        const float kt = h2f_at(rec + l.k_tok + 2 * tl);
        const float vsc = h2f_at(rec + l.v_scale + 2 * tl);
        const float vz = h2f_at(rec + l.v_zero + 2 * tl);
        const float vc = h2f_at(rec + l.v_ch + 2 * vcol);
        {
            float mk = fmaxf(fmaxf(fabsf(ks[0]), fabsf(ks[1])), fmaxf(fabsf(ks[2]), fabsf(ks[3])));
            float mv = fabsf(vsc);
            for (int o = 16; o; o >>= 1) {
                mk = fmaxf(mk, __shfl_xor_sync(0xFFFFFFFFu, mk, o));
                mv = fmaxf(mv, __shfl_xor_sync(0xFFFFFFFFu, mv, o));
            }
            if (lane == 0) { row[ROW_MAXK + warp] = mk; row[ROW_MAXV + warp] = mv; }
        }
        {
            const int t = tl, shift = (t & 8) ? 4 : 0;
            const uint8_t * kp = rec + l.k_payload;
            uint32_t colv[16];
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8) {
                const int c = 8 * half + c8;
                const uint4 w = *reinterpret_cast<const uint4 *>(kp + ((((t >> 4) * 16 + c) * 32) + 4 * (t & 7)) * 4);
                unpack16(w, shift, colv + 4 * (c8 & 3));
                if ((c8 & 3) == 3) tc::st_x16(tmem + lane_base + COL_AK + 32 * half + 16 * (c8 >> 2), colv);
            }
        }
        __syncthreads();                                                          // S1
        // ---- B: B_K = three s8 digits of round(Q' 2^e), zero-point partials ----
        {
            float maxk = 0.0f, cz[4];
#pragma unroll
            for (int w = 0; w < 8; ++w) maxk = fmaxf(maxk, row[ROW_MAXK + w]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = 4 * brg + i;
                const float bound = qmax[i] * maxk;
                const int e = (bound > 0.0f && bound < INFINITY) ? 21 - pow2_exp(bound) : 0;
                const float sc = pow2f(e);
                if (bg == 0) row[ROW_KINV + r] = pow2f(-e);
                // digits of the 4 channels (bytes 0..2 of z_j) transposed into one word per digit plane
                const uint32_t z0 = digits3(qv[i][0] * ks[0], sc), z1 = digits3(qv[i][1] * ks[1], sc);
                const uint32_t z2 = digits3(qv[i][2] * ks[2], sc), z3 = digits3(qv[i][3] * ks[3], sc);
                const uint32_t a = prmt(z0, z1, 0x5140u), b = prmt(z2, z3, 0x5140u);   // [z0.0 z1.0 z0.1 z1.1]
                const uint32_t off = b_off(r, 4 * bg);
                *reinterpret_cast<uint32_t *>(bk + off) = prmt(a, b, 0x5410u);
                *reinterpret_cast<uint32_t *>(bk + off + 256) = prmt(a, b, 0x7632u);
                *reinterpret_cast<uint32_t *>(bk + off + 512) = prmt(prmt(z0, z1, 0x0062u), prmt(z2, z3, 0x0062u), 0x5410u);
                cz[i] = (qv[i][0] * kz[0] + qv[i][1] * kz[1]) + (qv[i][2] * kz[2] + qv[i][3] * kz[3]);
            }
            const float c = warp_sum_rows4(cz[0], cz[1], cz[2], cz[3], lane);
            if ((lane & 7) == 0) red[RED_C + warp * 4 + (lane >> 3)] = c;
        }
        tc::wait_st();
        tc::fence_proxy_async();
        tc::fence_before_sync();
        __syncthreads();                                                          // S2
        tc::fence_after_sync();
        if (tid == 0) {
#pragma unroll 1
            for (int k = 0; k < D / 32; ++k)
                tc::mma_ts_i8(tmem + COL_S, tmem + COL_AK + 8 * k, tc::smem_desc(bk + 2 * BCH * k, BCH, 128), idesc, k ? 1u : 0u);
            tc::mma_commit(&bars[2]);
        }
        mma_pending = true;
        if (tid < NR) row[ROW_C + tid] = red[RED_C + (2 * (tid >> 2)) * 4 + (tid & 3)] + red[RED_C + (2 * (tid >> 2) + 1) * 4 + (tid & 3)];
        // ---- C: A_V (channel 128 half + tl over the 8 token tiles), overlapping the K MMAs ----
        {
            const int d = 128 * half + tl, shift = (d & 8) ? 4 : 0;
            const uint8_t * vp = rec + l.v_payload;
            uint32_t colv[16];
#pragma unroll
            for (int s8 = 0; s8 < 8; ++s8) {
                const uint4 w = *reinterpret_cast<const uint4 *>(vp + (((s8 * 16 + (d >> 4)) * 32) + 4 * (d & 7)) * 4);
                unpack16(w, shift, colv + 4 * (s8 & 3));
                if ((s8 & 3) == 3) tc::st_x16(tmem + lane_base + COL_AV + 32 * half + 16 * (s8 >> 2), colv);
            }
        }
        tc::wait_st();
        ok = __syncthreads_and(tc::mbar_wait(&bars[2], mma_phase));              // S3: K MMAs done
        if (!ok) break;
        mma_phase ^= 1u;
        mma_pending = false;
        tc::fence_after_sync();
        // ---- D: scores of token tl for rows 8 half .. 8 half + 7, log2 domain; row maxima ----
        float s2[8];
        {
            uint32_t a0[8], a1[8], a2[8];
            tc::ld_x8_u(tmem + lane_base + COL_S + 8 * half, a0);
            tc::ld_x8_u(tmem + lane_base + COL_S + 16 + 8 * half, a1);
            tc::ld_x8_u(tmem + lane_base + COL_S + 32 + 8 * half, a2);
            tc::wait_ld();
            const uint32_t pos = p.S + g * (uint32_t) G + (uint32_t) tl;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = 8 * half + i;
                const float S = fmaf(65536.0f, i2f(a2[i]), fmaf(256.0f, i2f(a1[i]), i2f(a0[i])));
                const float dot = kt * fmaf(S, row[ROW_KINV + r], row[ROW_C + r]);
                s2[i] = pos < qlim[i] ? dot * sl2 : -INFINITY;
            }
            const float mw = warp_rows8<true>(s2, lane);
            if ((lane & 3) == 0) red[RED_MAX + half * 32 + quarter * 8 + (lane >> 2)] = mw;
        }
        __syncthreads();                                                          // S4
        if (tid < NR) {
            const int hh = tid >> 3, rr = tid & 7;
            const float * mr = red + RED_MAX + hh * 32 + rr;
            const float mrec = fmaxf(fmaxf(mr[0], mr[8]), fmaxf(mr[16], mr[24]));
            const float mold = row[ROW_M2 + tid], mnew = fmaxf(mold, mrec);
            row[ROW_MNEW + tid] = mnew;
            row[ROW_ALPHA + tid] = mnew == -INFINITY ? 1.0f : ex2(mold - mnew);
            row[ROW_M2 + tid] = mnew;
            // P' = p Vscale of this row is at most ex2(mrec - mnew) * max Vscale: rescale it to < 2^21
            float maxv = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; ++w) maxv = fmaxf(maxv, row[ROW_MAXV + w]);
            const float bound = (mrec == -INFINITY ? 0.0f : ex2(mrec - mnew)) * maxv;
            const int ev = (bound > 0.0f && bound < INFINITY) ? 21 - pow2_exp(bound) : 0;
            row[ROW_VSCL + tid] = pow2f(ev);
            row[ROW_VINV + tid] = pow2f(-ev);
        }
        __syncthreads();                                                          // S5
        // ---- E: weights p, B_V = two s8 digits of round(P' 2^ev), row sums ----
        {
            float ls[8], zs[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = 8 * half + i;
                const float mnew = row[ROW_MNEW + r];
                const float pw = mnew == -INFINITY ? 0.0f : ex2(s2[i] - mnew);
                ls[i] = pw;
                zs[i] = pw * vz;
                const uint32_t z = digits3(pw * vsc, row[ROW_VSCL + r]);
                const uint32_t off = b_off(r, tl);
                bv[off] = (uint8_t) z;
                bv[off + 256] = (uint8_t) (z >> 8);
                bv[off + 512] = (uint8_t) (z >> 16);
            }
            const float lw = warp_rows8<false>(ls, lane);
            const float zw = warp_rows8<false>(zs, lane);
            if ((lane & 3) == 0) {
                red[RED_L + half * 32 + quarter * 8 + (lane >> 2)] = lw;
                red[RED_Z + half * 32 + quarter * 8 + (lane >> 2)] = zw;
            }
        }
        tc::fence_proxy_async();
        tc::fence_before_sync();
        __syncthreads();                                                          // S6
        tc::fence_after_sync();
        if (tid == 0) {
#pragma unroll 1
            for (int tile = 0; tile < 2; ++tile)
                for (int k = 0; k < G / 32; ++k)
                    tc::mma_ts_i8(tmem + COL_O + 48 * tile, tmem + COL_AV + 32 * tile + 8 * k,
                                  tc::smem_desc(bv + 2 * BCH * k, BCH, 128), idesc, k ? 1u : 0u);
            tc::mma_commit(&bars[2]);
        }
        mma_pending = true;
        if (tid < NR) {
            const int hh = tid >> 3, rr = tid & 7;
            const float * lr = red + RED_L + hh * 32 + rr;
            const float * zr = red + RED_Z + hh * 32 + rr;
            row[ROW_L + tid] = row[ROW_L + tid] * row[ROW_ALPHA + tid] + ((lr[0] + lr[8]) + (lr[16] + lr[24]));
            row[ROW_Z + tid] = (zr[0] + zr[8]) + (zr[16] + zr[24]);
        }
        ok = __syncthreads_and(tc::mbar_wait(&bars[2], mma_phase));              // S7: V MMAs done
        if (!ok) break;
        mma_phase ^= 1u;
        mma_pending = false;
        tc::fence_after_sync();
        // ---- F: epilogue, channel 128 half + tl ----
        {
            uint32_t o0[16], o1[16], o2[16];
            tc::ld_x16_u(tmem + lane_base + COL_O + 48 * half, o0);
            tc::ld_x16_u(tmem + lane_base + COL_O + 48 * half + 16, o1);
            tc::ld_x16_u(tmem + lane_base + COL_O + 48 * half + 32, o2);
            tc::wait_ld();
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const float O = fmaf(65536.0f, i2f(o2[r]), fmaf(256.0f, i2f(o1[r]), i2f(o0[r]))) * row[ROW_VINV + r];
                acc[r] = fmaf(acc[r], row[ROW_ALPHA + r], vc * (O + row[ROW_Z + r]));
            }
        }
        tc::fence_before_sync();
        __syncthreads();                                                          // S8
        tc::fence_after_sync();
    }

    // ---- drain: a timed-out CTA still waits (bounded) for its own copies and MMAs before releasing TMEM ----
    if (!ok) {
        if (load_pending >= 0) tc::mbar_wait(&bars[load_pending & 1], ((uint32_t) load_pending >> 1) & 1u);
        if (mma_pending) tc::mbar_wait(&bars[2], mma_phase);
    }
    // ---- partials (m in the natural-log domain, l, o[D]) per real query row ----
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

// ---- host side ---------------------------------------------------------------------------------------------

// Whether the tensor-core body path applies: 4-bit scalar records (fragment-ordered payload), D = 256,
// at most 16 query rows per KV head.
int sjk_tc_body_supported(const sjk_view * v, int n_q, int grp) {
    const sj_kvarn_layout & l = v->lay;
    return l.D == 256 && l.G == 128 && l.body == SJKVARN_BODY_SCALAR && l.bits_k == 4 && l.bits_v == 4 &&
           n_q * grp <= NR && l.bytes == REC_MAX;
}

int sjk_tc_body_splits(uint32_t n_rec, int n_kv, int * recs_per_split) {
    if (n_rec == 0) { *recs_per_split = 1; return 0; }
    const int target = (2 * 148 + n_kv - 1) / n_kv;            // two CTAs per SM over the call's KV heads
    int rps = (int) ((n_rec + (uint32_t) target - 1) / (uint32_t) target);
    if (rps < 1) rps = 1;
    *recs_per_split = rps;
    return (int) ((n_rec + (uint32_t) rps - 1) / (uint32_t) rps);
}

int sjk_tc_body_launch(const sjk_view * v, uint32_t n_rec, uint32_t qpos0, int n_q, int n_head, int kv0, int n_kv,
                       const float * q, float scale, float * part, int split0, int splits, int recs_per_split,
                       sjk_stream st) {
    TcParams p;
    p.lay = v->lay; p.body = v->body; p.blocks = v->blocks; p.H = v->n_head_kv; p.kv0 = kv0; p.S = v->S;
    p.n_rec = n_rec; p.qpos0 = qpos0; p.n_q = n_q; p.n_head = n_head; p.grp = n_head / n_kv; p.rows = n_q * p.grp;
    p.q = q; p.scale = scale; p.part = part; p.split0 = split0; p.recs_per_split = recs_per_split;
    cudaError_t e = cudaFuncSetAttribute(attend_body_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_TOTAL);
    if (e != cudaSuccess) return sjk_check(e);
    attend_body_tc_kernel<<<dim3((unsigned) splits, (unsigned) n_kv), NT, SMEM_TOTAL, st>>>(p);
    return sjk_check_launch();
}

extern "C" int sjk_device_status(void) {
    int v = 0, zero = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    if (cudaMemcpyFromSymbol(&v, sjk_dev_status, sizeof v) != cudaSuccess) return -1;
    cudaMemcpyToSymbol(sjk_dev_status, &zero, sizeof zero);
    return v;
}
