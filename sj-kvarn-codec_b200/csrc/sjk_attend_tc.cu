// sjk_attend_tc.cu - tensor-core (tcgen05, kind::i8) attention over the sealed body of a 4-bit scalar layer.
//
// Per record (128 tokens x 256 channels of one KV head) the query rows of the head (decode width x GQA
// group, padded to 16) meet the codes on the tensor core:
//
//   K side  S^T[t, r] = sum_d code_K[t, d] * Q'[r, d],   Q'[r, d] = q[r, d] * Kscale[d]
//           dot[t, r] = Ktok[t] * (S^T[t, r] + sum_d q[r, d] * Kzero[d])
//   V side  O^T[d, r] = sum_t code_V[d, t] * P'[r, t],   P'[r, t] = p[r, t] * Vscale[t]
//           out[d, r] = Vch[d] * (O^T[d, r] + sum_t p[r, t] * Vzero[t])
//
// i.e. the reference reconstruction K = (q*Ks + Kz)*Kt, V = (q*Vs + Vz)*Vc (sj_kvarn.h:1187-1207) regrouped
// so the 4-bit codes enter the tensor core as exact signed 8-bit integers (A operand in TMEM, unpacked from
// the fragment-ordered payload with LOP3/PRMT). Q' and P' are rounded to integers after an exact power-of-two
// rescale (Q' per query row below 2^21, P' per row and record below 2^20) and split into three signed 8-bit
// digits placed side by side in the MMA's N dimension (N = 3 x 16), so one MMA accumulates all three digit
// sums exactly in s32; the digits recombine in fp32 (scores) or in s32 (outputs, which stay below 2^31).
//
// The kernel is persistent and warp-specialized: one CTA (544 threads) per SM walks a contiguous range of
// records of one KV head with three roles that overlap consecutive records:
//   warp 16, lane 0  issuer   bulk copies of records into a 3-stage ring; the K MMAs of record g + 1 ahead of
//                             the V MMAs of record g; commits
//   warps 0-7        unpack   A_K / A_V (TMEM, double-buffered) and the B_K digits (shared, double-buffered)
//   warps 8-15       softmax  scores, online softmax, the B_V digits, and the epilogue of the previous record
// Warp w of a group works on TMEM lane quarter w % 4 and on half w / 4 of the rows, channels or tiles.
// linked by mbarriers. TMEM (512 columns): A_K[2] 0/64, A_V[2] 128/192, O[2] 256/352 (2 tiles x 48), S 448.
// Every wait is bounded (sjk_tc.cuh); a role whose wait runs out stops, the others run out in turn, and the
// issuer drains its own copies and MMAs before the TMEM is released.
#include "sjk_common.cuh"
#include "sjk_internal.h"
#include "sjk_tc.cuh"

namespace {

using namespace tc::num;

constexpr int NR = 16;                  // query rows per KV head, padded
constexpr int NB = 3 * NR;              // MMA N: three digit planes x 16 rows
constexpr int D = 256;
constexpr int G = 128;
constexpr int NT = 544;                 // 8 unpack warps, 8 softmax warps, 1 issuer warp
constexpr int NW = 8;                   // warps per group
constexpr uint32_t NS = 3;              // record stages
constexpr uint32_t TM_COLS = 512;
constexpr uint32_t COL_AK = 0, COL_AV = 128, COL_O = 256, COL_S = 448;

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

// B operands: K-major, no swizzle, N = 48 rows (n = 16 digit + query row), 8-row x 16-byte core matrices
// (SBO 128), one 16-element K chunk every BCH = 784 bytes (768 + 16: consecutive chunks start 4 banks apart,
// so the builders' stores are conflict-free); an MMA's 32-element K step spans two chunks (LBO = BCH).
constexpr uint32_t BCH = 784;
__device__ __forceinline__ uint32_t b_off(int n, int k) { return (uint32_t) (k >> 4) * BCH + (uint32_t) (n * 16 + (k & 15)); }

// shared memory (bytes)
constexpr uint32_t REC_MAX = 35072;
constexpr uint32_t OFF_REC = 0;                               // NS x record
constexpr uint32_t OFF_BK = OFF_REC + NS * REC_MAX;           // 2 x (16 chunks x BCH)
constexpr uint32_t OFF_BV = OFF_BK + 2 * 16 * BCH;            // 2 x (8 chunks x BCH)
constexpr uint32_t OFF_F = OFF_BV + 2 * 8 * BCH;              // float arrays below
enum : uint32_t {                                             // offsets in floats from OFF_F (16-byte aligned arrays)
    F_KINV = 0,        // [2][16]       2^-e of the Q' rescale per buffer
    F_CPART = 32,      // [2][8][4]     zero-point partials per unpack warp (warps 2i, 2i+1: rows 4i..4i+3)
    F_QMAX = 96,       // [8][4]        per-unpack-warp row maxima of |q|
    F_UMAX2 = 128,     // [2][8]        max |Kscale| per unpack warp, per buffer
    F_M2 = 144,        // [2][16]       running max (log2 domain) after the record of each buffer
    F_ALPHA = 176,     // [2][16]       rescale of the running sums when the record of each buffer arrived
    F_VINV = 208,      // [2][16]       2^-ev of the P' rescale per buffer
    F_RMAXV = 240,     // [2][8]        per-softmax-warp max |Vscale|
    F_RMAX = 256,      // [2][2][4][8]  row maxima of the scores per (buffer, row half, lane quarter)
    F_RL = 384,        // [2][2][4][8]  row sums of p
    F_RZ = 512,        // [2][2][4][8]  row sums of p Vzero
    F_LSUM = 640,      // [16]          running sums of p
    F_END = 656
};
constexpr uint32_t OFF_BAR = OFF_F + F_END * 4;
enum : uint32_t {                                             // mbarrier indices
    B_RFULL = 0, B_REMPTY = 3, B_AK = 6, B_AV = 8, B_SFULL = 10, B_SFREE = 11, B_BV = 12, B_VDONE = 14, B_OFREE = 16,
    B_COUNT = 18
};
constexpr uint32_t OFF_TMEM = OFF_BAR + B_COUNT * 8;
constexpr uint32_t SMEM_TOTAL = OFF_TMEM + 16;

// The 4-bit payloads are in 16x16-tile fragment order: the 4 words of one tile row group hold, for rows
// i and i + 8 (low / high nibbles), word j = elements {2j, 2j+8, 2j+1, 2j+9} of the tile's k index. The
// A operands keep that order - k position p of a tile holds element PI(p) - and the B operands are built
// with the same permutation of their k rows, which leaves every product sum unchanged.
__device__ __forceinline__ int pi_elem(int p) { return ((p >> 2) << 1) + ((p >> 1) & 1) + ((p & 1) << 3); }
__device__ __forceinline__ int pi_pos(int e) { return 2 * (e & 7) + (e >> 3); }     // inverse of pi_elem

// 16 k bytes (payload order) of the thread's row of one tile from its 4 fragment words
__device__ __forceinline__ void unpack16(uint4 w, int shift, uint32_t * col) {
    col[0] = (w.x >> shift) & 0x0F0F0F0Fu;
    col[1] = (w.y >> shift) & 0x0F0F0F0Fu;
    col[2] = (w.z >> shift) & 0x0F0F0F0Fu;
    col[3] = (w.w >> shift) & 0x0F0F0F0Fu;
}

// lane 0 of the warp arrives on `bar` once every lane of the warp got here (after their fences)
__device__ __forceinline__ void warp_arrive(uint64_t * bar, int lane) {
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(bar);
}

__global__ void __launch_bounds__(NT, 1) attend_body_tc_kernel(TcParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hl = blockIdx.y, h = p.kv0 + hl, split = blockIdx.x;
    const sj_kvarn_layout & l = p.lay;
    float * F = reinterpret_cast<float *>(sm + OFF_F);
    uint64_t * bars = reinterpret_cast<uint64_t *>(sm + OFF_BAR);
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(sm + OFF_TMEM);
    const uint32_t r_begin = (uint32_t) split * (uint32_t) p.recs_per_split;
    const uint32_t r_end = min(r_begin + (uint32_t) p.recs_per_split, p.n_rec);
    const uint32_t n = r_end > r_begin ? r_end - r_begin : 0u;

    if (warp == 2 * NW) { tc::tmem_alloc(tmem_slot, TM_COLS); tc::tmem_relinquish(); }
    if (tid == 2 * NW * 32) {
        for (uint32_t i = 0; i < NS; ++i) { tc::mbar_init(&bars[B_RFULL + i], 1); tc::mbar_init(&bars[B_REMPTY + i], 2 * NW); }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&bars[B_AK + i], NW); tc::mbar_init(&bars[B_AV + i], NW); tc::mbar_init(&bars[B_BV + i], NW);
            tc::mbar_init(&bars[B_VDONE + i], 1); tc::mbar_init(&bars[B_OFREE + i], NW);
        }
        tc::mbar_init(&bars[B_SFULL], 1); tc::mbar_init(&bars[B_SFREE], NW);
        tc::mbar_fence_init();
    }
    if (tid < 2 * NR) F[F_M2 + tid] = -INFINITY;
    if (tid < NR) F[F_LSUM + tid] = 0.0f;
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;

    if (warp < NW) {
        // ================= unpack: A_K, B_K (+ zero-point partials), A_V of record g =================
        const int u = tid, quarter = warp & 3, half = warp >> 2, tl = quarter * 32 + lane;
        const int bg = u & 63, brg = u >> 6;                     // B_K: k positions 4 bg.., rows 4 brg..
        int kch[4];                                              // channels at those k positions
#pragma unroll
        for (int j = 0; j < 4; ++j) kch[j] = 16 * (bg >> 2) + pi_elem(4 * (bg & 3) + j);
        const uint32_t lane_base = (uint32_t) (quarter * 32) << 16;
        float qv[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = 4 * brg + i;
#pragma unroll
            for (int j = 0; j < 4; ++j) qv[i][j] = 0.0f;
            if (r < p.rows) {
                const int iq = r / p.grp, hq = hl * p.grp + r % p.grp;
                const float * qr = p.q + ((size_t) iq * p.n_head + hq) * D;
#pragma unroll
                for (int j = 0; j < 4; ++j) qv[i][j] = qr[kch[j]];
            }
        }
        float qmax[4];
        {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float m = fmaxf(fmaxf(fabsf(qv[i][0]), fabsf(qv[i][1])), fmaxf(fabsf(qv[i][2]), fabsf(qv[i][3])));
                for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
                qmax[i] = m;
            }
            if (lane == 0)
                for (int i = 0; i < 4; ++i) F[F_QMAX + warp * 4 + i] = qmax[i];
            tc::nbar_sync(1, NW * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) qmax[i] = fmaxf(F[F_QMAX + (2 * brg) * 4 + i], F[F_QMAX + (2 * brg + 1) * 4 + i]);
        }
        int kcol[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) kcol[j] = sjk_k_ch(l, kch[j]);
        const int shift = (tl & 8) ? 4 : 0;                      // the thread's row nibbles (token tl / channel tl)
        for (uint32_t g = 0; g < n; ++g) {
            const uint32_t s = g % NS, b = g & 1u;
            const uint8_t * rec = sm + OFF_REC + s * REC_MAX;
            // A_K[b] and B_K[b] were last read by the K MMAs of record g - 2: done once those of g - 1 are
            bool w_ok = tc::mbar_wait(&bars[B_RFULL + s], (g / NS) & 1u);
            if (g >= 1) w_ok = w_ok && tc::mbar_wait(&bars[B_SFULL], (g - 1) & 1u);
            float ks[4], kz[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) { ks[j] = h2f_at(rec + l.k_scale + 2 * kcol[j]); kz[j] = h2f_at(rec + l.k_zero + 2 * kcol[j]); }
            {
                float mk = fmaxf(fmaxf(fabsf(ks[0]), fabsf(ks[1])), fmaxf(fabsf(ks[2]), fabsf(ks[3])));
                for (int o = 16; o; o >>= 1) mk = fmaxf(mk, __shfl_xor_sync(0xFFFFFFFFu, mk, o));
                if (lane == 0) F[F_UMAX2 + 8 * b + warp] = mk;
            }
            ok = tc::nbar_and(1, NW * 32, ok && w_ok);
            if (!ok) break;
            tc::fence_after_sync();
            float maxk = 0.0f;
#pragma unroll
            for (int w = 0; w < NW; ++w) maxk = fmaxf(maxk, F[F_UMAX2 + 8 * b + w]);
            // ---- A_K: token tl, channel tiles 8 half .. 8 half + 7 ----
            {
                const uint8_t * kp = rec + l.k_payload;
                uint32_t col[16];
#pragma unroll
                for (int c8 = 0; c8 < 8; ++c8) {
                    const int c = 8 * half + c8;
                    const uint4 w = *reinterpret_cast<const uint4 *>(kp + ((((tl >> 4) * 16 + c) * 32) + 4 * (tl & 7)) * 4);
                    unpack16(w, shift, col + 4 * (c8 & 3));
                    if ((c8 & 3) == 3) tc::st_x16(tmem + lane_base + COL_AK + 64 * b + 32 * half + 16 * (c8 >> 2), col);
                }
            }
            // ---- B_K: three s8 digits of round(Q' 2^e), zero-point partials ----
            {
                uint8_t * bk = sm + OFF_BK + b * 16 * BCH;
                float cz[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = 4 * brg + i;
                    const float bound = qmax[i] * maxk;
                    const int e = (bound > 0.0f && bound < INFINITY) ? 21 - pow2_exp(bound) : 0;
                    const float sc = pow2f(e);
                    if (bg == 0) F[F_KINV + 16 * b + r] = pow2f(-e);
                    const uint32_t z0 = digits3(qv[i][0] * ks[0], sc), z1 = digits3(qv[i][1] * ks[1], sc);
                    const uint32_t z2 = digits3(qv[i][2] * ks[2], sc), z3 = digits3(qv[i][3] * ks[3], sc);
                    const uint32_t a = prmt(z0, z1, 0x5140u), c = prmt(z2, z3, 0x5140u);   // [z0.0 z1.0 z0.1 z1.1]
                    const uint32_t off = b_off(r, 4 * bg);
                    *reinterpret_cast<uint32_t *>(bk + off) = prmt(a, c, 0x5410u);
                    *reinterpret_cast<uint32_t *>(bk + off + 256) = prmt(a, c, 0x7632u);
                    *reinterpret_cast<uint32_t *>(bk + off + 512) = prmt(prmt(z0, z1, 0x0062u), prmt(z2, z3, 0x0062u), 0x5410u);
                    cz[i] = (qv[i][0] * kz[0] + qv[i][1] * kz[1]) + (qv[i][2] * kz[2] + qv[i][3] * kz[3]);
                }
                const float cw = warp_sum_rows4(cz[0], cz[1], cz[2], cz[3], lane);
                if ((lane & 7) == 0) F[F_CPART + 32 * b + warp * 4 + (lane >> 3)] = cw;
            }
            tc::wait_st();
            tc::fence_proxy_async();
            tc::fence_before_sync();
            warp_arrive(&bars[B_AK + b], lane);
            // ---- A_V: channel 128 half + tl over the 8 token tiles; A_V[b] was last read by the V MMAs of g - 2 ----
            if (g >= 2) ok = __all_sync(0xFFFFFFFFu, tc::mbar_wait(&bars[B_VDONE + b], ((g - 2) >> 1) & 1u));
            tc::fence_after_sync();
            if (ok) {
                const uint8_t * vp = rec + l.v_payload;
                const int d = 128 * half + tl;
                uint32_t col[16];
#pragma unroll
                for (int s8 = 0; s8 < 8; ++s8) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(vp + (((s8 * 16 + (d >> 4)) * 32) + 4 * (d & 7)) * 4);
                    unpack16(w, shift, col + 4 * (s8 & 3));
                    if ((s8 & 3) == 3) tc::st_x16(tmem + lane_base + COL_AV + 64 * b + 32 * half + 16 * (s8 >> 2), col);
                }
                tc::wait_st();
                tc::fence_before_sync();
                warp_arrive(&bars[B_AV + b], lane);
            }
            warp_arrive(&bars[B_REMPTY + s], lane);
        }
    } else if (warp < 2 * NW) {
        // ===== softmax: scores and weights of record g, B_V digits, then the epilogue of record g - 1 =====
        // Thread (quarter, half, lane): token tl of the record for rows 8 half .. 8 half + 7, and channel
        // 128 half + tl of the output for all rows. Lane 0 of the quarter-0 warps keeps the running sums l.
        const int sw = warp - NW, quarter = sw & 3, half = sw >> 2, tl = quarter * 32 + lane;
        const bool keeper = quarter == 0 && lane == 0;
        const uint32_t lane_base = (uint32_t) (quarter * 32) << 16;
        const float sl2 = p.scale * LOG2E;
        uint32_t qlim[8];                                        // rows 8 half + i: positions < qlim are visible
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = 8 * half + i;
            qlim[i] = r < p.rows ? p.qpos0 + (uint32_t) (r / p.grp) + 1u : 0u;
        }
        const int vcol = sjk_v_ch(l, 128 * half + tl);           // epilogue channel 128 half + tl
        float acc[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
        float vc_n = 0.0f, vc_e = 0.0f;                          // Vch: newest record / record of the next epilogue
        for (uint32_t g = 0; g <= n; ++g) {                      // pass n only finishes record n - 1
            const uint32_t b = g & 1u, pb = b ^ 1u;
            if (g < n) {
                const uint32_t s = g % NS;
                const uint8_t * rec = sm + OFF_REC + s * REC_MAX;
                bool w_ok = tc::mbar_wait(&bars[B_RFULL + s], (g / NS) & 1u);
                w_ok = w_ok && tc::mbar_wait(&bars[B_SFULL], g & 1u);
                w_ok = w_ok && tc::mbar_wait(&bars[B_AK + b], (g >> 1) & 1u);
                tc::fence_after_sync();
                uint32_t a0[8], a1[8], a2[8];
                tc::ld_x8_u(tmem + lane_base + COL_S + 8 * half, a0);
                tc::ld_x8_u(tmem + lane_base + COL_S + 16 + 8 * half, a1);
                tc::ld_x8_u(tmem + lane_base + COL_S + 32 + 8 * half, a2);
                // per-row constants of the K side (buffer b is rewritten for record g + 2 after S is released)
                float kinv[8], cp0[8], cp1[8];
                ld8(F + F_KINV + 16 * b + 8 * half, kinv);
                ld8(F + F_CPART + 32 * b + 16 * half, cp0);      // rows 8 half + 0..3 (two warps), then 4..7
                ld8(F + F_CPART + 32 * b + 16 * half + 8, cp1);
                tc::wait_ld();
                tc::fence_before_sync();
                warp_arrive(&bars[B_SFREE], lane);
                const float kt = h2f_at(rec + l.k_tok + 2 * tl);
                const float vsc = h2f_at(rec + l.v_scale + 2 * tl), vz = h2f_at(rec + l.v_zero + 2 * tl);
                vc_e = vc_n;
                vc_n = h2f_at(rec + l.v_ch + 2 * vcol);
                warp_arrive(&bars[B_REMPTY + s], lane);
                // ---- scores of token tl for rows 8 half .. 8 half + 7 (log2 domain), row maxima, max |Vscale| ----
                float s2[8];
                {
                    const uint32_t pos = p.S + (r_begin + g) * (uint32_t) G + (uint32_t) tl;
                    const float kts = kt * sl2;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float C = i < 4 ? cp0[i] + cp0[i + 4] : cp1[i - 4] + cp1[i];
                        // digit sums: |a0|, |a1| < 2^19, so a0 + 256 a1 is exact in s32
                        const float S = fmaf(65536.0f, i2f(a2[i]), (float) ((int) a0[i] + ((int) a1[i] << 8)));
                        s2[i] = pos < qlim[i] ? kts * fmaf(S, kinv[i], C) : -INFINITY;
                    }
                    const float mw = warp_rows8<true>(s2, lane);
                    if ((lane & 3) == 0) F[F_RMAX + 64 * b + 32 * half + 8 * quarter + (lane >> 2)] = mw;
                    float mv = fabsf(vsc);
                    for (int o = 16; o; o >>= 1) mv = fmaxf(mv, __shfl_xor_sync(0xFFFFFFFFu, mv, o));
                    if (lane == 0) F[F_RMAXV + 8 * b + sw] = mv;
                }
                ok = tc::nbar_and(2, NW * 32, ok && w_ok);
                if (!ok) break;
                // ---- row statistics: lane i (mod 8) of each warp computes row 8 half + i, then broadcasts ----
                float mnew[8], vscl[8];
                {
                    const int i = lane & 7, r = 8 * half + i;
                    const float mold = F[F_M2 + 16 * pb + r];
                    const float * rm = F + F_RMAX + 64 * b + 32 * half + i;
                    const float mrec = fmaxf(fmaxf(rm[0], rm[8]), fmaxf(rm[16], rm[24]));
                    float mv0[8];
                    ld8(F + F_RMAXV + 8 * b, mv0);
                    const float maxv = fmaxf(fmaxf(fmaxf(mv0[0], mv0[1]), fmaxf(mv0[2], mv0[3])), fmaxf(fmaxf(mv0[4], mv0[5]), fmaxf(mv0[6], mv0[7])));
                    const float mn = fmaxf(mold, mrec);
                    // P' = p Vscale of this row is at most ex2(mrec - mnew) * max |Vscale|: rescale it below 2^20
                    const float bound = (mrec == -INFINITY ? 0.0f : ex2(mrec - mn)) * maxv;
                    const int ev = (bound > 0.0f && bound < INFINITY) ? 20 - pow2_exp(bound) : 0;
                    const float vs = pow2f(ev);
                    if (quarter == 0 && lane < 8) {                    // the keeper warp of this half records the row
                        if (g >= 1) {                                  // record g - 1 joins the running sum
                            const float * rl = F + F_RL + 64 * pb + 32 * half + i;
                            F[F_LSUM + r] = F[F_LSUM + r] * F[F_ALPHA + 16 * pb + r] + ((rl[0] + rl[8]) + (rl[16] + rl[24]));
                        }
                        F[F_M2 + 16 * b + r] = mn;
                        F[F_ALPHA + 16 * b + r] = mn == -INFINITY ? 1.0f : ex2(mold - mn);
                        F[F_VINV + 16 * b + r] = pow2f(-ev);
                    }
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        mnew[k] = __shfl_sync(0xFFFFFFFFu, mn, k);
                        vscl[k] = __shfl_sync(0xFFFFFFFFu, vs, k);
                    }
                }
                // ---- weights, B_V = three s8 digits of round(P' 2^ev), row sums ----
                {
                    uint8_t * bv = sm + OFF_BV + b * 8 * BCH + b_off(8 * half, (tl & ~15) + pi_pos(tl & 15));
                    float ls[8], zs[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float pw = mnew[i] == -INFINITY ? 0.0f : ex2(s2[i] - mnew[i]);
                        ls[i] = pw;
                        zs[i] = pw * vz;
                        const uint32_t z = digits3(pw * vsc, vscl[i]);
                        bv[16 * i] = (uint8_t) z;
                        bv[16 * i + 256] = (uint8_t) (z >> 8);
                        bv[16 * i + 512] = (uint8_t) (z >> 16);
                    }
                    tc::fence_proxy_async();
                    warp_arrive(&bars[B_BV + b], lane);
                    const float lw = warp_rows8<false>(ls, lane);
                    const float zw = warp_rows8<false>(zs, lane);
                    if ((lane & 3) == 0) {
                        F[F_RL + 64 * b + 32 * half + 8 * quarter + (lane >> 2)] = lw;
                        F[F_RZ + 64 * b + 32 * half + 8 * quarter + (lane >> 2)] = zw;
                    }
                }
            } else {
                vc_e = vc_n;
                tc::nbar_sync(2, NW * 32);                         // the last record's row sums are visible
                if (quarter == 0 && lane < 8 && n >= 1) {
                    const int r = 8 * half + lane;
                    const float * rl = F + F_RL + 64 * pb + 32 * half + lane;
                    F[F_LSUM + r] = F[F_LSUM + r] * F[F_ALPHA + 16 * pb + r] + ((rl[0] + rl[8]) + (rl[16] + rl[24]));
                }
            }
            // ---- epilogue of record g - 1 (buffer pb): channel 128 half + tl, all rows ----
            if (g >= 1) {
                const uint32_t pg = g - 1;
                // warp-uniform: the TMEM loads below are .sync.aligned
                const bool e_ok = __all_sync(0xFFFFFFFFu, tc::mbar_wait(&bars[B_VDONE + pb], (pg >> 1) & 1u));
                tc::fence_after_sync();
                if (e_ok) {
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh) {                // rows 8 hh .. 8 hh + 7
                        uint32_t o0[8], o1[8], o2[8];
                        const uint32_t oc = tmem + lane_base + COL_O + 96 * pb + 48 * half + 8 * hh;
                        tc::ld_x8_u(oc, o0);
                        tc::ld_x8_u(oc + 16, o1);
                        tc::ld_x8_u(oc + 32, o2);
                        float al[8], vi[8], za[8], zc[8], zd[8], ze[8];
                        ld8(F + F_ALPHA + 16 * pb + 8 * hh, al);
                        ld8(F + F_VINV + 16 * pb + 8 * hh, vi);
                        ld8(F + F_RZ + 64 * pb + 32 * hh, za); ld8(F + F_RZ + 64 * pb + 32 * hh + 8, zc);
                        ld8(F + F_RZ + 64 * pb + 32 * hh + 16, zd); ld8(F + F_RZ + 64 * pb + 32 * hh + 24, ze);
                        tc::wait_ld();
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            // |sum_t code P''| < 128 * 15 * 2^20 < 2^31: the digit sums recombine exactly in s32
                            const float O = (float) (int) (o0[i] + (o1[i] << 8) + (o2[i] << 16));
                            const float z = (za[i] + zc[i]) + (zd[i] + ze[i]);
                            acc[8 * hh + i] = fmaf(acc[8 * hh + i], al[i], vc_e * fmaf(O, vi[i], z));
                        }
                    }
                }
                tc::fence_before_sync();
                warp_arrive(&bars[B_OFREE + pb], lane);
                ok = ok && e_ok;
            }
        }
        ok = tc::nbar_and(2, NW * 32, ok);
        // ---- partials (m in the natural-log domain, l, o[D]) per real query row ----
        const uint32_t mb = n >= 1 ? (n - 1) & 1u : 1u;
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            if (r < p.rows) {
                const int iq = r / p.grp, hq = hl * p.grp + r % p.grp;
                float * dst = p.part + ((size_t) (p.split0 + split) * p.n_q * p.n_head + (size_t) iq * p.n_head + hq) * (D + 2);
                dst[2 + 128 * half + tl] = ok ? acc[r] : 0.0f;
            }
        }
        if (keeper) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = 8 * half + i;
                if (r < p.rows) {
                    const int iq = r / p.grp, hq = hl * p.grp + r % p.grp;
                    float * dst = p.part + ((size_t) (p.split0 + split) * p.n_q * p.n_head + (size_t) iq * p.n_head + hq) * (D + 2);
                    const float m2 = F[F_M2 + 16 * mb + r];
                    dst[0] = ok ? (m2 == -INFINITY ? m2 : m2 * LN2) : -INFINITY;
                    dst[1] = ok ? F[F_LSUM + r] : 0.0f;
                }
            }
        }
    } else if (lane == 0) {
        // ========================== issuer: record copies, MMAs, commits ==========================
        const uint32_t idesc = tc::idesc_s8(128, NB);
        auto blk_of = [&](uint32_t g) -> uint32_t { return p.blocks ? p.blocks[r_begin + g] : r_begin + g; };
        auto load = [&](uint32_t g, uint32_t blk) {
            const uint32_t s = g % NS;
            tc::mbar_expect_tx(&bars[B_RFULL + s], l.bytes);
            tc::bulk_g2s(sm + OFF_REC + s * REC_MAX, p.body + ((size_t) blk * p.H + h) * l.bytes, l.bytes, &bars[B_RFULL + s]);
        };
        // operand descriptors of buffer b; the k steps add compile-time offsets (a fully unrolled issue sequence
        // with constant offsets issues about 40 % faster than descriptors recomputed in a runtime loop)
        const uint64_t bk_desc0 = tc::smem_desc(sm + OFF_BK, BCH, 128), bv_desc0 = tc::smem_desc(sm + OFF_BV, BCH, 128);
        auto issue_k = [&](uint32_t g) {
            const uint32_t b = g & 1u;
            const uint64_t bd = bk_desc0 + (uint64_t) ((b * 16 * BCH) >> 4);
            const uint32_t a0 = tmem + COL_AK + 64 * b;
#pragma unroll
            for (int k = 0; k < D / 32; ++k)
                tc::mma_ts_i8(tmem + COL_S, a0 + 8 * k, bd + (uint64_t) ((2 * BCH * k) >> 4), idesc, k ? 1u : 0u);
            tc::mma_commit(&bars[B_SFULL]);
        };
        uint32_t loaded = 0, k_issued = 0, v_issued = 0;
        for (; loaded < n && loaded < NS; ++loaded) load(loaded, blk_of(loaded));
        uint32_t next_blk = loaded < n ? blk_of(loaded) : 0u;    // block of the next record to load, read ahead
        if (n) {
            ok = tc::mbar_wait(&bars[B_AK], 0u);
            if (ok) { tc::fence_after_sync(); issue_k(0); ++k_issued; }
        }
        for (uint32_t g = 0; g < n && ok; ++g) {
            const uint32_t b = g & 1u;
            // K MMAs of record g + 1, ahead of the V MMAs of record g
            if (g + 1 < n) {
                ok = tc::mbar_wait(&bars[B_AK + (b ^ 1u)], ((g + 1) >> 1) & 1u);
                if (ok) ok = tc::mbar_wait(&bars[B_SFREE], g & 1u);
                if (!ok) break;
                tc::fence_after_sync();
                issue_k(g + 1);
                ++k_issued;
            }
            ok = tc::mbar_wait(&bars[B_AV + b], (g >> 1) & 1u);
            if (ok) ok = tc::mbar_wait(&bars[B_BV + b], (g >> 1) & 1u);
            if (ok && g >= 2) ok = tc::mbar_wait(&bars[B_OFREE + b], ((g - 2) >> 1) & 1u);
            if (!ok) break;
            tc::fence_after_sync();
            {
                const uint64_t bd = bv_desc0 + (uint64_t) ((b * 8 * BCH) >> 4);
                const uint32_t d0 = tmem + COL_O + 96 * b, a0 = tmem + COL_AV + 64 * b;
#pragma unroll
                for (int tile = 0; tile < 2; ++tile)
#pragma unroll
                    for (int k = 0; k < G / 32; ++k)
                        tc::mma_ts_i8(d0 + 48 * tile, a0 + 32 * tile + 8 * k, bd + (uint64_t) ((2 * BCH * k) >> 4), idesc, k ? 1u : 0u);
                tc::mma_commit(&bars[B_VDONE + b]);
                ++v_issued;
            }
            // the stage of record g takes record g + NS once both consumer groups released it
            if (loaded < n) {
                ok = tc::mbar_wait(&bars[B_REMPTY + g % NS], (g / NS) & 1u);
                if (!ok) break;
                load(loaded, next_blk);
                ++loaded;
                if (loaded < n) next_blk = blk_of(loaded);
            }
        }
        if (!ok) {
            // drain (bounded): the last commits cover every MMA issued; the last NS copies may still be in flight
            if (k_issued) tc::mbar_wait(&bars[B_SFULL], (k_issued - 1) & 1u);
            if (v_issued) tc::mbar_wait(&bars[B_VDONE + ((v_issued - 1) & 1u)], ((v_issued - 1) >> 1) & 1u);
            for (uint32_t j = loaded > NS ? loaded - NS : 0u; j < loaded; ++j)
                tc::mbar_wait(&bars[B_RFULL + j % NS], (j / NS) & 1u);
        }
    }
    __syncwarp();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == 2 * NW) tc::tmem_dealloc(tmem, TM_COLS);
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

// one persistent CTA per SM over the call's KV heads
int sjk_tc_body_splits(uint32_t n_rec, int n_kv, int * recs_per_split) {
    if (n_rec == 0) { *recs_per_split = 1; return 0; }
    const int target = (148 + n_kv - 1) / n_kv;
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

SJK_STATUS_READER(sjk_tc_body_status_take)
