// sjk_attend_trellis.cu - tensor-core (tcgen05, kind::f16) attention over the sealed body of a trellis layer
// (3/3t, 3/2t, 2/2t records: sj_kvarn.h:1025-1109, 1176-1207).
//
// A trellis record stores, per channel d, the codes of its 128 tokens as one channel-major bit stream; the
// value of token t is a codebook entry picked by the window of its code and the 6 stream bits before it
// (sj_kvarn.h:879-900). The decoded rows are
//   K[t, d] = (cb_K[w_K(d, t)] Ks[d] + Kz[d]) Kt[t],      V[t, d] = (cb_V[w_V(d, t)] Vs[t] + Vz[t]) Vc[d]
// and regroup as in the 4-bit kernel:
//   S^T[t, r] = Kt[t] (sum_d cb_K[w_K(d, t)] Q'[r, d] + C[r]),   Q' = q Ks,  C = sum_d q Kz
//   O^T[d, r] = Vc[d] (sum_t cb_V[w_V(d, t)] P'[r, t] + z[r]),   P' = p Vs,  z = sum_t p Vz
// The codebook entries are fp16, so the A operands enter the tensor core exactly; Q' and P' enter as fp16
// hi + lo halves side by side in N (B = [hi | lo], N = 32): one MMA per k step leaves the hi and lo products in
// column groups 0..15 and 16..31, whose sum is the fp32 product to about 2^-22.
//
// Decoding follows the streams: a thread walks 64 codes of one channel with the stream words in registers, so
// every window is one shift and one mask at a compile-time offset. A_V is channel-major (lane = channel), so
// the V values go straight into the thread's TMEM lane; A_K is token-major (lane = token), so the K values go
// through a [token][channel] shared tile first. The codebooks sit in shared memory in 16 interleaved copies
// (lookups by different lanes rarely share a bank).
//
// One CTA (512 threads, 16 warps) per SM walks a contiguous range of one KV head's records; the next record's
// bytes arrive by cp.async.bulk (no multicast) while the current one is processed; the online softmax state
// (m, l, o) per query row goes to the split partials that the merge kernel combines. Waits are bounded.
#include <cuda_fp16.h>

#include "sjk_common.cuh"
#include "sjk_internal.h"
#include "sjk_tc.cuh"

namespace {

using namespace tc::num;

constexpr int NT = 512;
constexpr int NR = 16;
constexpr int NB = 2 * NR;              // B operands: hi rows 0..15, lo rows 16..31
constexpr int D = 256;
constexpr int G = 128;
constexpr uint32_t TM_COLS = 512;
constexpr uint32_t COL_AK = 0, COL_AV = 128, COL_S = 256, COL_O = 288;   // A_K (256 ch) | A_V (2 tiles x 128 t) | S | O0 O1
constexpr int MAX_SPLITS = 148;
constexpr uint32_t REC_MAX = 26880;     // largest trellis record at D = 256 (3/3t)
constexpr int CB_COPIES = 16;

struct TrellisParams {
    sjk_view v;
    int kv0;
    uint32_t S, B, N, qpos0, n_rec;
    int n_q, n_head, grp, rows;
    uint32_t row_iq[NR];        // r / grp
    int row_q[NR];              // iq n_head + r % grp (q row and partial row of r, less hl grp)
    const float * q;
    float scale;
    float * part;
    int split0;
    uint32_t rec_bounds[MAX_SPLITS + 1];
};

// B operand (K-major, no swizzle, 32 rows): element (n, k) at (k / 8) * HCH + n * 16 + (k % 8) * 2 with an
// 8-element K chunk every HCH = 528 bytes (consecutive chunks start 4 banks apart); 128 k per tile
constexpr uint32_t HCH = 528;
constexpr uint32_t TILE_B = 16 * HCH;
__device__ __forceinline__ uint32_t h_off(int n, int k) { return (uint32_t) (k >> 3) * HCH + (uint32_t) (n * 16 + (k & 7) * 2); }

// shared memory (bytes)
constexpr uint32_t TRS = 2 * D + 16;                            // [token][channel] fp16 tile row (conflict-free LDS.128)
constexpr uint32_t OFF_REC = 0;                                 // 2 x record
constexpr uint32_t OFF_TR = OFF_REC + 2 * REC_MAX;              // K values, [128 tokens][256 channels]
constexpr uint32_t OFF_BK = OFF_TR + G * TRS;                   // [Q' hi | Q' lo] over 256 channels: 2 x TILE_B
constexpr uint32_t OFF_BV = OFF_BK + 2 * TILE_B;                // [P' hi | P' lo] over 128 tokens: TILE_B
constexpr uint32_t OFF_CBK = OFF_BV + TILE_B;                   // u32 [512][16]: K codebook, 16 copies
constexpr uint32_t OFF_CBV = OFF_CBK + 512 * CB_COPIES * 4;     // u32 [512][16]: V codebook
constexpr uint32_t OFF_ROW = OFF_CBV + 512 * CB_COPIES * 4;     // per-row floats
constexpr uint32_t OFF_RED = OFF_ROW + 8 * NR * 4;              // reduction partials
constexpr uint32_t OFF_BAR = OFF_RED + 3 * 256 * 4;
constexpr uint32_t OFF_TMEM = OFF_BAR + 4 * 8;
constexpr uint32_t SMEM_TOTAL = OFF_TMEM + 16;
static_assert(SMEM_TOTAL <= 227 * 1024, "shared memory");
enum { ROW_M2 = 0, ROW_MNEW = 16, ROW_ALPHA = 32, ROW_L = 48, ROW_C = 64, ROW_Z = 80 };
enum { RED_MAX = 0, RED_L = 256, RED_Z = 512, RED_C = 512 };    // RED_C shares RED_Z's space (different phases)
enum { BAR_REC = 0, BAR_MMA = 2 };

// The codes of tokens [64 TH, 64 TH + 64) of one channel: stream words from bit 64 TH BITS - 32 on, the word
// before the channel's first reading as zero (the history before token 0). Token 64 TH + j then starts its
// window at bit 26 + j BITS of W for both halves and both widths, since the window is 6 + BITS bits long and
// ends with the token's code.
template <int BITS>
constexpr int window_words() { return (26 + 63 * BITS + 6 + BITS + 31) / 32; }

template <int BITS, int TH>
__device__ __forceinline__ void load_stream(const uint32_t * ch_words, uint32_t (&W)[window_words<BITS>()]) {
    constexpr int base = TH * 2 * BITS - 1;                     // word index of W[0] within the channel
#pragma unroll
    for (int i = 0; i < window_words<BITS>(); ++i) W[i] = (base + i < 0) ? 0u : ch_words[base + i];
}

template <int BITS>
__device__ __forceinline__ uint32_t window_of(const uint32_t (&W)[window_words<BITS>()], int j) {
    const int b = 26 + j * BITS, a = b >> 5, s = b & 31;
    constexpr uint32_t MASK = (1u << (6 + BITS)) - 1u;
    if (s + 6 + BITS <= 32) return (W[a] >> s) & MASK;
    return __funnelshift_r(W[a], W[a + 1], s) & MASK;
}

// fp16 bits of codebook entry idx (copy `c` of 16 interleaved copies)
__device__ __forceinline__ uint32_t cb_at(const uint32_t * tbl, uint32_t idx, int c) { return tbl[idx * CB_COPIES + c]; }

// K side: 64 tokens of channel d into the [token][channel] tile
template <int BITS, int TH>
__device__ __forceinline__ void decode_k(const uint32_t * ch_words, const uint32_t * tbl, int c, uint8_t * tr, int d) {
    uint32_t W[window_words<BITS>()];
    load_stream<BITS, TH>(ch_words, W);
#pragma unroll
    for (int j = 0; j < 64; ++j)
        *reinterpret_cast<uint16_t *>(tr + (64 * TH + j) * TRS + 2 * d) = (uint16_t) cb_at(tbl, window_of<BITS>(W, j), c);
}

// V side: 64 tokens of channel d as fp16 pairs (token 2i low) into the thread's TMEM lane
template <int BITS, int TH>
__device__ __forceinline__ void decode_v(const uint32_t * ch_words, const uint32_t * tbl, int c, uint32_t taddr) {
    uint32_t W[window_words<BITS>()];
    load_stream<BITS, TH>(ch_words, W);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint32_t col[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int j = 32 * h + 2 * i;
            col[i] = prmt(cb_at(tbl, window_of<BITS>(W, j), c), cb_at(tbl, window_of<BITS>(W, j + 1), c), 0x5410u);
        }
        tc::st_x16(taddr + 16 * h, col);
    }
}

template <int BK, int BV>
__global__ void __launch_bounds__(NT, 1) attend_trellis_tc_kernel(TrellisParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int quarter = warp & 3, grp = warp >> 2, tl = quarter * 32 + lane;
    const int hl = blockIdx.y, h = p.kv0 + hl, split = blockIdx.x;
    const sjk_view & v = p.v;
    const sj_kvarn_layout & l = v.lay;
    uint8_t * tr = sm + OFF_TR;
    uint8_t * bk = sm + OFF_BK;
    uint8_t * bv = sm + OFF_BV;
    uint32_t * cbk = reinterpret_cast<uint32_t *>(sm + OFF_CBK);
    uint32_t * cbv = reinterpret_cast<uint32_t *>(sm + OFF_CBV);
    float * row = reinterpret_cast<float *>(sm + OFF_ROW);
    float * red = reinterpret_cast<float *>(sm + OFF_RED);
    uint64_t * bars = reinterpret_cast<uint64_t *>(sm + OFF_BAR);
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(sm + OFF_TMEM);
    const uint32_t r_begin = p.rec_bounds[split], r_end = p.rec_bounds[split + 1];
    const uint32_t n = r_end > r_begin ? r_end - r_begin : 0u;
    const uint32_t rb = l.bytes;

    if (warp == 0) { tc::tmem_alloc(tmem_slot, TM_COLS); tc::tmem_relinquish(); }
    if (tid == 0) {
        tc::mbar_init(&bars[BAR_REC], 1); tc::mbar_init(&bars[BAR_REC + 1], 1); tc::mbar_init(&bars[BAR_MMA], 1);
        tc::mbar_fence_init();
    }
    uint32_t issued = 0;                                        // thread 0: records requested so far
    auto load = [&](uint32_t g) {                                // record g of the range into stage g % 2
        const uint32_t rec = r_begin + g, blk = v.blocks ? v.blocks[rec] : rec;
        tc::fence_proxy_async();
        tc::mbar_expect_tx(&bars[BAR_REC + (g & 1u)], rb);
        tc::bulk_g2s(sm + OFF_REC + (g & 1u) * REC_MAX, v.body + ((size_t) blk * v.n_head_kv + h) * rb, rb, &bars[BAR_REC + (g & 1u)]);
        ++issued;
    };
    // codebooks (16 interleaved copies) and the per-row state
    {
        const uint16_t * ck = sjk_codebook(BK, 0), * cv = sjk_codebook(BV, 1);
        for (int i = tid; i < (1 << (6 + BK)) * CB_COPIES; i += NT) cbk[i] = ck[i / CB_COPIES];
        for (int i = tid; i < (1 << (6 + BV)) * CB_COPIES; i += NT) cbv[i] = cv[i / CB_COPIES];
    }
    if (tid < NR) { row[ROW_M2 + tid] = -INFINITY; row[ROW_L + tid] = 0.0f; }
    // this thread's query values for the B_K build: channel tid % 256, rows 8 (tid / 256) ..
    const int bd = tid & 255, brh = tid >> 8;
    float q8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = 8 * brh + i;
        q8[i] = r < p.rows ? __ldg(p.q + (size_t) (p.row_q[r] + hl * p.grp) * D + bd) : 0.0f;
    }
    uint32_t qlim4[4];                                          // softmax rows 4 grp + i: positions < qlim4 are visible
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = 4 * grp + i;
        qlim4[i] = r < p.rows ? p.qpos0 + p.row_iq[r] + 1u : 0u;
    }
    if (tid == 0 && n) load(0);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = (uint32_t) (quarter * 32) << 16;
    const float sl2 = p.scale * LOG2E;
    const uint32_t idesc = tc::idesc_f16(128, NB);
    const int cc = lane & (CB_COPIES - 1);
    float acc[NR];                                              // warps 0..7: running output of channel 128 grp + tl
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
    bool ok = true, mma_pending = false;
    uint32_t mma_phase = 0;
    const uint32_t b_end = p.B < p.N ? p.B : p.N;
    // everyone: operand stores visible to the async proxy, then thread 0 issues; wait_mma: everyone waits
    auto issue = [&](bool k_side) {
        tc::wait_st();
        tc::fence_proxy_async();
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        if (tid == 0) {
            if (k_side) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const uint64_t db = tc::smem_desc(bk + TILE_B * (j >> 3), HCH, 128) + (uint64_t) ((2 * HCH * (j & 7)) >> 4);
                    tc::mma_ts(tmem + COL_S, tmem + COL_AK + 8 * j, db, idesc, j ? 1u : 0u);
                }
            } else {
#pragma unroll
                for (int tile = 0; tile < 2; ++tile)
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const uint64_t db = tc::smem_desc(bv, HCH, 128) + (uint64_t) ((2 * HCH * k) >> 4);
                        tc::mma_ts(tmem + COL_O + 32 * tile, tmem + COL_AV + 64 * tile + 8 * k, db, idesc, k ? 1u : 0u);
                    }
            }
            tc::mma_commit(&bars[BAR_MMA]);
        }
        mma_pending = true;
    };
    auto wait_mma = [&]() -> bool {
        const bool got = __syncthreads_and(tc::mbar_wait(&bars[BAR_MMA], mma_phase));
        if (got) { mma_phase ^= 1u; mma_pending = false; }
        tc::fence_after_sync();
        return got;
    };

    uint32_t arrived = 0;                                       // records whose bytes every thread has seen land
    for (uint32_t g = 0; g < n && ok; ++g) {
        const uint32_t s = g & 1u;
        const uint8_t * rec = sm + OFF_REC + s * REC_MAX;
        ok = __syncthreads_and(tc::mbar_wait(&bars[BAR_REC + s], (g >> 1) & 1u));
        if (!ok) break;
        arrived = g + 1;
        if (tid == 0 && g + 1 < n) load(g + 1);                 // the other stage was released at the end of g - 1
        const uint32_t gg = r_begin + g, p0 = p.S + gg * (uint32_t) G;
        const uint32_t len = min((uint32_t) G, b_end - p0);
        // ---- B_K = [Q' hi | Q' lo] (channel bd, rows 8 brh ..) and the zero-point partials ----
        {
            const float ks = h2f_at(rec + l.k_scale + 2 * bd), kz = h2f_at(rec + l.k_zero + 2 * bd);
            uint8_t * bt = bk + TILE_B * (bd >> 7);
            float cz[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = 8 * brh + i;
                const float x = q8[i] * ks;
                const __half hi = __float2half_rn(x);
                *reinterpret_cast<__half *>(bt + h_off(r, bd & 127)) = hi;
                *reinterpret_cast<__half *>(bt + h_off(NR + r, bd & 127)) = __float2half_rn(x - __half2float(hi));
                cz[i] = q8[i] * kz;
            }
            const float cw = warp_rows8<false>(cz, lane);
            if ((lane & 3) == 0) red[RED_C + warp * 8 + (lane >> 2)] = cw;
        }
        // ---- K values of channel bd, tokens 64 brh .. into the [token][channel] tile ----
        {
            const uint32_t * cw = reinterpret_cast<const uint32_t *>(rec + l.k_payload) + bd * (4 * BK);
            if (brh == 0) decode_k<BK, 0>(cw, cbk, cc, tr, bd);
            else decode_k<BK, 1>(cw, cbk, cc, tr, bd);
        }
        __syncthreads();
        if (tid < NR) {                                        // C[r]: the eight warps of the row's half
            const int r = tid, base = (r >> 3) * 8;
            float c = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; ++w) c += red[RED_C + (base + w) * 8 + (r & 7)];
            row[ROW_C + r] = c;
        }
        // ---- A_K: token tl, channels 64 grp .. 64 grp + 63 ----
        {
            const uint4 * src = reinterpret_cast<const uint4 *>(tr + tl * TRS + 128 * grp);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                uint32_t col[16];
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4) {
                    const uint4 x = src[4 * hh + c4];
                    col[4 * c4] = x.x; col[4 * c4 + 1] = x.y; col[4 * c4 + 2] = x.z; col[4 * c4 + 3] = x.w;
                }
                tc::st_x16(tmem + lane_base + COL_AK + 32 * grp + 16 * hh, col);
            }
        }
        issue(true);
        // ---- A_V (while the K MMAs run): channel 128 (grp / 2) + tl, tokens 64 (grp % 2) .. ----
        {
            const int d = 128 * (grp >> 1) + tl;
            const uint32_t * cw = reinterpret_cast<const uint32_t *>(rec + l.v_payload) + d * (4 * BV);
            const uint32_t ta = tmem + lane_base + COL_AV + 64 * (grp >> 1) + 32 * (grp & 1);
            if (grp & 1) decode_v<BV, 1>(cw, cbv, cc, ta);
            else decode_v<BV, 0>(cw, cbv, cc, ta);
        }
        ok = wait_mma();
        if (!ok) break;
        // ---- scores of token tl for rows 4 grp .. 4 grp + 3 (log2 domain), row maxima ----
        float s2[4];
        const float kt = h2f_at(rec + l.k_tok + 2 * tl), vsc = h2f_at(rec + l.v_scale + 2 * tl), vz = h2f_at(rec + l.v_zero + 2 * tl);
        {
            uint32_t a[4], al[4];
            tc::ld_x4_u(tmem + lane_base + COL_S + 4 * grp, a);
            tc::ld_x4_u(tmem + lane_base + COL_S + NR + 4 * grp, al);
            tc::wait_ld();
            const float kts = kt * sl2;
            const uint32_t pos = p0 + (uint32_t) tl;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float dot = kts * ((__uint_as_float(a[i]) + __uint_as_float(al[i])) + row[ROW_C + 4 * grp + i]);
                s2[i] = ((uint32_t) tl < len && pos < qlim4[i]) ? dot : -INFINITY;
            }
            const float mw = warp_rows4<true>(s2, lane);
            if ((lane & 7) == 0) red[RED_MAX + (grp * 4 + quarter) * 4 + (lane >> 3)] = mw;
        }
        __syncthreads();
        if (tid < NR) {
            const int r = tid, gq = (r >> 2) * 16 + (r & 3);
            const float mrec = fmaxf(fmaxf(red[RED_MAX + gq], red[RED_MAX + gq + 4]), fmaxf(red[RED_MAX + gq + 8], red[RED_MAX + gq + 12]));
            const float mold = row[ROW_M2 + r], mnew = fmaxf(mold, mrec);
            row[ROW_MNEW + r] = mnew;
            row[ROW_ALPHA + r] = mnew == -INFINITY ? 1.0f : ex2(mold - mnew);
            row[ROW_M2 + r] = mnew;
        }
        __syncthreads();
        // ---- P' = p Vscale as [hi | lo] (B of the V MMAs), row sums of p and p Vzero ----
        {
            float ls[4], zs[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = 4 * grp + i;
                const float mnew = row[ROW_MNEW + r];
                const float pw = mnew == -INFINITY ? 0.0f : ex2(s2[i] - mnew);
                ls[i] = pw;
                zs[i] = pw * vz;
                const float x = pw * vsc;
                const __half hi = __float2half_rn(x);
                *reinterpret_cast<__half *>(bv + h_off(r, tl)) = hi;
                *reinterpret_cast<__half *>(bv + h_off(NR + r, tl)) = __float2half_rn(x - __half2float(hi));
            }
            const float lw = warp_rows4<false>(ls, lane), zw = warp_rows4<false>(zs, lane);
            if ((lane & 7) == 0) {
                red[RED_L + (grp * 4 + quarter) * 4 + (lane >> 3)] = lw;
                red[RED_Z + (grp * 4 + quarter) * 4 + (lane >> 3)] = zw;
            }
        }
        issue(false);                                           // (its barrier makes the row sums visible)
        if (tid < NR) {
            const int r = tid, gq = (r >> 2) * 16 + (r & 3);
            const float lsum = (red[RED_L + gq] + red[RED_L + gq + 4]) + (red[RED_L + gq + 8] + red[RED_L + gq + 12]);
            row[ROW_L + r] = row[ROW_L + r] * row[ROW_ALPHA + r] + lsum;
            row[ROW_Z + r] = (red[RED_Z + gq] + red[RED_Z + gq + 4]) + (red[RED_Z + gq + 8] + red[RED_Z + gq + 12]);
        }
        ok = wait_mma();
        if (!ok) break;
        // ---- epilogue (warps 0..7): channel 128 grp + tl, all rows ----
        if (grp < 2) {
            const float vc = h2f_at(rec + l.v_ch + 2 * (128 * grp + tl));
            float o[16], ol[16];
            tc::ld_x16(tmem + lane_base + COL_O + 32 * grp, o);
            tc::ld_x16(tmem + lane_base + COL_O + 32 * grp + NR, ol);
            tc::wait_ld();
#pragma unroll
            for (int r = 0; r < NR; ++r) acc[r] = fmaf(acc[r], row[ROW_ALPHA + r], vc * ((o[r] + ol[r]) + row[ROW_Z + r]));
        }
        tc::fence_before_sync();
        __syncthreads();                                        // stage s, the B operands and TMEM free again
        tc::fence_after_sync();
    }
    if (mma_pending) tc::mbar_wait(&bars[BAR_MMA], mma_phase);  // a record that gave up: its MMAs first (bounded)
    if (tid == 0)                                               // and a copy still in flight lands before the CTA exits
        for (uint32_t j = arrived; j < issued; ++j) tc::mbar_wait(&bars[BAR_REC + (j & 1u)], (j >> 1) & 1u);
    __syncthreads();
    // ---- partials (m in the natural-log domain, l, o[D]) per real query row ----
    if (grp < 2) {
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            if (r < p.rows) {
                float * dst = p.part + ((size_t) (p.split0 + split) * p.n_q * p.n_head + (size_t) (p.row_q[r] + hl * p.grp)) * (D + 2);
                dst[2 + 128 * grp + tl] = ok ? acc[r] : 0.0f;
            }
        }
    }
    if (tid < p.rows) {
        const int r = tid;
        float * dst = p.part + ((size_t) (p.split0 + split) * p.n_q * p.n_head + (size_t) (p.row_q[r] + hl * p.grp)) * (D + 2);
        const float m2 = row[ROW_M2 + r];
        dst[0] = ok ? (m2 == -INFINITY ? m2 : m2 * LN2) : -INFINITY;
        dst[1] = ok ? row[ROW_L + r] : 0.0f;
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, TM_COLS);
}

}  // namespace

// ---- host side ---------------------------------------------------------------------------------------------

// Whether the tensor-core trellis path applies: trellis records of 2- or 3-bit codes, D = 256, G = 128, at most 16
// query rows per KV head.
int sjk_tc_trellis_supported(const sjk_view * v, int n_q, int grp) {
    const sj_kvarn_layout & l = v->lay;
    const bool bits_ok = (l.bits_k == 2 || l.bits_k == 3) && (l.bits_v == 2 || l.bits_v == 3);
    return l.D == D && l.G == G && l.body == SJKVARN_BODY_TRELLIS && bits_ok && n_q * grp <= NR && l.bytes <= REC_MAX &&
           l.bytes % 16 == 0 && l.k_payload % 16 == 0 && l.v_payload % 16 == 0;
}

// Splits (persistent CTAs) per KV head: one CTA per SM over the call's KV heads.
int sjk_tc_trellis_max_splits(int n_kv) {
    const int t = (148 + (n_kv > 0 ? n_kv : 1) - 1) / (n_kv > 0 ? n_kv : 1);
    return t < MAX_SPLITS ? t : MAX_SPLITS;
}

int sjk_tc_trellis_launch(const sjk_view * v, uint32_t B, uint32_t N, uint32_t n_rec, uint32_t qpos0, int n_q, int n_head,
                          int kv0, int n_kv, const float * q, float scale, float * part, int split0, int * splits_out,
                          sjk_stream st) {
    TrellisParams p;
    p.v = *v; p.kv0 = kv0; p.S = v->S; p.B = B; p.N = N; p.qpos0 = qpos0; p.n_rec = n_rec;
    p.n_q = n_q; p.n_head = n_head; p.grp = n_head / n_kv; p.rows = n_q * p.grp;
    for (int r = 0; r < NR; ++r) {
        const int iq = r < p.rows ? r / p.grp : 0, g = r < p.rows ? r % p.grp : 0;
        p.row_iq[r] = (uint32_t) iq;
        p.row_q[r] = iq * n_head + g;
    }
    p.q = q; p.scale = scale; p.part = part; p.split0 = split0;
    int splits = sjk_tc_trellis_max_splits(n_kv);
    if ((uint32_t) splits > n_rec) splits = (int) n_rec;
    *splits_out = splits;
    if (splits == 0) return 0;
    for (int s = 0; s <= splits; ++s) p.rec_bounds[s] = (uint32_t) (((uint64_t) n_rec * (uint32_t) s) / (uint32_t) splits);
    const int bk = v->lay.bits_k, bv = v->lay.bits_v;
    auto kfn = bk == 3 ? (bv == 3 ? attend_trellis_tc_kernel<3, 3> : attend_trellis_tc_kernel<3, 2>)
                       : (bv == 3 ? attend_trellis_tc_kernel<2, 3> : attend_trellis_tc_kernel<2, 2>);
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_TOTAL);
    if (e != cudaSuccess) return sjk_check(e);
    kfn<<<dim3((unsigned) splits, (unsigned) n_kv), NT, SMEM_TOTAL, st>>>(p);
    return sjk_check_launch();
}

SJK_STATUS_READER(sjk_tc_trellis_status_take)
