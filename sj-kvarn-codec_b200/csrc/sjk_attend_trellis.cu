// sjk_attend_trellis.cu - tensor-core (tcgen05, kind::f16) attention over the sealed body of trellis layers
// (3/3t, 3/2t, 2/2t records: sj_kvarn.h:1025-1109, 1176-1207), for one sequence or a batch of sequences.
//
// A trellis record stores, per channel d, the codes of its 128 tokens as one channel-major bit stream; the
// value of token t is a codebook entry picked by the window of its code and the 6 stream bits before it
// (sj_kvarn.h:879-900). The decoded rows are
//   K[t, d] = (cb_K[w_K(d, t)] Ks[d] + Kz[d]) Kt[t],      V[t, d] = (cb_V[w_V(d, t)] Vs[t] + Vz[t]) Vc[d]
// and regroup so the codebook entries (fp16, exact) are the tensor-core A operands:
//   S^T[t, r] = Kt[t] (sum_d cb_K[w_K(d, t)] Q'[r, d] + C[r]),   Q' = q Ks,  C = sum_d q Kz
//   O^T[d, r] = Vc[d] (sum_t cb_V[w_V(d, t)] P'[r, t] + z[r]),   P' = p Vs,  z = sum_t p Vz
// Q' and P' enter as fp16 hi + lo halves side by side in N (B = [hi | lo], N = 32): one MMA per k step leaves
// the hi and lo products in column groups 0..15 and 16..31, whose sum is the fp32 product to about 2^-22.
//
// Both A operands are decoded channel by channel, the order of the streams: a thread holds one channel's
// stream words in registers and looks each window up in a shared table. The table keeps 32 copies of every
// entry, one per bank, with the K codebook in the low and the V codebook in the high half of each word, so
// every lookup of a warp is one conflict-free wavefront and both sides share 64 KB. A_K (token rows, channel
// k) is stored MN-major in shared memory - a channel's 128 tokens are 16 contiguous 16-byte chunks - so the
// decoded pairs leave with 16-byte stores; A_V (channel rows, token k) goes straight into the thread's TMEM lane.
//
// The kernel is persistent and warp-specialized. Each CTA walks a list of work items (a contiguous record
// range of one KV head of one sequence), so one launch covers a single sequence split across the SMs or many
// sequences of a paged pool. Roles, linked only by mbarriers, overlap consecutive records:
//   warps 0-7    K side   B_K = [Q' hi | Q' lo] and the zero-point sums C, then A_K (shared, MN-major)
//   warps 8-15   V side   A_V into TMEM (double-buffered), then the epilogue of the previous record
//   warps 16-23  softmax  scores, online softmax per item, B_V = [P' hi | P' lo], the sums of p and p Vz
//                         (warps 16-19 at 4 or 8 query rows per KV head)
//   warp 24 (20) issuer   bulk copies of records into a 2-stage ring (no multicast), the MMAs, commits
// Every wait is bounded; a role whose wait runs out raises a CTA abort flag, the others stop at their next
// wait, and the issuer drains its own copies and MMAs before the TMEM is released.
#include <cuda_fp16.h>

#include "sjk_common.cuh"
#include "sjk_internal.h"
#include "sjk_plan.cuh"
#include "sjk_tc.cuh"

namespace {

using namespace tc::num;

constexpr int NR = 16;                  // most query rows per KV head (the kernels pad to 4, 8 or 16; B = [hi | lo] rows)
constexpr int D = 256;
constexpr int G = 128;
constexpr int W_V = 8, W_S = 16;       // 8 K-side warps, 8 V-side warps, then the softmax warps and 1 issuer warp
// softmax warps: 8 at 16 query rows (two per TMEM lane quarter, one half of the rows each), 4 at 4 or 8 rows
template <int R> constexpr int SW_N = R == 16 ? 8 : 4;
template <int R> constexpr int W_I = W_S + SW_N<R>;
template <int R> constexpr int NT = 32 * (W_I<R> + 1);
constexpr uint32_t TM_COLS = 512;
constexpr uint32_t COL_AV = 0, COL_S = 256, COL_O = 320;     // A_V [2 buffers][2 tiles][64] | S [2][32] | O [2 tiles][32]
constexpr uint32_t REC_MAX = 26880;     // largest trellis record at D = 256 (3/3t)
constexpr int MAX_SEQS = 128;
constexpr int MAX_ITEMS = 672;
constexpr int MAX_CTAS = 148;

struct TwSeq {                          // one sequence of the call
    const uint8_t * body;               // [blocks][n_head_kv][record]
    const uint32_t * blocks;            // block table (null: record g is block g)
    const float * q;                    // [n_q][n_head][D] rotated queries of this sequence
    uint32_t S;                         // sink length: record g covers positions S + 128 g ..
    uint32_t b_end;                     // min(B, N): positions at or past it are not in the body
    uint32_t qpos0;                     // position of the first query row
    uint32_t pad;
};
struct TwItem {                         // records [r0, r1) of KV head h of sequence seq, partial slot `slot`
    uint32_t seq_hl;                    // seq | hl << 16 (hl: head index inside q and the partial rows)
    uint32_t h_slot;                    // h | slot << 16
    uint32_t r0, r1;
};
struct TwParams {
    sj_kvarn_layout lay;
    int n_head_kv;
    int rows, grp, n_rows;              // query rows per KV head (n_q grp), GQA group, n_q n_head
    uint32_t row_iq[NR];                // r / grp
    int row_q[NR];                      // iq n_head + r % grp: q row and partial row of r, less hl grp
    float scale;
    float * part;                       // [slots][n_rows][D + 2]: m, l, o[D]
    int n_cta;
    uint16_t cta_item[MAX_CTAS + 1];    // items of CTA c: [cta_item[c], cta_item[c + 1])
    TwSeq seq[MAX_SEQS];
    TwItem item[MAX_ITEMS];
};

// B operand (K-major, no swizzle, 32 rows): element (n, k) at (k / 8) * HCH + n * 16 + (k % 8) * 2 with an
// 8-element K chunk every HCH = 528 bytes (consecutive chunks start 4 banks apart); 128 k per tile
constexpr uint32_t HCH = 528;
constexpr uint32_t TILE_B = 16 * HCH;
__device__ __forceinline__ uint32_t h_off(int n, int k) { return (uint32_t) (k >> 3) * HCH + (uint32_t) (n * 16 + (k & 7) * 2); }

// A_K, MN-major without swizzle: element (t, d) at (t / 8) * 128 + (d / 8) * 2048 + (d % 8) * 16 + (t % 8) * 2,
// i.e. 8 x 8 core matrices of 128 contiguous bytes, 128 bytes apart along t (SBO) and 2048 apart along d (LBO)
constexpr uint32_t AK_SBO = 128, AK_LBO = 2048;

// shared memory (bytes)
constexpr uint32_t OFF_TBL = 0;                                 // u32 [512][32]: cb_K | cb_V << 16, 32 copies
constexpr uint32_t OFF_AK = OFF_TBL + 512 * 32 * 4;             // 64 KB
constexpr uint32_t OFF_REC = OFF_AK + 32 * AK_LBO;              // 2 x record (bulk copies)
constexpr uint32_t OFF_BK = OFF_REC + 2 * REC_MAX;              // [Q' hi | Q' lo] over 256 channels: 2 x TILE_B
constexpr uint32_t OFF_BV = OFF_BK + 2 * TILE_B;                // [P' hi | P' lo] over 128 tokens: TILE_B
constexpr uint32_t OFF_F = OFF_BV + TILE_B;                     // floats below
enum : uint32_t {
    F_REDC = 0,         // [2][8 warps][8]   zero-point partials of the K side
    F_REDM = 128,       // [4 lane quarters][16] score maxima
    F_REDL = 192,       // [4][16]           sums of p
    F_REDZ = 256,       // [4][16]           sums of p Vz
    F_C = 320,          // [2][16]           C[r] per record parity
    F_MN = 352,         // [16]              running max after the current record (log2 domain)
    F_AL = 368,         // [3][16]           rescale of the running sums at the record (slot g % 3)
    F_Z = 416,          // [3][16]           z[r] of the record (slot g % 3)
    F_END = 464
};
constexpr uint32_t OFF_BAR = OFF_F + F_END * 4;
enum : uint32_t {       // mbarriers
    B_RFULL = 0, B_REMPTY = 2, B_AKFULL = 4, B_SFULL = 5, B_SFREE = 7, B_CFULL = 9, B_AZFULL = 11, B_AVFULL = 13,
    B_VDONE = 15, B_OFREE = 17, B_COUNT = 18
};
constexpr uint32_t OFF_TMEM = OFF_BAR + B_COUNT * 8;
constexpr uint32_t OFF_ABORT = OFF_TMEM + 4;
constexpr uint32_t SMEM_TOTAL = OFF_ABORT + 12;
static_assert(SMEM_TOTAL <= 227 * 1024, "shared memory");
static_assert(OFF_REC % 16 == 0 && REC_MAX % 16 == 0 && OFF_BK % 16 == 0 && OFF_BV % 16 == 0 && OFF_F % 16 == 0, "alignment");

// Wait for the phase of `bar` with the given parity (try_wait suspends the thread until the phase completes or
// about 1 us passes). Gives up when the CTA's abort flag is raised or after about 1 s of wall clock (then it raises
// the flag and records the timeout in the device status word).
__device__ __forceinline__ bool wait_bar(uint64_t * bar, uint32_t parity, volatile int * abort) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = tc::globaltimer();
    while (true) {
        if (tc::mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (tc::globaltimer() - t0 > SJK_WAIT_NS) {
            atomicExch(&sjk_dev_status, SJK_DEV_TIMEOUT);
            *abort = 1;
            return false;
        }
    }
}
// the same for a whole warp: true only if every lane saw the phase complete
__device__ __forceinline__ bool warp_wait(uint64_t * bar, uint32_t parity, volatile int * abort) {
    return __all_sync(0xFFFFFFFFu, wait_bar(bar, parity, abort));
}
__device__ __forceinline__ void warp_arrive(uint64_t * bar, int lane) {
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(bar);
}

// ---- record streams -----------------------------------------------------------------------------------------
// The CTA's work as a sequence of records over its items: cursor over (item, record)
struct Cursor {
    int it, it_end;
    uint32_t rec, r1;
    __device__ __forceinline__ void start(const TwParams & p, int i0, int i1) {
        it = i0; it_end = i1;
        if (it < it_end) { rec = p.item[it].r0; r1 = p.item[it].r1; }
    }
    __device__ __forceinline__ bool first(const TwParams & p) const { return rec == p.item[it].r0; }
    __device__ __forceinline__ bool last() const { return rec + 1 == r1; }
    __device__ __forceinline__ void next(const TwParams & p) {
        if (++rec == r1 && ++it < it_end) { rec = p.item[it].r0; r1 = p.item[it].r1; }
    }
};
// block id of the cursor's record (a load from the sequence's block table, or the record index itself)
__device__ __forceinline__ uint32_t blk_of(const TwParams & p, const Cursor & c) {
    const TwSeq & sq = p.seq[p.item[c.it].seq_hl & 0xFFFFu];
    return sq.blocks ? __ldg(sq.blocks + c.rec) : c.rec;
}
__device__ __forceinline__ const uint8_t * rec_ptr(const TwParams & p, const Cursor & c, uint32_t blk) {
    const TwItem & it = p.item[c.it];
    return p.seq[it.seq_hl & 0xFFFFu].body + ((size_t) blk * p.n_head_kv + (it.h_slot & 0xFFFFu)) * p.lay.bytes;
}

// The 4 BITS stream words of one channel (128 tokens), 16-byte aligned in shared memory.
template <int BITS>
__device__ __forceinline__ void load_words(const uint8_t * src, uint32_t (&w)[4 * BITS]) {
#pragma unroll
    for (int i = 0; i < BITS; ++i) {
        const uint4 x = reinterpret_cast<const uint4 *>(src)[i];
        w[4 * i] = x.x; w[4 * i + 1] = x.y; w[4 * i + 2] = x.z; w[4 * i + 3] = x.w;
    }
}

// ---- stream decoding ----------------------------------------------------------------------------------------
// 32 tokens are BITS whole stream words. Token j of the 32 starts its window (its code above the 6 stream bits
// before it, the bits before the stream reading as zero, sj_kvarn.h:879-900) at bit 26 + j BITS of
// win = {word before the 32 tokens, their BITS words}. Byte offset of the window's table row (copy `lane`):
// window * 128 + 4 lane, one shift and one LOP3 at a compile-time bit offset.
template <int BITS>
__device__ __forceinline__ uint32_t tbl_off(const uint32_t (&win)[BITS + 1], int j, uint32_t lane4) {
    const int b = 26 + j * BITS, a = b >> 5, s = b & 31;
    constexpr uint32_t M7 = ((1u << (6 + BITS)) - 1u) << 7;
    uint32_t y;
    if (s >= 7) y = (s + 6 + BITS <= 32) ? (win[a] >> (s - 7)) : __funnelshift_r(win[a], win[a + 1 <= BITS ? a + 1 : BITS], s - 7);
    else y = win[a] << (7 - s);
    return (y & M7) | lane4;
}
__device__ __forceinline__ uint32_t lds32(const uint8_t * base, uint32_t off) {
    return *reinterpret_cast<const uint32_t *>(base + off);
}
// fp16 pair of tokens j, j + 1 (token j low) from the table half selected by sel (0x5410 K, 0x7632 V)
template <int BITS>
__device__ __forceinline__ uint32_t pair_at(const uint8_t * tbl, const uint32_t (&win)[BITS + 1], int j, uint32_t lane4, uint32_t sel) {
    return prmt(lds32(tbl, tbl_off<BITS>(win, j, lane4)), lds32(tbl, tbl_off<BITS>(win, j + 1, lane4)), sel);
}

// K side, 32 tokens at a time: tokens 32 sc .. 32 sc + 31 of one channel as the fp16 pairs of its MN-major A_K
// chunks 4 sc .. 4 sc + 3 (prev: the stream word before them; w: their BITS words)
template <int BITS>
__device__ __forceinline__ void decode_k_sub(const uint8_t * tbl, uint32_t prev, const uint32_t * w, uint32_t lane4, uint32_t (&o)[16]) {
    uint32_t win[BITS + 1];
    win[0] = prev;
#pragma unroll
    for (int i = 0; i < BITS; ++i) win[1 + i] = w[i];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j] = pair_at<BITS>(tbl, win, 2 * j, lane4, 0x5410u);
}
__device__ __forceinline__ void store_k_sub(uint8_t * ak_ch, int sc, const uint32_t (&o)[16]) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4 *>(ak_ch + (4 * sc + c) * AK_SBO) = make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
}
// V side: the 128 tokens of one channel as fp16 pairs (token 2i low) into the thread's TMEM lane
template <int BITS>
__device__ __forceinline__ void decode_v(const uint8_t * tbl, uint32_t (&w)[4 * BITS], uint32_t lane4, uint32_t taddr) {
    uint32_t prev = 0;
#pragma unroll 1
    for (int sc = 0; sc < 4; ++sc) {
        uint32_t win[BITS + 1];
        win[0] = prev;
#pragma unroll
        for (int i = 0; i < BITS; ++i) win[1 + i] = w[i];
        uint32_t col[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) col[i] = pair_at<BITS>(tbl, win, 2 * i, lane4, 0x7632u);
        tc::st_x16(taddr + 16 * sc, col);
        prev = w[BITS - 1];
#pragma unroll
        for (int i = 0; i < 3 * BITS; ++i) w[i] = w[i + BITS];
    }
}

// Reduce R per-thread row values across the 32 lanes; afterwards lanes (32 / R) r .. hold row r.
template <int R, bool MAX>
__device__ __forceinline__ float warp_rows(const float (&v)[R], int lane) {
    if constexpr (R == 16) return warp_rows16<MAX>(v, lane);
    else if constexpr (R == 8) return warp_rows8<MAX>(v, lane);
    else if constexpr (R == 4) return warp_rows4<MAX>(v, lane);
    else {                                                      // R = 2: lanes 16 r .. 16 r + 15 hold row r
        const bool up = lane & 16;
        const float x = __shfl_xor_sync(0xFFFFFFFFu, up ? v[0] : v[1], 16);
        float c = MAX ? fmaxf(up ? v[1] : v[0], x) : (up ? v[1] : v[0]) + x;
#pragma unroll
        for (int o = 8; o; o >>= 1) {
            const float y = __shfl_xor_sync(0xFFFFFFFFu, c, o);
            c = MAX ? fmaxf(c, y) : c + y;
        }
        return c;
    }
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, one CTA
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u));
}

// R: query rows per KV head the kernel computes (4, 8 or 16, padded; the MMA N is 2 R, at least 16)
template <int BK, int BV, int R>
SJK_DEV void trellis_ws_body(const TwParams & p) {
    constexpr int RH = R / 2;                                   // B_K rows per thread (two row halves)
    constexpr int LPH = 32 / RH;                                // lanes per row after a warp_rows<RH>
    constexpr int NSW = SW_N<R>, WI = W_I<R>, NTH = NT<R>;
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const sj_kvarn_layout & l = p.lay;
    float * F = reinterpret_cast<float *>(sm + OFF_F);
    uint64_t * bars = reinterpret_cast<uint64_t *>(sm + OFF_BAR);
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(sm + OFF_TMEM);
    volatile int * abort = reinterpret_cast<volatile int *>(sm + OFF_ABORT);
    const int i0 = p.cta_item[blockIdx.x], i1 = p.cta_item[blockIdx.x + 1];
    uint32_t n = 0;
    for (int i = i0; i < i1; ++i) n += p.item[i].r1 - p.item[i].r0;

    if (warp == WI) { tc::tmem_alloc(tmem_slot, TM_COLS); tc::tmem_relinquish(); }
    if (tid == WI * 32) {
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&bars[B_RFULL + i], 1); tc::mbar_init(&bars[B_REMPTY + i], WI);
            tc::mbar_init(&bars[B_SFULL + i], 1); tc::mbar_init(&bars[B_SFREE + i], NSW);
            tc::mbar_init(&bars[B_CFULL + i], 1); tc::mbar_init(&bars[B_AZFULL + i], NSW);
            tc::mbar_init(&bars[B_AVFULL + i], 8); tc::mbar_init(&bars[B_VDONE + i], 1);
        }
        tc::mbar_init(&bars[B_AKFULL], 8); tc::mbar_init(&bars[B_OFREE], 8);
        *abort = 0;
        tc::mbar_fence_init();
    }
    // lookup table: word [idx][c] = cb_K[idx] | cb_V[idx] << 16 for every copy c (rows past a 2-bit table unused)
    {
        const uint16_t * ck = sjk_codebook(BK, 0), * cv = sjk_codebook(BV, 1);
        constexpr int NK = 1 << (6 + BK), NV = 1 << (6 + BV), NI = NK > NV ? NK : NV;
        for (int i = tid; i < NI * 8; i += NTH) {
            const int idx = i >> 3;
            const uint32_t w = (uint32_t) (idx < NK ? ck[idx] : 0) | ((uint32_t) (idx < NV ? cv[idx] : 0) << 16);
            reinterpret_cast<uint4 *>(sm + OFF_TBL)[i] = make_uint4(w, w, w, w);
        }
    }
    // the first two records of a sequence without a block table into L2 (a prefetch only: no load into the SM)
    if (tid == WI * 32 && i0 < i1) {
        const TwItem & it = p.item[i0];
        const TwSeq & sq = p.seq[it.seq_hl & 0xFFFFu];
        if (!sq.blocks)
            for (uint32_t g = it.r0; g < it.r1 && g < it.r0 + 2; ++g)
                tc::prefetch_l2(sq.body + ((size_t) g * p.n_head_kv + (it.h_slot & 0xFFFFu)) * p.lay.bytes, p.lay.bytes);
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // The grid may be launched as a programmatic dependent of the previous kernel in the stream (the previous call's
    // merge, say): the set-up above reads nothing another kernel writes, and this wait returns once that kernel has
    // completed. Only then may this grid's own dependents (the same call's staged-row kernel beside it, or its
    // merge) start, on the SMs it leaves free.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const uint32_t tmem = *tmem_slot;
    const uint8_t * tbl = sm + OFF_TBL;
    const uint32_t lane4 = (uint32_t) lane * 4u;
    Cursor cur;
    cur.start(p, i0, i1);

    if (warp < W_V) {
        // ================================ K side ================================
        const int jp = tid & 127, rh = tid >> 7;               // B_K: channels 2 jp, 2 jp + 1; rows RH rh ..
        const int d = tid;                                      // decoding: channel d
        uint8_t * bk = sm + OFF_BK + TILE_B * (jp >> 6) + h_off(0, (2 * jp) & 127);
        uint8_t * ak_ch = sm + OFF_AK + (d >> 3) * AK_LBO + (d & 7) * 16;
        float2 q2[RH];
        for (uint32_t g = 0; g < n; ++g, cur.next(p)) {
            const TwItem & itm = p.item[cur.it];
            if (cur.first(p)) {
                const TwSeq & sq = p.seq[itm.seq_hl & 0xFFFFu];
                const int hl = (int) (itm.seq_hl >> 16);
#pragma unroll
                for (int i = 0; i < RH; ++i) {
                    const int r = RH * rh + i;
                    q2[i] = r < p.rows ? __ldg(reinterpret_cast<const float2 *>(sq.q + (size_t) (p.row_q[r] + hl * p.grp) * D) + jp)
                                       : make_float2(0.0f, 0.0f);
                }
            }
            const uint32_t s = g & 1u;
            // every K warp reaches the group barrier below on every record, also after a wait gave up. What only
            // reads the record (the zero-point partials, the stream words, the first 32 tokens into registers) runs
            // before the wait for the previous record's K MMAs, which read B_K and A_K.
            bool ok = warp_wait(&bars[B_RFULL + s], (g >> 1) & 1u, abort);
            float2 ks = make_float2(0.0f, 0.0f);
            uint32_t w[4 * BK], o[16];
            if (ok) {
                tc::fence_after_sync();
                const uint8_t * rec = sm + OFF_REC + s * REC_MAX;
                ks = __half22float2(*reinterpret_cast<const __half2 *>(rec + l.k_scale + 4 * jp));
                const float2 kz = __half22float2(*reinterpret_cast<const __half2 *>(rec + l.k_zero + 4 * jp));
                float cz[RH];
#pragma unroll
                for (int i = 0; i < RH; ++i) cz[i] = fmaf(q2[i].y, kz.y, q2[i].x * kz.x);
                const float cw = warp_rows<RH, false>(cz, lane);
                if (lane % LPH == 0) F[F_REDC + s * 64 + warp * 8 + lane / LPH] = cw;
                load_words<BK>(rec + l.k_payload + d * (16 * BK), w);
                warp_arrive(&bars[B_REMPTY + s], lane);
                decode_k_sub<BK>(tbl, 0u, w, lane4, o);
            }
            ok = ok && (g == 0 || warp_wait(&bars[B_SFULL + ((g - 1) & 1u)], ((g - 1) >> 1) & 1u, abort));
            if (ok) {
                tc::fence_after_sync();
#pragma unroll
                for (int i = 0; i < RH; ++i) {
                    const int r = RH * rh + i;
                    const float2 x = make_float2(q2[i].x * ks.x, q2[i].y * ks.y);
                    const __half2 hi = __floats2half2_rn(x.x, x.y);
                    const float2 hf = __half22float2(hi);
                    const __half2 lo = __floats2half2_rn(x.x - hf.x, x.y - hf.y);
                    *reinterpret_cast<__half2 *>(bk + r * 16) = hi;
                    *reinterpret_cast<__half2 *>(bk + (R + r) * 16) = lo;
                }
                store_k_sub(ak_ch, 0, o);
#pragma unroll 1
                for (int sc = 1; sc < 4; ++sc) {
                    const uint32_t prev = w[BK - 1];
#pragma unroll
                    for (int i = 0; i < 3 * BK; ++i) w[i] = w[i + BK];
                    decode_k_sub<BK>(tbl, prev, w, lane4, o);
                    store_k_sub(ak_ch, sc, o);
                }
                tc::fence_proxy_async();
            }
            if (!tc::nbar_and(1, 256, ok)) break;               // zero-point partials of all K warps in place
            if (warp == 0 && lane < R) {
                const int r = lane, base = (r / RH) * 4;
                const float * rc = F + F_REDC + s * 64 + (r % RH);
                F[F_C + s * NR + r] = (rc[8 * base] + rc[8 * (base + 1)]) + (rc[8 * (base + 2)] + rc[8 * (base + 3)]);
            }
            if (warp == 0) warp_arrive(&bars[B_CFULL + s], lane);
            warp_arrive(&bars[B_AKFULL], lane);
        }
    } else if (warp < W_S) {
        // ================================ V side ================================
        const int vw = warp - W_V, tile = vw >> 2, quarter = warp & 3;
        const int d = 128 * tile + 32 * quarter + lane;
        const uint32_t lane_base = (uint32_t) (32 * quarter) << 16;
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = 0.0f;
        float vc_prev = 0.0f;
        Cursor ecur = cur;                                      // the epilogue's cursor lags one record
        uint32_t e3 = 0;                                        // e % 3: the softmax's alpha / z slot of record e
        // epilogue of record e: acc = acc alpha + Vc (O + z), in two halves of 8 rows; at the end of an item the
        // outputs leave as partials
        auto epilogue = [&](uint32_t e, float vc) -> bool {
            const uint32_t es = e & 1u;
            if (!warp_wait(&bars[B_VDONE + es], (e >> 1) & 1u, abort)) return false;
            if (!warp_wait(&bars[B_AZFULL + es], (e >> 1) & 1u, abort)) return false;
            tc::fence_after_sync();
            constexpr int EW = R < 8 ? R : 8;                   // rows per TMEM load
#pragma unroll
            for (int hh = 0; hh < R / EW; ++hh) {
                uint32_t o[EW], ol[EW];
                float al[EW], z[EW];
                if constexpr (EW == 8) {
                    tc::ld_x8_u(tmem + lane_base + COL_O + 32 * tile + 8 * hh, o);
                    tc::ld_x8_u(tmem + lane_base + COL_O + 32 * tile + R + 8 * hh, ol);
                } else {
                    tc::ld_x4_u(tmem + lane_base + COL_O + 32 * tile, o);
                    tc::ld_x4_u(tmem + lane_base + COL_O + 32 * tile + R, ol);
                }
#pragma unroll
                for (int i = 0; i < EW; i += 4) {
                    const float4 a4 = *reinterpret_cast<const float4 *>(F + F_AL + e3 * NR + EW * hh + i);
                    const float4 z4 = *reinterpret_cast<const float4 *>(F + F_Z + e3 * NR + EW * hh + i);
                    al[i] = a4.x; al[i + 1] = a4.y; al[i + 2] = a4.z; al[i + 3] = a4.w;
                    z[i] = z4.x; z[i + 1] = z4.y; z[i + 2] = z4.z; z[i + 3] = z4.w;
                }
                tc::wait_ld();
#pragma unroll
                for (int r = 0; r < EW; ++r)
                    acc[EW * hh + r] = fmaf(acc[EW * hh + r], al[r], vc * ((__uint_as_float(o[r]) + __uint_as_float(ol[r])) + z[r]));
            }
            tc::fence_before_sync();
            warp_arrive(&bars[B_OFREE], lane);
            e3 = e3 == 2 ? 0 : e3 + 1;
            if (ecur.last()) {
                const TwItem & itm = p.item[ecur.it];
                const int hl = (int) (itm.seq_hl >> 16), slot = (int) (itm.h_slot >> 16);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if (r < p.rows)
                        p.part[((size_t) slot * p.n_rows + (size_t) (p.row_q[r] + hl * p.grp)) * (D + 2) + 2 + d] = acc[r];
                    acc[r] = 0.0f;
                }
            }
            ecur.next(p);
            return true;
        };
        bool ok = true;
        for (uint32_t g = 0; g < n; ++g) {
            const uint32_t s = g & 1u;
            if (!warp_wait(&bars[B_RFULL + s], (g >> 1) & 1u, abort)) { ok = false; break; }
            if (g > 1 && !warp_wait(&bars[B_VDONE + s], ((g - 2) >> 1) & 1u, abort)) { ok = false; break; }
            tc::fence_after_sync();
            const uint8_t * rec = sm + OFF_REC + s * REC_MAX;
            uint32_t w[4 * BV];
            load_words<BV>(rec + l.v_payload + d * (16 * BV), w);
            const float vc = h2f_at(rec + l.v_ch + 2 * d);
            warp_arrive(&bars[B_REMPTY + s], lane);
            decode_v<BV>(tbl, w, lane4, tmem + lane_base + COL_AV + 128 * s + 64 * tile);
            tc::wait_st();
            tc::fence_before_sync();
            warp_arrive(&bars[B_AVFULL + s], lane);
            if (g > 0 && !epilogue(g - 1, vc_prev)) { ok = false; break; }
            vc_prev = vc;
        }
        if (ok && n > 0) epilogue(n - 1, vc_prev);
    } else if (warp < WI) {
        // ================================ softmax ================================
        // warp w reads the scores of TMEM lane quarter w % 4 (its 32 tokens) for RS of the R rows from r0 on
        constexpr int RS = R * 4 / NSW, LPS = 32 / RS;
        const int quarter = warp & 3, r0 = RS * ((warp - W_S) >> 2), t = 32 * quarter + lane;
        const uint32_t lane_base = (uint32_t) (32 * quarter) << 16;
        const float sl2 = p.scale * LOG2E;
        float M = -INFINITY, L = 0.0f;                          // warp W_S, lane r < 16: running max / sum of row r
        uint32_t g3 = 0;                                        // g % 3: slot of alpha / z (the epilogue of g - 3 is done)
        auto ldrs = [](const float * src, float (&v)[RS]) {
#pragma unroll
            for (int i = 0; i < RS; i += 4) {
                const float4 x = *reinterpret_cast<const float4 *>(src + i);
                v[i] = x.x; v[i + 1] = x.y; v[i + 2] = x.z; v[i + 3] = x.w;
            }
        };
        for (uint32_t g = 0; g < n; ++g, cur.next(p), g3 = g3 == 2 ? 0 : g3 + 1) {
            const TwItem & itm = p.item[cur.it];
            const TwSeq & sq = p.seq[itm.seq_hl & 0xFFFFu];
            if (cur.first(p)) { M = -INFINITY; L = 0.0f; }
            const uint32_t s = g & 1u;
            // every softmax warp reaches the group barriers below on every record, also after a wait gave up
            bool ok = warp_wait(&bars[B_SFULL + s], (g >> 1) & 1u, abort) && warp_wait(&bars[B_RFULL + s], (g >> 1) & 1u, abort) &&
                      warp_wait(&bars[B_CFULL + s], (g >> 1) & 1u, abort);
            float sc[RS], vsc = 0.0f, vz = 0.0f;
            if (ok) {
                tc::fence_after_sync();
                const uint8_t * rec = sm + OFF_REC + s * REC_MAX;
                const float kt = h2f_at(rec + l.k_tok + 2 * t);
                vsc = h2f_at(rec + l.v_scale + 2 * t);
                vz = h2f_at(rec + l.v_zero + 2 * t);
                float c[RS];
                ldrs(F + F_C + s * NR + r0, c);
                // the record stage and C[s] are rewritten only after this arrival (record g + 2)
                warp_arrive(&bars[B_REMPTY + s], lane);
                uint32_t a[RS], al[RS];
                static_assert(RS == 8 || RS == 4, "rows per softmax warp");
                if constexpr (RS == 8) {
                    tc::ld_x8_u(tmem + lane_base + COL_S + 32 * s + r0, a);
                    tc::ld_x8_u(tmem + lane_base + COL_S + 32 * s + R + r0, al);
                } else {
                    tc::ld_x4_u(tmem + lane_base + COL_S + 32 * s + r0, a);
                    tc::ld_x4_u(tmem + lane_base + COL_S + 32 * s + R + r0, al);
                }
                tc::wait_ld();
                tc::fence_before_sync();
                warp_arrive(&bars[B_SFREE + s], lane);
                const uint32_t pos = sq.S + cur.rec * (uint32_t) G + (uint32_t) t;
                const bool in = pos < sq.b_end;
                const float kts = kt * sl2;
#pragma unroll
                for (int i = 0; i < RS; ++i) {
                    const int r = r0 + i;
                    const bool vis = in && r < p.rows && pos < sq.qpos0 + p.row_iq[r] + 1u;
                    sc[i] = vis ? kts * ((__uint_as_float(a[i]) + __uint_as_float(al[i])) + c[i]) : -INFINITY;
                }
                const float mw = warp_rows<RS, true>(sc, lane);
                if (lane % LPS == 0) F[F_REDM + quarter * NR + r0 + lane / LPS] = mw;
            }
            if (!tc::nbar_and(2, 32 * NSW, ok)) break;
            if (warp == W_S && lane < R) {
                const int r = lane;
                const float mrec = fmaxf(fmaxf(F[F_REDM + r], F[F_REDM + NR + r]), fmaxf(F[F_REDM + 2 * NR + r], F[F_REDM + 3 * NR + r]));
                const float mnew = fmaxf(M, mrec);
                F[F_AL + g3 * NR + r] = mnew == -INFINITY ? 1.0f : ex2(M - mnew);
                F[F_MN + r] = mnew;
                M = mnew;
            }
            tc::nbar_sync(2, 32 * NSW);
            float mn[RS];
            ldrs(F + F_MN + r0, mn);
            // B_V is free once the V MMAs of the previous record completed
            ok = g == 0 || warp_wait(&bars[B_VDONE + (s ^ 1u)], ((g - 1) >> 1) & 1u, abort);
            if (ok) {
                uint8_t * bv = sm + OFF_BV;
                float ls[RS], zs[RS];
#pragma unroll
                for (int i = 0; i < RS; ++i) {
                    const int r = r0 + i;
                    const float pw = mn[i] == -INFINITY ? 0.0f : ex2(sc[i] - mn[i]);
                    ls[i] = pw;
                    zs[i] = pw * vz;
                    const float x = pw * vsc;
                    const __half hi = __float2half_rn(x);
                    *reinterpret_cast<__half *>(bv + h_off(r, t)) = hi;
                    *reinterpret_cast<__half *>(bv + h_off(R + r, t)) = __float2half_rn(x - __half2float(hi));
                }
                const float lw = warp_rows<RS, false>(ls, lane), zw = warp_rows<RS, false>(zs, lane);
                if (lane % LPS == 0) {
                    F[F_REDL + quarter * NR + r0 + lane / LPS] = lw;
                    F[F_REDZ + quarter * NR + r0 + lane / LPS] = zw;
                }
                tc::fence_proxy_async();
            }
            if (!tc::nbar_and(2, 32 * NSW, ok)) break;
            if (warp == W_S && lane < R) {
                const int r = lane;
                const float lsum = (F[F_REDL + r] + F[F_REDL + NR + r]) + (F[F_REDL + 2 * NR + r] + F[F_REDL + 3 * NR + r]);
                L = L * F[F_AL + g3 * NR + r] + lsum;
                F[F_Z + g3 * NR + r] = (F[F_REDZ + r] + F[F_REDZ + NR + r]) + (F[F_REDZ + 2 * NR + r] + F[F_REDZ + 3 * NR + r]);
                if (cur.last() && r < p.rows) {
                    const int hl = (int) (itm.seq_hl >> 16), slot = (int) (itm.h_slot >> 16);
                    float * dst = p.part + ((size_t) slot * p.n_rows + (size_t) (p.row_q[r] + hl * p.grp)) * (D + 2);
                    dst[0] = M == -INFINITY ? M : M * LN2;
                    dst[1] = L;
                }
            }
            warp_arrive(&bars[B_AZFULL + s], lane);
        }
    } else if (lane == 0) {
        // ================================ issuer ================================
        // In program order: the K MMAs of record g, the V MMAs of record g - 1, the bulk copy of record g + 2; each
        // after blocking waits. Records up to four ahead are prefetched into L2, so the bulk copies read from it.
        // MMA N = 2 R columns ([hi | lo]), at least 16: at R = 4 columns 8-15 read B rows nobody writes, and nobody
        // reads those columns back
        constexpr int NB = 2 * R < 16 ? 16 : 2 * R;
        const uint32_t idesc_k = tc::idesc_f16(128, NB) | (1u << 15);  // A MN-major (tokens contiguous per channel)
        const uint32_t idesc_v = tc::idesc_f16(128, NB);
        const uint32_t rb = l.bytes;
        Cursor pc = cur, lc = cur;                              // L2 prefetch and load cursors
        uint32_t np = 0, nl = 0;                                // records prefetched / loaded
        int last_commit = -1;                                   // barrier index and parity of the last commit
        uint32_t last_parity = 0;
        auto prefetch_to = [&](uint32_t upto) {
            for (; np < n && np < upto; ++np, pc.next(p)) tc::prefetch_l2(rec_ptr(p, pc, blk_of(p, pc)), rb);
        };
        auto mma_v = [&](uint32_t e) -> bool {
            if (!wait_bar(&bars[B_AZFULL + (e & 1u)], (e >> 1) & 1u, abort)) return false;
            if (!wait_bar(&bars[B_AVFULL + (e & 1u)], (e >> 1) & 1u, abort)) return false;
            if (e > 0 && !wait_bar(&bars[B_OFREE], (e - 1) & 1u, abort)) return false;
            tc::fence_after_sync();
#pragma unroll
            for (int tile = 0; tile < 2; ++tile)
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const uint64_t db = tc::smem_desc(sm + OFF_BV, HCH, 128) + (uint64_t) ((2 * HCH * k) >> 4);
                    tc::mma_ts(tmem + COL_O + 32 * tile, tmem + COL_AV + 128 * (e & 1u) + 64 * tile + 8 * k, db, idesc_v, k ? 1u : 0u);
                }
            tc::mma_commit(&bars[B_VDONE + (e & 1u)]);
            last_commit = (int) (B_VDONE + (e & 1u)); last_parity = (e >> 1) & 1u;
            return true;
        };
        // record j into stage j % 2, once the roles released record j - 2
        auto load_to = [&](uint32_t upto) -> bool {
            for (; nl < n && nl < upto; ++nl, lc.next(p)) {
                if (nl >= 2 && !wait_bar(&bars[B_REMPTY + (nl & 1u)], ((nl - 2) >> 1) & 1u, abort)) return false;
                tc::mbar_expect_tx(&bars[B_RFULL + (nl & 1u)], rb);
                tc::bulk_g2s(sm + OFF_REC + (nl & 1u) * REC_MAX, rec_ptr(p, lc, blk_of(p, lc)), rb, &bars[B_RFULL + (nl & 1u)]);
            }
            return true;
        };
        // the first two records are copied before anything is prefetched: their requests go first
        bool ok = load_to(2);
        for (; np < nl; ++np) pc.next(p);
        prefetch_to(4);
        for (uint32_t g = 0; g < n && ok; ++g) {
            prefetch_to(g + 5);
            ok = wait_bar(&bars[B_AKFULL], g & 1u, abort) && (g < 2 || wait_bar(&bars[B_SFREE + (g & 1u)], ((g - 2) >> 1) & 1u, abort));
            if (!ok) break;
            tc::fence_after_sync();
            const uint32_t dcol = tmem + COL_S + 32 * (g & 1u);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint64_t da = tc::smem_desc(sm + OFF_AK + 2 * AK_LBO * j, AK_LBO, AK_SBO);
                const uint64_t db = tc::smem_desc(sm + OFF_BK + TILE_B * (j >> 3), HCH, 128) + (uint64_t) ((2 * HCH * (j & 7)) >> 4);
                mma_ss(dcol, da, db, idesc_k, j ? 1u : 0u);
            }
            tc::mma_commit(&bars[B_SFULL + (g & 1u)]);
            last_commit = (int) (B_SFULL + (g & 1u)); last_parity = (g >> 1) & 1u;
            if (g > 0) ok = mma_v(g - 1);
            // record g + 2 into the stage of record g, as soon as the roles released it (the softmax reads its last
            // bytes right after the K MMAs above complete)
            if (ok) ok = load_to(g + 3);
        }
        if (ok && n > 0) mma_v(n - 1);
        // drain: the copies still in flight (at most the last two) and the MMAs behind the last commit
        for (uint32_t j = nl > 2 ? nl - 2 : 0; j < nl; ++j) tc::mbar_wait(&bars[B_RFULL + (j & 1u)], (j >> 1) & 1u);
        if (last_commit >= 0) tc::mbar_wait(&bars[last_commit], last_parity);
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (warp == WI) tc::tmem_dealloc(tmem, TM_COLS);
}

template <int BK, int BV, int R>
__global__ void __launch_bounds__(NT<R>, 1) attend_trellis_ws_kernel(const __grid_constant__ TwParams p) {
    trellis_ws_body<BK, BV, R>(p);
}

// the descriptor-driven form: the work list was planned on the device (trellis_dyn_plan_kernel); the grid covers
// the most CTAs a plan can use and the CTAs past the plan's return at once
template <int BK, int BV, int R>
__global__ void __launch_bounds__(NT<R>, 1) attend_trellis_ws_dyn_kernel(const TwParams * __restrict__ pp) {
    if ((int) blockIdx.x >= pp->n_cta) return;
    trellis_ws_body<BK, BV, R>(*pp);
}

template <int BK, int BV, int R>
int launch_kernel(const TwParams & p, const TwParams * dyn, sjk_stream st) {
    if (dyn) {
        auto kfn = attend_trellis_ws_dyn_kernel<BK, BV, R>;
        const cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_TOTAL);
        if (e != cudaSuccess) return sjk_check(e);
        kfn<<<(unsigned) p.n_cta, NT<R>, SMEM_TOTAL, st>>>(dyn);
        return sjk_check_launch();
    }
    auto kfn = attend_trellis_ws_kernel<BK, BV, R>;
    const cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_TOTAL);
    if (e != cudaSuccess) return sjk_check(e);
    // programmatic dependent launch: the set-up overlaps the previous kernel of the stream (trellis_ws_body waits)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) p.n_cta);
    cfg.blockDim = dim3(NT<R>);
    cfg.dynamicSmemBytes = SMEM_TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (sjk_check(cudaLaunchKernelEx(&cfg, kfn, p))) return SJK_ERR_DEVICE;
    return sjk_check_launch();
}

// p: the plan (host launches) or only its layout, rows and grid size (dyn: the plan in device memory)
template <int R>
int launch_rows(const TwParams & p, const TwParams * dyn, sjk_stream st) {
    const int bk = p.lay.bits_k, bv = p.lay.bits_v;
    if (bk == 3) return bv == 3 ? launch_kernel<3, 3, R>(p, dyn, st) : launch_kernel<3, 2, R>(p, dyn, st);
    return bv == 3 ? launch_kernel<2, 3, R>(p, dyn, st) : launch_kernel<2, 2, R>(p, dyn, st);
}

// the 4-row kernel for up to 4 query rows per KV head (decode width 1 at GQA 4), the 8-row one for up to 8, else
// the 16-row one
int launch(const TwParams & p, sjk_stream st, const TwParams * dyn = nullptr) {
    return p.rows <= 4 ? launch_rows<4>(p, dyn, st) : p.rows <= 8 ? launch_rows<8>(p, dyn, st) : launch_rows<16>(p, dyn, st);
}

SJK_HD void fill_rows(TwParams & p, int n_q, int n_head, int n_kv) {
    p.grp = n_head / n_kv;
    p.rows = n_q * p.grp;
    p.n_rows = n_q * n_head;
    for (int r = 0; r < NR; ++r) {
        const int iq = r < p.rows ? r / p.grp : 0, g = r < p.rows ? r % p.grp : 0;
        p.row_iq[r] = (uint32_t) iq;
        p.row_q[r] = iq * n_head + g;
    }
}

// One sequence: records [0, n_rec) of KV heads kv0 .. kv0 + n_kv - 1, each head split into `splits` contiguous ranges;
// item (head, split) is CTA hl * splits + split and writes partial slot split0 + split. Runs on the host (sjk_attend)
// and in the planner kernel of the descriptor-driven call.
SJK_HD void fill_single(TwParams & p, const sjk_view & v, uint32_t b_end, uint32_t n_rec, uint32_t qpos0, int n_q, int n_head,
                        int kv0, int n_kv, const float * q, float scale, float * part, int split0, int splits) {
    p.lay = v.lay; p.n_head_kv = v.n_head_kv; p.scale = scale; p.part = part;
    fill_rows(p, n_q, n_head, n_kv);
    p.seq[0].body = v.body; p.seq[0].blocks = v.blocks; p.seq[0].q = q; p.seq[0].S = v.S;
    p.seq[0].b_end = b_end; p.seq[0].qpos0 = qpos0; p.seq[0].pad = 0;
    int k = 0;
    for (int hl = 0; hl < n_kv; ++hl)
        for (int s = 0; s < splits; ++s, ++k) {
            TwItem & it = p.item[k];
            it.seq_hl = (uint32_t) hl << 16;
            it.h_slot = (uint32_t) (kv0 + hl) | ((uint32_t) (split0 + s) << 16);
            it.r0 = (uint32_t) (((uint64_t) n_rec * (uint32_t) s) / (uint32_t) splits);
            it.r1 = (uint32_t) (((uint64_t) n_rec * (uint32_t) (s + 1)) / (uint32_t) splits);
            p.cta_item[k] = (uint16_t) k;
        }
    p.cta_item[k] = (uint16_t) k;
    p.n_cta = k;
}

// planner of the descriptor-driven call: the plan of sjk_tc_trellis_launch for the counts in *ds
__global__ void trellis_dyn_plan_kernel(const sjk_dyn_state * __restrict__ ds, sjk_view v, int n_q, int n_head, int kv0, int n_kv,
                                        const float * q, float scale, float * part, TwParams * out) {
    if (threadIdx.x != 0) return;
    const sjk_dyn_state d = *ds;
    const uint32_t b_end = d.B < d.N ? d.B : d.N;
    fill_single(*out, v, b_end, d.n_tc, d.qpos0, n_q, n_head, kv0, n_kv, q, scale, part, 0, d.ok ? d.splits_tc : 0);
}

}  // namespace

// ---- host side ---------------------------------------------------------------------------------------------

// Whether the tensor-core trellis path applies: trellis records of 2- or 3-bit codes, D = 256, G = 128, at most 16
// query rows per KV head.
int sjk_tc_trellis_supported(const sjk_view * v, int n_q, int grp) {
    const sj_kvarn_layout & l = v->lay;
    const bool bits_ok = (l.bits_k == 2 || l.bits_k == 3) && (l.bits_v == 2 || l.bits_v == 3);
    return l.D == D && l.G == G && l.body == SJKVARN_BODY_TRELLIS && bits_ok && n_q * grp <= NR && l.bytes <= REC_MAX &&
           l.bytes % 16 == 0 && l.k_payload % 16 == 0 && l.v_payload % 16 == 0 && l.k_scale % 4 == 0 && l.k_zero % 4 == 0 &&
           v->n_head_kv <= MAX_CTAS;
}

// Splits (persistent CTAs) per KV head of a one-sequence call: one CTA per SM over the call's KV heads.
int sjk_tc_trellis_max_splits(int n_kv) {
    const int t = (MAX_CTAS + (n_kv > 0 ? n_kv : 1) - 1) / (n_kv > 0 ? n_kv : 1);
    return t < MAX_CTAS ? t : MAX_CTAS;
}

size_t sjk_tc_trellis_params_bytes(void) { return sizeof(TwParams); }

// One sequence: records [0, n_rec) of KV heads kv0 .. kv0 + n_kv - 1, each head split into `splits` contiguous
// ranges; item (head, split) is CTA hl * splits + split and writes partial slot split0 + split.
int sjk_tc_trellis_launch(const sjk_view * v, uint32_t B, uint32_t N, uint32_t n_rec, uint32_t qpos0, int n_q, int n_head,
                          int kv0, int n_kv, const float * q, float scale, float * part, int split0, int splits,
                          int * splits_out, sjk_stream st) {
    *splits_out = splits;
    if (splits <= 0) return 0;
    if (split0 + splits > 0xFFFF || splits * n_kv > MAX_CTAS) return SJK_ERR_UNSUPPORTED;
    static thread_local TwParams p;
    fill_single(p, *v, B < N ? B : N, n_rec, qpos0, n_q, n_head, kv0, n_kv, q, scale, part, split0, splits);
    return launch(p, st);
}

// Descriptor-driven form: the counts come from *ds (written on the device by the call's planner), this function's
// planner kernel writes the plan into `params` (sjk_tc_trellis_params_bytes() bytes of device memory) and the kernel
// reads it from there. The launch covers the most CTAs a plan can use.
int sjk_tc_trellis_dyn_launch(const sjk_view * v, int n_q, int n_head, int kv0, int n_kv, const float * q, float scale,
                              float * part, const sjk_dyn_state * ds, void * params, sjk_stream st) {
    TwParams * dp = static_cast<TwParams *>(params);
    trellis_dyn_plan_kernel<<<1, 32, 0, st>>>(ds, *v, n_q, n_head, kv0, n_kv, q, scale, part, dp);
    if (sjk_check_launch()) return SJK_ERR_DEVICE;
    static thread_local TwParams shape;        // only the layout, the rows and the grid size are read
    shape.lay = v->lay;
    fill_rows(shape, n_q, n_head, n_kv);
    int max_splits = sjk_tc_trellis_max_splits(n_kv);
    while (max_splits * n_kv > MAX_CTAS) --max_splits;
    shape.n_cta = max_splits * n_kv;
    if (shape.n_cta <= 0) return 0;
    return launch(shape, st, dp);
}

// Many sequences of one layer (same layout as views[0]): sequence s attends with query rows q + s n_q n_head D over its
// body records [0, ceil((min(B, N) - S) / 128)). The records of all (sequence, KV head) pairs, in that order, are cut
// into at most one contiguous range per SM, each range into items that stay inside one pair; items get partial slots
// slot0, slot0 + 1, ...; for pair (s, h) the items are slots first[s H + h] .. first[s H + h + 1] - 1.
int sjk_tc_trellis_batch_launch(const sjk_view * views, const uint32_t * B, const uint32_t * N, const uint32_t * qpos0,
                                int n_seq, int n_q, int n_head, const float * q, float scale, float * part, int slot0,
                                uint16_t * first, int * n_items, sjk_stream st) {
    const sjk_view & v0 = views[0];
    const int H = v0.n_head_kv;
    if (n_seq > MAX_SEQS || n_seq * H + MAX_CTAS > MAX_ITEMS) return SJK_ERR_UNSUPPORTED;
    static thread_local TwParams p;
    static thread_local uint32_t n_rec[MAX_SEQS];
    p.lay = v0.lay; p.n_head_kv = H; p.scale = scale; p.part = part;
    fill_rows(p, n_q, n_head, H);
    uint64_t total = 0;
    for (int s = 0; s < n_seq; ++s) {
        const uint32_t b_end = B[s] < N[s] ? B[s] : N[s];
        TwSeq & sq = p.seq[s];
        sq.body = views[s].body; sq.blocks = views[s].blocks; sq.q = q + (size_t) s * n_q * n_head * D;
        sq.S = v0.S; sq.b_end = b_end; sq.qpos0 = qpos0[s]; sq.pad = 0;
        n_rec[s] = b_end > v0.S ? (b_end - v0.S + 127u) / 128u : 0u;
        total += (uint64_t) n_rec[s] * (uint32_t) H;
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
                uint32_t r = 0;
                while (r < n_rec[s]) {
                    const uint32_t take = (uint32_t) (per - filled < (uint64_t) (n_rec[s] - r) ? per - filled : (uint64_t) (n_rec[s] - r));
                    if (k >= MAX_ITEMS || slot0 + k > 0xFFFF) return SJK_ERR_UNSUPPORTED;
                    TwItem & it = p.item[k++];
                    it.seq_hl = (uint32_t) s | ((uint32_t) h << 16);
                    it.h_slot = (uint32_t) h | ((uint32_t) (slot0 + k - 1) << 16);
                    it.r0 = r; it.r1 = r + take;
                    r += take;
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
    p.n_cta = cta;
    if (cta == 0) return 0;
    return launch(p, st);
}

SJK_STATUS_READER(sjk_tc_trellis_status_take)
