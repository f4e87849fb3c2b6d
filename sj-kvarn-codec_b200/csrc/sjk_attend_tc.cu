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
#include "sjk_fwht.cuh"
#include "sjk_internal.h"
#include "sjk_plan.cuh"
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

constexpr int MAX_SPLITS = 148;

struct TcParams {
    sj_kvarn_layout lay;
    const uint8_t * body;
    const uint32_t * blocks;
    int H, kv0;
    uint32_t S;                 // sink length: record g covers positions S + 128 g ..
    uint32_t n_rec;             // sealed records per head in [S, B)
    uint32_t qpos0;
    int n_q, n_head, grp, rows;
    // query row r (r < rows) of the KV head's group: position iq = r / grp, query head hl grp + r % grp; the
    // divisions are done once on the host
    uint32_t row_iq[NR];        // r / grp
    int row_q[NR];              // iq n_head + r % grp: q row (and partial row) of r, less hl grp
    const float * q;            // rotated queries, or model-basis ones for the QROT kernel (rotated on chip)
    float scale;
    float fwht_scale;           // 1/sqrt(D) of the query rotation (QROT kernel)
    float * part;               // [splits][n_q*n_head][D + 2]
    int split0;                 // partial slot of this kernel's first split
    int n_splits;               // splits per KV head (the descriptor-driven grid may be wider)
    // staged rows, taken by the same CTAs before their records: the sink [0, min(S, N)) and the staging ring
    // [max(B, S), N) in chunks of 128 positions (sink chunks first); chunk u of a head goes to split u % splits
    const uint8_t * sink;
    const uint8_t * ring;
    int staging, sink_type;
    uint32_t cap, stage_bytes, B, N;
    uint32_t n_sink_chunks, n_dense;
    uint32_t rec_bounds[MAX_SPLITS + 1];   // records of split s: [rec_bounds[s], rec_bounds[s + 1])
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
    F_ROWOFF = 128,    // [16] (u32)    offset of each query row's partial in p.part
    F_M2 = 144,        // [2][16]       running max (log2 domain) after the record of each buffer
    F_ALPHA = 176,     // [3][16]       rescale of the running sums when record g arrived (slot g % 3)
    F_VINV = 224,      // [3][16]       2^-ev of the P' rescale (slot g % 3)
    F_RMAXV = 272,     // [2][8]        per-softmax-warp max |Vscale|
    F_RMAX = 288,      // [2][2][4][8]  row maxima of the scores per (buffer, row half, lane quarter)
    F_RL = 416,        // [2][2][4][8]  row sums of p
    F_RZ = 544,        // [3][2][4][8]  row sums of p Vzero (slot g % 3)
    F_LSUM = 736,      // [16]          running sums of p
    F_OK = 752,        // [4]           per role: all its waits completed (unpack, softmax, issuer)
    F_BC = 768,        // [8][16]       per softmax warp: mnew and 2^ev of its 8 rows
    F_END = 896
};
constexpr uint32_t OFF_BAR = OFF_F + F_END * 4;
enum : uint32_t {                                             // mbarrier indices
    B_RFULL = 0, B_REMPTY = 3, B_AK = 6, B_AV = 8, B_SFULL = 10, B_SFREE = 11, B_BV = 12, B_VDONE = 14, B_OFREE = 16,
    B_DENSE = 18, B_EPI = 19, B_COUNT = 22
};
constexpr uint32_t OFF_TMEM = OFF_BAR + B_COUNT * 8;
// staged-row (dense) phase: rows staged in record stages 1..2, [q hi | q lo] in the B_K area, and its own
// [P' hi | P' lo] operands and bookkeeping
constexpr uint32_t HCH = 528;                                 // fp16 B operand: 8-element K chunk stride
constexpr uint32_t TILE_H = 16 * HCH;                         // one fp16 B operand over 128 k
constexpr uint32_t D_STG = OFF_REC + REC_MAX;                 // up to 2 REC_MAX bytes of staged rows
constexpr uint32_t D_STG_F16 = 528, D_STG_TQ6 = 2 * 2 * SJKVARN_TQ6_BLOCK_BYTES;   // staged row strides
constexpr uint32_t OFF_DBV = (OFF_TMEM + 16 + 127) & ~127u;   // 2 x TILE_H
constexpr uint32_t OFF_DM = OFF_DBV + 2 * TILE_H;             // dense bookkeeping (bytes below)
enum : uint32_t { DM_ROWP = 256, DM_NRM = 1280, DM_RED = 3328, DM_RED_L = 3584, DM_ROW = 3840, DM_QH = 4096,
                  DM_END = 5120 };
constexpr uint32_t OFF_DCODE = OFF_DM + DM_END;               // V codes of a chunk, [token][channel] bytes
constexpr uint32_t OFF_DCENT = OFF_DCODE + 128 * 256;        // centroid (fp16 hi | lo) table, one copy per bank
constexpr uint32_t SMEM_TOTAL = OFF_DCENT + 64 * 32 * 4;
// the kernel that takes model-basis queries (QROT) keeps the head's rotated query rows [16][256] after the rest
constexpr uint32_t OFF_QROT = SMEM_TOTAL;
constexpr uint32_t SMEM_TOTAL_QROT = OFF_QROT + NR * D * 4;
static_assert(SMEM_TOTAL_QROT <= 227 * 1024, "shared memory (QROT)");
constexpr uint32_t OFF_XF = OFF_DCODE;                        // [16][256] outputs on their way out (after the staged rows)
constexpr uint32_t DCOL_A = 0, DCOL_S = 256, DCOL_O = 320;   // dense TMEM: A (2 blocks x hi|lo), S (2 x 32), O (2 x 32)
static_assert(128 * D_STG_F16 <= 2 * REC_MAX && 128 * D_STG_TQ6 <= 2 * REC_MAX, "staged rows fit in stages 1..2");
static_assert(2 * TILE_H <= 2 * 16 * BCH, "[q hi | q lo] fits in the B_K area");

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

// QROT: p.q holds model-basis queries; each CTA rotates its KV head's rows on chip (the reference's FWHT, the same
// stage order and scale as sjk_hadamard) into shared memory before anything reads them
template <bool QROT>
SJK_DEV void body_tc_body(const TcParams & p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hl = blockIdx.y, h = p.kv0 + hl, split = blockIdx.x;
    const sj_kvarn_layout & l = p.lay;
    float * F = reinterpret_cast<float *>(sm + OFF_F);
    uint64_t * bars = reinterpret_cast<uint64_t *>(sm + OFF_BAR);
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(sm + OFF_TMEM);
    const uint32_t r_begin = p.rec_bounds[split], r_end = p.rec_bounds[split + 1];
    const uint32_t n = r_end > r_begin ? r_end - r_begin : 0u;

    if (warp == 2 * NW) { tc::tmem_alloc(tmem_slot, TM_COLS); tc::tmem_relinquish(); }
    if (tid == 2 * NW * 32) {
        for (uint32_t i = 0; i < NS; ++i) { tc::mbar_init(&bars[B_RFULL + i], 1); tc::mbar_init(&bars[B_REMPTY + i], 2 * NW); }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&bars[B_AK + i], NW); tc::mbar_init(&bars[B_AV + i], NW); tc::mbar_init(&bars[B_BV + i], NW);
            tc::mbar_init(&bars[B_VDONE + i], 1); tc::mbar_init(&bars[B_OFREE + i], NW);
        }
        tc::mbar_init(&bars[B_SFULL], 1); tc::mbar_init(&bars[B_SFREE], NW);
        tc::mbar_init(&bars[B_DENSE], 1);
        for (int i = 0; i < 3; ++i) tc::mbar_init(&bars[B_EPI + i], NW);
        tc::mbar_fence_init();
    }
    if (tid < 2 * NR) F[F_M2 + tid] = -INFINITY;
    if (tid < NR) {
        F[F_LSUM + tid] = 0.0f;
        reinterpret_cast<uint32_t *>(F + F_ROWOFF)[tid] =
            (uint32_t) (((size_t) (p.split0 + split) * p.n_q * p.n_head + (size_t) (p.row_q[tid] + hl * p.grp)) * (D + 2));
    }
    // staged-row chunk u of this head: first position, length, row format and the global K row of each token
    struct Chunk { uint32_t p0, len, side_off; bool f16, in_sink; };
    auto chunk_of = [&](uint32_t u) -> Chunk {
        Chunk c;
        const uint32_t s_eff = p.S < p.N ? p.S : p.N, t0 = p.B > p.S ? p.B : p.S;
        c.in_sink = u < p.n_sink_chunks;
        c.p0 = c.in_sink ? u * 128u : t0 + (u - p.n_sink_chunks) * 128u;
        c.len = min(128u, (c.in_sink ? s_eff : p.N) - c.p0);
        c.f16 = (c.in_sink && p.sink_type == SJKVARN_SINK_F16) || p.staging == SJKVARN_STAGING_F16;
        c.side_off = (c.in_sink && p.sink_type == SJKVARN_SINK_F16) ? 2u * D : p.stage_bytes;
        return c;
    };
    const uint8_t ** rowp = reinterpret_cast<const uint8_t **>(sm + OFF_DM + DM_ROWP);
    auto set_rowp = [&](const Chunk & c) {
        if (tid < 128) {
            const uint32_t pos = c.p0 + (uint32_t) min(tid, (int) c.len - 1);
            const uint8_t * r;
            if (c.in_sink && p.sink_type == SJKVARN_SINK_F16) r = p.sink + ((size_t) pos * p.H + h) * 4 * D;
            else if (c.in_sink) r = p.sink + ((size_t) pos * p.H + h) * 2 * p.stage_bytes;
            else r = p.ring + ((size_t) sjk_ring_slot(p.S, p.cap, pos) * p.H + h) * 2 * p.stage_bytes;
            rowp[tid] = r;
        }
    };
    // The grid may be launched as a programmatic dependent of the previous kernel in the stream (the merge of the
    // previous call, say), so that its set-up above overlaps that kernel's tail. Nothing above reads data another
    // kernel writes; the queries, the block table, the cache and the partials come after this wait, which returns
    // once the previous kernel has completed and its writes are visible (at once when there is none).
    if (tid == 2 * NW * 32 && !p.blocks)                   // the first records into L2 meanwhile (a prefetch only)
        for (uint32_t g = 0; g < 2 && g < n; ++g) tc::prefetch_l2(p.body + ((size_t) (r_begin + g) * p.H + h) * l.bytes, l.bytes);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    float qx[8];                                        // staged rows: this thread's q values (channel tid % 256)
    float * qrot = reinterpret_cast<float *>(sm + OFF_QROT);
    if ((uint32_t) split < p.n_dense) {
        set_rowp(chunk_of((uint32_t) split));
        if (!QROT) {
            const int d = tid & 255, r0 = (tid >> 8) * 8;
            const float * __restrict__ qg = p.q;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = r0 + i, rr = r < p.rows ? r : 0;
                qx[i] = tid < 512 ? __ldg(qg + (size_t) (p.row_q[rr] + hl * p.grp) * D + d) : 0.0f;
            }
        }
    }
    if (QROT && warp < NR) {                            // warp r rotates query row r of the head (zeros past rows)
        const int r = warp;
        float v[D / 32];
        const float * qr = p.q + (size_t) (p.row_q[r < p.rows ? r : 0] + hl * p.grp) * D + lane * (D / 32);
#pragma unroll
        for (int i = 0; i < D / 32; ++i) v[i] = r < p.rows ? __ldg(qr + i) : 0.0f;
        fwht_warp<D / 32>(v, lane, p.fwht_scale);
#pragma unroll
        for (int i = 0; i < D / 32; ++i) qrot[r * D + lane * (D / 32) + i] = v[i];
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    if (QROT && (uint32_t) split < p.n_dense) {
        const int d = tid & 255, r0 = (tid >> 8) * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) qx[i] = tid < 512 ? qrot[(r0 + i) * D + d] : 0.0f;
    }
    // the merge kernel that follows may be launched now; it waits for this grid on the device
    asm volatile("griddepcontrol.launch_dependents;");
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    float acc[NR];                                      // softmax warps: running output of their channel, all rows
#pragma unroll
    for (int r = 0; r < NR; ++r) acc[r] = 0.0f;
    // record 0 streams into stage 0 while the staged rows (stages 1..2) are processed
    const uint32_t pre_loaded = n >= 1 ? 1u : 0u;
    if (tid == 2 * NW * 32 && pre_loaded) {
        const uint32_t blk = p.blocks ? p.blocks[r_begin] : r_begin;
        tc::mbar_expect_tx(&bars[B_RFULL], l.bytes);
        tc::bulk_g2s(sm + OFF_REC, p.body + ((size_t) blk * p.H + h) * l.bytes, l.bytes, &bars[B_RFULL]);
    }

    if ((uint32_t) split < p.n_dense) {
        // ====== staged rows (sink, staging ring): chunks split, split + splits, .. of this head, one at a time ======
        // K side per block b:  S_b^T[t, r] = sum_{d in b} cent[code_K(t, d)] q[r, d],    dot = sum_b normK(t, b) S_b
        // V side per tile b:   O_b^T[d, r] = sum_t cent[code_V(t, d)] P'_b[r, t],        P'_b = p normV(t, b)
        // with fp16 hi + lo halves: A = centroid (hi | lo), B = [hi | lo] side by side in N (N = 32); two MMAs per
        // k step (A_hi x [hi | lo], A_lo x hi) leave hi*hi + lo*hi in columns 0..15 and hi*lo in 16..31. fp16 rows
        // enter with lo = 0. The chunk's scores join the CTA's running softmax state (m, l, acc) directly.
        // Warps 0..15: quarter w % 4, group w / 4 (block / tile w / 8, half (w / 4) % 2; score rows 4 (w / 4) ..).
        const int W = warp, quarter = W & 3, grp = W >> 2, tl = quarter * 32 + lane;
        const bool worker = W < 2 * NW;
        const uint32_t lane_base = (uint32_t) (quarter * 32) << 16;
        uint8_t * stg = sm + D_STG;
        uint8_t * dbq = sm + OFF_BK;
        uint8_t * dbv = sm + OFF_DBV;
        // centroid table, 32 copies interleaved by bank: entry c of lane L at word 32 c + L (conflict-free lookups)
        uint32_t * centr = reinterpret_cast<uint32_t *>(sm + OFF_DCENT);
        float * nrm = reinterpret_cast<float *>(sm + OFF_DM + DM_NRM);       // normK b*128+t, normV 256 + b*128+t
        float * dred = reinterpret_cast<float *>(sm + OFF_DM + DM_RED);      // [4 groups][4 quarters][4 rows]
        float * dredl = reinterpret_cast<float *>(sm + OFF_DM + DM_RED_L);
        float * drow = reinterpret_cast<float *>(sm + OFF_DM + DM_ROW);      // mnew[16], alpha[16]
        uint32_t * qh_lut = reinterpret_cast<uint32_t *>(sm + OFF_DM + DM_QH);
        uint8_t * vcodes = sm + OFF_DCODE;                                    // [token][channel] V codes
        auto hoff = [](int nn, int k) -> uint32_t { return (uint32_t) (k >> 3) * HCH + (uint32_t) (nn * 16 + (k & 7) * 2); };
        const float sl2 = p.scale * LOG2E;
        uint32_t qlim4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = 4 * grp + i;
            qlim4[i] = r < p.rows ? p.qpos0 + p.row_iq[r] + 1u : 0u;
        }
        uint32_t dphase = 0;
        bool d_pending = false;
        // all threads: operand stores visible, warp 16 lane 0 issues both blocks / tiles; dense_wait: everyone waits
        auto dense_issue = [&](const uint8_t * b_base, uint32_t d_col, bool f16) {
            tc::wait_st();
            tc::fence_proxy_async();
            tc::fence_before_sync();
            __syncthreads();
            tc::fence_after_sync();
            if (tid == 2 * NW * 32) {
                const uint32_t idesc32 = tc::idesc_f16(128, 2 * NR), idesc16 = tc::idesc_f16(128, NR);
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    const uint64_t db = tc::smem_desc(b_base + TILE_H * b, HCH, 128);
                    const uint32_t ah = tmem + DCOL_A + 128 * b, dc = tmem + d_col + 32 * b;
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        tc::mma_ts(dc, ah + 8 * k, db + (uint64_t) ((2 * HCH * k) >> 4), idesc32, k ? 1u : 0u);
                        if (!f16) tc::mma_ts(dc, ah + 64 + 8 * k, db + (uint64_t) ((2 * HCH * k) >> 4), idesc16, 1u);
                    }
                }
                tc::mma_commit(&bars[B_DENSE]);
            }
            d_pending = true;
        };
        auto dense_wait = [&]() -> bool {
            const bool got = __syncthreads_and(tc::mbar_wait(&bars[B_DENSE], dphase));
            if (got) { dphase ^= 1u; d_pending = false; }
            tc::fence_after_sync();
            return got;
        };
        for (uint32_t u = (uint32_t) split; u < p.n_dense && ok; u += (uint32_t) p.n_splits) {
            const Chunk ck = chunk_of(u);
            const uint32_t p0 = ck.p0, len = ck.len, side_off = ck.side_off;
            const bool f16 = ck.f16;
            const uint32_t sstride = f16 ? D_STG_F16 : D_STG_TQ6;
            if (u != (uint32_t) split) {                       // the first chunk's row addresses were set up front
                set_rowp(ck);
                __syncthreads();
            }
            // rows of the chunk (asynchronous copies, zeros past len), one warp per token: tq6_0 K and V rows
            // together (392 contiguous bytes, 49 x 8); fp16 rows one side at a time (512 bytes, 32 x 16)
            auto stage = [&](int side) {
                if (f16) {
                    const uint32_t so = side ? side_off : 0u;
                    for (int t = W; t < 128; t += 2 * NW)
                        tc::cp_async16(stg + t * D_STG_F16 + 16 * lane, rowp[t] + so + 16 * lane, (uint32_t) t < len ? 16u : 0u);
                } else {
                    for (int t = W; t < 128; t += 2 * NW) {
                        const uint8_t * src = rowp[t];
                        const uint32_t nb = (uint32_t) t < len ? 8u : 0u;
                        tc::cp_async8(stg + t * D_STG_TQ6 + 8 * lane, src + 8 * lane, nb);
                        if (lane < 17) tc::cp_async8(stg + t * D_STG_TQ6 + 256 + 8 * lane, src + 256 + 8 * lane, nb);
                    }
                }
            };
            if (worker) stage(0);
            if (u == (uint32_t) split) {
                // tables and [q hi | q lo], built while the first chunk's rows stream in
                if (tid < 256) {
                    const uint32_t y = (uint32_t) tid;
                    qh_lut[tid] = ((y & 3u) << 4) | (((y >> 2) & 3u) << 12) | (((y >> 4) & 3u) << 20) | (((y >> 6) & 3u) << 28);
                }
                for (int i = tid; i < 64 * 32; i += NT) {
                    const float c = sjk_tq6_cent[i >> 5];
                    const __half hi = __float2half_rn(c);
                    const __half2 hl2 = __floats2half2_rn(__half2float(hi), c - __half2float(hi));
                    centr[i] = *reinterpret_cast<const uint32_t *>(&hl2);
                }
                if (tid < 512) {                                   // [q hi | q lo]: channel tid % 256, rows 8 (tid / 256) ..
                    const int d = tid & 255, r0 = (tid >> 8) * 8;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int r = r0 + i;
                        const float xr = r < p.rows ? qx[i] : 0.0f;
                        const __half hi = __float2half_rn(xr);
                        *reinterpret_cast<__half *>(dbq + hoff(r, d)) = hi;
                        *reinterpret_cast<__half *>(dbq + hoff(NR + r, d)) = __float2half_rn(xr - __half2float(hi));
                    }
                }
            }
            if (worker) tc::cp_async_wait_all();
            tc::fence_before_sync();
            __syncthreads();
            tc::fence_after_sync();
            if (tid < 128) {
                const uint8_t * r0 = stg + tid * sstride;
                nrm[tid] = f16 ? 1.0f : h2f_at(r0);
                nrm[128 + tid] = f16 ? 1.0f : h2f_at(r0 + SJKVARN_TQ6_BLOCK_BYTES);
                nrm[256 + tid] = f16 ? 1.0f : h2f_at(r0 + 2 * SJKVARN_TQ6_BLOCK_BYTES);
                nrm[384 + tid] = f16 ? 1.0f : h2f_at(r0 + 3 * SJKVARN_TQ6_BLOCK_BYTES);
            }
            // ---- K side: block grp / 2, channels 64 ((grp % 2)) .. of token tl -> A (hi | lo) ----
            if (worker) {
                const int b = grp >> 1, half = grp & 1;
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
                        const uint2 cw = tq6_codes8(blk, 64 * half + 8 * g, qh_lut);    // elements 64 half + 8 g ..
#pragma unroll
                        for (int pp = 0; pp < 4; ++pp) {
                            const uint32_t w = pp < 2 ? cw.x : cw.y, sh = 16 * (pp & 1);
                            const uint32_t e0 = centr[32 * ((w >> sh) & 0xFFu) + lane];
                            const uint32_t e1 = centr[32 * ((w >> (sh + 8)) & 0xFFu) + lane];
                            ch[4 * g + pp] = prmt(e0, e1, 0x5410u);
                            cl[4 * g + pp] = prmt(e0, e1, 0x7632u);
                        }
                    }
                    tc::st_x16(tmem + lane_base + DCOL_A + 128 * b + 64 + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(cl));
                    tc::st_x16(tmem + lane_base + DCOL_A + 128 * b + 64 + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(cl + 16));
                }
                tc::st_x16(tmem + lane_base + DCOL_A + 128 * b + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(ch));
                tc::st_x16(tmem + lane_base + DCOL_A + 128 * b + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(ch + 16));
            }
            dense_issue(dbq, DCOL_S, f16);
            // tq6_0 (while the K MMAs run): V codes of the chunk in natural order (token, 8 channels per item) for
            // the channel-wise A build
            if (!f16 && worker) {
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int it = tid + 512 * k, t = it >> 5, gch = it & 31;          // channels 8 gch ..
                    const uint8_t * vblk = stg + t * D_STG_TQ6 + 2 * SJKVARN_TQ6_BLOCK_BYTES + SJKVARN_TQ6_BLOCK_BYTES * (gch >> 4);
                    *reinterpret_cast<uint2 *>(vcodes + t * 256 + 8 * gch) = tq6_codes8(vblk, 8 * (gch & 15), qh_lut);
                }
            }
            ok = dense_wait();
            if (!ok) break;
            // ---- scores of token tl for rows 4 grp .. 4 grp + 3 (log2 domain), row maxima ----
            float s2[4];
            if (worker) {
                uint32_t a0[4], a0l[4], a1[4], a1l[4];
                tc::ld_x4_u(tmem + lane_base + DCOL_S + 4 * grp, a0);
                tc::ld_x4_u(tmem + lane_base + DCOL_S + 16 + 4 * grp, a0l);
                tc::ld_x4_u(tmem + lane_base + DCOL_S + 32 + 4 * grp, a1);
                tc::ld_x4_u(tmem + lane_base + DCOL_S + 48 + 4 * grp, a1l);
                tc::wait_ld();
                const float nk0 = nrm[tl] * sl2, nk1 = nrm[128 + tl] * sl2;
                const uint32_t pos = p0 + (uint32_t) tl;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float dot = nk0 * (__uint_as_float(a0[i]) + __uint_as_float(a0l[i])) +
                                      nk1 * (__uint_as_float(a1[i]) + __uint_as_float(a1l[i]));
                    s2[i] = ((uint32_t) tl < len && pos < qlim4[i]) ? dot : -INFINITY;
                }
                const float mw = warp_rows4<true>(s2, lane);
                if ((lane & 7) == 0) dred[(grp * 4 + quarter) * 4 + (lane >> 3)] = mw;
            }
            tc::fence_before_sync();
            __syncthreads();
            if (tid < NR) {
                const int r = tid, gq = (r >> 2) * 16 + (r & 3);
                const float mrec = fmaxf(fmaxf(dred[gq], dred[gq + 4]), fmaxf(dred[gq + 8], dred[gq + 12]));
                const float mold = F[F_M2 + NR + r], mnew = fmaxf(mold, mrec);
                drow[r] = mnew;
                drow[NR + r] = mnew == -INFINITY ? 1.0f : ex2(mold - mnew);
                F[F_M2 + NR + r] = mnew;
            }
            if (f16 && worker) stage(1);                          // fp16: the V rows replace the K rows
            __syncthreads();
            // ---- P'_b = p normV(t, b) as [hi | lo] per tile, row sums ----
            if (worker) {
                if (f16) tc::cp_async_wait_all();
                const float nv0 = nrm[256 + tl], nv1 = nrm[384 + tl];
                float ls[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = 4 * grp + i;
                    const float mnew = drow[r];
                    const float pw = mnew == -INFINITY ? 0.0f : ex2(s2[i] - mnew);
                    ls[i] = pw;
                    const float x0 = pw * nv0, x1 = pw * nv1;
                    const __half2 hh = __floats2half2_rn(x0, x1);
                    const float2 hf = __half22float2(hh);
                    const __half2 ll = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
                    const uint32_t o = hoff(r, tl);
                    *reinterpret_cast<__half *>(dbv + o) = __low2half(hh);
                    *reinterpret_cast<__half *>(dbv + o + 256) = __low2half(ll);
                    *reinterpret_cast<__half *>(dbv + TILE_H + o) = __high2half(hh);
                    *reinterpret_cast<__half *>(dbv + TILE_H + o + 256) = __high2half(ll);
                }
                const float lw = warp_rows4<false>(ls, lane);
                if ((lane & 7) == 0) dredl[(grp * 4 + quarter) * 4 + (lane >> 3)] = lw;
            }
            __syncthreads();
            if (tid < NR) {
                const int r = tid, gq = (r >> 2) * 16 + (r & 3);
                F[F_LSUM + r] = F[F_LSUM + r] * drow[NR + r] + ((dredl[gq] + dredl[gq + 4]) + (dredl[gq + 8] + dredl[gq + 12]));
            }
            // ---- V side: tile grp / 2, channel 128 (grp / 2) + tl, tokens 64 (grp % 2) .. -> A (hi | lo) ----
            if (worker) {
                const int t = grp >> 1, half = grp & 1, d = 128 * t + tl;
                const uint8_t * vbase = f16 ? stg : stg + 2 * SJKVARN_TQ6_BLOCK_BYTES;   // tq6_0: V row follows K row
                uint32_t ch[32], cl[32];
                if (f16) {
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        const uint8_t * ra = vbase + (64 * half + 2 * c) * D_STG_F16;
                        const uint32_t x0 = *reinterpret_cast<const uint16_t *>(ra + 2 * d);
                        const uint32_t x1 = *reinterpret_cast<const uint16_t *>(ra + D_STG_F16 + 2 * d);
                        ch[c] = x0 | (x1 << 16);
                    }
                } else {
                    const uint8_t * col = vcodes + (64 * half) * 256 + d;
#pragma unroll
                    for (int c = 0; c < 32; ++c) {
                        const uint32_t e0 = centr[32 * col[(2 * c) * 256] + lane], e1 = centr[32 * col[(2 * c + 1) * 256] + lane];
                        ch[c] = prmt(e0, e1, 0x5410u);
                        cl[c] = prmt(e0, e1, 0x7632u);
                    }
                    tc::st_x16(tmem + lane_base + DCOL_A + 128 * t + 64 + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(cl));
                    tc::st_x16(tmem + lane_base + DCOL_A + 128 * t + 64 + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(cl + 16));
                }
                tc::st_x16(tmem + lane_base + DCOL_A + 128 * t + 32 * half, *reinterpret_cast<uint32_t (*)[16]>(ch));
                tc::st_x16(tmem + lane_base + DCOL_A + 128 * t + 32 * half + 16, *reinterpret_cast<uint32_t (*)[16]>(ch + 16));
            }
            dense_issue(dbv, DCOL_O, f16);
            ok = dense_wait();
            if (!ok) break;
            // ---- epilogue (unpack warps, which hold the outputs): channel 128 half + tl, all rows ----
            if (warp < NW) {
                const int half = warp >> 2;
                float o[16], ol[16];
                tc::ld_x16(tmem + lane_base + DCOL_O + 32 * half, o);
                tc::ld_x16(tmem + lane_base + DCOL_O + 32 * half + 16, ol);
                tc::wait_ld();
#pragma unroll
                for (int r = 0; r < NR; ++r) acc[r] = fmaf(acc[r], drow[NR + r], o[r] + ol[r]);
            }
            tc::fence_before_sync();
            __syncthreads();
            tc::fence_after_sync();
        }
        if (d_pending) tc::mbar_wait(&bars[B_DENSE], dphase);      // a chunk that gave up: its MMAs first (bounded)
        __syncthreads();                                          // B_K area and TMEM free for the records
    }

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
                const float * qr = QROT ? qrot + r * D : p.q + (size_t) (p.row_q[r] + hl * p.grp) * D;
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
        const int vcol = sjk_v_ch(l, 128 * half + tl);           // output channel 128 half + tl (epilogue)
        float vc_m1 = 0.0f, vc_m2 = 0.0f;                        // its Vch in records g - 1 and g - 2
        // epilogue of record e (O buffer e % 2, softmax slot e % 3): channel 128 half + tl, all rows. The caller
        // has waited for the record's V MMAs (B_VDONE) and for alpha, 2^-ev and z from the softmax warps (B_EPI).
        auto wait_epi = [&](uint32_t e) -> bool {
            return __all_sync(0xFFFFFFFFu, tc::mbar_wait2(&bars[B_VDONE + (e & 1u)], (e >> 1) & 1u, &bars[B_EPI + e % 3u], (e / 3u) & 1u));
        };
        auto epilogue = [&](uint32_t e, float vc) {
            const uint32_t eb = e & 1u, e3 = e % 3u;
            {
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {                // rows 8 hh .. 8 hh + 7
                    uint32_t o0[8], o1[8], o2[8];
                    const uint32_t oc = tmem + lane_base + COL_O + 96 * eb + 48 * half + 8 * hh;
                    tc::ld_x8_u(oc, o0);
                    tc::ld_x8_u(oc + 16, o1);
                    tc::ld_x8_u(oc + 32, o2);
                    float al[8], vi[8], za[8], zc[8], zd[8], ze[8];
                    ld8(F + F_ALPHA + 16 * e3 + 8 * hh, al);
                    ld8(F + F_VINV + 16 * e3 + 8 * hh, vi);
                    ld8(F + F_RZ + 64 * e3 + 32 * hh, za); ld8(F + F_RZ + 64 * e3 + 32 * hh + 8, zc);
                    ld8(F + F_RZ + 64 * e3 + 32 * hh + 16, zd); ld8(F + F_RZ + 64 * e3 + 32 * hh + 24, ze);
                    tc::wait_ld();
#pragma unroll
                    for (int i = 0; i < 8; i += 2) {           // rows in pairs: packed fp32 arithmetic
                        // |sum_t code P''| < 128 * 15 * 2^20 < 2^31: the digit sums recombine exactly in s32
                        const float2 O = make_float2((float) (int) (o0[i] + (o1[i] << 8) + (o2[i] << 16)),
                                                     (float) (int) (o0[i + 1] + (o1[i + 1] << 8) + (o2[i + 1] << 16)));
                        const float2 z = add2(add2(make_float2(za[i], za[i + 1]), make_float2(zc[i], zc[i + 1])),
                                              add2(make_float2(zd[i], zd[i + 1]), make_float2(ze[i], ze[i + 1])));
                        const float2 t = mul2(make_float2(vc, vc), fma2(O, make_float2(vi[i], vi[i + 1]), z));
                        const float2 r = fma2(make_float2(acc[8 * hh + i], acc[8 * hh + i + 1]), make_float2(al[i], al[i + 1]), t);
                        acc[8 * hh + i] = r.x;
                        acc[8 * hh + i + 1] = r.y;
                    }
                }
            }
            tc::fence_before_sync();
            warp_arrive(&bars[B_OFREE + eb], lane);
        };
        for (uint32_t g = 0; g < n; ++g) {
            const uint32_t s = g % NS, b = g & 1u;
            const uint8_t * rec = sm + OFF_REC + s * REC_MAX;
            // A_K[b] and B_K[b] were last read by the K MMAs of record g - 2: done once those of g - 1 are
            const bool w_ok = g >= 1 ? tc::mbar_wait2(&bars[B_RFULL + s], (g / NS) & 1u, &bars[B_SFULL], (g - 1) & 1u)
                                     : tc::mbar_wait(&bars[B_RFULL + s], (g / NS) & 1u);
            ok = __all_sync(0xFFFFFFFFu, ok && w_ok);
            if (!ok) break;
            tc::fence_after_sync();
            float ks[4], kz[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) { ks[j] = h2f_at(rec + l.k_scale + 2 * kcol[j]); kz[j] = h2f_at(rec + l.k_zero + 2 * kcol[j]); }
            const float vc_g = h2f_at(rec + l.v_ch + 2 * vcol);
            const float maxk = absmax256_h(rec + l.k_scale, lane);  // max |Kscale| of the record (every warp on its own)
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
                    const uint2 z01 = digits3x2(mul2(make_float2(qv[i][0], qv[i][1]), make_float2(ks[0], ks[1])), make_float2(sc, sc));
                    const uint2 z23 = digits3x2(mul2(make_float2(qv[i][2], qv[i][3]), make_float2(ks[2], ks[3])), make_float2(sc, sc));
                    const uint32_t z0 = z01.x, z1 = z01.y, z2 = z23.x, z3 = z23.y;
                    const uint32_t a = prmt(z0, z1, 0x5140u), c = prmt(z2, z3, 0x5140u);   // [z0.0 z1.0 z0.1 z1.1]
                    const uint32_t off = b_off(r, 4 * bg);
                    *reinterpret_cast<uint32_t *>(bk + off) = prmt(a, c, 0x5410u);
                    *reinterpret_cast<uint32_t *>(bk + off + 256) = prmt(a, c, 0x7632u);
                    *reinterpret_cast<uint32_t *>(bk + off + 512) = prmt(prmt(z0, z1, 0x0062u), prmt(z2, z3, 0x0062u), 0x5410u);
                    const float2 c2 = fma2(make_float2(qv[i][0], qv[i][2]), make_float2(kz[0], kz[2]),
                                           mul2(make_float2(qv[i][1], qv[i][3]), make_float2(kz[1], kz[3])));
                    cz[i] = c2.x + c2.y;
                }
                const float cw = warp_sum_rows4(cz[0], cz[1], cz[2], cz[3], lane);
                if ((lane & 7) == 0) F[F_CPART + 32 * b + warp * 4 + (lane >> 3)] = cw;
            }
            tc::wait_st();
            tc::fence_proxy_async();
            tc::fence_before_sync();
            warp_arrive(&bars[B_AK + b], lane);
            // ---- A_V: channel 128 half + tl over the 8 token tiles; A_V[b] was last read by the V MMAs of g - 2 ----
            if (g >= 2) ok = wait_epi(g - 2);
            tc::fence_after_sync();
            if (ok && g >= 2) epilogue(g - 2, vc_m2);                // record g - 2 out of O[b] before V(g) reuses it
            vc_m2 = vc_m1;
            vc_m1 = vc_g;
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
        // the last two records' epilogues (their V MMAs may still be running)
        for (uint32_t e = n >= 2 ? n - 2 : 0u; ok && e < n; ++e) {
            ok = wait_epi(e);
            tc::fence_after_sync();
            if (ok) epilogue(e, e + 2 == n ? vc_m2 : vc_m1);
        }
        ok = tc::nbar_and(1, NW * 32, ok);
        {                                                      // the outputs go out through shared memory
            float * xf = reinterpret_cast<float *>(sm + OFF_XF);
#pragma unroll
            for (int r = 0; r < NR; ++r) xf[r * D + 128 * half + tl] = acc[r];
        }
        if (lane == 0) F[F_OK] = ok ? 1.0f : 0.0f;             // (read after the CTA barrier below)
    } else if (warp < 2 * NW) {
        // ===== softmax: scores and weights of record g, B_V digits, row sums; the unpack warps run the epilogue =====
        // Thread (quarter, half, lane): token tl of the record for rows 8 half .. 8 half + 7. Lanes 0..7 of the
        // quarter-0 warps keep the running max / sums of their half's rows.
        const int sw = warp - NW, quarter = sw & 3, half = sw >> 2, tl = quarter * 32 + lane;
        const uint32_t lane_base = (uint32_t) (quarter * 32) << 16;
        const float sl2 = p.scale * LOG2E;
        uint32_t qlim[8];                                        // rows 8 half + i: positions < qlim are visible
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int r = 8 * half + i;
            qlim[i] = r < p.rows ? p.qpos0 + p.row_iq[r] + 1u : 0u;
        }
        for (uint32_t g = 0; g <= n; ++g) {                      // pass n only finishes record n - 1
            const uint32_t b = g & 1u, pb = b ^ 1u, s3 = g % 3u, ps3 = (g + 2u) % 3u;   // ps3: slot of record g - 1
            if (g < n) {
                const uint32_t s = g % NS;
                const uint8_t * rec = sm + OFF_REC + s * REC_MAX;
                const bool w_ok = tc::mbar_wait3(&bars[B_RFULL + s], (g / NS) & 1u, &bars[B_SFULL], g & 1u, &bars[B_AK + b], (g >> 1) & 1u);
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
                warp_arrive(&bars[B_REMPTY + s], lane);
                // ---- scores of token tl for rows 8 half .. 8 half + 7 (log2 domain), row maxima, max |Vscale| ----
                float s2[8];
                {
                    const uint32_t pos = p.S + (r_begin + g) * (uint32_t) G + (uint32_t) tl;
                    const float kts = kt * sl2;
#pragma unroll
                    for (int i = 0; i < 8; i += 2) {                   // rows in pairs: packed fp32 arithmetic
                        const float2 C = i < 4 ? add2(make_float2(cp0[i], cp0[i + 1]), make_float2(cp0[i + 4], cp0[i + 5]))
                                               : add2(make_float2(cp1[i - 4], cp1[i - 3]), make_float2(cp1[i], cp1[i + 1]));
                        // digit sums: |a0|, |a1| < 2^19, so a0 + 256 a1 is exact in s32; a2 through the magic constant
                        const float2 hi = add2(make_float2(__uint_as_float(a2[i] + MAGIC_BITS), __uint_as_float(a2[i + 1] + MAGIC_BITS)),
                                               make_float2(-MAGIC, -MAGIC));
                        const float2 lo = make_float2((float) ((int) a0[i] + ((int) a1[i] << 8)), (float) ((int) a0[i + 1] + ((int) a1[i + 1] << 8)));
                        const float2 S = fma2(make_float2(65536.0f, 65536.0f), hi, lo);
                        const float2 v = mul2(make_float2(kts, kts), fma2(S, make_float2(kinv[i], kinv[i + 1]), C));
                        s2[i] = pos < qlim[i] ? v.x : -INFINITY;
                        s2[i + 1] = pos < qlim[i + 1] ? v.y : -INFINITY;
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
                            F[F_LSUM + r] = F[F_LSUM + r] * F[F_ALPHA + 16 * ps3 + r] + ((rl[0] + rl[8]) + (rl[16] + rl[24]));
                        }
                        F[F_M2 + 16 * b + r] = mn;
                        F[F_ALPHA + 16 * s3 + r] = mn == -INFINITY ? 1.0f : ex2(mold - mn);
                        F[F_VINV + 16 * s3 + r] = pow2f(-ev);
                    }
                    float * bc = F + F_BC + 16 * sw;
                    __syncwarp();
                    if (lane < 8) { bc[lane] = mn; bc[8 + lane] = vs; }
                    __syncwarp();
                    ld8(bc, mnew);
                    ld8(bc + 8, vscl);
                }
                // ---- weights, B_V = three s8 digits of round(P' 2^ev), row sums ----
                {
                    uint8_t * bv = sm + OFF_BV + b * 8 * BCH + b_off(8 * half, (tl & ~15) + pi_pos(tl & 15));
                    float ls[8], zs[8];
#pragma unroll
                    for (int i = 0; i < 8; i += 2) {                   // rows in pairs: packed fp32 arithmetic
                        const float2 d = add2(make_float2(s2[i], s2[i + 1]), make_float2(-mnew[i], -mnew[i + 1]));
                        const float2 pw = make_float2(mnew[i] == -INFINITY ? 0.0f : ex2(d.x), mnew[i + 1] == -INFINITY ? 0.0f : ex2(d.y));
                        ls[i] = pw.x;
                        ls[i + 1] = pw.y;
                        const float2 zz = mul2(pw, make_float2(vz, vz));
                        zs[i] = zz.x;
                        zs[i + 1] = zz.y;
                        const uint2 z = digits3x2(mul2(pw, make_float2(vsc, vsc)), make_float2(vscl[i], vscl[i + 1]));
                        bv[16 * i] = (uint8_t) z.x;
                        bv[16 * i + 256] = (uint8_t) (z.x >> 8);
                        bv[16 * i + 512] = (uint8_t) (z.x >> 16);
                        bv[16 * i + 16] = (uint8_t) z.y;
                        bv[16 * i + 16 + 256] = (uint8_t) (z.y >> 8);
                        bv[16 * i + 16 + 512] = (uint8_t) (z.y >> 16);
                    }
                    tc::fence_proxy_async();
                    const float lw = warp_rows8<false>(ls, lane);
                    const float zw = warp_rows8<false>(zs, lane);
                    if ((lane & 3) == 0) {
                        F[F_RL + 64 * b + 32 * half + 8 * quarter + (lane >> 2)] = lw;
                        F[F_RZ + 64 * s3 + 32 * half + 8 * quarter + (lane >> 2)] = zw;
                    }
                    warp_arrive(&bars[B_BV + b], lane);
                    warp_arrive(&bars[B_EPI + s3], lane);            // alpha, 2^-ev and z of record g for the epilogue
                }
            } else {
                tc::nbar_sync(2, NW * 32);                         // the last record's row sums are visible
                if (quarter == 0 && lane < 8 && n >= 1) {
                    const int r = 8 * half + lane;
                    const float * rl = F + F_RL + 64 * pb + 32 * half + lane;
                    F[F_LSUM + r] = F[F_LSUM + r] * F[F_ALPHA + 16 * ps3 + r] + ((rl[0] + rl[8]) + (rl[16] + rl[24]));
                }
            }
        }
        ok = tc::nbar_and(2, NW * 32, ok);
        if (lane == 0) F[F_OK + 1] = ok ? 1.0f : 0.0f;        // (read after the CTA barrier below)
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
        uint32_t loaded = pre_loaded, k_issued = 0, v_issued = 0;   // record 0 was issued before the staged rows
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
                ok = tc::mbar_wait2(&bars[B_AK + (b ^ 1u)], ((g + 1) >> 1) & 1u, &bars[B_SFREE], g & 1u);
                if (!ok) break;
                tc::fence_after_sync();
                issue_k(g + 1);
                ++k_issued;
            }
            // the stage of record g takes record g + NS once both consumer groups released it (the softmax warps do
            // right after reading S of record g, long before its B_V is ready: load early, ahead of V(g))
            if (loaded < n) {
                ok = tc::mbar_wait(&bars[B_REMPTY + g % NS], (g / NS) & 1u);
                if (!ok) break;
                load(loaded, next_blk);
                ++loaded;
                if (loaded < n) next_blk = blk_of(loaded);
            }
            ok = g >= 2 ? tc::mbar_wait3(&bars[B_AV + b], (g >> 1) & 1u, &bars[B_BV + b], (g >> 1) & 1u, &bars[B_OFREE + b], ((g - 2) >> 1) & 1u)
                        : tc::mbar_wait2(&bars[B_AV + b], (g >> 1) & 1u, &bars[B_BV + b], (g >> 1) & 1u);
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
        }
        F[F_OK + 2] = ok ? 1.0f : 0.0f;
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
    // ---- partials (m in the natural-log domain, l, o[D]) per real query row, valid only if every role finished ----
    {
        const bool all_ok = F[F_OK] != 0.0f && F[F_OK + 1] != 0.0f && F[F_OK + 2] != 0.0f && ok;
        const uint32_t * rowoff = reinterpret_cast<const uint32_t *>(F + F_ROWOFF);
        const float * xf = reinterpret_cast<const float *>(sm + OFF_XF);
        for (int i = tid; i < p.rows * (D / 2); i += NT) {     // outputs: pairs of channels, coalesced
            const int r = i / (D / 2), c = 2 * (i % (D / 2));
            const float2 v = all_ok ? make_float2(xf[r * D + c], xf[r * D + c + 1]) : make_float2(0.0f, 0.0f);
            *reinterpret_cast<float2 *>(p.part + rowoff[r] + 2 + c) = v;
        }
        if (tid < p.rows) {                                    // m and l
            const int r = tid;
            const uint32_t mb = n >= 1 ? (n - 1) & 1u : 1u;
            const float m2 = F[F_M2 + 16 * mb + r];
            float * dst = p.part + rowoff[r];
            dst[0] = all_ok ? (m2 == -INFINITY ? m2 : m2 * LN2) : -INFINITY;
            dst[1] = all_ok ? F[F_LSUM + r] : 0.0f;
        }
    }
    if (warp == 2 * NW) tc::tmem_dealloc(tmem, TM_COLS);
}

template <bool QROT>
__global__ void __launch_bounds__(NT, 1) attend_body_tc_kernel(const __grid_constant__ TcParams p) { body_tc_body<QROT>(p); }

// the descriptor-driven form: the plan was made on the device (body_tc_dyn_plan_kernel); the grid covers the most
// splits a plan can use and the CTAs past the plan's return at once
__global__ void __launch_bounds__(NT, 1) attend_body_tc_dyn_kernel(const TcParams * __restrict__ pp) {
    if ((int) blockIdx.x >= pp->n_splits) return;
    body_tc_body<false>(*pp);
}

// fp64 steps of the record balancing, rounded as written (the device form must not contract them into fma)
SJK_HD double d_mul(double a, double b) {
#ifdef __CUDA_ARCH__
    return __dmul_rn(a, b);
#else
    return a * b;
#endif
}
SJK_HD double d_add(double a, double b) {
#ifdef __CUDA_ARCH__
    return __dadd_rn(a, b);
#else
    return a + b;
#endif
}
SJK_HD double d_div(double a, double b) {
#ifdef __CUDA_ARCH__
    return __ddiv_rn(a, b);
#else
    return a / b;
#endif
}

// A staged-row chunk costs about DENSE_WEIGHT sealed records of CTA time; the record ranges are balanced so that
// the CTAs that also take a chunk get fewer records.
constexpr double DENSE_WEIGHT = 4.5;

// The plan of one call (records [0, n_rec) of KV heads kv0 .., plus the staged rows of dense_regions). Returns the
// splits per KV head. Runs on the host (sjk_tc_body_launch) and in the descriptor-driven call's planner kernel.
SJK_HD int fill_plan(TcParams & p, const sjk_view & v, uint32_t B, uint32_t N, uint32_t n_rec, int dense_regions, uint32_t qpos0,
                     int n_q, int n_head, int kv0, int n_kv, const float * q, float scale, float * part, int split0,
                     bool enabled, int max_ctas) {
    p.lay = v.lay; p.body = v.body; p.blocks = v.blocks; p.H = v.n_head_kv; p.kv0 = kv0; p.S = v.S;
    p.n_rec = n_rec; p.qpos0 = qpos0; p.n_q = n_q; p.n_head = n_head; p.grp = n_head / n_kv; p.rows = n_q * p.grp;
    for (int r = 0; r < NR; ++r) {
        const int iq = r < p.rows ? r / p.grp : 0, g = r < p.rows ? r % p.grp : 0;
        p.row_iq[r] = (uint32_t) iq;
        p.row_q[r] = iq * n_head + g;
    }
    p.q = q; p.scale = scale; p.fwht_scale = 0.0f; p.part = part; p.split0 = split0;
    p.sink = v.sink; p.ring = v.ring; p.staging = v.staging; p.sink_type = v.sink_type; p.cap = v.cap;
    p.stage_bytes = (uint32_t) v.stage_bytes; p.B = B; p.N = N;
    p.n_sink_chunks = 0; p.n_dense = 0;
    if (dense_regions) {
        const uint32_t s_end = v.S < N ? v.S : N, t0 = B > v.S ? B : v.S;
        p.n_sink_chunks = (dense_regions & 1) ? (s_end + 127u) / 128u : 0u;
        p.n_dense = p.n_sink_chunks + ((dense_regions & 2) && N > t0 ? (N - t0 + 127u) / 128u : 0u);
    }
    const int splits = enabled ? sjk_tcbody_split_count(n_kv, n_rec, p.n_dense, max_ctas) : 0;
    p.n_splits = splits;
    if (splits == 0) return 0;
    // record ranges: split s takes d(s) chunks (u = s, s + splits, ..) and about target - DENSE_WEIGHT d(s) records
    double want[MAX_SPLITS], total = 0.0;
    const double target = d_div(d_add((double) n_rec, d_mul(DENSE_WEIGHT, (double) p.n_dense)), (double) splits);
    for (int s = 0; s < splits; ++s) {
        const uint32_t d = p.n_dense > (uint32_t) s ? (p.n_dense - 1u - (uint32_t) s) / (uint32_t) splits + 1u : 0u;
        const double w = d_add(target, -d_mul(DENSE_WEIGHT, (double) d));
        want[s] = w > 0.0 ? w : 0.0;
        total = d_add(total, want[s]);
    }
    double run = 0.0;
    p.rec_bounds[0] = 0;
    for (int s = 0; s < splits; ++s) {
        run = d_add(run, want[s]);
        uint32_t b = total > 0.0 ? (uint32_t) d_add(d_mul(d_div(run, total), (double) n_rec), 0.5) : 0u;
        if (b > n_rec) b = n_rec;
        if (b < p.rec_bounds[s]) b = p.rec_bounds[s];
        p.rec_bounds[s + 1] = b;
    }
    p.rec_bounds[splits] = n_rec;
    return splits;
}

// planner of the descriptor-driven call: the plan of sjk_tc_body_launch for the counts in *ds
__global__ void body_tc_dyn_plan_kernel(const sjk_dyn_state * __restrict__ ds, sjk_view v, int n_q, int n_head, int kv0, int n_kv,
                                        const float * q, float scale, float * part, TcParams * out) {
    if (threadIdx.x != 0) return;
    const sjk_dyn_state d = *ds;
    fill_plan(*out, v, d.B, d.N, d.n_tc, (int) d.dense_regions, d.qpos0, n_q, n_head, kv0, n_kv, q, scale, part, 0, d.ok != 0,
              148 - d.dense_sms);
}

}  // namespace

// ---- host side ---------------------------------------------------------------------------------------------

// Whether the tensor-core body path applies: 4-bit scalar records (fragment-ordered payload), D = 256,
// at most 16 query rows per KV head.
int sjk_tc_body_supported(const sjk_view * v, int n_q, int grp) {
    const sj_kvarn_layout & l = v->lay;
    return l.D == 256 && l.G == 128 && l.body == SJKVARN_BODY_SCALAR && l.bits_k == 4 && l.bits_v == 4 &&
           n_q * grp <= NR && l.bytes == REC_MAX && l.k_scale % 16 == 0;
}

// Splits (persistent CTAs) per KV head: one CTA per SM over the call's KV heads, at most one per work item.
int sjk_tc_body_max_splits(int n_kv) {
    const int t = (148 + (n_kv > 0 ? n_kv : 1) - 1) / (n_kv > 0 ? n_kv : 1);
    return t < MAX_SPLITS ? t : MAX_SPLITS;
}

int sjk_tc_body_launch(const sjk_view * v, uint32_t B, uint32_t N, uint32_t n_rec, int dense_regions, uint32_t qpos0, int n_q,
                       int n_head, int kv0, int n_kv, const float * q, float scale, float * part, int split0, int max_ctas,
                       bool q_model, int * splits_out, sjk_stream st) {
    TcParams p;
    const int splits = fill_plan(p, *v, B, N, n_rec, dense_regions, qpos0, n_q, n_head, kv0, n_kv, q, scale, part, split0, true,
                                 max_ctas);
    p.fwht_scale = sjk_fwht_scale(D);
    *splits_out = splits;
    if (splits == 0) return 0;
    const dim3 grid((unsigned) splits, (unsigned) n_kv);
    // programmatic dependent launch: the CTAs may start while the previous kernel of the stream finishes and wait
    // for it on the device before they read anything (body_tc_body)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = q_model ? SMEM_TOTAL_QROT : SMEM_TOTAL;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (q_model) {
        cudaError_t e = cudaFuncSetAttribute(attend_body_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_TOTAL_QROT);
        if (e != cudaSuccess) return sjk_check(e);
        if (sjk_check(cudaLaunchKernelEx(&cfg, attend_body_tc_kernel<true>, p))) return SJK_ERR_DEVICE;
        return sjk_check_launch();
    }
    cudaError_t e = cudaFuncSetAttribute(attend_body_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_TOTAL);
    if (e != cudaSuccess) return sjk_check(e);
    if (sjk_check(cudaLaunchKernelEx(&cfg, attend_body_tc_kernel<false>, p))) return SJK_ERR_DEVICE;
    return sjk_check_launch();
}

size_t sjk_tc_body_params_bytes(void) { return sizeof(TcParams); }

// Descriptor-driven form: the counts come from *ds (written on the device by the call's planner), this function's
// planner kernel writes the plan into `params` (sjk_tc_body_params_bytes() bytes of device memory) and the kernel
// reads it there. The grid covers the most splits a plan can use.
int sjk_tc_body_dyn_launch(const sjk_view * v, int n_q, int n_head, int kv0, int n_kv, const float * q, float scale,
                           float * part, const sjk_dyn_state * ds, void * params, sjk_stream st) {
    TcParams * dp = static_cast<TcParams *>(params);
    body_tc_dyn_plan_kernel<<<1, 32, 0, st>>>(ds, *v, n_q, n_head, kv0, n_kv, q, scale, part, dp);
    if (sjk_check_launch()) return SJK_ERR_DEVICE;
    const int max_splits = sjk_tc_body_max_splits(n_kv);
    cudaError_t e = cudaFuncSetAttribute(attend_body_tc_dyn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_TOTAL);
    if (e != cudaSuccess) return sjk_check(e);
    attend_body_tc_dyn_kernel<<<dim3((unsigned) max_splits, (unsigned) n_kv), NT, SMEM_TOTAL, st>>>(dp);
    return sjk_check_launch();
}

SJK_STATUS_READER(sjk_tc_body_status_take)
