// sjk_merge.cuh - the merge of attention partials (m, l, o[D]) shared by the split merge of one call, the merge of
// context slices (sjk_attend_merge) and the exchange over peer memory (sjk_xchg_exchange, sjk_attend_partial_xchg),
// so that every path combines the same partials with the same arithmetic, in the same order.
//
//   out[row] = sum_i o_i w_i / sum_i l_i w_i,   w_i = e^(m_i - m), m = max_i m_i   (splits i in index order)
//
// One CTA of 256 threads per (row, 64-channel tile).
//
// Exchange over peer memory: rank r's CTA (row, tile) stores its tile of the rank's triple (m, l, o[64]) into slot
// [parity][r][row] of every rank's exchange buffer (plain 8-byte stores through CUDA IPC mappings of the other GPUs'
// buffers; no TMA, no multicast), then waits (bounded) until the tile's words of every rank's slot in its own buffer
// carry the epoch, copies them to shared memory and merges the world triples in rank order there - the all-gather +
// merge of the same triples, in one kernel. Every word holds a value in its low half and the epoch that wrote it in
// its high half; 8-byte stores and loads are single-copy atomic, so a word is either the old or the new one, and no
// fence or separate flag is needed (each word validates itself).
// Exchange buffer: u64 words [2][world][n_rows][D + 2] (m, l, o[D] per row). Consecutive epochs alternate parities;
// a rank publishes epoch e + 2 only after its merge of e + 1 saw every rank's words of e + 1, written after those
// ranks' merges of e completed (stream order), so a slot is never overwritten while it is read.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sjk.h"

namespace sjkm {

constexpr int MERGE_SPLITS = 768;         // >= the most splits a call can make (148 + 296 + 296)
constexpr int MERGE_PRE = 24;             // outputs per thread loaded ahead of the weights
constexpr uint64_t XCHG_WAIT_NS = 1000000000ull;   // 1 s of wall clock per exchange wait

__host__ __device__ inline int merge_tiles(int D) { return (D + 63) / 64; }
__host__ __device__ inline size_t xchg_words_bytes(int world, int n_rows, int D) {
    return (size_t) 2 * world * n_rows * (size_t) (D + 2) * sizeof(uint64_t);
}

// Combines `splits` partial sets part[splits][n_rows][D + 2] for (row, channels d0 .. d0 + 63). On return every thread
// holds m and t = sum l w; the tile's unnormalized outputs are acc_o(wts + splits, tid) for tid < 64. wts: shared
// memory of at least splits + 256 floats; s_red: 16 floats.
__device__ __forceinline__ void merge_tile(const float * part, int splits, int n_rows, int D, int row, int d0, float * wts,
                                           float * s_red, float & m_out, float & t_out) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
    m_out = m;
    t_out = t;
}

__device__ __forceinline__ float acc_o(const float * acc, int tid) {
    return (acc[tid] + acc[64 + tid]) + (acc[128 + tid] + acc[192 + tid]);
}

// the normalized output of the tile (threads 0..63)
__device__ __forceinline__ void store_out(const float * acc, float t, int D, int row, int d0, float * out) {
    const int tid = threadIdx.x;
    const float s_inv = t == 0.0f ? 0.0f : 1.0f / t;
    if (tid < 64 && d0 + tid < D) out[(size_t) row * D + d0 + tid] = acc_o(acc, tid) * s_inv;
}

// the kernels' view of the ranks' exchange buffers
struct XchgArgs {
    uint8_t * buf[SJK_XCHG_MAX_WORLD];    // every rank's buffer as this process maps it; buf[rank] is its own
    int world, rank;
    uint32_t epoch;
};

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

constexpr int XCHG_TILE_WORDS = 66;        // m, l and 64 outputs of one (row, tile)

// Publish this rank's triple tile (m, t, and o = my_o of threads 0..63) of (row, tile) to every rank, and gather every
// rank's tile of the same (row, tile) into stage[world][66] (shared memory: m, l, o[64]); returns false (in every
// thread) when a wait ran out. n_rows, D: the shape of the exchange.
__device__ __forceinline__ bool xchg_publish_gather(const XchgArgs & x, int n_rows, int D, int row, int tile, float m, float t,
                                                    float my_o, float * stage) {
    const int tid = threadIdx.x, d0 = 64 * tile;
    const uint32_t par = x.epoch & 1u;
    const uint64_t tag = (uint64_t) x.epoch << 32;
    const size_t row_words = (size_t) (D + 2);
    // thread j < 64: o[d0 + j]; thread 64: m; thread 65: l (every tile's CTA writes the row's m and l: same values)
    if (tid < XCHG_TILE_WORDS) {
        const int w = tid < 64 ? 2 + d0 + tid : tid - 64;
        if (w < D + 2) {
            const float val = tid < 64 ? my_o : (tid == 64 ? m : t);
            const uint64_t word = tag | __float_as_uint(val);
            const size_t off = ((((size_t) par * x.world + x.rank) * n_rows + row) * row_words + (size_t) w) * sizeof(uint64_t);
            for (int dst = 0; dst < x.world; ++dst)
                asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(x.buf[dst] + off), "l"(word) : "memory");
        }
    }
    // gather: word j of source src's tile, polled in this rank's own buffer until it carries the epoch
    bool ok = true;
    const uint8_t * own = x.buf[x.rank];
    for (int i = tid; i < x.world * XCHG_TILE_WORDS; i += blockDim.x) {
        const int src = i / XCHG_TILE_WORDS, j = i - src * XCHG_TILE_WORDS;
        const int w = j < 2 ? j : 2 + d0 + (j - 2);
        float v = 0.0f;
        if (w < D + 2 && ok) {                                // after a wait ran out, the rest read as zeros
            const uint64_t * p = reinterpret_cast<const uint64_t *>(own) + (((size_t) par * x.world + src) * n_rows + row) * row_words + w;
            uint64_t word;
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(word) : "l"(p) : "memory");
            if ((word >> 32) != x.epoch) {
                const uint64_t t0 = gtimer();
                do {
                    __nanosleep(32);
                    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(word) : "l"(p) : "memory");
                } while ((word >> 32) != x.epoch && gtimer() - t0 < XCHG_WAIT_NS);
            }
            ok = ok && (word >> 32) == x.epoch;
            v = __uint_as_float((uint32_t) word);
        }
        stage[i] = v;
    }
    return __syncthreads_and(ok) != 0;
}

}  // namespace sjkm
