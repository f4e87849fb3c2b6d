// sjk_merge.cuh - the merge of attention partials (m, l, o[D]) shared by the split merge of one call, the merge of
// context slices (sjk_attend_merge) and the exchange over peer memory (sjk_xchg_exchange, sjk_attend_partial_xchg),
// so that every path combines the same partials with the same arithmetic, in the same order.
//
//   out[row] = sum_i o_i w_i / sum_i l_i w_i,   w_i = e^(m_i - m), m = max_i m_i   (splits i in index order)
//
// One CTA of 256 threads per (row, 64-channel tile).
//
// Exchange over peer memory: rank r's CTA (row, tile) stores its tile of the rank's triple (m, l, o[64]) into slot
// [parity][r][row] of every rank's exchange buffer (plain stores through CUDA IPC mappings of the other GPUs'
// buffers; no TMA, no multicast), raises flag [parity][r][row][tile] = epoch in each buffer with a release store at
// system scope, then waits (bounded) until the flags [parity][src][row][tile] of its own buffer all hold the epoch
// and merges the world slots of its (row, tile) in rank order - the all-gather + merge of the same triples, in one
// kernel.
// Exchange buffer: flags u32 [2][SJK_XCHG_MAX_WORLD][n_rows][tiles] (rounded up to 256 bytes), then slots
// float [2][world][n_rows][D + 2]. Consecutive epochs alternate parities; a rank publishes epoch e + 2 only after its
// merge of e + 1 saw every rank's flags of e + 1, raised after those ranks' merges of e completed (stream order), so
// a slot is never overwritten while it is read.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sjk.h"

namespace sjkm {

constexpr int MERGE_SPLITS = 768;         // >= the most splits a call can make (148 + 296 + 296)
constexpr int MERGE_PRE = 24;             // outputs per thread loaded ahead of the weights
constexpr uint64_t XCHG_WAIT_NS = 1000000000ull;   // 1 s of wall clock per exchange wait

__host__ __device__ inline int merge_tiles(int D) { return (D + 63) / 64; }
__host__ __device__ inline size_t xchg_flag_bytes(int n_rows, int D) {
    return ((size_t) 2 * SJK_XCHG_MAX_WORLD * n_rows * merge_tiles(D) * sizeof(uint32_t) + 255) & ~(size_t) 255;
}

// Combines `splits` partial sets part[splits][n_rows][D + 2] for (row, channels d0 .. d0 + 63). On return every thread
// holds m and t = sum l w; the tile's unnormalized outputs are acc_o(wts + splits, tid) for tid < 64. wts: shared
// memory of at least splits + 256 floats; s_red: 16 floats.
// CG: read the partials through L2 only (partials that other GPUs wrote during this kernel)
template <bool CG = false>
__device__ __forceinline__ float ldp(const float * p) { return CG ? __ldcg(p) : *p; }
template <bool CG = false>
__device__ __forceinline__ float2 ldp2(const float * p) {
    return CG ? __ldcg(reinterpret_cast<const float2 *>(p)) : *reinterpret_cast<const float2 *>(p);
}

template <bool CG = false>
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
        xo[k] = i < splits ? ldp<CG>(src + (size_t) i * step) : 0.0f;
    }
    // one pass over (m, l) of the splits this thread owns (at most MERGE_SPLITS / 256)
    float mi[MERGE_SPLITS / 256], li[MERGE_SPLITS / 256];
#pragma unroll
    for (int k = 0; k < MERGE_SPLITS / 256; ++k) {
        const int i = tid + 256 * k;
        mi[k] = -INFINITY; li[k] = 0.0f;
        if (i < splits) {
            const float2 ml = ldp2<CG>(part + ((size_t) i * n_rows + row) * (D + 2));
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
    for (int i = grp4 + 4 * MERGE_PRE; i < splits; i += 4) o = fmaf(ldp<CG>(src + (size_t) i * step), wts[i], o);
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

// Publish this rank's triple tile (m, t, and o = my_o for threads 0..63) of (row, tile) to every rank, then wait for
// every rank's; returns false (in every thread) when a wait ran out. n_rows, D: the shape of the exchange.
__device__ __forceinline__ bool xchg_publish_wait(const XchgArgs & x, int n_rows, int D, int row, int tile, float m, float t,
                                                  float my_o) {
    const int tid = threadIdx.x, d0 = 64 * tile, tiles = merge_tiles(D);
    const uint32_t par = x.epoch & 1u;
    const size_t fb = xchg_flag_bytes(n_rows, D);
    const size_t slot_off = (((size_t) par * x.world + x.rank) * n_rows + row) * (D + 2);
    for (int dst = 0; dst < x.world; ++dst) {
        float * slot = reinterpret_cast<float *>(x.buf[dst] + fb) + slot_off;
        if (tid < 64 && d0 + tid < D) slot[2 + d0 + tid] = my_o;
        if (tid == 64) { slot[0] = m; slot[1] = t; }          // every tile's CTA writes the row's (m, l): same values
    }
    // the CTA barrier orders every thread's slot stores before the flag stores below, and a release at system scope
    // is cumulative: it makes the stores it is ordered after visible to a peer that acquires the flag
    __syncthreads();
    const size_t fidx_src = (((size_t) par * SJK_XCHG_MAX_WORLD + x.rank) * n_rows + row) * tiles + tile;
    if (tid < x.world) {
        uint32_t * flag = reinterpret_cast<uint32_t *>(x.buf[tid]) + fidx_src;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(x.epoch) : "memory");
    }
    bool ok = true;
    if (tid < x.world) {
        const uint32_t * flag = reinterpret_cast<const uint32_t *>(x.buf[x.rank]) +
                                (((size_t) par * SJK_XCHG_MAX_WORLD + tid) * n_rows + row) * tiles + tile;
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v != x.epoch) {
            const uint64_t t0 = gtimer();
            do {
                __nanosleep(100);
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
            } while (v != x.epoch && gtimer() - t0 < XCHG_WAIT_NS);
        }
        ok = v == x.epoch;
    }
    ok = __syncthreads_and(ok) != 0;
    __threadfence();
    return ok;
}

// the local slots of the epoch's parity: [world][n_rows][D + 2]
__device__ __forceinline__ const float * xchg_slots(const XchgArgs & x, int n_rows, int D) {
    return reinterpret_cast<const float *>(x.buf[x.rank] + xchg_flag_bytes(n_rows, D)) +
           (size_t) (x.epoch & 1u) * x.world * n_rows * (D + 2);
}

}  // namespace sjkm
