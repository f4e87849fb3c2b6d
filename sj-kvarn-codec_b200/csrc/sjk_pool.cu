// sjk_pool.cu - the paged record pool's bookkeeping on the device: block reservation and release for many
// sequences in one launch, and truncation of many (sequence, layer) caches in one scrub launch plus one release
// launch (the batched server paths of the reference's pool mode, sj_kvarn.h:1581-1603, 1643-1675, 1716-1739).
//
// The device pool is a stack of free block ids in device memory, the same stack the host pool keeps
// (sj_kvarn_pool.free_ids / n_free): sjk_pool_dev_load copies a host pool's stack in, sjk_pool_dev_store copies it
// back. Requests are served in order with the host's semantics, so a batch leaves exactly the block tables and the
// stack that the same calls on the host pool leave:
//   reserve [g0, g1) of a block table: every NO_BLOCK entry, in group order, takes the id on top of the stack; a
//     request that needs more blocks than are free takes none and reports SJKVARN_ERR_POOL_FULL
//     (sj_kvarn__seq_reserve: it releases what it took, which restores the stack);
//   release [g0, g1): every entry that holds a block pushes it, in group order (while the stack has room), and
//     becomes NO_BLOCK (sj_kvarn__seq_release).
// One CTA walks the requests in order; inside a request the groups are split over its threads with a block-wide
// prefix sum.
//
// Truncation scrub (sj_kvarn_layer_truncate for a batch): per request, the records of the dropped groups
// [ (B_new - S) / G, (B_old - S) / G ) (through the block table when there is one, skipping NO_BLOCK), the sink rows
// of [resume, min(n_old, S)) and the ring rows of the last cap positions of [max(resume, S), n_old) are zeroed;
// grid: blockIdx.y = request, the CTAs of a request split its words.
#include <cuda_runtime.h>
#include <stdint.h>

#include "sjk_common.cuh"
#include "sjk_internal.h"

namespace {

constexpr int NT = 256;

struct DevPool {                        // device layout (sjk_pool_dev_bytes)
    uint32_t n_free, n_blocks, pad0, pad1;
    uint32_t ids[1];                    // [n_blocks]
};

struct ReqList {
    int n;
    sjk_block_req req[SJK_POOL_MAX_REQ];
};

// exclusive prefix sum of v over the CTA (NT threads); *total gets the sum. s: NT / 32 + 1 ints of shared memory.
__device__ __forceinline__ int cta_scan(int v, int * s, int * total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < NT / 32 ? s[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < NT / 32) s[lane] = w;                    // inclusive prefix of the warp sums
    }
    __syncthreads();
    const int before = (warp ? s[warp - 1] : 0) + x - v;
    *total = s[NT / 32 - 1];
    __syncthreads();                                          // s is reused by the next call
    return before;
}

__global__ void __launch_bounds__(NT) pool_reserve_kernel(DevPool * pool, const __grid_constant__ ReqList rl, int * status) {
    __shared__ int s_scan[NT / 32 + 1];
    __shared__ uint32_t s_free;
    if (threadIdx.x == 0) s_free = pool->n_free;
    __syncthreads();
    for (int r = 0; r < rl.n; ++r) {
        const sjk_block_req q = rl.req[r];
        // blocks the request needs
        int need = 0;
        for (uint32_t g = q.g0 + threadIdx.x; g < q.g1; g += NT) need += q.blocks[g] == SJKVARN_NO_BLOCK ? 1 : 0;
        int total;
        cta_scan(need, s_scan, &total);
        const uint32_t n_free = s_free;
        if ((uint32_t) total > n_free) {
            if (threadIdx.x == 0) status[r] = SJKVARN_ERR_POOL_FULL;
            continue;                                         // nothing taken: the stack is as it was
        }
        // the k-th NO_BLOCK entry in group order takes ids[n_free - 1 - k]
        int base = 0;
        for (uint32_t g0 = q.g0; g0 < q.g1; g0 += NT) {
            const uint32_t g = g0 + threadIdx.x;
            const int take = g < q.g1 && q.blocks[g] == SJKVARN_NO_BLOCK ? 1 : 0;
            int chunk;
            const int k = base + cta_scan(take, s_scan, &chunk);
            if (take) q.blocks[g] = pool->ids[n_free - 1u - (uint32_t) k];
            base += chunk;
        }
        __syncthreads();
        if (threadIdx.x == 0) { s_free = n_free - (uint32_t) total; status[r] = 0; }
        __syncthreads();
    }
    if (threadIdx.x == 0) pool->n_free = s_free;
}

__global__ void __launch_bounds__(NT) pool_release_kernel(DevPool * pool, const __grid_constant__ ReqList rl) {
    __shared__ int s_scan[NT / 32 + 1];
    __shared__ uint32_t s_free;
    if (threadIdx.x == 0) s_free = pool->n_free;
    __syncthreads();
    const uint32_t cap = pool->n_blocks;
    for (int r = 0; r < rl.n; ++r) {
        const sjk_block_req q = rl.req[r];
        for (uint32_t g0 = q.g0; g0 < q.g1; g0 += NT) {
            const uint32_t g = g0 + threadIdx.x;
            const uint32_t id = g < q.g1 ? q.blocks[g] : SJKVARN_NO_BLOCK;
            const int push = id != SJKVARN_NO_BLOCK ? 1 : 0;
            int chunk;
            const uint32_t n_free = s_free;
            const uint32_t pos = n_free + (uint32_t) cta_scan(push, s_scan, &chunk);
            if (push && pos < cap) pool->ids[pos] = id;       // the host pushes while the stack has room
            if (g < q.g1) q.blocks[g] = SJKVARN_NO_BLOCK;
            if (threadIdx.x == 0) s_free = n_free + (uint32_t) chunk < cap ? n_free + (uint32_t) chunk : cap;
            __syncthreads();
        }
    }
    if (threadIdx.x == 0) pool->n_free = s_free;
}

struct TruncList {
    int n;
    sjk_trunc_req req[SJK_TRUNC_MAX_REQ];
};

// the spans a truncation request zeroes: dropped groups (one span of H records per group), the sink rows, at most
// two runs of ring rows
struct TruncSpans {
    uint32_t g0, g1;                    // dropped groups
    uint32_t grp_words;                 // 32-bit words of one group's records (all KV heads)
    uint32_t sink_words;                // words of the sink rows, from sink_off
    size_t sink_off;
    uint32_t ring_words[2];             // words of the ring runs, from ring_off
    size_t ring_off[2];
};

__device__ __forceinline__ TruncSpans trunc_spans(const sjk_trunc_req & q) {
    TruncSpans t = {};
    const uint32_t S = q.S, G = q.group, H = q.n_head_kv;
    if (q.B_new < q.B_old) { t.g0 = (q.B_new - S) / G; t.g1 = (q.B_old - S) / G; }
    t.grp_words = (uint32_t) ((size_t) H * q.rec_bytes / 4u);
    if (q.resume < q.n_old && q.resume < S) {
        const uint32_t end = q.n_old < S ? q.n_old : S;
        t.sink_off = (size_t) q.resume * H * q.sink_entry_bytes;
        t.sink_words = (uint32_t) ((size_t) (end - q.resume) * H * q.sink_entry_bytes / 4u);
    }
    uint32_t from = q.resume > S ? q.resume : S;
    if (q.n_old > from && q.n_old - from > q.cap) from = q.n_old - q.cap;
    const size_t row = (size_t) H * 2u * q.stage_bytes;
    for (int k = 0; k < 2 && from < q.n_old; ++k) {
        const uint32_t slot = sjk_ring_slot(S, q.cap, from);
        uint32_t run = q.cap - slot;
        if (run > q.n_old - from) run = q.n_old - from;
        t.ring_off[k] = (size_t) slot * row;
        t.ring_words[k] = (uint32_t) (run * row / 4u);
        from += run;
    }
    return t;
}

__global__ void __launch_bounds__(NT) trunc_scrub_kernel(const __grid_constant__ TruncList tl) {
    const sjk_trunc_req & q = tl.req[blockIdx.y];
    const TruncSpans t = trunc_spans(q);
    const uint64_t w_groups = (uint64_t) (t.g1 - t.g0) * t.grp_words;
    const uint64_t total = w_groups + t.sink_words + t.ring_words[0] + t.ring_words[1];
    for (uint64_t w = (uint64_t) blockIdx.x * NT + threadIdx.x; w < total; w += (uint64_t) gridDim.x * NT) {
        uint32_t * dst;
        if (w < w_groups) {
            const uint32_t g = t.g0 + (uint32_t) (w / t.grp_words), off = (uint32_t) (w % t.grp_words);
            const uint32_t blk = q.blocks ? q.blocks[g] : g;
            if (blk == SJKVARN_NO_BLOCK) continue;
            dst = reinterpret_cast<uint32_t *>(q.body + (size_t) blk * t.grp_words * 4u) + off;
        } else if (w < w_groups + t.sink_words) {
            dst = reinterpret_cast<uint32_t *>(q.sink + t.sink_off) + (w - w_groups);
        } else if (w < w_groups + t.sink_words + t.ring_words[0]) {
            dst = reinterpret_cast<uint32_t *>(q.ring + t.ring_off[0]) + (w - w_groups - t.sink_words);
        } else {
            dst = reinterpret_cast<uint32_t *>(q.ring + t.ring_off[1]) + (w - w_groups - t.sink_words - t.ring_words[0]);
        }
        *dst = 0u;
    }
}

}  // namespace

extern "C" size_t sjk_pool_dev_bytes(uint32_t n_blocks) { return 16u + (size_t) n_blocks * sizeof(uint32_t); }

extern "C" int sjk_pool_dev_load(void * dev, const sj_kvarn_pool * pool, sjk_stream st) {
    if (!dev || !pool || !pool->free_ids) return SJKVARN_ERR_ARG;
    const uint32_t hdr[4] = {pool->n_free, pool->n_blocks, 0u, 0u};
    if (sjk_check(cudaMemcpyAsync(dev, hdr, sizeof hdr, cudaMemcpyHostToDevice, st))) return SJK_ERR_DEVICE;
    if (sjk_check(cudaMemcpyAsync(static_cast<uint8_t *>(dev) + 16, pool->free_ids, (size_t) pool->n_blocks * sizeof(uint32_t),
                                  cudaMemcpyHostToDevice, st)))
        return SJK_ERR_DEVICE;
    return sjk_check(cudaStreamSynchronize(st)) ? SJK_ERR_DEVICE : 0;
}

extern "C" int sjk_pool_dev_store(const void * dev, sj_kvarn_pool * pool, sjk_stream st) {
    if (!dev || !pool || !pool->free_ids) return SJKVARN_ERR_ARG;
    uint32_t hdr[4];
    if (sjk_check(cudaMemcpyAsync(hdr, dev, sizeof hdr, cudaMemcpyDeviceToHost, st))) return SJK_ERR_DEVICE;
    if (sjk_check(cudaMemcpyAsync(pool->free_ids, static_cast<const uint8_t *>(dev) + 16, (size_t) pool->n_blocks * sizeof(uint32_t),
                                  cudaMemcpyDeviceToHost, st)))
        return SJK_ERR_DEVICE;
    if (sjk_check(cudaStreamSynchronize(st))) return SJK_ERR_DEVICE;
    if (hdr[1] != pool->n_blocks) return SJKVARN_ERR_ARG;
    pool->n_free = hdr[0];
    return 0;
}

extern "C" int sjk_pool_reserve_batch(void * dev, const sjk_block_req * reqs, int n, int * status, sjk_stream st) {
    if (!dev || n < 0 || n > SJK_POOL_MAX_REQ || (n && (!reqs || !status))) return SJKVARN_ERR_ARG;
    if (n == 0) return 0;
    static thread_local ReqList rl;
    rl.n = n;
    for (int i = 0; i < n; ++i) {
        if (!reqs[i].blocks || reqs[i].g1 < reqs[i].g0) return SJKVARN_ERR_ARG;
        rl.req[i] = reqs[i];
    }
    pool_reserve_kernel<<<1, NT, 0, st>>>(static_cast<DevPool *>(dev), rl, status);
    return sjk_check_launch();
}

extern "C" int sjk_pool_release_batch(void * dev, const sjk_block_req * reqs, int n, sjk_stream st) {
    if (!dev || n < 0 || n > SJK_POOL_MAX_REQ || (n && !reqs)) return SJKVARN_ERR_ARG;
    if (n == 0) return 0;
    static thread_local ReqList rl;
    rl.n = n;
    for (int i = 0; i < n; ++i) {
        if (!reqs[i].blocks || reqs[i].g1 < reqs[i].g0) return SJKVARN_ERR_ARG;
        rl.req[i] = reqs[i];
    }
    pool_release_kernel<<<1, NT, 0, st>>>(static_cast<DevPool *>(dev), rl);
    return sjk_check_launch();
}

extern "C" int sjk_truncate_batch(const sjk_trunc_req * reqs, int n, void * dev, sjk_stream st) {
    if (n < 0 || n > SJK_TRUNC_MAX_REQ || (n && !reqs)) return SJKVARN_ERR_ARG;
    if (n == 0) return 0;
    static thread_local TruncList tl;
    static thread_local ReqList rel;
    tl.n = n;
    rel.n = 0;
    uint64_t most = 0;
    for (int i = 0; i < n; ++i) {
        const sjk_trunc_req & q = reqs[i];
        if (!q.body || !q.sink || !q.ring || q.group == 0 || q.cap == 0 || q.B_old < q.S || q.B_new < q.S || q.B_new > q.B_old ||
            q.rec_bytes % 4 || q.sink_entry_bytes % 4 || q.stage_bytes % 2)
            return SJKVARN_ERR_ARG;
        tl.req[i] = q;
        const uint64_t w = (uint64_t) (q.B_old - q.B_new) / q.group * q.n_head_kv * q.rec_bytes / 4u +
                           (uint64_t) (q.S + q.cap) * q.n_head_kv * (q.sink_entry_bytes + 2u * q.stage_bytes) / 4u;
        if (w > most) most = w;
        if (q.release && q.blocks && q.B_new < q.B_old) {
            if (!dev || rel.n >= SJK_POOL_MAX_REQ) return SJKVARN_ERR_ARG;
            sjk_block_req & r = rel.req[rel.n++];
            r.blocks = q.blocks;
            r.g0 = (q.B_new - q.S) / q.group;
            r.g1 = (q.B_old - q.S) / q.group;
        }
    }
    // enough CTAs per request for a few words per thread, at most about a wave over all requests
    uint64_t per = (most + (uint64_t) NT * 16u - 1u) / ((uint64_t) NT * 16u);
    const uint64_t cap_x = (2u * 148u + (uint64_t) n - 1u) / (uint64_t) n;
    if (per > cap_x) per = cap_x;
    if (per < 1) per = 1;
    trunc_scrub_kernel<<<dim3((unsigned) per, (unsigned) n), NT, 0, st>>>(tl);
    if (sjk_check_launch()) return SJK_ERR_DEVICE;
    if (rel.n) {
        pool_release_kernel<<<1, NT, 0, st>>>(static_cast<DevPool *>(dev), rel);
        return sjk_check_launch();
    }
    return 0;
}
