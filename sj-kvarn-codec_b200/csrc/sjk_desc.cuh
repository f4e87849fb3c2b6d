// sjk_desc.cuh - the per-ubatch cache descriptor read at run time by the descriptor-driven calls (sjk_*_dyn).
//
// The descriptor is the reference's ggml op input (INTEGRATION_LLAMACPP.md:52-70 of the reference): 16 int32 entries
// in device memory, set per ubatch, so a captured CUDA graph of a decode step replays unchanged while only the
// descriptor's values move. The kernels check its static entries against the cache they were launched on; a
// descriptor that fails a check makes the call do nothing and sets SJK_DEVICE_DESC in the device status word.
#pragma once
#include <stdint.h>

#include "../../include/sjk.h"

#ifndef SJK_HD
#ifdef __CUDACC__
#define SJK_HD __host__ __device__ __forceinline__
#else
#define SJK_HD inline
#endif
#endif

// the static description of a cache that a descriptor has to match (taken from a view on the host)
struct sjk_desc_ref {
    uint32_t S, cap, G, D, rec_bytes, H;
    int staging, body, sink_type;
};

// the entries that change per ubatch
struct sjk_desc_vals {
    uint32_t B, N, qpos0, B_old;
};

inline sjk_desc_ref sjk_desc_ref_of(const sjk_view & v) {
    sjk_desc_ref r;
    r.S = v.S; r.cap = v.cap; r.G = (uint32_t) v.lay.G; r.D = (uint32_t) v.lay.D; r.rec_bytes = v.lay.bytes;
    r.H = (uint32_t) v.n_head_kv; r.staging = v.staging; r.body = v.lay.body; r.sink_type = v.sink_type;
    return r;
}

// Checks a descriptor's entries e[0..15] against the cache: the static entries equal the cache's, every entry is
// non-negative, B and B_OLD lie on group boundaries at or past the sink with B_OLD <= B, and the staged positions
// [max(B, S), N) fit in the ring. Returns false for a descriptor that fails a check.
SJK_HD bool sjk_desc_check(const int32_t * e, const sjk_desc_ref & r, sjk_desc_vals * o) {
    for (int i = 0; i < SJK_DESC_N_ENTRIES; ++i)
        if (e[i] < 0) return false;
    if ((uint32_t) e[SJK_DESC_S] != r.S || (uint32_t) e[SJK_DESC_CAP] != r.cap || (uint32_t) e[SJK_DESC_G] != r.G ||
        (uint32_t) e[SJK_DESC_D] != r.D || (uint32_t) e[SJK_DESC_RECBYTES] != r.rec_bytes || (uint32_t) e[SJK_DESC_HKV] != r.H ||
        e[SJK_DESC_TYPE_K] != r.staging || e[SJK_DESC_TYPE_V] != r.staging || e[SJK_DESC_BODY_TYPE] != r.body ||
        e[SJK_DESC_SINK_TYPE] != r.sink_type)
        return false;
    const uint32_t B = (uint32_t) e[SJK_DESC_B], N = (uint32_t) e[SJK_DESC_N], B_old = (uint32_t) e[SJK_DESC_B_OLD];
    if (r.G == 0 || B < r.S || (B - r.S) % r.G != 0 || B_old < r.S || (B_old - r.S) % r.G != 0 || B_old > B) return false;
    const uint32_t t0 = B > r.S ? B : r.S;
    if (N > t0 && N - t0 > r.cap) return false;
    o->B = B; o->N = N; o->qpos0 = (uint32_t) e[SJK_DESC_QPOS0]; o->B_old = B_old;
    return true;
}

#ifdef __CUDACC__
// descriptor faults of this translation unit's kernels (SJK_DEVICE_DESC); read and cleared by the reader below
static __device__ int sjk_desc_status;
#define SJK_DESC_STATUS_READER(name)                                                      \
    int name(void) {                                                                      \
        int v_ = 0, zero_ = 0;                                                            \
        if (cudaMemcpyFromSymbol(&v_, sjk_desc_status, sizeof v_) != cudaSuccess) return -1; \
        if (cudaMemcpyToSymbol(sjk_desc_status, &zero_, sizeof zero_) != cudaSuccess) return -1; \
        return v_;                                                                        \
    }

// the same, reading the descriptor from device memory
__device__ inline bool sjk_desc_read(const int32_t * desc, const sjk_desc_ref & r, sjk_desc_vals * o) {
    int32_t e[SJK_DESC_N_ENTRIES];
#pragma unroll
    for (int i = 0; i < SJK_DESC_N_ENTRIES; ++i) e[i] = desc[i];
    return sjk_desc_check(e, r, o);
}
#endif

#ifdef __CUDACC__
__device__ inline void sjk_desc_fault() { atomicOr(&sjk_desc_status, (int) SJK_DEVICE_DESC); }
#endif
