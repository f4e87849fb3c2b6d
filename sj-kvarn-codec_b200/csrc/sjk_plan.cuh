// sjk_plan.cuh - how one attention call over one cache is cut into work: which kernel takes which region, how
// many partial slots each writes. Shared by the host launchers (sjk_attend) and by the planner kernels of the
// descriptor-driven calls (sjk_attend_dyn), which evaluate the same functions on the device when B, N and qpos0
// are known only there, so both make identical launches for identical values.
#pragma once
#include <stdint.h>

#include "sjk_desc.cuh"

// upper bound of the split count of the CUDA-core and dense kernels: about two CTAs per SM over the call's KV heads
SJK_HD int sjk_split_target(int n_kv) {
    const int H = n_kv > 0 ? n_kv : 1;
    const int t = (2 * 148 + H - 1) / H;
    return t < 1 ? 1 : t;
}

// the dense (staged-row) kernel: n_chunks chunks per KV head in items of *cps chunks; returns the item count
SJK_HD int sjk_dense_split_count(uint32_t n_chunks, int n_kv, int * cps) {
    if (n_chunks == 0) { *cps = 1; return 0; }
    const int target = (2 * 148 + n_kv - 1) / n_kv;
    int c = (int) ((n_chunks + (uint32_t) target - 1) / (uint32_t) target);
    if (c < 1) c = 1;
    *cps = c;
    return (int) ((n_chunks + (uint32_t) c - 1) / (uint32_t) c);
}

// the trellis body kernel (persistent, one CTA per SM over the call's KV heads): splits per KV head
SJK_HD int sjk_trellis_split_count(int n_kv, uint32_t n_rec) {
    const int n = n_kv > 0 ? n_kv : 1;
    int t = (148 + n - 1) / n;
    if (t > 148) t = 148;
    if ((uint32_t) t > n_rec) t = (int) n_rec;
    while (t * n_kv > 148) --t;
    return t;
}

// the 4-bit tensor-core body kernel: splits per KV head over n_rec records and n_dense staged chunks
SJK_HD int sjk_tcbody_split_count(int n_kv, uint32_t n_rec, uint32_t n_dense) {
    const int n = n_kv > 0 ? n_kv : 1;
    int t = (148 + n - 1) / n;
    if (t > 148) t = 148;
    if ((uint32_t) t > n_rec + n_dense) t = (int) (n_rec + n_dense);
    return t;
}

// The CUDA-core kernel's chunks: the body after the first body_skip records, plus the sink and the staging ring
// unless the dense tensor-core kernel takes them (no_staged).
struct sjk_plan_v1 {
    int splits, chunks_per_split, n_chunks;
    uint32_t n_sink, n_body;
};
SJK_HD sjk_plan_v1 sjk_make_plan_v1(uint32_t S, uint32_t B, uint32_t N, int n_kv, uint32_t body_skip, bool no_staged,
                                           unsigned regions) {
    sjk_plan_v1 pl;
    const uint32_t s_end = S < N ? S : N;
    pl.n_sink = (no_staged || !(regions & SJK_REGION_SINK)) ? 0u : (s_end + 127u) / 128u;
    const uint32_t b_end = B < N ? B : N;
    pl.n_body = (b_end > S && (regions & SJK_REGION_BODY)) ? (b_end - S + 127u) / 128u : 0u;
    pl.n_body = pl.n_body > body_skip ? pl.n_body - body_skip : 0u;
    const uint32_t t0 = B > S ? B : S;
    const uint32_t n_tail = (N > t0 && !no_staged && (regions & SJK_REGION_RING)) ? (N - t0 + 127u) / 128u : 0u;
    pl.n_chunks = (int) (pl.n_sink + pl.n_body + n_tail);
    const int target = sjk_split_target(n_kv);
    pl.chunks_per_split = (pl.n_chunks + target - 1) / target;
    if (pl.chunks_per_split < 1) pl.chunks_per_split = 1;
    pl.splits = pl.n_chunks > 0 ? (pl.n_chunks + pl.chunks_per_split - 1) / pl.chunks_per_split : 1;
    return pl;
}

// Which kernels an attention call uses: fixed by the layout, the formats and the query shape.
struct sjk_paths {
    bool tc_body;       // 4-bit scalar records on tensor cores
    bool tc_trellis;    // trellis records on tensor cores
    bool dense;         // the staged rows on tensor cores
    bool fused;         // tc_body && dense: the body kernel also takes the staged rows
};

// Everything an attention call decides once B, N and qpos0 are known: the records of the tensor-core body kernel,
// the dense kernel's chunks, the CUDA-core kernel's plan, and the partial slots of each kernel (tensor-core body
// first, then dense, then CUDA-core). Written by the planner kernel of sjk_attend_dyn into the call's scratch.
struct sjk_dyn_state {
    int ok;                     // 0: the descriptor failed its checks; nothing is attended (a zero output)
    uint32_t B, N, qpos0;
    uint32_t n_tc;              // records [0, n_tc) to the tensor-core body kernel
    uint32_t dense_regions;     // fused: bit 0 the sink, bit 1 the ring also go to the body kernel
    int splits_tc;              // its partial slots [0, splits_tc)
    uint32_t n_sink_d, n_dense; // the dense kernel's chunks (sink chunks first)
    int cps_d, splits_d;        // chunks per item; slots [splits_tc, splits_tc + splits_d)
    sjk_plan_v1 v1;             // the CUDA-core kernel; slots after those
    int splits_v1;
    int splits;                 // all partial slots of the call
};

SJK_HD void sjk_plan_counts(const sjk_paths & pa, uint32_t S, uint32_t B, uint32_t N, unsigned regions, int n_kv,
                                   sjk_dyn_state * d) {
    const uint32_t b_end = B < N ? B : N;
    const bool body_on = (regions & SJK_REGION_BODY) != 0;
    d->B = B; d->N = N;
    d->n_tc = ((pa.tc_body || pa.tc_trellis) && body_on && b_end > S) ? (b_end - S) / 128u : 0u;
    d->n_sink_d = 0; d->n_dense = 0;
    if (pa.dense && !pa.fused) {
        const uint32_t s_end = S < N ? S : N, t0 = B > S ? B : S;
        d->n_sink_d = (regions & SJK_REGION_SINK) ? (s_end + 127u) / 128u : 0u;
        d->n_dense = d->n_sink_d + ((regions & SJK_REGION_RING) && N > t0 ? (N - t0 + 127u) / 128u : 0u);
    }
    d->cps_d = 1;
    d->splits_d = (pa.dense && !pa.fused) ? sjk_dense_split_count(d->n_dense, n_kv, &d->cps_d) : 0;
    d->v1 = sjk_make_plan_v1(S, B, N, n_kv, d->n_tc, pa.dense, regions);
    d->splits_v1 = d->v1.n_chunks > 0 ? d->v1.splits : 0;
    d->dense_regions = pa.fused ? ((regions & SJK_REGION_SINK) ? 1u : 0u) | ((regions & SJK_REGION_RING) ? 2u : 0u) : 0u;
    const unsigned staged = regions & (SJK_REGION_SINK | SJK_REGION_RING);
    d->splits_tc = 0;
    if (pa.tc_body && (d->n_tc > 0 || (pa.fused && staged))) {
        uint32_t n_dense_b = 0;
        if (d->dense_regions) {
            const uint32_t s_end = S < N ? S : N, t0 = B > S ? B : S;
            n_dense_b = (d->dense_regions & 1) ? (s_end + 127u) / 128u : 0u;
            n_dense_b += (d->dense_regions & 2) && N > t0 ? (N - t0 + 127u) / 128u : 0u;
        }
        d->splits_tc = sjk_tcbody_split_count(n_kv, d->n_tc, n_dense_b);
    } else if (pa.tc_trellis && d->n_tc > 0) {
        d->splits_tc = sjk_trellis_split_count(n_kv, d->n_tc);
    }
    d->splits = d->splits_tc + d->splits_d + d->splits_v1;
}
