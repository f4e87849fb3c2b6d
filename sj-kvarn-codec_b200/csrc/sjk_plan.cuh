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

// the dense (staged-row) kernel: n_chunks chunks per KV head in items of *cps chunks, the items of all KV heads on at
// most max_ctas SMs (one CTA per SM, one wave); returns the items per KV head
SJK_HD int sjk_dense_split_count(uint32_t n_chunks, int n_kv, int * cps, int max_ctas = 148) {
    if (n_chunks == 0) { *cps = 1; return 0; }
    const int target = n_kv > 0 && n_kv <= max_ctas ? max_ctas / n_kv : 1;
    int c = (int) ((n_chunks + (uint32_t) target - 1) / (uint32_t) target);
    if (c < 1) c = 1;
    *cps = c;
    return (int) ((n_chunks + (uint32_t) c - 1) / (uint32_t) c);
}

// the trellis body kernel (persistent, one CTA per SM over the call's KV heads, on at most max_ctas SMs): splits per
// KV head
SJK_HD int sjk_trellis_split_count(int n_kv, uint32_t n_rec, int max_ctas = 148) {
    const int n = n_kv > 0 ? n_kv : 1;
    int t = max_ctas / n;
    if (t < 1) t = 1;
    if ((uint32_t) t > n_rec) t = (int) n_rec;
    return t;
}

// When one call has both sealed trellis records and staged rows, the trellis kernel and the dense kernel run side by
// side on disjoint SMs (the dense kernel is a programmatic dependent that starts at once on the SMs the trellis kernel
// leaves free). A staged chunk costs about 3.2 trellis records of CTA time (a dense chunk about 17 K cycles, a trellis
// record about 6.5 K in steady state, plus the trellis kernel's longer pipeline fill; tuned on config 2's shapes); the
// SMs are shared in proportion, with at least one CTA per KV head on each side. Returns the dense kernel's SMs (0: the
// call has only one of the two); the trellis kernel takes at most the others.
// (4-bit scalar layers do not use this: their body kernel takes the staged chunks itself, spread over all SMs, which
// measured faster than the dense kernel beside it: 65.5 against 80.5 us on config 1.)
constexpr uint32_t SJK_CHUNK_W10 = 32;   // chunk weight in tenths of a trellis record
SJK_HD int sjk_dense_side_sms(int n_kv, uint32_t n_rec, uint32_t n_chunks, uint32_t w10 = SJK_CHUNK_W10) {
    if (n_rec == 0 || n_chunks == 0 || n_kv <= 0 || 2 * n_kv > 148) return 0;
    const uint64_t wt = (uint64_t) n_rec * 10u, wd = (uint64_t) n_chunks * w10;
    int k = (int) ((148u * wd + (wt + wd) / 2u) / (wt + wd));
    if (k < n_kv) k = n_kv;
    if (k > 148 - n_kv) k = 148 - n_kv;
    return k;
}

// the 4-bit tensor-core body kernel: splits per KV head over n_rec records and n_dense staged chunks
SJK_HD int sjk_tcbody_split_count(int n_kv, uint32_t n_rec, uint32_t n_dense, int max_ctas = 148) {
    const int n = n_kv > 0 ? n_kv : 1;
    int t = max_ctas >= 148 ? (148 + n - 1) / n : max_ctas / n;
    if (t > 148) t = 148;
    if (t < 1) t = 1;
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
    int dense_sms;              // > 0: the dense kernel runs beside the trellis kernel on this many SMs
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
    // trellis records and staged rows in one call: the two kernels share the SMs and run side by side
    const uint32_t n_tc_t = (pa.tc_trellis && !pa.tc_body) ? d->n_tc : 0u;
    d->dense_sms = (pa.dense && !pa.fused) ? sjk_dense_side_sms(n_kv, n_tc_t, d->n_dense) : 0;
    d->splits_d = (pa.dense && !pa.fused) ? sjk_dense_split_count(d->n_dense, n_kv, &d->cps_d, d->dense_sms ? d->dense_sms : 148) : 0;
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
        d->splits_tc = sjk_tcbody_split_count(n_kv, d->n_tc, n_dense_b, 148 - d->dense_sms);
    } else if (pa.tc_trellis && d->n_tc > 0) {
        d->splits_tc = sjk_trellis_split_count(n_kv, d->n_tc, 148 - d->dense_sms);
    }
    d->splits = d->splits_tc + d->splits_d + d->splits_v1;
}
