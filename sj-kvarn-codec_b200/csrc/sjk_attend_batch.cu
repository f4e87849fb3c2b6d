// sjk_attend_batch.cu - decode attention of many sequences of one layer in one call: the decode step of a paged
// record pool (sj_kvarn.h:1645-1739 sequences over one slab), where every sequence attends with its own query rows
// over its own sink, staging ring and block table.
//
// Trellis layers run as three launches for the whole batch, whatever the number of sequences:
//   body     attend_trellis_ws_kernel over work items that cut the records of all (sequence, KV head) pairs into
//            one balanced range per SM (sjk_attend_trellis.cu)
//   staged   attend_dense_tc_kernel over items of at most a few 128-position chunks of the sinks and staging
//            rings (sjk_attend_dense.cu)
//   merge    one CTA per (sequence, query row, query head) combines the (m, l, o) partials of that pair's items
// Other bodies (scalar codes) take one sjk_attend call per sequence on the same stream and scratch.
#include <cuda_runtime.h>

#include "sjk_common.cuh"
#include "sjk_internal.h"

int sjk_tc_trellis_batch_launch(const sjk_view * views, const uint32_t * B, const uint32_t * N, const uint32_t * qpos0,
                                int n_seq, int n_q, int n_head, const float * q, float scale, float * part, int slot0,
                                uint16_t * first, int * n_items, sjk_stream st);
int sjk_tc_dense_batch_launch(const sjk_view * views, const uint32_t * B, const uint32_t * N, const uint32_t * qpos0,
                              int n_seq, int n_q, int n_head, const float * q, float scale, float * part, int slot0,
                              uint16_t * first, int * n_items, sjk_stream st);

namespace {

constexpr int MAX_SEQS = 128;
constexpr int MAX_PAIRS = 512;
constexpr int MAX_SLOTS = 672 + 768;            // body items + staged-row items of one call
constexpr int D = 256;

struct MergeParams {
    const float * part;                         // [slots][n_rows][D + 2]
    float * out;                                // [n_seq][n_rows][D]
    int n_rows, n_head, grp, H;
    uint16_t body_first[MAX_PAIRS + 1];         // slots of pair (s, h): [body_first[p], body_first[p + 1])
    uint16_t dense_first[MAX_PAIRS + 1];        //                  and [dense_first[p], dense_first[p + 1])
};

// out[s][row] = sum_i exp(m_i - m) o_i / sum_i exp(m_i - m) l_i over the partial slots of the row's (sequence,
// KV head) pair, in slot order; a row that saw no position gets zeros.
__global__ void __launch_bounds__(D) attend_batch_merge_kernel(const __grid_constant__ MergeParams p) {
    const int b = blockIdx.x, s = b / p.n_rows, row = b - s * p.n_rows, d = threadIdx.x;
    const int pr = s * p.H + (row % p.n_head) / p.grp;
    const int a0 = p.body_first[pr], a1 = p.body_first[pr + 1], c0 = p.dense_first[pr], c1 = p.dense_first[pr + 1];
    const size_t step = (size_t) p.n_rows * (D + 2);
    const float * base = p.part + (size_t) row * (D + 2);
    float m = -INFINITY;
    for (int i = a0; i < a1; ++i) m = fmaxf(m, base[(size_t) i * step]);
    for (int i = c0; i < c1; ++i) m = fmaxf(m, base[(size_t) i * step]);
    float den = 0.0f, o = 0.0f;
    if (m != -INFINITY) {
        for (int i = a0; i < a1; ++i) {
            const float * x = base + (size_t) i * step;
            const float w = x[0] == -INFINITY ? 0.0f : expf(x[0] - m);
            den = fmaf(x[1], w, den);
            o = fmaf(x[2 + d], w, o);
        }
        for (int i = c0; i < c1; ++i) {
            const float * x = base + (size_t) i * step;
            const float w = x[0] == -INFINITY ? 0.0f : expf(x[0] - m);
            den = fmaf(x[1], w, den);
            o = fmaf(x[2 + d], w, o);
        }
    }
    p.out[((size_t) s * p.n_rows + row) * D + d] = den > 0.0f ? o * (1.0f / den) : 0.0f;
}

bool same_format(const sjk_view & a, const sjk_view & b) {
    const sj_kvarn_layout & x = a.lay, & y = b.lay;
    return x.D == y.D && x.G == y.G && x.bits_k == y.bits_k && x.bits_v == y.bits_v && x.body == y.body && x.bytes == y.bytes &&
           a.n_head_kv == b.n_head_kv && a.staging == b.staging && a.sink_type == b.sink_type && a.S == b.S && a.cap == b.cap &&
           a.stage_bytes == b.stage_bytes;
}

}  // namespace

extern "C" size_t sjk_attend_batch_scratch_bytes(const sjk_view * v, int n_seq, int n_q, int n_head) {
    if (!v || n_seq <= 0 || n_q <= 0 || n_head <= 0) return 0;
    const size_t batched = (size_t) MAX_SLOTS * n_q * n_head * (v->lay.D + 2) * sizeof(float);
    const size_t single = sjk_attend_scratch_bytes(v, 0, n_q, n_head);
    return batched > single ? batched : single;
}

extern "C" int sjk_attend_batch(const sjk_view * views, const uint32_t * B, const uint32_t * N, const uint32_t * qpos0, int n_seq,
                                int n_q, int n_head, const float * q, float scale, float * out, void * scratch,
                                size_t scratch_bytes, sjk_stream st) {
    if (!views || !B || !N || !qpos0 || !q || !out || n_seq <= 0 || n_q <= 0 || n_head <= 0) return SJKVARN_ERR_ARG;
    const sjk_view & v0 = views[0];
    const int H = v0.n_head_kv;
    if (H <= 0 || n_head % H) return SJKVARN_ERR_ARG;
    for (int s = 0; s < n_seq; ++s) {
        if (!same_format(views[s], v0)) return SJKVARN_ERR_ARG;
        if (B[s] < v0.S) return SJKVARN_ERR_ARG;
    }
    if (!scratch || scratch_bytes < sjk_attend_batch_scratch_bytes(&v0, n_seq, n_q, n_head)) return SJKVARN_ERR_ARG;
    const int grp = n_head / H;
    const size_t per_seq = (size_t) n_q * n_head * v0.lay.D;
    const bool batched = sjk_tc_trellis_supported(&v0, n_q, grp) && sjk_tc_dense_supported(&v0, n_q, grp) && n_seq <= MAX_SEQS &&
                         n_seq * H <= MAX_PAIRS && v0.lay.D == D;
    if (!batched) {
        // one call per sequence: stream order makes the shared scratch safe to reuse
        for (int s = 0; s < n_seq; ++s) {
            const int rc = sjk_attend(&views[s], B[s], N[s], qpos0[s], n_q, n_head, q + (size_t) s * per_seq, scale,
                                      out + (size_t) s * per_seq, scratch, scratch_bytes, st);
            if (rc) return rc;
        }
        return 0;
    }
    static thread_local MergeParams mp;
    float * part = (float *) scratch;
    int n_body = 0, n_dense = 0;
    int rc = sjk_tc_trellis_batch_launch(views, B, N, qpos0, n_seq, n_q, n_head, q, scale, part, 0, mp.body_first, &n_body, st);
    if (rc) return rc;
    rc = sjk_tc_dense_batch_launch(views, B, N, qpos0, n_seq, n_q, n_head, q, scale, part, n_body, mp.dense_first, &n_dense, st);
    if (rc) return rc;
    mp.part = part; mp.out = out; mp.n_rows = n_q * n_head; mp.n_head = n_head; mp.grp = grp; mp.H = H;
    attend_batch_merge_kernel<<<(unsigned) (n_seq * n_q * n_head), D, 0, st>>>(mp);
    return sjk_check_launch();
}
