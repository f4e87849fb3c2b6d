// sjk_attend.cu - causal decode attention over the three regions of an SJ-KVaRN layer cache
// (fp16 sink [0, S), sealed body [S, B), staging ring [B, N)), flash-decoding style:
//
//   split kernel  grid (splits, KV heads). Each CTA walks a contiguous range of 128-position chunks
//                 (a chunk never straddles two regions; a body chunk is one record), decodes the K/V rows
//                 of 32 positions at a time into shared memory exactly as the reference decoders do, and
//                 keeps a running (max, sum, output) per query row of its KV head (all GQA heads x rows).
//   merge kernel  one CTA per (query row, query head) combines the splits' partials.
//
// Scores use the reference's sequential fp32 dot (sj_kvarn.h:1288-1293) on identically decoded rows, so
// they are bit-equal to the reference's; only the softmax accumulation order differs (chunk-wise online
// softmax + merge instead of one position-ordered pass), which the 1e-3 relative contract covers.
#include <mutex>

#include <cooperative_groups.h>

#include "sjk_common.cuh"
#include "sjk_fwht.cuh"
#include "sjk_internal.h"
#include "sjk_merge.cuh"
#include "sjk_plan.cuh"

namespace {

constexpr int NT = 256;
constexpr int SUB = 32;             // positions decoded per step
constexpr int MAXROWS = 16;         // query rows per KV head handled by one CTA (n_q * GQA group)

struct AttnParams {
    sjk_view v;
    int kv0;                        // first KV head of the call (grid.y walks kv0 .. kv0 + n_kv - 1)
    uint32_t B, N, qpos0;
    int n_q, n_head, grp, rows;     // rows = n_q * grp
    const float * q;
    float scale;
    float * part;                   // [splits][n_q*n_head][D + 2]: m, l, o[D]
    int split0;                     // partial slot of this kernel's first split
    int chunks_per_split, n_chunks;
    uint32_t n_sink_chunks, n_body_chunks;
    uint32_t body_skip;             // leading body records handled by the tensor-core kernel
    int n_splits;                   // splits per KV head (the descriptor-driven grid may be wider)
};

struct Chunk { int region; uint32_t p0, len, g; };   // region 0 sink, 1 body, 2 ring

SJK_DEV Chunk chunk_of(const AttnParams & p, uint32_t ci) {
    Chunk c;
    const uint32_t S = p.v.S;
    const uint32_t s_end = S < p.N ? S : p.N;
    if (ci < p.n_sink_chunks) {
        c.region = 0; c.p0 = ci * 128u; c.len = min(128u, s_end - c.p0); c.g = 0;
    } else if (ci < p.n_sink_chunks + p.n_body_chunks) {
        const uint32_t b_end = p.B < p.N ? p.B : p.N;      // a query over a prefix may end inside a record
        c.region = 1; c.g = p.body_skip + ci - p.n_sink_chunks; c.p0 = S + c.g * 128u; c.len = min(128u, b_end - c.p0);
    } else {
        const uint32_t k = ci - p.n_sink_chunks - p.n_body_chunks;
        const uint32_t b0 = p.B > S ? p.B : S;
        c.region = 2; c.p0 = b0 + k * 128u; c.len = min(128u, p.N - c.p0); c.g = 0;
    }
    return c;
}

// Decode rows [t0, t0+n) of a chunk into K/V shared tiles [SUB][D+1] (sj_kvarn.h:1516-1533).
template <int D>
SJK_DEV void load_rows(const AttnParams & p, const Chunk & c, uint32_t t0, uint32_t n, int h, float * Ks, float * Vs,
                       const float * sc, const float * cbk, const float * cbv) {
    const sjk_view & v = p.v;
    const sj_kvarn_layout & l = v.lay;
    const int H = v.n_head_kv;
    for (int e = threadIdx.x; e < (int) n * D; e += NT) {
        const int t = e / D, d = e % D;
        const uint32_t pos = c.p0 + t0 + (uint32_t) t;
        float kv, vv;
        if (c.region == 1) {
            const uint32_t blk = v.blocks ? v.blocks[c.g] : c.g;
            const uint8_t * rec = v.body + ((size_t) blk * H + h) * l.bytes;
            const int tt = (int) (t0 + (uint32_t) t);
            float qk, qv;
            if (l.body == SJKVARN_BODY_TRELLIS) {
                qk = cbk[sjk_window(rec + l.k_payload, l.bits_k, d, tt, 128)];
                qv = cbv[sjk_window(rec + l.v_payload, l.bits_v, d, tt, 128)];
            } else {
                qk = (float) sjk_get_bits(rec + l.k_payload, sjk_code_bit(l, tt, d, 0), l.bits_k);
                qv = (float) sjk_get_bits(rec + l.v_payload, sjk_code_bit(l, tt, d, 1), l.bits_v);
            }
            // sc: ks[D], kz[D], vc[D], kt[128], vs[128], vz[128] of this record, natural order
            kv = __fmul_rn(__fadd_rn(__fmul_rn(qk, sc[d]), sc[D + d]), sc[3 * D + tt]);
            vv = __fmul_rn(__fadd_rn(__fmul_rn(qv, sc[3 * D + 128 + tt]), sc[3 * D + 256 + tt]), sc[2 * D + d]);
        } else if (c.region == 0 && v.sink_type == SJKVARN_SINK_F16) {
            const uint8_t * row = v.sink + ((size_t) pos * H + h) * 4 * D;
            kv = sjk_h2f(sjk_ld_u16(row + 2 * d));
            vv = sjk_h2f(sjk_ld_u16(row + 2 * D + 2 * d));
        } else {
            const uint8_t * row = c.region == 0 ? v.sink + ((size_t) pos * H + h) * 2 * v.stage_bytes
                                                : v.ring + ((size_t) sjk_ring_slot(v.S, v.cap, pos) * H + h) * 2 * v.stage_bytes;
            if (v.staging == SJKVARN_STAGING_F16) {
                kv = sjk_h2f(sjk_ld_u16(row + 2 * d));
                vv = sjk_h2f(sjk_ld_u16(row + v.stage_bytes + 2 * d));
            } else {
                const int j = d & 127;
                const uint8_t * bk = row + (d >> 7) * SJKVARN_TQ6_BLOCK_BYTES;
                const uint8_t * bv = bk + v.stage_bytes;
                const int ck = ((bk[2 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((bk[66 + (j >> 2)] >> (2 * (j & 3))) & 3) << 4);
                const int cv = ((bv[2 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((bv[66 + (j >> 2)] >> (2 * (j & 3))) & 3) << 4);
                kv = __fmul_rn(sjk_tq6_cent[ck], sjk_h2f(sjk_ld_u16(bk)));
                vv = __fmul_rn(sjk_tq6_cent[cv], sjk_h2f(sjk_ld_u16(bv)));
            }
        }
        Ks[t * (D + 1) + d] = kv;
        Vs[t * (D + 1) + d] = vv;
    }
}

template <int D>
SJK_DEV void split_body(const AttnParams & p) {
    extern __shared__ __align__(16) float sm[];
    float * Ks = sm;                                  // [SUB][D+1]
    float * Vs = Ks + SUB * (D + 1);                  // [SUB][D+1]
    float * Qs = Vs + SUB * (D + 1);                  // [MAXROWS][D]
    float * Ss = Qs + MAXROWS * D;                    // [MAXROWS][SUB] scores -> weights
    float * sc = Ss + MAXROWS * SUB;                  // record scales: 3D + 384
    float * cbk = sc + 3 * D + 384;                   // 512
    float * cbv = cbk + 512;                          // 512
    float * rowm = cbv + 512;                         // [MAXROWS] running max
    float * rowl = rowm + MAXROWS;                    // [MAXROWS] running sum
    float * rowa = rowl + MAXROWS;                    // [MAXROWS] rescale factor of the current step
    const int hl = blockIdx.y, h = p.kv0 + hl, split = blockIdx.x;   // hl: head index inside q / out
    const sj_kvarn_layout & l = p.v.lay;
    const int R = p.rows;

    // query rows of this KV head: row r = iq * grp + j  <->  query head h*grp + j, row iq
    for (int e = threadIdx.x; e < R * D; e += NT) {
        const int r = e / D, d = e % D;
        const int iq = r / p.grp, hq = hl * p.grp + r % p.grp;
        Qs[e] = p.q[((size_t) iq * p.n_head + hq) * D + d];
    }
    if (l.body == SJKVARN_BODY_TRELLIS) {
        const uint16_t * ck = sjk_codebook(l.bits_k, 0), * cv = sjk_codebook(l.bits_v, 1);
        for (int i = threadIdx.x; i < (1 << (6 + l.bits_k)); i += NT) cbk[i] = sjk_h2f(ck[i]);
        for (int i = threadIdx.x; i < (1 << (6 + l.bits_v)); i += NT) cbv[i] = sjk_h2f(cv[i]);
    }
    if (threadIdx.x < MAXROWS) { rowm[threadIdx.x] = -__int_as_float(0x7F800000); rowl[threadIdx.x] = 0.0f; }
    // accumulator: thread owns row r_own for channels d = g + 16 i (i < D/16)
    const int r_own = threadIdx.x / 16, g_own = threadIdx.x % 16;
    float acc[D / 16];
#pragma unroll
    for (int i = 0; i < D / 16; ++i) acc[i] = 0.0f;
    __syncthreads();

    const int c_begin = split * p.chunks_per_split;
    const int c_end = min(p.n_chunks, c_begin + p.chunks_per_split);
    for (int ci = c_begin; ci < c_end; ++ci) {
        const Chunk c = chunk_of(p, (uint32_t) ci);
        if (c.region == 1) {
            const uint32_t blk = p.v.blocks ? p.v.blocks[c.g] : c.g;
            const uint8_t * rec = p.v.body + ((size_t) blk * p.v.n_head_kv + h) * l.bytes;
            __syncthreads();
            for (int d = threadIdx.x; d < D; d += NT) {
                const int kc = sjk_k_ch(l, d), vc = sjk_v_ch(l, d);
                sc[d] = sjk_h2f(sjk_ld_u16(rec + l.k_scale + 2 * kc));
                sc[D + d] = sjk_h2f(sjk_ld_u16(rec + l.k_zero + 2 * kc));
                sc[2 * D + d] = sjk_h2f(sjk_ld_u16(rec + l.v_ch + 2 * vc));
            }
            for (int t = threadIdx.x; t < 128; t += NT) {
                sc[3 * D + t] = sjk_h2f(sjk_ld_u16(rec + l.k_tok + 2 * t));
                sc[3 * D + 128 + t] = sjk_h2f(sjk_ld_u16(rec + l.v_scale + 2 * t));
                sc[3 * D + 256 + t] = sjk_h2f(sjk_ld_u16(rec + l.v_zero + 2 * t));
            }
        }
        for (uint32_t t0 = 0; t0 < c.len; t0 += SUB) {
            const uint32_t n = min((uint32_t) SUB, c.len - t0);
            __syncthreads();
            load_rows<D>(p, c, t0, n, h, Ks, Vs, sc, cbk, cbv);
            __syncthreads();
            // scores: the reference's sequential dot, then x scale; masked beyond each row's causal end
            for (int e = threadIdx.x; e < R * SUB; e += NT) {
                const int r = e / SUB, t = e % SUB;
                const uint32_t pos = c.p0 + t0 + (uint32_t) t;
                const uint32_t qpos = p.qpos0 + (uint32_t) (r / p.grp);
                float s = -__int_as_float(0x7F800000);
                if ((uint32_t) t < n && pos <= qpos) {
                    const float * qr = Qs + r * D;
                    const float * kr = Ks + t * (D + 1);
                    float dot = 0.0f;
                    for (int d = 0; d < D; ++d) dot = __fadd_rn(dot, __fmul_rn(qr[d], kr[d]));
                    s = __fmul_rn(dot, p.scale);
                }
                Ss[r * SUB + t] = s;
            }
            __syncthreads();
            // online softmax per row over this step's positions
            if (threadIdx.x < R) {
                const int r = threadIdx.x;
                float mx = rowm[r];
                for (int t = 0; t < SUB; ++t) mx = fmaxf(mx, Ss[r * SUB + t]);
                float alpha = 1.0f, sum = 0.0f;
                if (mx == -__int_as_float(0x7F800000)) {
                    for (int t = 0; t < SUB; ++t) Ss[r * SUB + t] = 0.0f;
                } else {
                    alpha = expf(rowm[r] - mx);
                    for (int t = 0; t < SUB; ++t) {
                        const float w = expf(Ss[r * SUB + t] - mx);
                        Ss[r * SUB + t] = w;
                        sum += w;
                    }
                    rowm[r] = mx;
                }
                rowl[r] = rowl[r] * alpha + sum;
                rowa[r] = alpha;
            }
            __syncthreads();
            if (r_own < R) {
                const float alpha = rowa[r_own];
#pragma unroll
                for (int i = 0; i < D / 16; ++i) acc[i] *= alpha;
                for (int t = 0; t < (int) n; ++t) {
                    const float w = Ss[r_own * SUB + t];
                    const float * vr = Vs + t * (D + 1) + g_own;
#pragma unroll
                    for (int i = 0; i < D / 16; ++i) acc[i] = fmaf(w, vr[16 * i], acc[i]);
                }
            }
        }
    }
    // partials: (m, l, o[D]) per (row, query head)
    __syncthreads();
    if (r_own < R) {
        const int iq = r_own / p.grp, hq = hl * p.grp + r_own % p.grp;
        float * dst = p.part + ((size_t) (p.split0 + split) * p.n_q * p.n_head + (size_t) iq * p.n_head + hq) * (D + 2);
        if (g_own == 0) { dst[0] = rowm[r_own]; dst[1] = rowl[r_own]; }
#pragma unroll
        for (int i = 0; i < D / 16; ++i) dst[2 + g_own + 16 * i] = acc[i];
    }
}

template <int D>
__global__ void __launch_bounds__(NT) attend_split_kernel(const __grid_constant__ AttnParams p) { split_body<D>(p); }

// the descriptor-driven form: the plan was made on the device (attend_dyn_plan_kernel)
template <int D>
__global__ void __launch_bounds__(NT) attend_split_dyn_kernel(const AttnParams * __restrict__ pp) {
    if ((int) blockIdx.x >= pp->n_splits) return;
    split_body<D>(*pp);
}

// out[row, head] = sum_i o_i e^(m_i - m) / sum_i l_i e^(m_i - m) (sjk_merge.cuh). Grid (query row x head, channel tiles
// of 64); each CTA recomputes the split weights (cheap) into shared memory and sums its 64 channels.
using sjkm::MERGE_SPLITS;

// part_out (optional): instead of out, write the combined partial (m, l, o[D]) of each row (o not normalized), the
// form sjk_attend_partial returns
// splits_dev (optional): read the split count from device memory (the descriptor-driven call's plan)
__global__ void __launch_bounds__(256) attend_merge_kernel(const float * part, int splits, int n_rows, int D, float * out,
                                                           float * part_out, const int * splits_dev) {
    extern __shared__ float wts[];                     // [max(splits, ranks)] weights, then [4][64] partial sums
    __shared__ float s_red[16];
    const int row = blockIdx.x, d0 = blockIdx.y * 64;
    const int tid = threadIdx.x;
    // launched as a programmatic dependent of the kernels that write the partials: wait until they completed; a
    // kernel launched as this one's dependent (the exchange of sjk_attend_partial_xchg) may be set up meanwhile
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    if (splits_dev) splits = *splits_dev;
    float m, t;
    sjkm::merge_tile(part, splits, n_rows, D, row, d0, wts, s_red, m, t);
    const float * acc = wts + splits;
    if (part_out) {
        if (tid < 64 && d0 + tid < D) part_out[(size_t) row * (D + 2) + 2 + d0 + tid] = sjkm::acc_o(acc, tid);
        if (blockIdx.y == 0 && tid == 0) { part_out[(size_t) row * (D + 2)] = m; part_out[(size_t) row * (D + 2) + 1] = t; }
    } else {
        sjkm::store_out(acc, t, D, row, d0, out);
    }
}

// The merge for outputs in the model basis (sjk_attend_model): the D / 64 tile CTAs of a row form one cluster; each
// normalises its 64 outputs as attend_merge_kernel does and stores them into the shared row of the cluster's first
// CTA, which applies the rotation (the reference's FWHT, an involution at scale 1/sqrt(D)) and writes the row.
template <int D>
__global__ void __launch_bounds__(256) attend_merge_rot_kernel(const float * part, int splits, int n_rows, float * out,
                                                               float fwht_scale) {
    namespace cg = cooperative_groups;
    extern __shared__ float wts[];
    __shared__ float s_red[16];
    __shared__ __align__(16) float rowbuf[D];
    const int row = blockIdx.x, d0 = blockIdx.y * 64, tid = threadIdx.x;
    // launched as a programmatic dependent of the kernels that write the partials: wait until they completed; the
    // next call's body kernel, launched as this one's dependent, may be set up meanwhile
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    float m, t;
    sjkm::merge_tile(part, splits, n_rows, D, row, d0, wts, s_red, m, t);
    cg::cluster_group cl = cg::this_cluster();
    float * dst = cl.map_shared_rank(rowbuf, 0);
    if (tid < 64) {
        const float s_inv = t == 0.0f ? 0.0f : 1.0f / t;
        dst[d0 + tid] = sjkm::acc_o(wts + splits, tid) * s_inv;
    }
    cl.sync();
    if (cl.block_rank() == 0 && tid < 32) {
        constexpr int VPL = D / 32;
        float v[VPL];
#pragma unroll
        for (int i = 0; i < VPL; ++i) v[i] = rowbuf[tid * VPL + i];
        fwht_warp<VPL>(v, tid, fwht_scale);
#pragma unroll
        for (int i = 0; i < VPL; ++i) out[(size_t) row * D + tid * VPL + i] = v[i];
    }
}

// model-basis queries of a call rotated into the call's scratch (the calls whose kernels other than the 4-bit body
// kernel read q): one warp per row, the reference's FWHT
template <int D>
__global__ void __launch_bounds__(256) rotate_rows_kernel(const float * src, float * dst, int n_rows, float fwht_scale) {
    constexpr int VPL = D / 32;
    const int lane = threadIdx.x & 31, row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= n_rows) return;
    float v[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) v[i] = src[(size_t) row * D + lane * VPL + i];
    fwht_warp<VPL>(v, lane, fwht_scale);
#pragma unroll
    for (int i = 0; i < VPL; ++i) dst[(size_t) row * D + lane * VPL + i] = v[i];
}

template <int D>
size_t split_smem() {
    return (size_t) (2 * SUB * (D + 1) + MAXROWS * D + MAXROWS * SUB + 3 * D + 384 + 1024 + 3 * MAXROWS) * sizeof(float);
}

}  // namespace

size_t sjk_attend_heads_scratch_bytes(const sjk_view * v, int n_q, int n_head, int n_kv) {
    if (!v || n_q <= 0 || n_head <= 0) return 0;
    // CUDA-core, tensor-core body and tensor-core staged-row splits, each bounded by the per-call target
    return (size_t) 3 * sjk_split_target(n_kv) * n_q * n_head * (v->lay.D + 2) * sizeof(float);
}

// bytes of the rank's own partial in sjk_attend_partial_xchg's scratch (after the split partials), 256-aligned
static size_t xchg_part_bytes(const sjk_view * v, int n_q, int n_head) {
    return ((size_t) n_q * n_head * (v->lay.D + 2) * sizeof(float) + 255) & ~(size_t) 255;
}

extern "C" size_t sjk_attend_scratch_bytes(const sjk_view * v, uint32_t N, int n_q, int n_head) {
    (void) N;
    if (!v || n_q <= 0 || n_head <= 0) return 0;
    // the split partials, plus room for the call's own partial (sjk_attend_partial_xchg)
    return sjk_attend_heads_scratch_bytes(v, n_q, n_head, v->n_head_kv) + xchg_part_bytes(v, n_q, n_head);
}

namespace {

sjk_paths paths_of(const sjk_view * v, int n_q, int grp) {
    sjk_paths pa;
    pa.tc_body = sjk_tc_body_supported(v, n_q, grp) != 0;
    pa.tc_trellis = !pa.tc_body && sjk_tc_trellis_supported(v, n_q, grp) != 0;
    pa.dense = sjk_tc_dense_supported(v, n_q, grp) != 0;
    pa.fused = pa.tc_body && pa.dense;
    return pa;
}

// the CUDA-core kernel over the chunks of p (grid: splits x KV heads); dyn: its plan in device memory instead
int launch_split(const AttnParams & p, const AttnParams * dyn, int splits, int n_kv, sjk_stream st) {
    const dim3 grid((unsigned) splits, (unsigned) n_kv);
    cudaError_t e = cudaSuccess;
    switch (p.v.lay.D) {
        case 128: {
            const size_t sm = split_smem<128>();
            if (dyn) {
                e = cudaFuncSetAttribute(attend_split_dyn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) sm);
                if (e == cudaSuccess) attend_split_dyn_kernel<128><<<grid, NT, sm, st>>>(dyn);
            } else {
                e = cudaFuncSetAttribute(attend_split_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) sm);
                if (e == cudaSuccess) attend_split_kernel<128><<<grid, NT, sm, st>>>(p);
            }
            break;
        }
        case 256: {
            const size_t sm = split_smem<256>();
            if (dyn) {
                e = cudaFuncSetAttribute(attend_split_dyn_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) sm);
                if (e == cudaSuccess) attend_split_dyn_kernel<256><<<grid, NT, sm, st>>>(dyn);
            } else {
                e = cudaFuncSetAttribute(attend_split_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) sm);
                if (e == cudaSuccess) attend_split_kernel<256><<<grid, NT, sm, st>>>(p);
            }
            break;
        }
        default: return SJK_ERR_UNSUPPORTED;
    }
    if (sjk_check(e)) return SJK_ERR_DEVICE;
    return sjk_check_launch() ? SJK_ERR_DEVICE : 0;
}

// Programmatic dependent launch: the merge grid is set up while the partial kernels run and waits for them on the
// device (griddepcontrol.wait), so the launch gap between the two kernels disappears. splits_dev: the split count
// is read from device memory (shared memory sized for max_splits).
// rot_out: out in the model basis (attend_merge_rot_kernel, clusters of the D / 64 tiles of a row)
int launch_merge(const float * part, int splits, const int * splits_dev, int max_splits, int n_rows, int D, float * out,
                 float * part_out, sjk_stream st, bool rot_out = false) {
    const int n_w = splits_dev ? max_splits : splits;
    if (rot_out) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned) n_rows, (unsigned) (D / 64));
        cfg.blockDim = dim3(256);
        cfg.dynamicSmemBytes = (size_t) (splits + 256) * sizeof(float);
        cfg.stream = st;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 1; attr[1].val.clusterDim.y = (unsigned) (D / 64); attr[1].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        const float sc = sjk_fwht_scale(D);
        cudaError_t e;
        switch (D) {
            case 128: e = cudaLaunchKernelEx(&cfg, attend_merge_rot_kernel<128>, part, splits, n_rows, out, sc); break;
            case 256: e = cudaLaunchKernelEx(&cfg, attend_merge_rot_kernel<256>, part, splits, n_rows, out, sc); break;
            case 512: e = cudaLaunchKernelEx(&cfg, attend_merge_rot_kernel<512>, part, splits, n_rows, out, sc); break;
            default: return SJK_ERR_UNSUPPORTED;
        }
        if (sjk_check(e)) return SJK_ERR_DEVICE;
        return sjk_check_launch();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) n_rows, (unsigned) ((D + 63) / 64));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = (size_t) (n_w + 256) * sizeof(float);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, attend_merge_kernel, part, splits, n_rows, D, out, part_out, splits_dev);
    if (sjk_check(e))
        return SJK_ERR_DEVICE;
    return sjk_check_launch();
}

}  // namespace

namespace {
// model: q in the model basis and out in the model basis (sjk_attend_model); otherwise both rotated
int attend_heads_impl(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, int kv_head0, int n_kv,
                      const float * q, float scale, float * out, void * scratch, size_t scratch_bytes, sjk_stream st,
                      unsigned regions, float * part_out, bool model) {
    if (!v || !q || !(out || part_out) || n_q <= 0 || n_head <= 0 || n_kv <= 0 || kv_head0 < 0 || kv_head0 + n_kv > v->n_head_kv ||
        n_head % n_kv)
        return SJKVARN_ERR_ARG;
    if (B < v->S) return SJKVARN_ERR_ARG;
    const int grp = n_head / n_kv;
    if (n_q * grp > MAXROWS) return SJK_ERR_UNSUPPORTED;
    // sealed records [0, n_tc) go to the tensor-core kernel when it supports the body format; when it also supports
    // the staged-row formats, the same kernel takes the sink and the staging ring, else the dense kernel does
    const sjk_paths pa = paths_of(v, n_q, grp);
    sjk_dyn_state d;
    sjk_plan_counts(pa, v->S, B, N, regions, n_kv, &d);
    // the tensor-core kernel's split count is known after its launch plan; bound it for the scratch check
    const unsigned staged = regions & (SJK_REGION_SINK | SJK_REGION_RING);
    const int splits_tc_max = (pa.tc_body && (d.n_tc > 0 || (pa.fused && staged))) ? sjk_tc_body_max_splits(n_kv)
                              : (pa.tc_trellis && d.n_tc > 0)                       ? sjk_tc_trellis_max_splits(n_kv)
                                                                                    : 0;
    const size_t need = (size_t) (splits_tc_max + d.splits_d + d.splits_v1) * n_q * n_head * (v->lay.D + 2) * sizeof(float);
    if (!scratch || scratch_bytes < need) return SJKVARN_ERR_ARG;
    if (splits_tc_max + d.splits_d + d.splits_v1 > MERGE_SPLITS) return SJK_ERR_UNSUPPORTED;
    // model-basis queries: the 4-bit body kernel rotates them on chip when it is the call's only reader of q; otherwise
    // they are rotated once into the end of the scratch, which sjk_attend_scratch_bytes() sizes for it
    bool q_on_chip = false;
    if (model) {
        const int D = v->lay.D;
        if (D != 128 && D != 256 && D != 512) return SJK_ERR_UNSUPPORTED;
        q_on_chip = pa.tc_body && splits_tc_max > 0 && d.splits_d == 0 && d.splits_v1 == 0 && D == 256;
        if (!q_on_chip) {
            const size_t qb = (size_t) n_q * n_head * D * sizeof(float);
            const size_t off = scratch_bytes >= qb ? (scratch_bytes - qb) & ~(size_t) 255 : 0;
            if (scratch_bytes < qb || off < need) return SJKVARN_ERR_ARG;
            float * qr = reinterpret_cast<float *>(static_cast<uint8_t *>(scratch) + off);
            const dim3 grid((unsigned) ((n_q * n_head + 7) / 8)), block(256);
            const float sc = sjk_fwht_scale(D);
            if (D == 128) rotate_rows_kernel<128><<<grid, block, 0, st>>>(q, qr, n_q * n_head, sc);
            else if (D == 256) rotate_rows_kernel<256><<<grid, block, 0, st>>>(q, qr, n_q * n_head, sc);
            else rotate_rows_kernel<512><<<grid, block, 0, st>>>(q, qr, n_q * n_head, sc);
            if (sjk_check_launch()) return SJK_ERR_DEVICE;
            q = qr;
        }
    }
    int splits_tc = 0;
    if (splits_tc_max) {
        const int rc = pa.tc_body ? sjk_tc_body_launch(v, B, N, d.n_tc, (int) d.dense_regions, qpos0, n_q, n_head, kv_head0, n_kv, q,
                                                       scale, (float *) scratch, 0, 148 - d.dense_sms, q_on_chip, &splits_tc, st)
                                  : sjk_tc_trellis_launch(v, B, N, d.n_tc, qpos0, n_q, n_head, kv_head0, n_kv, q, scale,
                                                          (float *) scratch, 0, d.splits_tc, &splits_tc, st);
        if (rc) return rc;
    }
    const int splits = splits_tc + d.splits_d + d.splits_v1;
    // nothing to attend to: a zero output; an empty partial (m = -inf, l = 0, o = 0) comes from the merge kernel
    if (splits == 0 && !part_out) return sjk_check(cudaMemsetAsync(out, 0, (size_t) n_q * n_head * v->lay.D * sizeof(float), st));
    if (d.splits_d) {
        const int rc = sjk_tc_dense_launch(v, B, N, qpos0, n_q, n_head, kv_head0, n_kv, q, scale, (float *) scratch,
                                           splits_tc, d.splits_d, d.n_sink_d, d.n_dense, d.cps_d,
                                           d.dense_sms > 0 && splits_tc > 0, st);
        if (rc) return rc;
    }
    AttnParams p;
    p.v = *v; p.kv0 = kv_head0; p.B = B; p.N = N; p.qpos0 = qpos0; p.n_q = n_q; p.n_head = n_head; p.grp = grp;
    p.rows = n_q * grp; p.q = q; p.scale = scale; p.part = (float *) scratch; p.split0 = splits_tc + d.splits_d;
    p.chunks_per_split = d.v1.chunks_per_split; p.n_chunks = d.v1.n_chunks; p.n_sink_chunks = d.v1.n_sink;
    p.n_body_chunks = d.v1.n_body; p.body_skip = d.n_tc; p.n_splits = d.splits_v1;
    if (d.splits_v1) {
        const int rc = launch_split(p, nullptr, d.splits_v1, n_kv, st);
        if (rc) return rc;
    }
    return launch_merge(p.part, splits, nullptr, 0, n_q * n_head, v->lay.D, out, part_out, st, model && !part_out);
}
}  // namespace

int sjk_attend_heads(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, int kv_head0, int n_kv,
                     const float * q, float scale, float * out, void * scratch, size_t scratch_bytes, sjk_stream st,
                     unsigned regions, float * part_out) {
    return attend_heads_impl(v, B, N, qpos0, n_q, n_head, kv_head0, n_kv, q, scale, out, scratch, scratch_bytes, st, regions,
                             part_out, false);
}

// ---- descriptor-driven attention (the reference's region-aware flash attention op, INTEGRATION_LLAMACPP.md:50) ----
// The call's scratch: the device-side plan (counts, then each kernel's launch plan), then the split partials.
namespace {

constexpr size_t DYN_ALIGN = 256;
size_t dyn_align(size_t x) { return (x + DYN_ALIGN - 1) & ~(DYN_ALIGN - 1); }
struct DynLayout { size_t state, v1, body, dense, part, total_hdr; };
DynLayout dyn_layout() {
    DynLayout L;
    L.state = 0;
    L.v1 = dyn_align(sizeof(sjk_dyn_state));
    L.body = L.v1 + dyn_align(sizeof(AttnParams));
    const size_t tb = sjk_tc_body_params_bytes(), tt = sjk_tc_trellis_params_bytes();
    L.dense = L.body + dyn_align(tb > tt ? tb : tt);
    L.part = L.dense + dyn_align(sjk_tc_dense_params_bytes());
    L.total_hdr = L.part;
    return L;
}

// The counts of the call from the descriptor (sjk_plan_counts, as sjk_attend_heads makes them on the host) and the
// CUDA-core kernel's plan. A descriptor that fails its checks plans no work (a zero output).
__global__ void attend_dyn_plan_kernel(const int32_t * desc, sjk_desc_ref ref, sjk_paths pa, int n_kv, AttnParams tmpl,
                                       sjk_dyn_state * ds, AttnParams * v1) {
    if (threadIdx.x != 0) return;
    sjk_desc_vals dv;
    sjk_dyn_state d;
    memset(&d, 0, sizeof d);
    if (sjk_desc_read(desc, ref, &dv)) {
        d.ok = 1;
        sjk_plan_counts(pa, ref.S, dv.B, dv.N, SJK_REGION_ALL, n_kv, &d);
        d.qpos0 = dv.qpos0;
    } else {
        sjk_desc_fault();
        d.B = ref.S; d.N = 0;
    }
    *ds = d;
    AttnParams p = tmpl;
    p.B = d.B; p.N = d.N; p.qpos0 = d.qpos0; p.split0 = d.splits_tc + d.splits_d;
    p.chunks_per_split = d.v1.chunks_per_split; p.n_chunks = d.v1.n_chunks; p.n_sink_chunks = d.v1.n_sink;
    p.n_body_chunks = d.v1.n_body; p.body_skip = d.n_tc; p.n_splits = d.ok ? d.splits_v1 : 0;
    *v1 = p;
}

}  // namespace

extern "C" size_t sjk_attend_dyn_scratch_bytes(const sjk_view * v, int n_q, int n_head) {
    if (!v || n_q <= 0 || n_head <= 0) return 0;
    return dyn_layout().total_hdr + sjk_attend_heads_scratch_bytes(v, n_q, n_head, v->n_head_kv);
}

extern "C" int sjk_desc_fill(const sjk_view * v, uint32_t B_old, uint32_t B, uint32_t N, uint32_t qpos0, int32_t * desc) {
    if (!v || !desc || B_old > 0x7FFFFFFFu || B > 0x7FFFFFFFu || N > 0x7FFFFFFFu || qpos0 > 0x7FFFFFFFu) return SJKVARN_ERR_ARG;
    int32_t e[SJK_DESC_N_ENTRIES] = {0};
    e[SJK_DESC_S] = (int32_t) v->S; e[SJK_DESC_CAP] = (int32_t) v->cap; e[SJK_DESC_B] = (int32_t) B; e[SJK_DESC_N] = (int32_t) N;
    e[SJK_DESC_QPOS0] = (int32_t) qpos0; e[SJK_DESC_G] = v->lay.G; e[SJK_DESC_D] = v->lay.D;
    e[SJK_DESC_RECBYTES] = (int32_t) v->lay.bytes; e[SJK_DESC_HKV] = v->n_head_kv; e[SJK_DESC_B_OLD] = (int32_t) B_old;
    e[SJK_DESC_TYPE_K] = v->staging; e[SJK_DESC_TYPE_V] = v->staging; e[SJK_DESC_BODY_TYPE] = v->lay.body;
    e[SJK_DESC_SINK_TYPE] = v->sink_type;
    sjk_desc_vals dv;
    if (!sjk_desc_check(e, sjk_desc_ref_of(*v), &dv)) return SJKVARN_ERR_ARG;
    memcpy(desc, e, sizeof e);
    return 0;
}

// Launch shapes depend only on the cache, n_q and n_head: the planner kernel writes the counts and every kernel's
// plan into the scratch, each kernel reads its plan there and its CTAs past the plan return at once.
extern "C" int sjk_attend_dyn(const sjk_view * v, const int32_t * desc, int n_q, int n_head, const float * q, float scale,
                              float * out, void * scratch, size_t scratch_bytes, sjk_stream st) {
    if (!v || !desc || !q || !out || n_q <= 0 || n_head <= 0 || v->n_head_kv <= 0 || n_head % v->n_head_kv) return SJKVARN_ERR_ARG;
    const int n_kv = v->n_head_kv, grp = n_head / n_kv;
    if (n_q * grp > MAXROWS) return SJK_ERR_UNSUPPORTED;
    if (!scratch || scratch_bytes < sjk_attend_dyn_scratch_bytes(v, n_q, n_head)) return SJKVARN_ERR_ARG;
    if (((uintptr_t) scratch) % DYN_ALIGN) return SJKVARN_ERR_ARG;
    const sjk_paths pa = paths_of(v, n_q, grp);
    const DynLayout L = dyn_layout();
    uint8_t * base = static_cast<uint8_t *>(scratch);
    sjk_dyn_state * ds = reinterpret_cast<sjk_dyn_state *>(base + L.state);
    AttnParams * v1p = reinterpret_cast<AttnParams *>(base + L.v1);
    float * part = reinterpret_cast<float *>(base + L.part);
    AttnParams t;
    memset(&t, 0, sizeof t);
    t.v = *v; t.kv0 = 0; t.n_q = n_q; t.n_head = n_head; t.grp = grp; t.rows = n_q * grp; t.q = q; t.scale = scale; t.part = part;
    attend_dyn_plan_kernel<<<1, 32, 0, st>>>(desc, sjk_desc_ref_of(*v), pa, n_kv, t, ds, v1p);
    if (sjk_check_launch()) return SJK_ERR_DEVICE;
    int rc = 0;
    if (pa.tc_body) rc = sjk_tc_body_dyn_launch(v, n_q, n_head, 0, n_kv, q, scale, part, ds, base + L.body, st);
    else if (pa.tc_trellis) rc = sjk_tc_trellis_dyn_launch(v, n_q, n_head, 0, n_kv, q, scale, part, ds, base + L.body, st);
    if (rc) return rc;
    const int target = sjk_split_target(n_kv);
    if (pa.dense && !pa.fused) {
        // the most items a plan can have: the dense split count never exceeds the target, nor the chunks of the sink
        // and of a full ring (plus one for a ring range that straddles a chunk boundary)
        const uint32_t max_chunks = (v->S + 127u) / 128u + (v->cap + 127u) / 128u + 1u;
        const int per_head = (uint32_t) target < max_chunks ? target : (int) max_chunks;
        rc = sjk_tc_dense_dyn_launch(v, n_q, n_head, 0, n_kv, q, scale, part, ds, base + L.dense, per_head * n_kv, st);
        if (rc) return rc;
    }
    // the CUDA-core kernel: with both tensor-core paths it only takes the partly visible record of a query over a
    // prefix (at most one chunk per KV head); otherwise up to the target
    const int v1_max = ((pa.tc_body || pa.tc_trellis) && pa.dense) ? 1 : target;
    rc = launch_split(t, v1p, v1_max, n_kv, st);
    if (rc) return rc;
    const int max_splits = (pa.tc_body ? sjk_tc_body_max_splits(n_kv) : pa.tc_trellis ? sjk_tc_trellis_max_splits(n_kv) : 0) +
                           2 * target;
    return launch_merge(part, 0, &ds->splits, max_splits, n_q * n_head, v->lay.D, out, nullptr, st);
}

// Attention over a subset of the regions, as one partial (m, l, o[D]) per (query row, query head). The
// partials of disjoint region sets, or of context slices held by different GPUs, combine with sjk_attend_merge.
extern "C" int sjk_attend_partial(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                                  unsigned regions, const float * q, float scale, float * part_out, void * scratch,
                                  size_t scratch_bytes, sjk_stream st) {
    if (!v || !part_out || (regions & ~(unsigned) SJK_REGION_ALL)) return SJKVARN_ERR_ARG;
    return sjk_attend_heads(v, B, N, qpos0, n_q, n_head, 0, v->n_head_kv, q, scale, nullptr, scratch, scratch_bytes, st,
                            regions, part_out);
}

// sjk_attend_partial whose partials go straight to every rank over peer memory: the call's merge kernel writes the
// rank's triples to the end of the scratch, and one exchange launch (sjk_xchg_exchange) stores them into every rank's
// exchange buffer, gathers every rank's and writes the merge of all of them to out[n_q * n_head][D] - the all-gather +
// sjk_attend_merge of the same triples. (The exchange inside the merge kernel itself measured slower on 2 GPUs: 251.7
// against 241.3 us per config-4 call.)
extern "C" int sjk_attend_partial_xchg(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                                       unsigned regions, const float * q, float scale, void * scratch, size_t scratch_bytes,
                                       const sjk_xchg_peers * x, uint32_t epoch, float * out, sjk_stream st) {
    if (!v || !out || !x || (regions & ~(unsigned) SJK_REGION_ALL) || epoch == 0 || x->world <= 0 ||
        x->world > SJK_XCHG_MAX_WORLD || x->rank < 0 || x->rank >= x->world)
        return SJKVARN_ERR_ARG;
    for (int i = 0; i < x->world; ++i)
        if (!x->buf[i] || ((uintptr_t) x->buf[i] & 255)) return SJKVARN_ERR_ARG;
    const size_t own = xchg_part_bytes(v, n_q, n_head);
    if (!scratch || scratch_bytes < own + 256) return SJKVARN_ERR_ARG;
    const size_t split_bytes = (scratch_bytes - own) & ~(size_t) 255;
    float * part = reinterpret_cast<float *>(static_cast<uint8_t *>(scratch) + split_bytes);
    const int rc = sjk_attend_heads(v, B, N, qpos0, n_q, n_head, 0, v->n_head_kv, q, scale, nullptr, scratch, split_bytes, st,
                                    regions, part);
    if (rc) return rc;
    return sjk_xchg_exchange(x, part, n_q * n_head, v->lay.D, epoch, out, st);
}

// out[n_rows][D] from n_parts partial sets parts[n_parts][n_rows][D + 2], combined in index order
extern "C" int sjk_attend_merge(const float * parts, int n_parts, int n_rows, int D, float * out, sjk_stream st) {
    if (!parts || !out || n_parts <= 0 || n_rows <= 0 || D <= 0 || n_parts > MERGE_SPLITS) return SJKVARN_ERR_ARG;
    attend_merge_kernel<<<dim3((unsigned) n_rows, (unsigned) ((D + 63) / 64)), 256, (size_t) (n_parts + 256) * sizeof(float), st>>>(
        parts, n_parts, n_rows, D, out, nullptr, nullptr);
    return sjk_check_launch();
}

SJK_DESC_STATUS_READER(attend_desc_status_take)

// status words of every kernel with bounded waits (SJK_DEVICE_TIMEOUT) and of the descriptor-driven calls
// (SJK_DEVICE_DESC) since the last call
extern "C" int sjk_device_status(void) {
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    const int a = sjk_tc_body_status_take(), b = sjk_tc_dense_status_take(), c = sjk_tc_trellis_status_take();
    const int d = attend_desc_status_take(), e = sjk_seal_desc_status_take(), f = sjk_stage_desc_status_take();
    const int x = sjk_xchg_status_take();
    if (a < 0 || b < 0 || c < 0 || d < 0 || e < 0 || f < 0 || x < 0) return -1;
    return a | b | c | d | e | f | x;
}

extern "C" int sjk_attend(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head, const float * q,
                          float scale, float * out, void * scratch, size_t scratch_bytes, sjk_stream st) {
    if (!v) return SJKVARN_ERR_ARG;
    return sjk_attend_heads(v, B, N, qpos0, n_q, n_head, 0, v->n_head_kv, q, scale, out, scratch, scratch_bytes, st,
                            SJK_REGION_ALL, nullptr);
}

// sjk_attend with queries and outputs in the model basis: the rotation happens inside the call (on chip in the 4-bit
// body kernel and in the merge kernel's clusters, or one rotation launch for the other kernels' queries)
extern "C" int sjk_attend_model(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                                const float * q, float scale, float * out, void * scratch, size_t scratch_bytes, sjk_stream st) {
    if (!v || !out) return SJKVARN_ERR_ARG;
    return attend_heads_impl(v, B, N, qpos0, n_q, n_head, 0, v->n_head_kv, q, scale, out, scratch, scratch_bytes, st,
                             SJK_REGION_ALL, nullptr, true);
}

// ---- attention for callers that cannot allocate ------------------------------------------------------------
// sjk_attend_static: sjk_attend with its split-partial scratch in a fixed device array instead of a caller
// buffer. Capacity SJK_STATIC_SCRATCH_BYTES (16 MiB): every GPU that loads this library holds the array until
// the process exits. The array's host-side name is only a stand-in for its device address, so the address is
// looked up once per device (cudaGetSymbolAddress, with that device current) on the first call there and
// cached; that first call should therefore come before any stream capture. Shapes whose scratch bound
// (sjk_attend_scratch_bytes) exceeds the capacity are rejected with SJK_ERR_SCRATCH_LIMIT. Every call
// writes all the partials it later reads, so nothing needs clearing between calls; calls that overlap on
// the GPU (other streams, other host threads) share the array and race.
#define SJK_STATIC_SCRATCH_BYTES ((size_t) 16 << 20)
static __device__ __align__(256) unsigned char sjk_static_scratch[SJK_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_static_mu;
void * g_static_ptr[256];                    // device address of sjk_static_scratch, per device ordinal
}

extern "C" int sjk_attend_static(const sjk_view * v, uint32_t B, uint32_t N, uint32_t qpos0, int n_q, int n_head,
                                 const float * q, float scale, float * out, sjk_stream st) {
    if (!v || n_q <= 0 || n_head <= 0) return SJKVARN_ERR_ARG;
    const size_t need = sjk_attend_heads_scratch_bytes(v, n_q, n_head, v->n_head_kv);   // the split partials of one call
    if (need > SJK_STATIC_SCRATCH_BYTES) return SJK_ERR_SCRATCH_LIMIT;
    int dev = 0;
    if (sjk_check(cudaGetDevice(&dev))) return SJK_ERR_DEVICE;
    if (dev < 0 || dev >= 256) return SJK_ERR_UNSUPPORTED;
    void * ptr = NULL;
    {
        std::lock_guard<std::mutex> lk(g_static_mu);
        ptr = g_static_ptr[dev];
        if (!ptr) {
            if (sjk_check(cudaGetSymbolAddress(&ptr, sjk_static_scratch))) return SJK_ERR_DEVICE;
            g_static_ptr[dev] = ptr;
        }
    }
    return sjk_attend_heads(v, B, N, qpos0, n_q, n_head, 0, v->n_head_kv, q, scale, out, ptr, SJK_STATIC_SCRATCH_BYTES, st,
                            SJK_REGION_ALL, nullptr);
}
