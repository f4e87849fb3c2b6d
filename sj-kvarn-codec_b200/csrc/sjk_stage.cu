// sjk_stage.cu - K/V cache write: per-head Hadamard rotation fused with tq6_0 / fp16 staging into the
// fp16 sink or the staging ring (sj_kvarn.h:735-752, 1211-1284, 1475-1492), plus the standalone
// rotate / stage / unstage kernels of the device layer.
//
// One warp owns one (position, head, K|V) row of D values; lane l holds the D/32 contiguous values
// [l*D/32, (l+1)*D/32). The FWHT runs its first log2(D/32) butterfly stages inside each lane and the
// rest across lanes with shuffles, keeping the reference's stage order so each output is the same
// add/sub tree. The tq6_0 norm is a SEQUENTIAL fp32 sum over the block's 128 values (bit-exactness
// needs that order): it is carried lane to lane through the block with shuffles. The packed 98-byte
// blocks of a whole position are assembled in shared memory and leave in 16-byte stores, because a
// position's slot ([H][K row | V row], 1568 B at D=256, H=4) is contiguous and 16-byte aligned.
#include "sjk_common.cuh"
#include "sjk_fwht.cuh"
#include "sjk_desc.cuh"

namespace {

constexpr unsigned FULL = 0xFFFFFFFFu;

struct StoreParams {
    const float * k;
    const float * v;
    uint8_t * sink;
    uint8_t * ring;
    uint32_t pos0, S, cap;
    int H;
    int staging;        // SJKVARN_STAGING_*
    int sink_f16;       // 1: positions < S go to the fp16 sink; 0: to staging rows in the sink
    int rotate;
    float fwht_scale;   // 1/sqrt(D), computed on the host with the reference's operations
    uint32_t stage_bytes;
    const int32_t * desc;   // sjk_store_dyn: pos0 is the descriptor's QPOS0, read when the kernel runs
    sjk_desc_ref dref;
};

// code = number of decision midpoints not above v, as the reference's binary search
// (sj_kvarn.h:1211-1219); NaN compares false everywhere and ends on 63
SJK_DEV int tq6_code(float v, const float * mid) {
    int idx = 0;
#pragma unroll
    for (int step = 32; step >= 1; step >>= 1) {
        const int probe = idx + step - 1;
        if (probe < 63 && !(v < mid[probe])) idx += step;
    }
    return idx;
}

// Sequential sum over the 128 values of a block, in value order, carried across the LPB lanes of the block.
template <int VPL>
SJK_DEV float block_chain_sum(const float (&sq)[VPL], int lane) {
    constexpr int LPB = 128 / VPL;     // lanes per 128-value block
    const int first = lane & ~(LPB - 1), j = lane & (LPB - 1);
    float acc = 0.0f;
#pragma unroll
    for (int s = 0; s < LPB; ++s) {
        const float in = __shfl_sync(FULL, acc, first | ((s + LPB - 1) & (LPB - 1)));
        if (j == s) {
            float a = s == 0 ? 0.0f : in;
#pragma unroll
            for (int i = 0; i < VPL; ++i) a = __fadd_rn(a, sq[i]);
            acc = a;
        }
    }
    return __shfl_sync(FULL, acc, first | (LPB - 1));
}

// Quantize the warp's row (already rotated) to tq6_0 blocks written at dst (shared or global bytes).
template <int VPL>
SJK_DEV void tq6_row(const float (&x)[VPL], int lane, uint8_t * dst, const float * mid, const float * cent) {
    constexpr int LPB = 128 / VPL;
    float sq[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) sq[i] = __fmul_rn(x[i], x[i]);
    const float norm = sqrtf(block_chain_sum<VPL>(sq, lane));
    const bool live = norm > 1e-10f;
    const float inv = live ? __fdiv_rn(1.0f, norm) : 0.0f;
    int code[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        code[i] = tq6_code(live ? __fmul_rn(x[i], inv) : 0.0f, mid);
        const float c = cent[code[i]];
        sq[i] = __fmul_rn(c, c);
    }
    const float rn = sqrtf(block_chain_sum<VPL>(sq, lane));
    const uint16_t hn = sjk_f2h(rn > 1e-10f ? __fdiv_rn(norm, rn) : norm);
    const int blk = lane / LPB, j = lane & (LPB - 1);
    uint8_t * b = dst + blk * SJKVARN_TQ6_BLOCK_BYTES;
    if (j == 0) { b[0] = (uint8_t) hn; b[1] = (uint8_t) (hn >> 8); }
    // value i of the block = j*VPL + k: low nibble in qs[i/2] at bit 4(i%2), top bits in qh[i/4] at 2(i%4)
#pragma unroll
    for (int k = 0; k < VPL; k += 2)
        b[2 + (j * VPL + k) / 2] = (uint8_t) ((code[k] & 15) | ((code[k + 1] & 15) << 4));
#pragma unroll
    for (int k = 0; k < VPL; k += 4)
        b[66 + (j * VPL + k) / 4] = (uint8_t) (((code[k] >> 4) & 3) | (((code[k + 1] >> 4) & 3) << 2) |
                                               (((code[k + 2] >> 4) & 3) << 4) | (((code[k + 3] >> 4) & 3) << 6));
}

template <int VPL>
SJK_DEV void f16_row(const float (&x)[VPL], int lane, uint8_t * dst) {
    // VPL halves per lane: 2*VPL bytes at dst + lane*2*VPL (16-byte aligned rows)
    uint32_t w[VPL / 2];
#pragma unroll
    for (int i = 0; i < VPL / 2; ++i) w[i] = (uint32_t) sjk_f2h(x[2 * i]) | ((uint32_t) sjk_f2h(x[2 * i + 1]) << 16);
    uint32_t * o = reinterpret_cast<uint32_t *>(dst + (size_t) lane * 2 * VPL);
    if constexpr (VPL % 8 == 0) {
#pragma unroll
        for (int i = 0; i < VPL / 2; i += 4) *reinterpret_cast<uint4 *>(o + i) = make_uint4(w[i], w[i + 1], w[i + 2], w[i + 3]);
    } else {
#pragma unroll
        for (int i = 0; i < VPL / 2; ++i) o[i] = w[i];
    }
}

template <int VPL>
SJK_DEV void load_row(const float * src, int lane, float (&x)[VPL]) {
    const float4 * s = reinterpret_cast<const float4 *>(src + (size_t) lane * VPL);
#pragma unroll
    for (int i = 0; i < VPL / 4; ++i) {
        const float4 t = __ldg(s + i);
        x[4 * i] = t.x; x[4 * i + 1] = t.y; x[4 * i + 2] = t.z; x[4 * i + 3] = t.w;
    }
}

// Copy n bytes from shared to global with the widest stores both addresses allow.
SJK_DEV void copy_out(uint8_t * dst, const uint8_t * src, uint32_t n, int tid, int nthr) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(dst);
    if ((a & 15u) == 0 && (n & 15u) == 0) {
        for (uint32_t i = (uint32_t) tid; i < n / 16; i += (uint32_t) nthr)
            reinterpret_cast<uint4 *>(dst)[i] = reinterpret_cast<const uint4 *>(src)[i];
    } else if ((a & 3u) == 0 && (n & 3u) == 0) {
        for (uint32_t i = (uint32_t) tid; i < n / 4; i += (uint32_t) nthr)
            reinterpret_cast<uint32_t *>(dst)[i] = reinterpret_cast<const uint32_t *>(src)[i];
    } else {
        for (uint32_t i = (uint32_t) tid; i < n; i += (uint32_t) nthr) dst[i] = src[i];
    }
}

// Batched cache write (sjk_store_batch): one position per item, each in its own cache (sink and ring of one layer of
// one sequence); the rows of item i are k, v + i H D.
constexpr int STORE_BATCH_MAX = 1024;
// The store is latency-bound (two sequential 128-value norm sums per tq6_0 block): six resident CTAs per SM
// (40 registers a thread) hide more of it than three at the unconstrained 72 registers (8,320 positions:
// 76 against 107 us).
constexpr int STORE_MIN_CTAS = 6;
struct StoreBatchParams {
    StoreParams c;                          // shared fields (k, v, formats, S, cap, H); sink / ring / pos0 per item
    uint8_t * sink[STORE_BATCH_MAX];
    uint8_t * ring[STORE_BATCH_MAX];
    uint32_t pos[STORE_BATCH_MAX];
};

// One CTA per position: its 2H rows (head-major, K then V) are rotated, staged and written.
template <int D>
__global__ void __launch_bounds__(256, STORE_MIN_CTAS) store_kernel(StoreParams p);
template <int D>
__device__ __forceinline__ void store_position(const StoreParams & p, uint32_t pos, uint8_t * sink, uint8_t * ring,
                                               size_t row0);

template <int D>
__global__ void __launch_bounds__(256, STORE_MIN_CTAS) store_batch_kernel(const __grid_constant__ StoreBatchParams b) {
    store_position<D>(b.c, b.pos[blockIdx.x], b.sink[blockIdx.x], b.ring[blockIdx.x], blockIdx.x);
}

template <int D>
__global__ void __launch_bounds__(256, STORE_MIN_CTAS) store_kernel(StoreParams p) {
    uint32_t pos0 = p.pos0;
    if (p.desc) {
        sjk_desc_vals dv;
        if (!sjk_desc_read(p.desc, p.dref, &dv)) {
            if (blockIdx.x == 0 && threadIdx.x == 0) sjk_desc_fault();
            return;
        }
        pos0 = dv.qpos0;
    }
    store_position<D>(p, pos0 + blockIdx.x, p.sink, p.ring, blockIdx.x);
}

// Position pos of one cache; its rows are row0 .. of k and v ([*][H][D]).
template <int D>
__device__ __forceinline__ void store_position(const StoreParams & p, uint32_t pos, uint8_t * sink, uint8_t * ring,
                                               size_t row0) {
    constexpr int VPL = D / 32;
    extern __shared__ __align__(16) uint8_t smem[];
    float * mid = reinterpret_cast<float *>(smem);
    float * cent = mid + 64;
    uint8_t * rows = smem + 128 * sizeof(float);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    if (threadIdx.x < 63) mid[threadIdx.x] = sjk_tq6_mid[threadIdx.x];
    if (threadIdx.x < 64) cent[threadIdx.x] = sjk_tq6_cent[threadIdx.x];
    __syncthreads();
    const bool in_sink = pos < p.S;
    const bool f16_out = in_sink ? p.sink_f16 || p.staging == SJKVARN_STAGING_F16 : p.staging == SJKVARN_STAGING_F16;
    const uint32_t row_bytes = (in_sink && p.sink_f16) ? (uint32_t) D * 2u : p.stage_bytes;
    uint8_t * base = in_sink ? sink + (size_t) pos * p.H * 2 * row_bytes
                             : ring + (size_t) sjk_ring_slot(p.S, p.cap, pos) * p.H * 2 * row_bytes;
    for (int r = warp; r < 2 * p.H; r += nwarp) {
        const int h = r >> 1, side = r & 1;
        float x[VPL];
        load_row<VPL>((side ? p.v : p.k) + (row0 * p.H + h) * D, lane, x);
        if (p.rotate) fwht_warp<VPL>(x, lane, p.fwht_scale);
        if (f16_out) f16_row<VPL>(x, lane, base + (size_t) r * row_bytes);
        else tq6_row<VPL>(x, lane, rows + (size_t) r * row_bytes, mid, cent);
    }
    if (!f16_out) {
        __syncthreads();
        copy_out(base, rows, (uint32_t) (2 * p.H) * row_bytes, threadIdx.x, blockDim.x);
    }
}

// Standalone staging of rotated rows: one warp per row, staged bytes at dst + row*dst_row_bytes.
template <int D>
__global__ void __launch_bounds__(256) stage_rows_kernel(int staging, const float * x, uint8_t * dst, size_t dst_row_bytes,
                                                         int n_rows) {
    constexpr int VPL = D / 32;
    __shared__ float mid[64], cent[64];
    __shared__ __align__(16) uint8_t rowbuf[8][(D / 128) * SJKVARN_TQ6_BLOCK_BYTES + 16];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x < 63) mid[threadIdx.x] = sjk_tq6_mid[threadIdx.x];
    if (threadIdx.x < 64) cent[threadIdx.x] = sjk_tq6_cent[threadIdx.x];
    __syncthreads();
    const int row = blockIdx.x * 8 + warp;
    if (row >= n_rows) return;
    float v[VPL];
    load_row<VPL>(x + (size_t) row * D, lane, v);
    uint8_t * out = dst + (size_t) row * dst_row_bytes;
    if (staging == SJKVARN_STAGING_F16) {
        if ((reinterpret_cast<uintptr_t>(out) & 15u) == 0) { f16_row<VPL>(v, lane, out); return; }
        for (int i = 0; i < VPL; ++i) {
            const uint16_t hv = sjk_f2h(v[i]);
            out[2 * (lane * VPL + i)] = (uint8_t) hv; out[2 * (lane * VPL + i) + 1] = (uint8_t) (hv >> 8);
        }
        return;
    }
    tq6_row<VPL>(v, lane, rowbuf[warp], mid, cent);
    __syncwarp();
    constexpr int NB = (D / 128) * SJKVARN_TQ6_BLOCK_BYTES;
    for (int i = lane; i < NB; i += 32) out[i] = rowbuf[warp][i];
}

// Widen staged rows: one thread per value (sj_kvarn.h:1249-1260, 1276-1284).
__global__ void unstage_rows_kernel(int staging, const uint8_t * src, size_t src_row_bytes, float * x, int D, int n_rows) {
    const size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t) n_rows * D) return;
    const size_t row = i / (size_t) D;
    const int c = (int) (i % (size_t) D);
    const uint8_t * r = src + row * src_row_bytes;
    if (staging == SJKVARN_STAGING_F16) { x[i] = sjk_h2f(sjk_ld_u16(r + 2 * c)); return; }
    const uint8_t * b = r + (c >> 7) * SJKVARN_TQ6_BLOCK_BYTES;
    const int j = c & 127;
    const int code = ((b[2 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((b[66 + (j >> 2)] >> (2 * (j & 3))) & 3) << 4);
    x[i] = __fmul_rn(sjk_tq6_cent[code], sjk_h2f(sjk_ld_u16(b)));
}

template <int D>
__global__ void __launch_bounds__(256) hadamard_kernel(float * x, int n_rows, float scale) {
    constexpr int VPL = D / 32;
    const int lane = threadIdx.x & 31, row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= n_rows) return;
    float v[VPL];
    float * r = x + (size_t) row * D;
#pragma unroll
    for (int i = 0; i < VPL; ++i) v[i] = r[lane * VPL + i];
    fwht_warp<VPL>(v, lane, scale);
#pragma unroll
    for (int i = 0; i < VPL; ++i) r[lane * VPL + i] = v[i];
}


}  // namespace

// ---- host entry points --------------------------------------------------------------------------------------

extern "C" int sjk_hadamard(float * x, int n_rows, int n, sjk_stream st) {
    if (!x || n_rows < 0) return SJKVARN_ERR_ARG;
    if (n_rows == 0) return 0;
    const dim3 grid((unsigned) ((n_rows + 7) / 8)), block(256);
    const float s = sjk_fwht_scale(n);
    switch (n) {
        case 128: hadamard_kernel<128><<<grid, block, 0, st>>>(x, n_rows, s); break;
        case 256: hadamard_kernel<256><<<grid, block, 0, st>>>(x, n_rows, s); break;
        case 512: hadamard_kernel<512><<<grid, block, 0, st>>>(x, n_rows, s); break;
        case 1024: hadamard_kernel<1024><<<grid, block, 0, st>>>(x, n_rows, s); break;
        default: return SJK_ERR_UNSUPPORTED;
    }
    return sjk_check_launch();
}

extern "C" int sjk_stage_rows(int staging, const float * x_rot, uint8_t * dst, size_t dst_row_bytes, int D, int n_rows,
                              sjk_stream st) {
    if (!x_rot || !dst || n_rows < 0 || (staging != 0 && staging != 1)) return SJKVARN_ERR_ARG;
    if (n_rows == 0) return 0;
    const dim3 grid((unsigned) ((n_rows + 7) / 8)), block(256);
    switch (D) {
        case 128: stage_rows_kernel<128><<<grid, block, 0, st>>>(staging, x_rot, dst, dst_row_bytes, n_rows); break;
        case 256: stage_rows_kernel<256><<<grid, block, 0, st>>>(staging, x_rot, dst, dst_row_bytes, n_rows); break;
        case 512: stage_rows_kernel<512><<<grid, block, 0, st>>>(staging, x_rot, dst, dst_row_bytes, n_rows); break;
        default: return SJK_ERR_UNSUPPORTED;
    }
    return sjk_check_launch();
}

extern "C" int sjk_unstage_rows(int staging, const uint8_t * src, size_t src_row_bytes, float * x, int D, int n_rows,
                                sjk_stream st) {
    if (!src || !x || n_rows < 0 || D <= 0 || (D & 127)) return SJKVARN_ERR_ARG;
    if (n_rows == 0) return 0;
    const size_t n = (size_t) n_rows * D;
    unstage_rows_kernel<<<(unsigned) ((n + 255) / 256), 256, 0, st>>>(staging, src, src_row_bytes, x, D, n_rows);
    return sjk_check_launch();
}

// One position in each of n_items caches (the decode step's cache write across layers and sequences): item i
// stores rows k, vv + i H D at position pos[i] of views[i]'s sink / ring. Batches above STORE_BATCH_MAX take several
// launches.
extern "C" int sjk_store_batch(const sjk_view * views, const uint32_t * pos, int n_items, const float * k, const float * vv,
                               int rotate, sjk_stream st) {
    if (!views || !pos || !k || !vv || n_items < 0) return SJKVARN_ERR_ARG;
    if (n_items == 0) return 0;
    const sjk_view & v0 = views[0];
    if (v0.n_head_kv <= 0 || v0.cap == 0) return SJKVARN_ERR_ARG;
    for (int i = 0; i < n_items; ++i) {
        const sjk_view & v = views[i];
        if (!v.sink || !v.ring || v.lay.D != v0.lay.D || v.n_head_kv != v0.n_head_kv || v.staging != v0.staging ||
            v.sink_type != v0.sink_type || v.S != v0.S || v.cap != v0.cap || v.stage_bytes != v0.stage_bytes)
            return SJKVARN_ERR_ARG;
    }
    static thread_local StoreBatchParams b;
    StoreParams & p = b.c;
    p.S = v0.S; p.cap = v0.cap; p.H = v0.n_head_kv; p.pos0 = 0;
    p.staging = v0.staging; p.sink_f16 = v0.sink_type == SJKVARN_SINK_F16; p.rotate = rotate;
    p.fwht_scale = sjk_fwht_scale(v0.lay.D); p.stage_bytes = (uint32_t) v0.stage_bytes;
    p.sink = nullptr; p.ring = nullptr;
    const int warps = 2 * p.H < 8 ? 2 * p.H : 8;
    const size_t smem = 128 * sizeof(float) + (size_t) 2 * p.H * p.stage_bytes;
    if (smem > 48 * 1024) return SJK_ERR_UNSUPPORTED;
    const size_t row = (size_t) p.H * v0.lay.D;
    for (int i0 = 0; i0 < n_items; i0 += STORE_BATCH_MAX) {
        const int n = n_items - i0 < STORE_BATCH_MAX ? n_items - i0 : STORE_BATCH_MAX;
        p.k = k + (size_t) i0 * row; p.v = vv + (size_t) i0 * row;
        for (int i = 0; i < n; ++i) {
            b.sink[i] = const_cast<uint8_t *>(views[i0 + i].sink);
            b.ring[i] = const_cast<uint8_t *>(views[i0 + i].ring);
            b.pos[i] = pos[i0 + i];
        }
        switch (v0.lay.D) {
            case 128: store_batch_kernel<128><<<n, 32 * warps, smem, st>>>(b); break;
            case 256: store_batch_kernel<256><<<n, 32 * warps, smem, st>>>(b); break;
            case 512: store_batch_kernel<512><<<n, 32 * warps, smem, st>>>(b); break;
            default: return SJK_ERR_UNSUPPORTED;
        }
        const int rc = sjk_check_launch();
        if (rc) return rc;
    }
    return 0;
}

namespace {
int store_launch(const sjk_view * v, uint8_t * sink, uint8_t * ring, uint32_t pos0, uint32_t n_pos, const float * k,
                 const float * vv, int rotate, const int32_t * desc, sjk_stream st) {
    if (!v || !k || !vv || !sink || !ring || v->n_head_kv <= 0 || v->cap == 0) return SJKVARN_ERR_ARG;
    if (n_pos == 0) return 0;
    StoreParams p;
    p.desc = desc; p.dref = sjk_desc_ref_of(*v);
    p.k = k; p.v = vv; p.sink = sink; p.ring = ring; p.pos0 = pos0; p.S = v->S; p.cap = v->cap; p.H = v->n_head_kv;
    p.staging = v->staging; p.sink_f16 = v->sink_type == SJKVARN_SINK_F16; p.rotate = rotate;
    p.fwht_scale = sjk_fwht_scale(v->lay.D); p.stage_bytes = (uint32_t) v->stage_bytes;
    const int warps = 2 * p.H < 8 ? 2 * p.H : 8;
    const size_t smem = 128 * sizeof(float) + (size_t) 2 * p.H * p.stage_bytes;
    if (smem > 48 * 1024) return SJK_ERR_UNSUPPORTED;
    switch (v->lay.D) {
        case 128: store_kernel<128><<<n_pos, 32 * warps, smem, st>>>(p); break;
        case 256: store_kernel<256><<<n_pos, 32 * warps, smem, st>>>(p); break;
        case 512: store_kernel<512><<<n_pos, 32 * warps, smem, st>>>(p); break;
        default: return SJK_ERR_UNSUPPORTED;
    }
    return sjk_check_launch();
}
}  // namespace

extern "C" int sjk_store(const sjk_view * v, uint8_t * sink, uint8_t * ring, uint32_t pos0, uint32_t n_pos,
                         const float * k, const float * vv, int rotate, sjk_stream st) {
    return store_launch(v, sink, ring, pos0, n_pos, k, vv, rotate, nullptr, st);
}

// Descriptor-driven store (the reference's staged set_rows, INTEGRATION_LLAMACPP.md:48): positions QPOS0 ..
// QPOS0 + n_pos - 1 of the descriptor, read when the kernel runs.
extern "C" int sjk_store_dyn(const sjk_view * v, const int32_t * desc, uint32_t n_pos, const float * k, const float * vv,
                             int rotate, sjk_stream st) {
    if (!v || !desc) return SJKVARN_ERR_ARG;
    return store_launch(v, const_cast<uint8_t *>(v->sink), const_cast<uint8_t *>(v->ring), 0, n_pos, k, vv, rotate, desc, st);
}

SJK_DESC_STATUS_READER(sjk_stage_desc_status_take)
