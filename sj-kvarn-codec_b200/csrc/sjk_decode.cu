// sjk_decode.cu - record decode to float rows (sj_kvarn.h:1176-1207), the device layer's
// sjk_decode (the B200 counterpart of sj_kvarn_cuda_decode_kernel, sj_kvarn_cuda.cuh:57-66).
//
// One CTA per record. The record (<= 35 KB at D = 256) is copied to shared memory with 16-byte loads,
// the per-channel / per-token fp16 scales are widened once into float tables in natural channel order,
// and each thread then emits 4 consecutive channels of one token with a 16-byte store. Each value is
// ((q * scale) + zero) * column_scale with one rounding per operation, as the reference.
#include "sjk_common.cuh"
#include "sjk_internal.h"

namespace {

struct DecodeParams {
    sj_kvarn_layout lay;
    const uint8_t * body;
    float * out_k;
    float * out_v;
};

template <int D>
__global__ void __launch_bounds__(256) decode_kernel(DecodeParams p) {
    const sj_kvarn_layout & l = p.lay;
    constexpr int G = 128;
    extern __shared__ __align__(16) uint8_t smem[];
    float * ks = reinterpret_cast<float *>(smem);        // [D] K scale, natural channel order
    float * kz = ks + D;                                  // [D] K zero
    float * kt = kz + D;                                  // [G] K token scale
    float * vc = kt + G;                                  // [D] V channel scale
    float * vs = vc + D;                                  // [G] V scale
    float * vz = vs + G;                                  // [G] V zero
    float * cbk = vz + G;                                 // [512] trellis codebooks as float
    float * cbv = cbk + 512;
    uint8_t * rec = reinterpret_cast<uint8_t *>(cbv + 512);
    const uint8_t * grec = p.body + (size_t) blockIdx.x * l.bytes;
    // record -> smem (records are multiples of 16 bytes at every supported shape)
    for (uint32_t i = threadIdx.x; i < l.bytes / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(rec)[i] = __ldg(reinterpret_cast<const uint4 *>(grec) + i);
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        const int kc = sjk_k_ch(l, d), vcx = sjk_v_ch(l, d);
        ks[d] = sjk_h2f(sjk_ld_u16(rec + l.k_scale + 2 * kc));
        kz[d] = sjk_h2f(sjk_ld_u16(rec + l.k_zero + 2 * kc));
        vc[d] = sjk_h2f(sjk_ld_u16(rec + l.v_ch + 2 * vcx));
    }
    for (int t = threadIdx.x; t < G; t += blockDim.x) {
        kt[t] = sjk_h2f(sjk_ld_u16(rec + l.k_tok + 2 * t));
        vs[t] = sjk_h2f(sjk_ld_u16(rec + l.v_scale + 2 * t));
        vz[t] = sjk_h2f(sjk_ld_u16(rec + l.v_zero + 2 * t));
    }
    const bool trellis = l.body == SJKVARN_BODY_TRELLIS;
    if (trellis) {
        const uint16_t * ck = sjk_codebook(l.bits_k, 0), * cv = sjk_codebook(l.bits_v, 1);
        for (int i = threadIdx.x; i < (1 << (6 + l.bits_k)); i += blockDim.x) cbk[i] = sjk_h2f(ck[i]);
        for (int i = threadIdx.x; i < (1 << (6 + l.bits_v)); i += blockDim.x) cbv[i] = sjk_h2f(cv[i]);
    }
    __syncthreads();
    const uint8_t * kp = rec + l.k_payload, * vp = rec + l.v_payload;
    float * ok = p.out_k + (size_t) blockIdx.x * G * D;
    float * ov = p.out_v + (size_t) blockIdx.x * G * D;
    for (int i = threadIdx.x; i < G * D / 4; i += blockDim.x) {
        const int t = (4 * i) / D, d0 = (4 * i) % D;
        float rk[4], rv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int d = d0 + j;
            float qk, qv;
            if (trellis) {
                qk = cbk[sjk_window(kp, l.bits_k, d, t, G)];
                qv = cbv[sjk_window(vp, l.bits_v, d, t, G)];
            } else {
                qk = (float) sjk_get_bits(kp, sjk_code_bit(l, t, d, 0), l.bits_k);
                qv = (float) sjk_get_bits(vp, sjk_code_bit(l, t, d, 1), l.bits_v);
            }
            rk[j] = __fmul_rn(__fadd_rn(__fmul_rn(qk, ks[d]), kz[d]), kt[t]);
            rv[j] = __fmul_rn(__fadd_rn(__fmul_rn(qv, vs[t]), vz[t]), vc[d]);
        }
        reinterpret_cast<float4 *>(ok)[i] = make_float4(rk[0], rk[1], rk[2], rk[3]);
        reinterpret_cast<float4 *>(ov)[i] = make_float4(rv[0], rv[1], rv[2], rv[3]);
    }
}

}  // namespace

extern "C" int sjk_decode(const sj_kvarn_layout * lay, const uint8_t * body, int n_rec, float * out_k, float * out_v,
                          sjk_stream st) {
    if (!lay || !body || !out_k || !out_v || n_rec < 0 || lay->G != 128 || (lay->bytes & 15u)) return SJKVARN_ERR_ARG;
    if (n_rec == 0) return 0;
    DecodeParams p;
    p.lay = *lay; p.body = body; p.out_k = out_k; p.out_v = out_v;
    const size_t smem = (size_t) (3 * lay->D + 3 * 128 + 1024) * sizeof(float) + lay->bytes;
    cudaError_t e = cudaSuccess;
    switch (lay->D) {
        case 128:
            e = cudaFuncSetAttribute(decode_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
            if (e == cudaSuccess) decode_kernel<128><<<n_rec, 256, smem, st>>>(p);
            break;
        case 256:
            e = cudaFuncSetAttribute(decode_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
            if (e == cudaSuccess) decode_kernel<256><<<n_rec, 256, smem, st>>>(p);
            break;
        default: return SJK_ERR_UNSUPPORTED;
    }
    if (sjk_check(e)) return SJK_ERR_DEVICE;
    return sjk_check_launch();
}

// ---- single rows (the reference's decode_k_row / decode_v_row and layer_kv_row on device pointers) -----------
namespace {

SJK_DEV float decode_value(const sj_kvarn_layout & l, const uint8_t * rec, int t, int d, int is_v) {
    const int bits = is_v ? l.bits_v : l.bits_k;
    const uint8_t * payload = rec + (is_v ? l.v_payload : l.k_payload);
    float q;
    if (l.body == SJKVARN_BODY_TRELLIS) q = sjk_h2f(sjk_codebook(bits, is_v)[sjk_window(payload, bits, d, t, l.G)]);
    else q = (float) sjk_get_bits(payload, sjk_code_bit(l, t, d, is_v), bits);
    if (!is_v) {
        const int kc = sjk_k_ch(l, d);
        return __fmul_rn(__fadd_rn(__fmul_rn(q, sjk_h2f(sjk_ld_u16(rec + l.k_scale + 2 * kc))), sjk_h2f(sjk_ld_u16(rec + l.k_zero + 2 * kc))),
                         sjk_h2f(sjk_ld_u16(rec + l.k_tok + 2 * t)));
    }
    return __fmul_rn(__fadd_rn(__fmul_rn(q, sjk_h2f(sjk_ld_u16(rec + l.v_scale + 2 * t))), sjk_h2f(sjk_ld_u16(rec + l.v_zero + 2 * t))),
                     sjk_h2f(sjk_ld_u16(rec + l.v_ch + 2 * sjk_v_ch(l, d))));
}

__global__ void decode_row_kernel(sj_kvarn_layout l, const uint8_t * rec, int t, int is_v, float * out) {
    for (int d = threadIdx.x; d < l.D; d += blockDim.x) out[d] = decode_value(l, rec, t, d, is_v);
}

SJK_DEV float staged_value(int staging, const uint8_t * row, int d) {
    if (staging == SJKVARN_STAGING_F16) return sjk_h2f(sjk_ld_u16(row + 2 * d));
    const uint8_t * b = row + (d >> 7) * SJKVARN_TQ6_BLOCK_BYTES;
    const int j = d & 127;
    const int code = ((b[2 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((b[66 + (j >> 2)] >> (2 * (j & 3))) & 3) << 4);
    return __fmul_rn(sjk_tq6_cent[code], sjk_h2f(sjk_ld_u16(b)));
}

__global__ void kv_row_kernel(sjk_view v, uint32_t B, uint32_t pos, int h, float * k, float * vo) {
    const sj_kvarn_layout & l = v.lay;
    const int D = l.D, H = v.n_head_kv;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        if (pos >= v.S && pos < B) {
            const uint32_t g = (pos - v.S) / (uint32_t) l.G, t = (pos - v.S) % (uint32_t) l.G;
            const uint32_t blk = v.blocks ? v.blocks[g] : g;
            const uint8_t * rec = v.body + ((size_t) blk * H + h) * l.bytes;
            k[d] = decode_value(l, rec, (int) t, d, 0);
            vo[d] = decode_value(l, rec, (int) t, d, 1);
        } else if (pos < v.S && v.sink_type == SJKVARN_SINK_F16) {
            const uint8_t * row = v.sink + ((size_t) pos * H + h) * 4 * D;
            k[d] = sjk_h2f(sjk_ld_u16(row + 2 * d));
            vo[d] = sjk_h2f(sjk_ld_u16(row + 2 * D + 2 * d));
        } else {
            const uint8_t * row = pos < v.S ? v.sink + ((size_t) pos * H + h) * 2 * v.stage_bytes
                                            : v.ring + ((size_t) sjk_ring_slot(v.S, v.cap, pos) * H + h) * 2 * v.stage_bytes;
            k[d] = staged_value(v.staging, row, d);
            vo[d] = staged_value(v.staging, row + v.stage_bytes, d);
        }
    }
}

}  // namespace

namespace {
// The reference's attention helpers on one record (sj_kvarn.h:1288-1311), with its arithmetic order: each score is
// the sequential fp32 sum over channels of q[d] * K[t, d] (one rounding per multiply and per add; one thread per
// token), and each output channel adds w[t] * V[t, d] in token order (one thread per channel).
__global__ void record_scores_kernel(sj_kvarn_layout l, const uint8_t * rec, const float * q, int n, float * scores) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n) return;
    float s = 0.0f;
    for (int d = 0; d < l.D; ++d) s = __fadd_rn(s, __fmul_rn(q[d], decode_value(l, rec, t, d, 0)));
    scores[t] = s;
}

__global__ void record_accum_v_kernel(sj_kvarn_layout l, const uint8_t * rec, const float * w, int n, float * acc) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    if (d >= l.D) return;
    float a = acc[d];
    for (int t = 0; t < n; ++t) a = __fadd_rn(a, __fmul_rn(w[t], decode_value(l, rec, t, d, 1)));
    acc[d] = a;
}
}  // namespace

int sjk_record_scores(const sj_kvarn_layout * lay, const uint8_t * rec, const float * q, int n, float * scores, sjk_stream st) {
    if (!lay || !rec || !q || !scores || n < 0 || n > lay->G) return SJKVARN_ERR_ARG;
    if (n == 0) return 0;
    record_scores_kernel<<<(n + 127) / 128, 128, 0, st>>>(*lay, rec, q, n, scores);
    return sjk_check_launch();
}

int sjk_record_accum_v(const sj_kvarn_layout * lay, const uint8_t * rec, const float * w, int n, float * acc, sjk_stream st) {
    if (!lay || !rec || !w || !acc || n < 0 || n > lay->G) return SJKVARN_ERR_ARG;
    if (n == 0) return 0;
    record_accum_v_kernel<<<(lay->D + 127) / 128, 128, 0, st>>>(*lay, rec, w, n, acc);
    return sjk_check_launch();
}

int sjk_decode_row(const sj_kvarn_layout * lay, const uint8_t * rec, int t, int is_v, float * out, sjk_stream st) {
    if (!lay || !rec || !out || t < 0 || t >= lay->G) return SJKVARN_ERR_ARG;
    decode_row_kernel<<<1, 256, 0, st>>>(*lay, rec, t, is_v, out);
    return sjk_check_launch();
}

int sjk_kv_row(const sjk_view * v, uint32_t B, uint32_t pos, int h, float * k, float * vo, sjk_stream st) {
    if (!v || !k || !vo || h < 0 || h >= v->n_head_kv) return SJKVARN_ERR_ARG;
    kv_row_kernel<<<1, 256, 0, st>>>(*v, B, pos, h, k, vo);
    return sjk_check_launch();
}

// ---- record groups moved through a block table (state save / restore, truncation) ----------------------------
// Group g (the n_head_kv records of one 128-token group of a layer) lives at body + blk(g) * group_bytes with
// blk(g) = blocks ? blocks[g] : g (sj_kvarn.h:1429-1432, 1706-1739). One CTA per group moves it in words of T
// (16, 4 or 1 bytes, the widest that divides group_bytes): op 0 gathers groups [g0, g0 + n) into buf (group order),
// op 1 scatters buf into them, op 2 zeroes them; groups whose block is SJKVARN_NO_BLOCK are skipped (op 0 writes
// zeros for them).
namespace {
template <typename T>
__global__ void __launch_bounds__(256) group_move_kernel(uint8_t * body, const uint32_t * blocks, uint32_t g0, size_t group_bytes,
                                                         uint8_t * buf, int op) {
    const uint32_t g = g0 + blockIdx.x;
    const uint32_t blk = blocks ? blocks[g] : g;
    const size_t nw = group_bytes / sizeof(T);
    T * b = reinterpret_cast<T *>(buf + (size_t) blockIdx.x * group_bytes);
    const T zero{};
    if (blk == SJKVARN_NO_BLOCK) {
        if (op == 0)
            for (size_t i = threadIdx.x; i < nw; i += blockDim.x) b[i] = zero;
        return;
    }
    T * d = reinterpret_cast<T *>(body + (size_t) blk * group_bytes);
    for (size_t i = threadIdx.x; i < nw; i += blockDim.x) {
        if (op == 0) b[i] = d[i];
        else if (op == 1) d[i] = b[i];
        else d[i] = zero;
    }
}
}  // namespace

int sjk_group_move(uint8_t * body, const uint32_t * blocks, uint32_t g0, uint32_t n, size_t group_bytes, uint8_t * buf, int op,
                   sjk_stream st) {
    if (n == 0) return 0;
    if (!body || (op != 2 && !buf) || op < 0 || op > 2) return SJKVARN_ERR_ARG;
    if (group_bytes % 16 == 0) group_move_kernel<uint4><<<n, 256, 0, st>>>(body, blocks, g0, group_bytes, buf, op);
    else if (group_bytes % 4 == 0) group_move_kernel<uint32_t><<<n, 256, 0, st>>>(body, blocks, g0, group_bytes, buf, op);
    else group_move_kernel<uint8_t><<<n, 256, 0, st>>>(body, blocks, g0, group_bytes, buf, op);
    return sjk_check_launch();
}
