// sjk_common.cuh - shared device helpers of the B200 SJ-KVaRN kernels: exact fp16
// conversion, record-layout arithmetic, format tables and the status plumbing.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sjk.h"
#include "sjk_tables.h"

#define SJK_DEV __device__ __forceinline__
#define SJK_HD __host__ __device__ __forceinline__

// ---- status plumbing (host) ----------------------------------------------------------------------------
// set_cuda_error records the CUDA error of a failed call; the entry points turn it into SJK_ERR_DEVICE.
void sjk_set_cuda_error(cudaError_t e);
void sjk_set_sticky(int status);
static inline int sjk_check(cudaError_t e) {
    if (e != cudaSuccess) { sjk_set_cuda_error(e); return SJK_ERR_DEVICE; }
    return 0;
}
static inline int sjk_check_launch(void) { return sjk_check(cudaGetLastError()); }

// ---- format tables in device memory (a private copy per translation unit; a few KB) ----------------------
static __device__ const uint16_t sjk_cb3_k[512] = SJK_CB3_K_INIT;
static __device__ const uint16_t sjk_cb3_v[512] = SJK_CB3_V_INIT;
static __device__ const uint16_t sjk_cb2_k[256] = SJK_CB2_K_INIT;
static __device__ const uint16_t sjk_cb2_v[256] = SJK_CB2_V_INIT;
static __device__ const float sjk_tq6_cent[64] = SJK_TQ6_CENT_INIT;
static __device__ const float sjk_tq6_mid[63] = SJK_TQ6_MID_INIT;

SJK_DEV const uint16_t * sjk_codebook(int bits, int is_v) {
    return bits == 3 ? (is_v ? sjk_cb3_v : sjk_cb3_k) : (is_v ? sjk_cb2_v : sjk_cb2_k);
}

// ---- fp16 ------------------------------------------------------------------------------------------------
// Round-to-nearest-even float -> half in integer arithmetic, NaN -> 0x7E00 with the sign kept (the
// reference's converter, sj_kvarn.h:693-711, produces exactly these bits). Integer code keeps the result
// independent of the conversion instruction's NaN handling.
SJK_HD uint16_t sjk_f2h(float f) {
    uint32_t w;
#ifdef __CUDA_ARCH__
    w = __float_as_uint(f);
#else
    __builtin_memcpy(&w, &f, 4);
#endif
    const uint32_t sign = (w >> 16) & 0x8000u, a = w & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (uint16_t) (sign | 0x7E00u);
    if (a >= 0x477FF000u) return (uint16_t) (sign | 0x7C00u);
    if (a < 0x38800000u) {
        if (a < 0x33000000u) return (uint16_t) sign;
        const int sh = 126 - (int) (a >> 23);
        const uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
        uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t) (sign | q);
    }
    uint32_t q = (a - 0x38000000u) >> 13;
    const uint32_t rem = a & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t) (sign | q);
}

// Exact half -> float for every encoding, NaN payloads included (sj_kvarn.h:713-731).
SJK_HD float sjk_h2f(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 31u;
    uint32_t m = h & 0x3FFu, w;
    if (e == 31u) w = sign | 0x7F800000u | (m << 13);
    else if (e) w = sign | ((e + 112u) << 23) | (m << 13);
    else if (!m) w = sign;
    else {
#ifdef __CUDA_ARCH__
        const int lz = __clz(m) - 21;              // shifts that bring bit 10 to the top of the mantissa
#else
        const int lz = __builtin_clz(m) - 21;
#endif
        m <<= lz;
        w = sign | ((uint32_t) (113 - lz) << 23) | ((m & 0x3FFu) << 13);
    }
#ifdef __CUDA_ARCH__
    return __uint_as_float(w);
#else
    float f; __builtin_memcpy(&f, &w, 4); return f;
#endif
}

// ---- record layout (sj_kvarn.h:800-849) ----------------------------------------------------------------------
SJK_HD int sjk_frag(const sj_kvarn_layout & l, int bits) {
    return l.body == SJKVARN_BODY_SCALAR && bits == 4 && (l.D & 15) == 0 && (l.G & 15) == 0;
}

// bit offset of code (token t, channel d) in the K (is_v = 0) or V payload
SJK_HD uint32_t sjk_code_bit(const sj_kvarn_layout & l, int t, int d, int is_v) {
    const int bits = is_v ? l.bits_v : l.bits_k;
    if (l.body == SJKVARN_BODY_TRELLIS) return ((uint32_t) d * (uint32_t) l.G + (uint32_t) t) * (uint32_t) bits;
    if (!sjk_frag(l, bits)) return ((uint32_t) t * (uint32_t) l.D + (uint32_t) d) * (uint32_t) bits;
    const int row = is_v ? (d & 15) : (t & 15);   // MMA operand row inside the 16x16 tile
    const int col = is_v ? (t & 15) : (d & 15);   // its k index
    const uint32_t tile = (uint32_t) ((t >> 4) * (l.D >> 4) + (d >> 4));
    const uint32_t lane = (uint32_t) (4 * (row & 7) + ((col >> 1) & 3));
    const uint32_t nib = (uint32_t) ((row >> 3) + 2 * (col >> 3) + 4 * (col & 1));
    return (tile * 32u + lane) * 32u + nib * 4u;
}

// Inverse of the fragment order: nibble `nib` (0..7) of payload word w -> (t, d).
SJK_HD void sjk_frag_pos(const sj_kvarn_layout & l, uint32_t w, int nib, int is_v, int * t, int * d) {
    const int tile = (int) (w >> 5), lane = (int) (w & 31u);
    const int tiles_d = l.D >> 4;
    const int s = tile / tiles_d, c = tile % tiles_d;
    const int rr = nib & 3, e = nib >> 2;
    const int row = (lane >> 2) + 8 * (rr & 1);
    const int col = 2 * (lane & 3) + 8 * (rr >> 1) + e;
    if (!is_v) { *t = 16 * s + row; *d = 16 * c + col; }
    else       { *d = 16 * c + row; *t = 16 * s + col; }
}

SJK_HD int sjk_k_ch(const sj_kvarn_layout & l, int d) {
    if (!sjk_frag(l, l.bits_k)) return d;
    const int dd = d & 15, pair = dd >> 1;
    return (pair & 3) * (l.D >> 2) + (d >> 4) * 4 + (pair >> 2) * 2 + (dd & 1);
}

SJK_HD int sjk_v_ch(const sj_kvarn_layout & l, int d) {
    if (!sjk_frag(l, l.bits_v)) return d;
    const int dd = d & 15;
    return (dd & 7) * (l.D >> 3) + (d >> 4) * 2 + (dd >> 3);
}

SJK_DEV uint32_t sjk_get_bits(const uint8_t * p, uint32_t bit, int bits) {
    uint32_t w = p[bit >> 3];
    if ((bit & 7u) + (uint32_t) bits > 8u) w |= (uint32_t) p[(bit >> 3) + 1] << 8;
    return (w >> (bit & 7u)) & ((1u << bits) - 1u);
}

// trellis window of code i of channel seq: current code above the previous 6 stream bits (sj_kvarn.h:879-900)
SJK_DEV uint32_t sjk_window(const uint8_t * payload, int bits, int seq, int i, int seq_len) {
    const int hist = (6 + bits - 1) / bits;
    const uint32_t base = (uint32_t) seq * (uint32_t) seq_len * (uint32_t) bits;
    uint32_t w = 0;
    for (int k = 0; k <= hist && k <= i; ++k)
        w |= sjk_get_bits(payload, base + (uint32_t) (i - k) * (uint32_t) bits, bits) << (6 - k * bits);
    return w & ((1u << (6 + bits)) - 1u);
}

SJK_HD uint32_t sjk_ring_slot(uint32_t S, uint32_t cap, uint32_t pos) { return (pos - S) % cap; }

SJK_DEV uint16_t sjk_ld_u16(const uint8_t * p) { return (uint16_t) (p[0] | (p[1] << 8)); }
