// sjk_fwht.cuh - the normalised fast Walsh-Hadamard transform of one row, in the reference's stage order
// (sj_kvarn.h:735-759): shared by the cache write (sjk_stage.cu), sjk_hadamard, and the attention calls that take
// queries and return outputs in the model basis (sjk_attend_model). The transform with scale 1/sqrt(n) is its own
// inverse up to rounding.
#pragma once
#include <cuda_runtime.h>
#include <math.h>

// One row of 32 VPL values in a warp: lane L holds elements L VPL .. L VPL + VPL - 1.
template <int VPL>
__device__ __forceinline__ void fwht_warp(float (&x)[VPL], int lane, float scale) {
    // stages inside a lane: partners j, j+h with h < VPL
#pragma unroll
    for (int h = 1; h < VPL; h <<= 1) {
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            if ((j & h) == 0) {
                const float a = x[j], b = x[j + h];
                x[j] = __fadd_rn(a, b);
                x[j + h] = __fsub_rn(a, b);
            }
        }
    }
    // stages across lanes: partner lane ^ m holds index +- h (h = m*VPL)
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int j = 0; j < VPL; ++j) {
            const float o = __shfl_xor_sync(0xFFFFFFFFu, x[j], m);
            x[j] = upper ? __fsub_rn(o, x[j]) : __fadd_rn(x[j], o);
        }
    }
#pragma unroll
    for (int j = 0; j < VPL; ++j) x[j] = __fmul_rn(x[j], scale);
}

// 1/sqrt(n) rounded as the reference computes it: FDIV(1, sqrtf(n)) (sj_kvarn.h:747)
static inline float sjk_fwht_scale(int n) {
    volatile float s = sqrtf((float) n);
    volatile float r = 1.0f / s;
    return r;
}
