// sjk_synth.cu - the seeded synthetic K/V/Q generator of the benchmark configurations on the device (the same
// arithmetic as the host side, sjk_synth.h, so both produce identical bits). Input generation for the benchmark and
// the configuration parity tests; no counterpart in the reference, which ships no generator for these shapes.
#include <cuda_runtime.h>

#include "sjk_internal.h"
#include "sjk_synth.h"

namespace {

__global__ void synth_scales_kernel(uint64_t seed, int layer0, int n_layers, int H, int D, float * scale) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;          // (layer, head)
    if (i >= n_layers * H) return;
    const int il = i / H, h = i % H;
    sjk_syn_scales_head(seed, (uint32_t) (layer0 + il), h, D, scale + (size_t) i * D);
}

// one thread per element pair; k, v: [n][H][D] of positions pos0 ..; scale: [H][D]
__global__ void __launch_bounds__(256) synth_kv_kernel(uint64_t kk, uint64_t vk, uint64_t ck, int heavy, const float * scale,
                                                       uint64_t j0, uint64_t n_pairs, uint32_t hd, float * k, float * v) {
    for (uint64_t p = (uint64_t) blockIdx.x * blockDim.x + threadIdx.x; p < n_pairs; p += (uint64_t) gridDim.x * blockDim.x) {
        const uint64_t e = j0 + 2 * p;
        const uint32_t c = (uint32_t) (e % hd);
        float k0, k1, v0, v1;
        sjk_syn_kv_pair(kk, vk, ck, heavy, e >> 1, __ldg(scale + c), __ldg(scale + c + 1), &k0, &k1, &v0, &v1);
        reinterpret_cast<float2 *>(k)[p] = make_float2(k0, k1);
        reinterpret_cast<float2 *>(v)[p] = make_float2(v0, v1);
    }
}

__global__ void synth_q_kernel(uint64_t key, uint64_t n_pairs, float * q) {
    for (uint64_t p = (uint64_t) blockIdx.x * blockDim.x + threadIdx.x; p < n_pairs; p += (uint64_t) gridDim.x * blockDim.x) {
        float a, b;
        sjk_syn_q_pair(key, p, &a, &b);
        reinterpret_cast<float2 *>(q)[p] = make_float2(a, b);
    }
}

int launch_status() {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        sjk_set_cuda_error(e);
        return SJK_ERR_DEVICE;
    }
    return 0;
}

}  // namespace

extern "C" int sjk_synth_scales(uint64_t seed, int layer0, int n_layers, int H, int D, float * scale, sjk_stream st) {
    if (n_layers <= 0 || H <= 0 || D <= 0 || D > 1024 || (D & 1) || !scale || layer0 < 0) return SJKVARN_ERR_ARG;
    const int n = n_layers * H;
    synth_scales_kernel<<<(n + 63) / 64, 64, 0, st>>>(seed, layer0, n_layers, H, D, scale);
    return launch_status();
}

extern "C" int sjk_synth_kv(uint64_t seed, int layer, int H, int D, int heavy, const float * scale, uint32_t pos0,
                            uint32_t n, float * k, float * v, sjk_stream st) {
    if (H <= 0 || D <= 0 || ((H * D) & 1) || !scale || !k || !v || layer < 0) return SJKVARN_ERR_ARG;
    if (((uintptr_t) k | (uintptr_t) v) & 7) return SJKVARN_ERR_ARG;
    if (n == 0) return 0;
    const uint64_t hd = (uint64_t) H * (uint64_t) D;
    const uint64_t n_pairs = (uint64_t) n * hd / 2;
    const uint64_t blocks = (n_pairs + 255) / 256;
    const unsigned grid = (unsigned) (blocks < 148ull * 64 ? blocks : 148ull * 64);
    synth_kv_kernel<<<grid, 256, 0, st>>>(sjk_syn_key(seed, (uint32_t) layer, SJK_SYN_K),
                                          sjk_syn_key(seed, (uint32_t) layer, SJK_SYN_V),
                                          sjk_syn_key(seed, (uint32_t) layer, SJK_SYN_CHI), heavy ? 1 : 0, scale,
                                          (uint64_t) pos0 * hd, n_pairs, (uint32_t) hd, k, v);
    return launch_status();
}

extern "C" int sjk_synth_q(uint64_t seed, int layer, uint32_t n_rows, int D, float * q, sjk_stream st) {
    if (D <= 0 || (D & 1) || !q || layer < 0 || ((uintptr_t) q & 7)) return SJKVARN_ERR_ARG;
    if (n_rows == 0) return 0;
    const uint64_t n_pairs = (uint64_t) n_rows * (uint64_t) D / 2;
    const uint64_t blocks = (n_pairs + 255) / 256;
    synth_q_kernel<<<(unsigned) (blocks < 4096 ? blocks : 4096), 256, 0, st>>>(sjk_syn_key(seed, (uint32_t) layer, SJK_SYN_Q),
                                                                               n_pairs, q);
    return launch_status();
}
