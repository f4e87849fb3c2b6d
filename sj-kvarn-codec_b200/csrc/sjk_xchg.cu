// sjk_xchg.cu - exchange buffers of attention partials between the GPUs that hold context slices of one sequence
// (allocation, CUDA IPC mapping) and the stand-alone exchange of given triples. The kernels' exchange protocol and the
// buffer layout are in sjk_merge.cuh, shared with the merge kernel of sjk_attend_partial_xchg.
#include <cuda_runtime.h>
#include <string.h>

#include "sjk_common.cuh"
#include "sjk_internal.h"
#include "sjk_merge.cuh"

namespace {

__device__ int xchg_status;                  // SJK_DEVICE_TIMEOUT when an exchange gave up waiting

// grid (rows, 64-channel tiles): publish the tile of the given triples, wait for every rank's, merge in rank order
__global__ void __launch_bounds__(256) xchg_exchange_kernel(const float * __restrict__ part, int n_rows, int D, float * out,
                                                            const __grid_constant__ sjkm::XchgArgs x) {
    extern __shared__ float wts[];
    __shared__ float s_red[16];
    __shared__ __align__(16) float stage[SJK_XCHG_MAX_WORLD * sjkm::XCHG_TILE_WORDS];
    const int row = blockIdx.x, tile = blockIdx.y, d0 = 64 * tile, tid = threadIdx.x;
    // launched as a programmatic dependent of the kernel that writes part (sjk_attend_partial_xchg's merge): wait for
    // it; the next call's body kernel, launched as this one's dependent, may be set up meanwhile
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const float * pr = part + (size_t) row * (D + 2);
    const float my_o = (tid < 64 && d0 + tid < D) ? pr[2 + d0 + tid] : 0.0f;
    if (!sjkm::xchg_publish_gather(x, n_rows, D, row, tile, pr[0], pr[1], my_o, stage)) {
        if (tid < 64 && d0 + tid < D) out[(size_t) row * D + d0 + tid] = 0.0f;
        if (tid == 0) atomicOr(&xchg_status, (int) SJK_DEVICE_TIMEOUT);
        return;
    }
    float m, t;
    sjkm::merge_tile(stage, x.world, 1, sjkm::XCHG_TILE_WORDS - 2, 0, 0, wts, s_red, m, t);
    sjkm::store_out(wts + x.world, t, D, row, d0, out);
}

bool valid(const sjk_xchg_peers * x) {
    if (!x || x->world <= 0 || x->world > SJK_XCHG_MAX_WORLD || x->rank < 0 || x->rank >= x->world) return false;
    for (int i = 0; i < x->world; ++i)
        if (!x->buf[i] || ((uintptr_t) x->buf[i] & 255)) return false;
    return true;
}

}  // namespace

extern "C" size_t sjk_xchg_bytes(int world, int n_rows, int D) {
    if (world <= 0 || world > SJK_XCHG_MAX_WORLD || n_rows <= 0 || D <= 0 || (D & 1)) return 0;
    return sjkm::xchg_words_bytes(world, n_rows, D);
}

extern "C" int sjk_xchg_alloc(size_t bytes, void ** buf, void * ipc_handle) {
    if (!buf || bytes == 0) return SJKVARN_ERR_ARG;
    *buf = nullptr;
    void * p = nullptr;
    if (sjk_check(cudaMalloc(&p, bytes))) return SJK_ERR_DEVICE;
    if (sjk_check(cudaMemset(p, 0, bytes))) { cudaFree(p); return SJK_ERR_DEVICE; }
    if (ipc_handle) {
        cudaIpcMemHandle_t h;
        if (sjk_check(cudaIpcGetMemHandle(&h, p))) { cudaFree(p); return SJK_ERR_DEVICE; }
        static_assert(sizeof(cudaIpcMemHandle_t) == SJK_XCHG_HANDLE_BYTES, "IPC handle size");
        memcpy(ipc_handle, &h, sizeof h);
    }
    if (sjk_check(cudaDeviceSynchronize())) { cudaFree(p); return SJK_ERR_DEVICE; }
    *buf = p;
    return 0;
}

extern "C" int sjk_xchg_free(void * buf) {
    if (!buf) return 0;
    return sjk_check(cudaFree(buf));
}

extern "C" int sjk_xchg_open(const void * ipc_handle, void ** peer_buf) {
    if (!ipc_handle || !peer_buf) return SJKVARN_ERR_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof h);
    *peer_buf = nullptr;
    return sjk_check(cudaIpcOpenMemHandle(peer_buf, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int sjk_xchg_close(void * peer_buf) {
    if (!peer_buf) return 0;
    return sjk_check(cudaIpcCloseMemHandle(peer_buf));
}

extern "C" int sjk_xchg_exchange(const sjk_xchg_peers * x, const float * part, int n_rows, int D, uint32_t epoch, float * out,
                                 sjk_stream st) {
    if (!valid(x) || !part || !out || n_rows <= 0 || D <= 0 || (D & 1) || epoch == 0) return SJKVARN_ERR_ARG;
    sjkm::XchgArgs xa = {};
    xa.world = x->world; xa.rank = x->rank; xa.epoch = epoch;
    for (int i = 0; i < x->world; ++i) xa.buf[i] = reinterpret_cast<uint8_t *>(x->buf[i]);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) n_rows, (unsigned) sjkm::merge_tiles(D));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = (size_t) (x->world + 256) * sizeof(float);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (sjk_check(cudaLaunchKernelEx(&cfg, xchg_exchange_kernel, part, n_rows, D, out, xa))) return SJK_ERR_DEVICE;
    return sjk_check_launch();
}

int sjk_xchg_status_take(void) {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, xchg_status, sizeof v) != cudaSuccess) return -1;
    if (cudaMemcpyToSymbol(xchg_status, &zero, sizeof zero) != cudaSuccess) return -1;
    return v;
}
