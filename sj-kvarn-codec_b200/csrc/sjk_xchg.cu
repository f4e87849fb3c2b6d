// sjk_xchg.cu - exchange of attention partials between the GPUs that hold context slices of one sequence, over
// peer memory (NVLink P2P stores; no collective library, no TMA, no multicast).
//
// Every rank owns one exchange buffer (cudaMalloc'd here, shared with the other ranks through CUDA IPC handles):
//
//   flags  uint32 [2 parities][SJK_XCHG_MAX_WORLD sources][XCH_CHUNKS]     (512 bytes)
//   slots  float  [2 parities][world sources][n_rows][D + 2]
//
// Layer call `epoch` uses parity epoch & 1. sjk_xchg_publish (on rank r) writes r's partial triples (m, l, o[D]) into
// slot r of every rank's buffer with plain stores, then raises flag [parity][r][chunk] = epoch in each, one flag per
// publishing CTA, after a system-scope fence. sjk_xchg_merge (on every rank) waits, bounded, until every flag of the
// parity holds the epoch in its OWN buffer, then merges the world slots in rank order with the same kernel as
// sjk_attend_merge, so its output equals an all-gather + sjk_attend_merge of the same partials bit for bit.
//
// Two parities suffice: a rank publishes call e + 2 (parity e & 1 again) only after its merge of call e + 1 saw
// every peer's flag for e + 1, which every peer raised after its own merge of call e had completed (stream order).
// A wait that runs out (a peer that never publishes) leaves the output zero and records SJK_DEVICE_TIMEOUT.
#include <cuda_runtime.h>
#include <string.h>

#include "sjk_common.cuh"
#include "sjk_internal.h"

#define SJK_XCHG_WAIT_NS 1000000000ull      // 1 s of wall clock

namespace {

constexpr int XCH_CHUNKS = 4;                // publishing CTAs per destination
constexpr size_t XCH_FLAG_BYTES = 2 * SJK_XCHG_MAX_WORLD * XCH_CHUNKS * sizeof(uint32_t);

__device__ int xchg_status;                  // SJK_DEVICE_TIMEOUT when a merge gave up waiting

size_t slot_floats(int n_rows, int D) { return (size_t) n_rows * (size_t) (D + 2); }

struct Peers { float * base[SJK_XCHG_MAX_WORLD]; };

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// grid (world destinations, XCH_CHUNKS): CTA (dst, c) copies chunk c of the partials into slot `rank` of dst's
// buffer, then raises flag [parity][rank][c] there
__global__ void __launch_bounds__(512) xchg_publish_kernel(Peers peers, int rank, const float4 * __restrict__ part,
                                                           size_t n4, size_t slot_f, uint32_t epoch) {
    const int dst = blockIdx.x, c = blockIdx.y;
    const uint32_t par = epoch & 1u;
    uint8_t * base = reinterpret_cast<uint8_t *>(peers.base[dst]);
    float4 * slot = reinterpret_cast<float4 *>(base + XCH_FLAG_BYTES) + ((size_t) par * gridDim.x + (size_t) rank) * (slot_f / 4);
    const size_t per = (n4 + XCH_CHUNKS - 1) / XCH_CHUNKS, i0 = (size_t) c * per, i1 = min(n4, i0 + per);
    for (size_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) slot[i] = __ldg(part + i);
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t * flag = reinterpret_cast<uint32_t *>(base) + ((size_t) par * SJK_XCHG_MAX_WORLD + (size_t) rank) * XCH_CHUNKS + c;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(epoch) : "memory");
    }
}

// one CTA: wait until all world x XCH_CHUNKS flags of the parity hold `epoch` (bounded); on time-out zero the slots of
// the parity so that the merge writes zeros, and record the time-out
__global__ void xchg_wait_kernel(uint8_t * buf, int world, size_t slot_f, uint32_t epoch) {
    const uint32_t par = epoch & 1u;
    const int n = world * XCH_CHUNKS;
    bool ok = true;
    if ((int) threadIdx.x < n) {
        const int src = threadIdx.x / XCH_CHUNKS, c = threadIdx.x % XCH_CHUNKS;
        const uint32_t * flag = reinterpret_cast<const uint32_t *>(buf) + ((size_t) par * SJK_XCHG_MAX_WORLD + src) * XCH_CHUNKS + c;
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if (v != epoch) {
            const uint64_t t0 = gtimer();
            do {
                __nanosleep(200);
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
            } while (v != epoch && gtimer() - t0 < SJK_XCHG_WAIT_NS);
        }
        ok = v == epoch;
    }
    ok = __syncthreads_and(ok);
    if (!ok) {
        float * slots = reinterpret_cast<float *>(buf + XCH_FLAG_BYTES) + (size_t) par * world * slot_f;
        for (size_t i = threadIdx.x; i < (size_t) world * slot_f; i += blockDim.x) slots[i] = 0.0f;
        if (threadIdx.x == 0) atomicOr(&xchg_status, (int) SJK_DEVICE_TIMEOUT);
    }
    __threadfence();
}

}  // namespace

extern "C" size_t sjk_xchg_bytes(int world, int n_rows, int D) {
    if (world <= 0 || world > SJK_XCHG_MAX_WORLD || n_rows <= 0 || D <= 0 || (D & 1)) return 0;
    return XCH_FLAG_BYTES + 2 * (size_t) world * slot_floats(n_rows, D) * sizeof(float);
}

extern "C" int sjk_xchg_alloc(size_t bytes, void ** buf, void * ipc_handle) {
    if (!buf || bytes < XCH_FLAG_BYTES) return SJKVARN_ERR_ARG;
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

extern "C" int sjk_xchg_publish(void * const * peers, int world, int rank, const float * part, int n_rows, int D,
                                uint32_t epoch, sjk_stream st) {
    if (!peers || !part || world <= 0 || world > SJK_XCHG_MAX_WORLD || rank < 0 || rank >= world || n_rows <= 0 ||
        D <= 0 || (D & 1) || epoch == 0)
        return SJKVARN_ERR_ARG;
    const size_t slot_f = slot_floats(n_rows, D);
    if ((slot_f & 3) || ((uintptr_t) part & 15)) return SJKVARN_ERR_ARG;
    Peers pp = {};
    for (int i = 0; i < world; ++i) {
        if (!peers[i] || ((uintptr_t) peers[i] & 255)) return SJKVARN_ERR_ARG;
        pp.base[i] = reinterpret_cast<float *>(peers[i]);
    }
    xchg_publish_kernel<<<dim3((unsigned) world, XCH_CHUNKS), 512, 0, st>>>(pp, rank, reinterpret_cast<const float4 *>(part),
                                                                           slot_f / 4, slot_f, epoch);
    return sjk_check_launch();
}

extern "C" int sjk_xchg_merge(void * local_buf, int world, int n_rows, int D, uint32_t epoch, float * out, sjk_stream st) {
    if (!local_buf || !out || world <= 0 || world > SJK_XCHG_MAX_WORLD || n_rows <= 0 || D <= 0 || (D & 1) || epoch == 0)
        return SJKVARN_ERR_ARG;
    const size_t slot_f = slot_floats(n_rows, D);
    uint8_t * buf = reinterpret_cast<uint8_t *>(local_buf);
    xchg_wait_kernel<<<1, 128, 0, st>>>(buf, world, slot_f, epoch);
    if (sjk_check_launch()) return SJK_ERR_DEVICE;
    const float * slots = reinterpret_cast<const float *>(buf + XCH_FLAG_BYTES) + (size_t) (epoch & 1u) * world * slot_f;
    return sjk_attend_merge(slots, world, n_rows, D, out, st);
}

int sjk_xchg_status_take(void) {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, xchg_status, sizeof v) != cudaSuccess) return -1;
    if (cudaMemcpyToSymbol(xchg_status, &zero, sizeof zero) != cudaSuccess) return -1;
    return v;
}
