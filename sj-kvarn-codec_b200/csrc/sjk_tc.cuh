// sjk_tc.cuh - thin inline-PTX wrappers for the sm_100a tensor-core path: TMEM allocation, tcgen05.mma
// (A from TMEM, B from shared memory), tcgen05.ld / st, commits, fences, mbarriers and 1-D bulk copies.
// Every wait is bounded: a wait that runs out records SJK_DEV_TIMEOUT in the device status word and
// returns false, so a kernel can skip its remaining work, release its TMEM and exit instead of hanging.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define SJK_DEV_TIMEOUT 1
#define SJK_WAIT_NS 1000000000ull          // 1 s of wall clock per wait

// device status word of the including translation unit (read and cleared by sjk_device_status())
static __device__ int sjk_dev_status;

// defines `int name(void)` returning and clearing this translation unit's device status word (-1: CUDA error)
#define SJK_STATUS_READER(name)                                                          \
    int name(void) {                                                                     \
        int v_ = 0, zero_ = 0;                                                           \
        if (cudaMemcpyFromSymbol(&v_, sjk_dev_status, sizeof v_) != cudaSuccess) return -1; \
        if (cudaMemcpyToSymbol(sjk_dev_status, &zero_, sizeof zero_) != cudaSuccess) return -1; \
        return v_;                                                                       \
    }

namespace tc {

__device__ __forceinline__ uint32_t smem_addr(const void * p) { return (uint32_t) __cvta_generic_to_shared(p); }

// ---- TMEM -----------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t * dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::); }
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// generic-proxy shared-memory writes -> visible to the async proxy (tcgen05.mma operand reads)
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 lanes x 32 bits, 8 / 16 consecutive columns per thread (the warp's lane quarter)
__device__ __forceinline__ void st_x8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void ld_x16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
                   "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void st_x16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
                 ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
                 "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
                 : "memory");
}
__device__ __forceinline__ void ld_x4_u(uint32_t taddr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void ld_x8_u(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void ld_x16_u(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
                   "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr)
                 : "memory");
}

// ---- MMA: D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16, one CTA ------------------------------------------------
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u));
}
// D[tmem] (+)= A[tmem] * B[smem]^T, kind::i8 (s8 x s8 -> s32), one CTA
__device__ __forceinline__ void mma_ts_i8(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u));
}
// arrive on the mbarrier once every MMA issued so far by this thread has completed
__device__ __forceinline__ void mma_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// instruction descriptor, kind::f16: fp16 A and B (both K-major), fp32 accumulate, shape M x N
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t) (N >> 3) << 17) | ((uint32_t) (M >> 4) << 24);
}

// instruction descriptor, kind::i8: signed 8-bit A and B (K-major), s32 accumulate, shape M x N
__host__ __device__ constexpr uint32_t idesc_s8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (N >> 3) << 17) | ((uint32_t) (M >> 4) << 24);
}

// shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core matrices; `lbo` bytes between
// the two 8-element K halves of an instruction, `sbo` bytes between consecutive 8-row groups
__device__ __forceinline__ uint64_t smem_desc(const void * base, uint32_t lbo, uint32_t sbo) {
    const uint32_t a = smem_addr(base);
    return (uint64_t) ((a >> 4) & 0x3FFFu) | ((uint64_t) ((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// ---- mbarriers and bulk copies ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    // suspend-time hint of 1 us per try: the wall-clock bound below stays tight
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// wait for the phase with the given parity to complete, for at most SJK_WAIT_NS of wall clock
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (globaltimer() - t0 < SJK_WAIT_NS)
        if (mbar_try_wait(bar, parity)) return true;
    atomicExch(&sjk_dev_status, SJK_DEV_TIMEOUT);
    return false;
}
// non-blocking test of a phase (acquire at CTA scope when it reports completion)
__device__ __forceinline__ bool mbar_test(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
                 : "=r"(ok)
                 : "r"(smem_addr(bar)), "r"(parity)
                 : "memory");
    return ok != 0;
}
// wait for two / three phases: all are tested back to back, and only those not complete yet take the bounded
// wait, so phases that completed earlier cost one round trip together instead of one each
__device__ __forceinline__ bool mbar_wait2(uint64_t * b0, uint32_t p0, uint64_t * b1, uint32_t p1) {
    const bool r0 = mbar_test(b0, p0), r1 = mbar_test(b1, p1);
    return (r0 || mbar_wait(b0, p0)) && (r1 || mbar_wait(b1, p1));
}
__device__ __forceinline__ bool mbar_wait3(uint64_t * b0, uint32_t p0, uint64_t * b1, uint32_t p1, uint64_t * b2, uint32_t p2) {
    const bool r0 = mbar_test(b0, p0), r1 = mbar_test(b1, p1), r2 = mbar_test(b2, p2);
    return (r0 || mbar_wait(b0, p0)) && (r1 || mbar_wait(b1, p1)) && (r2 || mbar_wait(b2, p2));
}
// plain arrival (count 1) on an mbarrier, release semantics at CTA scope
__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// named barrier over `n` threads (a multiple of 32; every warp arrives whole)
__device__ __forceinline__ void nbar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// named barrier that also returns the AND of `v` over the `n` participating threads
__device__ __forceinline__ bool nbar_and(int id, int n, bool v) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}\n"
                 : "=r"(r)
                 : "r"((uint32_t) v), "r"(id), "r"(n)
                 : "memory");
    return r != 0;
}
// 1-D bulk copy global -> own shared memory, completion counted in bytes on `bar` (no multicast)
__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// global -> L2 prefetch of `bytes` (a multiple of 16) at a 16-byte aligned address
__device__ __forceinline__ void prefetch_l2(const void * src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// the same for any byte range: widened to 16-byte boundaries
__device__ __forceinline__ void prefetch_l2_span(const void * src, uint32_t bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(src), a0 = a & ~(uintptr_t) 15, a1 = (a + bytes + 15) & ~(uintptr_t) 15;
    prefetch_l2(reinterpret_cast<const void *>(a0), (uint32_t) (a1 - a0));
}

// asynchronous global -> shared copies of 4 / 16 bytes; src_bytes = 0 writes zeros (src is not read)
__device__ __forceinline__ void cp_async4(void * dst, const void * src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async8(void * dst, const void * src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async16(void * dst, const void * src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// close the thread's group of asynchronous copies issued since the last commit (an empty group is fine)
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// wait until at most N of the thread's committed groups are still in flight
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ---- numeric helpers shared by the tensor-core kernels ------------------------------------------------
namespace num {
constexpr float MAGIC = 12582912.0f;    // 1.5 * 2^23: v + MAGIC holds round(v) in the low mantissa bits
constexpr uint32_t MAGIC_BITS = 0x4B400000u;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

__device__ __forceinline__ int pow2_exp(float x) { return (int) ((__float_as_uint(x) >> 23) & 0xFF) - 126; }  // x < 2^e
__device__ __forceinline__ float pow2f(int e) {
    e = e < -126 ? -126 : (e > 127 ? 127 : e);
    return __uint_as_float((uint32_t) (e + 127) << 23);
}
// fp16 -> fp32 (exact for every half)
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ float h2f_at(const uint8_t * p) { return h2f(*reinterpret_cast<const uint16_t *>(p)); }
// float -> nearest integer and back (|v| < 2^22) without the conversion pipe
__device__ __forceinline__ int f2i(float v) { return (int) (__float_as_uint(v + MAGIC) - MAGIC_BITS); }
__device__ __forceinline__ float i2f(uint32_t x) { return __uint_as_float(x + MAGIC_BITS) - MAGIC; }
__device__ __forceinline__ int sext8(int x) { return (x << 24) >> 24; }
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}
__device__ __forceinline__ float ex2(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
// Packed fp32 pairs (sm_100 f32x2 instructions): each lane computes both halves with the rounding of the
// scalar instruction, so results are identical to two scalar operations at half the issue slots.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
// lane-wise max of two pairs of unsigned 16-bit values
__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// Largest |x| over 256 consecutive fp16 values (16-byte aligned), for every lane of the warp: lane L reads
// values 8L .. 8L + 7. The magnitude bits of finite values and infinities order like unsigned integers; a NaN
// counts as infinity.
__device__ __forceinline__ float absmax256_h(const uint8_t * p, int lane) {
    const uint4 w = *reinterpret_cast<const uint4 *>(p + 16 * lane);
    uint32_t m = max_u16x2(max_u16x2(w.x & 0x7FFF7FFFu, w.y & 0x7FFF7FFFu), max_u16x2(w.z & 0x7FFF7FFFu, w.w & 0x7FFF7FFFu));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = max_u16x2(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    uint32_t h = (m & 0xFFFFu) > (m >> 16) ? (m & 0xFFFFu) : (m >> 16);
    h = h < 0x7C00u ? h : 0x7C00u;
    return __half2float(__ushort_as_half((unsigned short) h));
}

// 8 consecutive floats of shared memory (16-byte aligned) into / from registers
__device__ __forceinline__ void ld8(const float * p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4 *>(p)[0], b = reinterpret_cast<const float4 *>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void st8(float * p, const float (&v)[8]) {
    reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// Reduce 8 per-thread values across the 32 lanes; afterwards lanes 4r..4r+3 hold row r.
template <bool MAX>
__device__ __forceinline__ float warp_rows8(const float (&v)[8], int lane) {
    float a[4], b[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const bool up = lane & 16;
        const float send = up ? v[i] : v[i + 4], keep = up ? v[i + 4] : v[i];
        const float r = __shfl_xor_sync(0xFFFFFFFFu, send, 16);
        a[i] = MAX ? fmaxf(keep, r) : keep + r;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const bool up = lane & 8;
        const float send = up ? a[i] : a[i + 2], keep = up ? a[i + 2] : a[i];
        const float r = __shfl_xor_sync(0xFFFFFFFFu, send, 8);
        b[i] = MAX ? fmaxf(keep, r) : keep + r;
    }
    const bool up = lane & 4;
    const float send = up ? b[0] : b[1], keep = up ? b[1] : b[0];
    float r = __shfl_xor_sync(0xFFFFFFFFu, send, 4);
    float c = MAX ? fmaxf(keep, r) : keep + r;
    r = __shfl_xor_sync(0xFFFFFFFFu, c, 2);
    c = MAX ? fmaxf(c, r) : c + r;
    r = __shfl_xor_sync(0xFFFFFFFFu, c, 1);
    return MAX ? fmaxf(c, r) : c + r;
}

// Reduce 16 per-thread values (rows 0..15) across the 32 lanes; afterwards lanes 2r, 2r+1 hold row r.
template <bool MAX>
__device__ __forceinline__ float warp_rows16(const float (&v)[16], int lane) {
    float a[8], b[4], c[2];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const bool up = lane & 16;
        const float send = up ? v[i] : v[i + 8], keep = up ? v[i + 8] : v[i];
        const float r = __shfl_xor_sync(0xFFFFFFFFu, send, 16);
        a[i] = MAX ? fmaxf(keep, r) : keep + r;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const bool up = lane & 8;
        const float send = up ? a[i] : a[i + 4], keep = up ? a[i + 4] : a[i];
        const float r = __shfl_xor_sync(0xFFFFFFFFu, send, 8);
        b[i] = MAX ? fmaxf(keep, r) : keep + r;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const bool up = lane & 4;
        const float send = up ? b[i] : b[i + 2], keep = up ? b[i + 2] : b[i];
        const float r = __shfl_xor_sync(0xFFFFFFFFu, send, 4);
        c[i] = MAX ? fmaxf(keep, r) : keep + r;
    }
    const bool up = lane & 2;
    const float send = up ? c[0] : c[1], keep = up ? c[1] : c[0];
    float r = __shfl_xor_sync(0xFFFFFFFFu, send, 2);
    const float d = MAX ? fmaxf(keep, r) : keep + r;
    r = __shfl_xor_sync(0xFFFFFFFFu, d, 1);
    return MAX ? fmaxf(d, r) : d + r;
}

// Reduce 4 per-thread values (rows 0..3) across the 32 lanes; afterwards lanes 8r..8r+7 hold row r.
template <bool MAX>
__device__ __forceinline__ float warp_rows4(const float (&v)[4], int lane) {
    const bool u16 = lane & 16, u8 = lane & 8;
    float r0 = __shfl_xor_sync(0xFFFFFFFFu, u16 ? v[0] : v[2], 16), r1 = __shfl_xor_sync(0xFFFFFFFFu, u16 ? v[1] : v[3], 16);
    const float a0 = MAX ? fmaxf(u16 ? v[2] : v[0], r0) : (u16 ? v[2] : v[0]) + r0;
    const float a1 = MAX ? fmaxf(u16 ? v[3] : v[1], r1) : (u16 ? v[3] : v[1]) + r1;
    const float r = __shfl_xor_sync(0xFFFFFFFFu, u8 ? a0 : a1, 8);
    float c = MAX ? fmaxf(u8 ? a1 : a0, r) : (u8 ? a1 : a0) + r;
#pragma unroll
    for (int o = 4; o; o >>= 1) {
        const float x = __shfl_xor_sync(0xFFFFFFFFu, c, o);
        c = MAX ? fmaxf(c, x) : c + x;
    }
    return c;
}

// Sum 4 per-thread values (rows 0..3) across the 32 lanes; afterwards lanes 8r..8r+7 hold row r.
__device__ __forceinline__ float warp_sum_rows4(float v0, float v1, float v2, float v3, int lane) {
    const bool u16 = lane & 16, u8 = lane & 8;
    const float a0 = (u16 ? v2 : v0) + __shfl_xor_sync(0xFFFFFFFFu, u16 ? v0 : v2, 16);
    const float a1 = (u16 ? v3 : v1) + __shfl_xor_sync(0xFFFFFFFFu, u16 ? v1 : v3, 16);
    float c = (u8 ? a1 : a0) + __shfl_xor_sync(0xFFFFFFFFu, u8 ? a0 : a1, 8);
    c += __shfl_xor_sync(0xFFFFFFFFu, c, 4);
    c += __shfl_xor_sync(0xFFFFFFFFu, c, 2);
    return c + __shfl_xor_sync(0xFFFFFFFFu, c, 1);
}

// Balanced base-256 digits of round(v * sc), |v * sc| < 2^22: byte i (i = 0, 1, 2) of the result is the signed
// digit d_i in [-128, 127] with round(v * sc) = d0 + 256 d1 + 65536 d2. fmaf(v, sc, MAGIC) holds the rounded
// integer x in its low mantissa bits (bits = MAGIC_BITS + x); adding 128 to every digit position maps the digits
// to the bytes of x + 0x808080 (each in [0, 255]), and flipping bit 7 of each byte maps them back to signed.
__device__ __forceinline__ uint32_t digits3(float v, float sc) {
    return (__float_as_uint(fmaf(v, sc, MAGIC)) + (0x00808080u - MAGIC_BITS)) ^ 0x00808080u;
}
// digits3 of two values (packed fp32 arithmetic, same results)
__device__ __forceinline__ uint2 digits3x2(float2 v, float2 sc) {
    const float2 f = fma2(v, sc, make_float2(MAGIC, MAGIC));
    return make_uint2((__float_as_uint(f.x) + (0x00808080u - MAGIC_BITS)) ^ 0x00808080u,
                      (__float_as_uint(f.y) + (0x00808080u - MAGIC_BITS)) ^ 0x00808080u);
}

// The 6-bit codes of elements j0 .. j0 + 7 (j0 % 8 == 0) of a tq6_0 block (norm, qs[64] nibbles, qh[32] 2-bit
// fields, sj_kvarn.h:1249-1284) as 8 bytes: nibble pairs spread with one PRMT, the high bits from a 256-entry
// table qh_lut[y] = (2-bit fields of y) << 4 in bytes 0..3.
__device__ __forceinline__ uint2 tq6_codes8(const uint8_t * blk, int j0, const uint32_t * qh_lut) {
    const uint32_t qs = (uint32_t) *reinterpret_cast<const uint16_t *>(blk + 2 + j0 / 2) |
                        ((uint32_t) *reinterpret_cast<const uint16_t *>(blk + 4 + j0 / 2) << 16);
    const uint32_t qh = *reinterpret_cast<const uint16_t *>(blk + 66 + j0 / 4);
    const uint32_t a = qs & 0x0F0F0F0Fu, b = (qs >> 4) & 0x0F0F0F0Fu;          // nibbles 0 2 4 6 / 1 3 5 7
    return make_uint2(prmt(a, b, 0x5140u) | qh_lut[qh & 0xFFu], prmt(a, b, 0x7362u) | qh_lut[qh >> 8]);
}

}  // namespace num

}  // namespace tc
