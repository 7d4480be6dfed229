// voxq_common.cuh -- shared device helpers for the voxq sm_100a library.
//
// Everything here is hand-written for sm_100a: bulk-copy / mbarrier / tcgen05
// inline PTX, packed f32x2 arithmetic, and the binary16 conversions the
// quantizer needs.  No CUDA math-library internals are restated here.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "voxq.h"

#define VOXQ_QBLK 32

// ---------------------------------------------------------------------------
// Host-side error plumbing: every CUDA failure maps to VOXCPM_ERR_INTERNAL with
// a stderr line, as the reference's CUDA_CHECK does (src/tensor_cuda.cu:20-27).
// ---------------------------------------------------------------------------
#define VOXQ_CUDA_TRY(call)                                                            \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess) {                                                       \
            fprintf(stderr, "[voxq] %s:%d: %s (%d)\n", __FILE__, __LINE__,              \
                    cudaGetErrorString(e_), (int)e_);                                  \
            return VOXCPM_ERR_INTERNAL;                                                \
        }                                                                              \
    } while (0)

namespace voxq {

// Row payload bytes of the device layout.
__host__ __device__ inline int64_t codes_row_bytes(int K, int qtype) {
    return qtype == VOXQ_Q4 ? (int64_t)K / 2 : (int64_t)K;
}
__host__ __device__ inline int scale_bytes(int qtype) { return qtype == VOXQ_Q4 ? 4 : 8; }
__host__ __device__ inline int block_bytes(int qtype) { return qtype == VOXQ_Q4 ? 20 : 40; }
// The scales buffer of a packed weight holds, in order:
//   trailers  [N][K/32] (scale, min)
//   rowmul    [N] float at the next 16-byte boundary: 2^e with
//             max_k |w[n][k]| * 2^e in [2^13, 2^14), the exact power-of-two
//             row scale the tensor-core path uses to stay in fp16 range
//   16 bytes of padding, so 16-byte copy windows over the trailers never
//   leave the buffer.
__host__ __device__ inline size_t trailer_bytes(int N, int K, int qtype) {
    return (size_t)N * (size_t)(K / VOXQ_QBLK) * (size_t)scale_bytes(qtype);
}
__host__ __device__ inline size_t rowmul_offset(int N, int K, int qtype) {
    return (trailer_bytes(N, K, qtype) + 15) & ~(size_t)15;
}
#define VOXQ_TRAILER_PAD 16
__host__ __device__ inline size_t scales_buffer_bytes(int N, int K, int qtype) {
    return rowmul_offset(N, K, qtype) + 4 * (size_t)N + VOXQ_TRAILER_PAD;
}

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

// 16-byte streaming load that skips L1 (weights are read exactly once).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float4 ldg_f4(const float* p) {
    return __ldg(reinterpret_cast<const float4*>(p));
}

// Read-only load whose issue stays where it is written (an asm volatile is not
// moved across other asm volatile statements, e.g. barrier waits), so a value
// wanted later can be fetched ahead of a wait.  __ldg may be sunk to its use.
__device__ __forceinline__ float ldg_ordered(const float* p) {
    float r;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(r) : "l"(p));
    return r;
}

// Shared-memory accesses of a fixed width at a 32-bit shared address.  Used
// where the compiler cannot prove the alignment of a runtime-aligned base and
// would otherwise split a vector access into narrower ones (whose bank pattern
// differs from the intended conflict-free one).  Volatile: these read buffers
// that asynchronous copies rewrite, so they must stay behind the barrier waits.
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// 16-byte global -> shared copy that completes asynchronously (cp.async
// groups); both addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(dst_smem))),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Packed fp32 pair arithmetic (sm_100 f32x2 forms).
struct f2 {
    float x, y;
};
__device__ __forceinline__ uint64_t pk(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void upk(uint64_t v, float& a, float& b) {
    asm("mov.b64 {%0,%1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// Programmatic dependent launch controls (no-ops when launched without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Shared-memory barriers and bulk copies (sm_90+ PTX, used on sm_100a).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Device-side error word (one int per device, passed to the kernels): a
// bounded wait that gives up records its site there; voxq_device_error reads
// and clears it.  Kernels never trap or hang.
enum : int { VOXQ_DEVERR_NONE = 0, VOXQ_DEVERR_WAIT_FULL = 1, VOXQ_DEVERR_WAIT_EMPTY = 2,
             VOXQ_DEVERR_WAIT_MMA = 3, VOXQ_DEVERR_WAIT_TMEM = 4 };

// try_wait that lets the hardware suspend the warp (instead of spinning)
// for up to `ns` nanoseconds while the phase is incomplete.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Waits for a barrier phase for at most `limit` suspended polls of up to
// 1 ms each (about a second); returns false and records `site` when the phase
// never completes.  A waiting warp is parked by the hardware, so waiting costs
// no issue slots of the warps doing the work.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int site, int* err,
                                                  uint32_t limit = 1000u) {
    if (mbar_try_wait(bar, parity)) return true;
    for (uint32_t i = 0; i < limit; i++) {
        if (mbar_try_wait_suspend(bar, parity, 1000000u)) return true;
        // once any wait has given up, later waits return at once so a
        // failing kernel ends quickly instead of timing out per wait
        if (i == 2 && site != VOXQ_DEVERR_NONE && *reinterpret_cast<volatile int*>(err) != 0) return false;
    }
    if (site != VOXQ_DEVERR_NONE) atomicCAS(err, 0, site);
    return false;
}

// Bounded wait for phases that are expected to take long (a whole main loop):
// polls with a short sleep in between so the waiting warp leaves the issue
// slots to the warps doing the work.  Gives up after about a second of clock.
__device__ __forceinline__ bool mbar_wait_sleepy(uint64_t* bar, uint32_t parity, int site, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t i = 0;; i++) {
        __nanosleep(200);
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 63) {
            if (*reinterpret_cast<volatile int*>(err) != 0) return false;
            if (clock64() - t0 > 2000000000ll) break;
        }
    }
    atomicCAS(err, 0, site);
    return false;
}

// Global -> shared bulk copy completing on an mbarrier (16-byte aligned
// addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// Same with an L2 evict-first hint for data that is read exactly once.
__device__ __forceinline__ void bulk_g2s_stream(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// binary64 -> binary16, round to nearest even, from the double directly.
// Integer restatement of IEEE 754 rounding (same rule as the CPU checker).
__host__ __device__ inline uint16_t double_to_half_rn(double d) {
    uint64_t bits;
#ifdef __CUDA_ARCH__
    bits = (uint64_t)__double_as_longlong(d);
#else
    memcpy(&bits, &d, 8);
#endif
    uint16_t sign = (uint16_t)((bits >> 48) & 0x8000u);
    int exp = (int)((bits >> 52) & 0x7ff);
    uint64_t mant = bits & ((1ull << 52) - 1);
    if (exp == 0x7ff) {
        if (mant == 0) return sign | 0x7c00u;
        uint16_t m = (uint16_t)(mant >> 42);
        if (m == 0) m = 0x200;
        return sign | 0x7c00u | m;
    }
    if (exp == 0) return sign;
    int e = exp - 1023;
    if (e > 15) return sign | 0x7c00u;
    if (e >= -14) {
        uint64_t hm = mant >> 42;
        uint64_t rem = mant & ((1ull << 42) - 1);
        uint64_t half = 1ull << 41;
        uint32_t h = ((uint32_t)(e + 15) << 10) + (uint32_t)hm;
        if (rem > half || (rem == half && (hm & 1))) h += 1;
        if (h >= 0x7c00u) h = 0x7c00u;
        return sign | (uint16_t)h;
    }
    int s = 28 - e;
    if (s > 53) return sign;
    uint64_t sig = mant | (1ull << 52);
    uint64_t hm = sig >> s;
    uint64_t rem = sig & ((1ull << s) - 1);
    uint64_t half = 1ull << (s - 1);
    if (rem > half || (rem == half && (hm & 1))) hm += 1;
    return sign | (uint16_t)hm;
}

// binary16 -> binary32 keeping NaN payloads the way the reference's
// fp16_to_fp32 (include/tensor.h:350-371) and x86 F16C do: mantissa << 13.
// (The GPU conversion returns its canonical NaN instead.)  Finite values go
// through the exact hardware conversion.
__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    if ((h & 0x7c00u) == 0x7c00u)
        return __uint_as_float(((uint32_t)(h & 0x8000u) << 16) | 0x7f800000u | ((uint32_t)(h & 0x3ffu) << 13));
    return __half2float(__ushort_as_half(h));
}

}  // namespace voxq
