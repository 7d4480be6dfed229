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

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

}  // namespace voxq
