// voxq_gemm.cu -- quantized matmul for M > 8 activation rows on the sm_100a
// tensor cores (tcgen05.mma, accumulators in tensor memory).
//
// out[m, n] = sum_k A[m, k] * W[n, k], W in the packed Q4/Q8 layout (voxq.h),
// i.e. the prefill / DiT-patch / batched regime of the reference's
// tensor_matmul_nt (src/tensor.c:617-678; its GPU path src/tensor_cuda.cu:
// 192-333 is an fp32 cuBLAS SGEMM on widened weights).
//
// Operands are fp16 with fp32 accumulation.  fp16 keeps 11 significant bits
// (bf16 only 8, which would break the 5e-3 per-element bar), and its range is
// handled exactly by powers of two: every activation row is scaled by 2^a and
// every weight row by 2^w (rowmul of the packed layout) so that its largest
// entry sits in [2^13, 2^14); the epilogue multiplies by 2^-(a+w).
//
// Orientation (swap-AB): the MMA's M dimension is 128 weight rows, its N
// dimension BN activation rows, so skinny batches (M = 16 .. 256) still fill
// the 128-lane accumulator.  Persistent CTAs walk 128 x BN output tiles (tiles
// sharing a weight slice are adjacent, so it is read from HBM once):
//   warp 0       TMA producer: raw code + trailer tiles (2-D tensor maps) into
//                a 4-deep ring, fp16 activation tiles (128-byte swizzle) into
//                their own 4-deep ring
//   warp 1       allocates tensor memory (two accumulators) and issues
//                tcgen05.mma (one thread); tcgen05.commit releases stages and
//                hands a finished accumulator to the epilogue
//   warps 2-9    dequantize codes -> fp16 straight into the UMMA K-major
//                128-byte-swizzled layout (3-deep ring)
//   warps 10-13  epilogue: tcgen05.ld, row/column scaling, bias / residual /
//                SwiGLU, coalesced fp32 stores -- overlapping the next tile's
//                main loop through the second accumulator.
// Every wait is bounded; a wait that gives up records the error word.
#include <cuda.h>

#include <mutex>

#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

constexpr int kBM = 128;       // weight rows per tile (MMA M)
constexpr int kBK = 64;        // fp16 K per operand stage (one 128-byte swizzle atom)
constexpr int kRaw = 4;        // raw code/trailer stages
constexpr int kOpsA = 3;       // fp16 weight operand stages
constexpr int kOpsB = 4;       // fp16 activation operand stages
constexpr int kDeqWarps = 8;   // dequant warps
constexpr int kEpiWarps = 4;   // epilogue warps (one per tensor-memory lane quarter)
constexpr int kThreads = (2 + kDeqWarps + kEpiWarps) * 32;
constexpr int kRawCodes = kBM * 64;   // bytes: 128 rows x 64 code bytes
constexpr int kRawTr = kBM * 16;      // bytes: 128 rows x 16 trailer bytes
constexpr int kA16 = kBM * kBK * 2;   // 16 KB fp16 weight operand

// ---------------------------------------------------------------------------
// Activation prepass: fp32 rows -> fp16 rows scaled by a power of two.
// One warp per row; ainv[m] = 2^-a.
// ---------------------------------------------------------------------------
__global__ void act_f16_kernel(const float* __restrict__ a, int M, int K, int64_t lda, __half* __restrict__ a16,
                               float* __restrict__ ainv) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    for (int m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; m < M; m += (gridDim.x * blockDim.x) >> 5) {
        const float* row = a + (int64_t)m * lda;
        float mx = 0.0f;
        for (int k = lane * 4; k < K; k += 128) {
            const float4 v = *reinterpret_cast<const float4*>(row + k);
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        int e = 0;
        if (mx > 0.0f && isfinite(mx)) {
            int x;
            frexpf(mx, &x);
            e = min(max(14 - x, -120), 120);
        }
        const float mul = ldexpf(1.0f, e);
        __half2* dst = reinterpret_cast<__half2*>(a16 + (int64_t)m * K);
        for (int k = lane * 4; k < K; k += 128) {
            const float4 v = *reinterpret_cast<const float4*>(row + k);
            dst[k / 2] = __floats2half2_rn(v.x * mul, v.y * mul);
            dst[k / 2 + 1] = __floats2half2_rn(v.z * mul, v.w * mul);
        }
        if (lane == 0) ainv[m] = ldexpf(1.0f, -e);
    }
}

// ---------------------------------------------------------------------------
// tcgen05 / TMA helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// K-major operand, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t umma_desc(const void* smem_ptr) {
    const uint32_t a = smem_u32(smem_ptr);
    return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
           ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: fp16 A and B (K-major), fp32 D, M = 128.
__host__ __device__ constexpr uint32_t umma_idesc(int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

struct GemmArgs {
    CUtensorMap tm_codes;   // u8 [N][rowb], box {64, 128}
    CUtensorMap tm_tr;      // u8 [N][srow], box {16, 128}
    CUtensorMap tm_act;     // f16 [M][K], box {64, BN}, 128-byte swizzle
    const float* rowmul;    // [N]
    const float* ainv;      // [M]
    float* out;
    const float* bias;
    const float* residual;
    const float* gate;      // SwiGLU: out = silu(gate) * (A W^T)
    int64_t ldo, ldr, ldg;
    int M, N, K;
    int q8_signed;
    int* err;
};

// Dequantizes 8 codes of one row into one 16-byte chunk of fp16 (q*s' + m'),
// fp32 arithmetic on packed pairs: codes become exact floats 2^23 + q by byte
// permutes / masks, 2^23 comes off with add.f32x2, then fma.f32x2 and one
// fp16x2 conversion per pair.
template <int QT, bool SIGNED>
__device__ __forceinline__ uint4 deq8(uint32_t lo, uint32_t hi, float s, float m) {
    uint64_t w[4];
    if (QT == VOXQ_Q8) {
        const uint32_t x = SIGNED ? 0x80808080u : 0u;
        const uint32_t w0 = lo ^ x, w1 = hi ^ x;
        const uint64_t bias = SIGNED ? 0xCB000080CB000080ull : 0xCB000000CB000000ull;  // -(2^23 [+128])
        const uint64_t S2 = pk(s, s), M2 = pk(m, m);
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const uint32_t v = i ? w1 : w0;
            const float f0 = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7440));
            const float f1 = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7441));
            const float f2 = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7442));
            const float f3 = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7443));
            w[2 * i] = fma2(add2(pk(f0, f1), bias), S2, M2);
            w[2 * i + 1] = fma2(add2(pk(f2, f3), bias), S2, M2);
        }
    } else {
        // byte i = code[2i] << 4 | code[2i+1]: the even code stays in place as
        // 16 * code and is scaled by s / 16 (exact)
        const uint64_t bias = 0xCB000000CB000000ull;
        const uint64_t S2 = pk(s * 0.0625f, s), M2 = pk(m, m);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t v = __byte_perm(lo, 0x4B000000u, 0x7440 + i);  // 2^23 + byte
            const float fe = __uint_as_float(v & 0x4B0000F0u);             // 2^23 + 16 * even
            const float fo = __uint_as_float(v & 0x4B00000Fu);             // 2^23 + odd
            w[i] = fma2(add2(pk(fe, fo), bias), S2, M2);
        }
    }
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float a, b;
        upk(w[i], a, b);
        __half2 t = __floats2half2_rn(a, b);
        h[i] = *reinterpret_cast<uint32_t*>(&t);
    }
    return make_uint4(h[0], h[1], h[2], h[3]);
}

// Ring position helper: slot and parity of the c-th use of a ring of S slots.
struct Ring {
    uint32_t c = 0;
    template <int S>
    __device__ __forceinline__ int slot() const { return (int)(c % S); }
    template <int S>
    __device__ __forceinline__ uint32_t phase() const { return (c / S) & 1u; }
};

template <int QT, int BN, bool SIGNED>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ GemmArgs g) {
    constexpr int RK = (QT == VOXQ_Q4) ? 2 : 1;  // operand stages per raw stage
    constexpr int kB = BN * kBK * 2;             // fp16 activation operand bytes
    constexpr int TC = BN < 32 ? 32 : BN;        // tensor-memory columns per accumulator
    constexpr uint32_t IDESC = umma_idesc(BN);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* opA = base;                 // kOpsA x 16 KB (fp16 weights, SW128)
    uint8_t* opB = opA + kOpsA * kA16;   // kOpsB x kB (fp16 activations, SW128)
    uint8_t* raw = opB + kOpsB * kB;     // kRaw x (codes + trailers)
    __shared__ uint64_t full_raw[kRaw], empty_raw[kRaw], full_a[kOpsA], empty_a[kOpsA], full_b[kOpsB],
        empty_b[kOpsB], acc_full[2], acc_empty[2];
    __shared__ uint32_t tmem_slot;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KU = g.K / kBK;  // operand stages along K
    const int mt = (g.M + BN - 1) / BN, ntl = (g.N + kBM - 1) / kBM;
    const int tiles = mt * ntl;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRaw; i++) {
            mbar_init(&full_raw[i], 1);
            mbar_init(&empty_raw[i], kDeqWarps);
        }
        for (int i = 0; i < kOpsA; i++) {
            mbar_init(&full_a[i], kDeqWarps);
            mbar_init(&empty_a[i], 1);
        }
        for (int i = 0; i < kOpsB; i++) {
            mbar_init(&full_b[i], 1);
            mbar_init(&empty_b[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kEpiWarps);
        }
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(2 * TC)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        // Weight tiles may stream before the kernel waits on its predecessor
        // (the activation prepass of this call, which waited on its own
        // predecessor before it let this kernel start); activation tiles may not.
        if (lane == 0) {
            Ring rr, rb;
            bool waited = false;
            for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
                const int m0 = (t % mt) * BN, n0 = (t / mt) * kBM;
                for (int u = 0; u < KU; u++) {
                    if (u % RK == 0) {
                        const int s = rr.slot<kRaw>();
                        if (rr.c >= kRaw) mbar_wait_bounded(&empty_raw[s], rr.phase<kRaw>() ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
                        mbar_arrive_expect_tx(&full_raw[s], kRawCodes + kRawTr);
                        uint8_t* rs = raw + s * (kRawCodes + kRawTr);
                        tma_load_2d(rs, &g.tm_codes, (u / RK) * 64, n0, &full_raw[s]);
                        tma_load_2d(rs + kRawCodes, &g.tm_tr, (u / RK) * 16, n0, &full_raw[s]);
                        rr.c++;
                    }
                    if (!waited) {
                        pdl_wait();
                        pdl_launch_dependents();
                        waited = true;
                    }
                    const int s = rb.slot<kOpsB>();
                    if (rb.c >= kOpsB) mbar_wait_bounded(&empty_b[s], rb.phase<kOpsB>() ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
                    mbar_arrive_expect_tx(&full_b[s], kB);
                    tma_load_2d(opB + s * kB, &g.tm_act, u * kBK, m0, &full_b[s]);
                    rb.c++;
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            Ring ra, rb;
            int it = 0;
            for (int t = blockIdx.x; t < tiles; t += gridDim.x, it++) {
                const int as = it & 1;
                if (it >= 2) mbar_wait_bounded(&acc_empty[as], ((it >> 1) & 1) ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(as * TC);
                for (int u = 0; u < KU; u++) {
                    const int sa = ra.slot<kOpsA>(), sb = rb.slot<kOpsB>();
                    mbar_wait_bounded(&full_a[sa], ra.phase<kOpsA>(), VOXQ_DEVERR_WAIT_FULL, g.err);
                    mbar_wait_bounded(&full_b[sb], rb.phase<kOpsB>(), VOXQ_DEVERR_WAIT_FULL, g.err);
                    tc_fence_after();
                    const uint64_t ad = umma_desc(opA + sa * kA16);
                    const uint64_t bd = umma_desc(opB + sb * kB);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; kk++)  // +32 bytes = 16 fp16 along K
                        umma_f16(acc, ad + 2 * kk, bd + 2 * kk, IDESC, (u > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(&empty_a[sa]);
                    umma_commit(&empty_b[sb]);
                    ra.c++;
                    rb.c++;
                }
                umma_commit(&acc_full[as]);
            }
        }
    } else if (warp < 2 + kDeqWarps) {
        // ---------------- dequant ----------------
        const int t8 = threadIdx.x - 64;  // 0 .. 255
        const int j = t8 & 7;             // 16-byte chunk (8 codes) of the 64-wide K slice
        // reads only weights (rowmul, codes via shared memory): no predecessor wait
        Ring rr, ra;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
            const int n0 = (t / mt) * kBM;
            float rmul[kBM / 32];
#pragma unroll
            for (int i = 0; i < kBM / 32; i++) {
                const int n = n0 + t8 / 8 + 32 * i;
                rmul[i] = n < g.N ? g.rowmul[n] : 1.0f;
            }
            for (int u = 0; u < KU; u++) {
                const int h = u % RK;
                const int s = rr.slot<kRaw>();
                if (h == 0) mbar_wait_bounded(&full_raw[s], rr.phase<kRaw>(), VOXQ_DEVERR_WAIT_FULL, g.err);
                const int sa = ra.slot<kOpsA>();
                if (ra.c >= kOpsA) mbar_wait_bounded(&empty_a[sa], ra.phase<kOpsA>() ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
                const uint8_t* rc = raw + s * (kRawCodes + kRawTr);
                const uint8_t* rt = rc + kRawCodes;
                uint8_t* dstA = opA + sa * kA16;
#pragma unroll
                for (int i = 0; i < kBM / 32; i++) {
                    const int row = t8 / 8 + 32 * i;
                    float sc, mn;
                    uint32_t lo, hi = 0;
                    if (QT == VOXQ_Q8) {
                        const uint2 c = *reinterpret_cast<const uint2*>(rc + row * 64 + 8 * j);
                        lo = c.x;
                        hi = c.y;
                        const float2 tr = *reinterpret_cast<const float2*>(rt + row * 16 + 8 * (j >> 2));
                        sc = tr.x;
                        mn = tr.y;
                    } else {
                        lo = *reinterpret_cast<const uint32_t*>(rc + row * 64 + 32 * h + 4 * j);
                        const float2 tr =
                            __half22float2(*reinterpret_cast<const __half2*>(rt + row * 16 + 4 * (2 * h + (j >> 2))));
                        sc = tr.x;
                        mn = tr.y;
                    }
                    const uint4 v = deq8<QT, SIGNED>(lo, hi, sc * rmul[i], mn * rmul[i]);
                    // K-major 128-byte swizzle: chunk j of row `row` lands at j ^ (row & 7)
                    *reinterpret_cast<uint4*>(dstA + row * 128 + ((j ^ (row & 7)) << 4)) = v;
                }
                // make the generic-proxy writes visible to the tensor core
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&full_a[sa]);
                    if (h == RK - 1) mbar_arrive(&empty_raw[s]);
                }
                ra.c++;
                if (h == RK - 1) rr.c++;
            }
        }
    } else {
        // ---------------- epilogue ----------------
        pdl_wait();  // row scales of the prepass; residual / output of earlier work
        pdl_launch_dependents();
        const int q = warp & 3;  // tensor-memory lane quarter of this warp
        int it = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, it++) {
            const int m0 = (t % mt) * BN, n0 = (t / mt) * kBM;
            const int as = it & 1;
            mbar_wait_bounded(&acc_full[as], (it >> 1) & 1, VOXQ_DEVERR_WAIT_MMA, g.err);
            tc_fence_after();
            const int nrow = n0 + q * 32 + lane;  // weight row = output column n
            const bool nok = nrow < g.N;
            const float rinv = nok ? 1.0f / g.rowmul[nrow] : 0.0f;
            const float bias = (nok && g.bias) ? g.bias[nrow] : 0.0f;
            for (int c0 = 0; c0 < BN; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(as * TC + c0), v);
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const int m = m0 + c0 + i;
                    if (m < g.M && nok) {
                        float y = __uint_as_float(v[i]) * (rinv * g.ainv[m]);
                        if (g.gate) y = silu_f(g.gate[(int64_t)m * g.ldg + nrow]) * y;
                        y += bias;
                        if (g.residual) y += g.residual[(int64_t)m * g.ldr + nrow];
                        g.out[(int64_t)m * g.ldo + nrow] = y;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[as]);
        }
    }
    // dequant / epilogue roles touch global outputs only after the wait below
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * TC) : "memory");
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

static bool make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, uint64_t inner, uint64_t rows,
                     uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

static size_t act_bytes(int M, int K) { return align256((size_t)M * K * 2) + align256((size_t)M * 4); }

size_t gemm_workspace_bytes(int M, int N, int K, bool swiglu) {
    // fp16 activations + their row scales (+ the SwiGLU gate result)
    return act_bytes(M, K) + (swiglu ? align256((size_t)M * N * 4) : 0);
}

static int pick_bn(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256; }

template <int QT, int BN, bool SIGNED>
static VoxCPMError launch_gemm_t(const GemmArgs& a, cudaStream_t st) {
    constexpr int kB = BN * kBK * 2;
    constexpr int smem = 1024 + kOpsA * kA16 + kOpsB * kB + kRaw * (kRawCodes + kRawTr);
    constexpr int TC = BN < 32 ? 32 : BN;
    auto kern = gemm_kernel<QT, BN, SIGNED>;
    static int occ = 1;
    static std::once_flag once;
    std::call_once(once, [&] {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem);
        const int tmem_cap = 512 / (2 * TC);  // co-resident CTAs must fit tensor memory
        if (occ > tmem_cap) occ = tmem_cap;
        if (occ < 1) occ = 1;
    });
    const int tiles = ((a.M + BN - 1) / BN) * ((a.N + kBM - 1) / kBM);
    const int cap = device_sm_count() * occ;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(tiles < cap ? tiles : cap);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
    return VOXCPM_SUCCESS;
}

template <int QT>
static VoxCPMError launch_bn(const GemmArgs& a, int bn, bool sgn, cudaStream_t st) {
    switch (bn) {
        case 16: return sgn ? launch_gemm_t<QT, 16, true>(a, st) : launch_gemm_t<QT, 16, false>(a, st);
        case 32: return sgn ? launch_gemm_t<QT, 32, true>(a, st) : launch_gemm_t<QT, 32, false>(a, st);
        case 64: return sgn ? launch_gemm_t<QT, 64, true>(a, st) : launch_gemm_t<QT, 64, false>(a, st);
        case 128: return sgn ? launch_gemm_t<QT, 128, true>(a, st) : launch_gemm_t<QT, 128, false>(a, st);
        default: return sgn ? launch_gemm_t<QT, 256, true>(a, st) : launch_gemm_t<QT, 256, false>(a, st);
    }
}

// Whether the tensor-core path takes this shape (else the GEMV path runs in
// groups of 8 rows).
static bool gemm_supported(int K, int qtype, int64_t lda) {
    if (qtype == VOXQ_Q8 && K % 64) return false;
    if (qtype == VOXQ_Q4 && K % 128) return false;
    return K > 0 && (lda % 4) == 0;
}

static VoxCPMError gemm_by_rows(const float* a, int M, int64_t lda, const voxq_qweight* w, float* out, int64_t ldo,
                                const voxq_epilogue* epi, cudaStream_t st) {
    for (int m0 = 0; m0 < M; m0 += 8) {
        voxq_gemv_item it = {};
        it.w = *w;
        it.a = a + m0 * lda;
        it.out = out + m0 * ldo;
        it.M = M - m0 < 8 ? M - m0 : 8;
        it.lda = (int32_t)lda;
        it.ldo = (int32_t)ldo;
        if (epi) {
            it.bias = epi->bias;
            it.residual = epi->residual ? epi->residual + m0 * epi->ldr : nullptr;
            it.ldr = (int32_t)epi->ldr;
            if (epi->up) {
                it.up_codes = epi->up->codes;
                it.up_scales = epi->up->scales;
            }
        }
        VoxCPMError e = gemv_launch(&it, 1, st);
        if (e) return e;
    }
    return VOXCPM_SUCCESS;
}

// One GEMM launch: out = epilogue(A W^T) with optional gate (SwiGLU second half).
static VoxCPMError gemm_one(const float* ainv, const __half* a16, int M, const voxq_qweight* w, float* out,
                            int64_t ldo, const float* bias, const float* residual, int64_t ldr, const float* gate,
                            int64_t ldg, cudaStream_t st) {
    const int N = w->N, K = w->K, qt = w->qtype;
    const int bn = pick_bn(M);
    static thread_local GemmArgs ga;
    const uint64_t rowb = (uint64_t)codes_row_bytes(K, qt);
    const uint64_t srow = (uint64_t)(K / VOXQ_QBLK) * scale_bytes(qt);
    if (!make_map(&ga.tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->codes, rowb, (uint64_t)N, rowb, 64, kBM,
                  CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map(&ga.tm_tr, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->scales, srow, (uint64_t)N, srow, 16, kBM,
                  CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map(&ga.tm_act, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a16, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, kBK,
                  (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_128B))
        return VOXCPM_ERR_INTERNAL;
    ga.rowmul = reinterpret_cast<const float*>(static_cast<const uint8_t*>(w->scales) + rowmul_offset(N, K, qt));
    ga.ainv = ainv;
    ga.out = out;
    ga.bias = bias;
    ga.residual = residual;
    ga.gate = gate;
    ga.ldo = ldo;
    ga.ldr = ldr;
    ga.ldg = ldg;
    ga.M = M;
    ga.N = N;
    ga.K = K;
    ga.q8_signed = w->q8_signed;
    ga.err = device_error_word();
    return qt == VOXQ_Q4 ? launch_bn<VOXQ_Q4>(ga, bn, false, st) : launch_bn<VOXQ_Q8>(ga, bn, w->q8_signed != 0, st);
}

VoxCPMError gemm_launch(const float* a, int M, int64_t lda, const voxq_qweight* w, float* out, int64_t ldo,
                        const voxq_epilogue* epi, void* ws, cudaStream_t st) {
    const int N = w->N, K = w->K;
    if (w->qtype != VOXQ_Q4 && w->qtype != VOXQ_Q8) return VOXCPM_ERR_UNSUPPORTED;
    if (M <= 0 || N <= 0) return VOXCPM_SUCCESS;
    if (K % VOXQ_QBLK) return VOXCPM_ERR_SHAPE_MISMATCH;
    if (!gemm_supported(K, w->qtype, lda) || (reinterpret_cast<uintptr_t>(a) & 15))
        return gemm_by_rows(a, M, lda, w, out, ldo, epi, st);
    if ((reinterpret_cast<uintptr_t>(w->codes) & 15) || (reinterpret_cast<uintptr_t>(w->scales) & 15))
        return VOXCPM_ERR_UNSUPPORTED;
    uint8_t* wsb = static_cast<uint8_t*>(ws);
    __half* a16 = reinterpret_cast<__half*>(wsb);
    float* ainv = reinterpret_cast<float*>(wsb + align256((size_t)M * K * 2));
    {
        cudaLaunchConfig_t cfg = {};
        const int blocks = (M + 7) / 8;
        cfg.gridDim = dim3(blocks < 1 ? 1 : blocks);
        cfg.blockDim = dim3(256);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, act_f16_kernel, a, M, K, lda, a16, ainv));
    }
    const float* bias = epi ? epi->bias : nullptr;
    const float* res = epi ? epi->residual : nullptr;
    const int64_t ldr = epi ? epi->ldr : 0;
    if (epi && epi->up) {
        // SwiGLU: gate into the workspace, then up with silu(gate) * y fused
        float* gbuf = reinterpret_cast<float*>(wsb + act_bytes(M, K));
        VoxCPMError e = gemm_one(ainv, a16, M, w, gbuf, N, nullptr, nullptr, 0, nullptr, 0, st);
        if (e) return e;
        return gemm_one(ainv, a16, M, epi->up, out, ldo, bias, res, ldr, gbuf, N, st);
    }
    return gemm_one(ainv, a16, M, w, out, ldo, bias, res, ldr, nullptr, 0, st);
}

}  // namespace voxq
