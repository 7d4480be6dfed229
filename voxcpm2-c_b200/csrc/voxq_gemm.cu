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
// the 128-lane accumulator.  One CTA computes a 128 x BN tile over all K:
//   warp 0      TMA producer: raw code + trailer tiles (2-D tensor maps) into
//               a 4-deep ring; fp16 activation tiles (128-byte swizzle) into
//               the operand ring
//   warp 1      allocates tensor memory and issues tcgen05.mma (one thread);
//               tcgen05.commit releases operand stages and signals the end
//   warps 2-9   dequantize codes -> fp16 straight into the UMMA K-major
//               128-byte-swizzled layout (codes never touch HBM twice), then
//               run the epilogue: tcgen05.ld, row/column scaling, bias /
//               residual / SwiGLU, coalesced fp32 stores.
// Every wait is bounded; a wait that gives up records the error word.
#include <cuda.h>

#include <mutex>

#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

constexpr int kBM = 128;       // weight rows per tile (MMA M)
constexpr int kBK = 64;        // fp16 K per operand stage (one 128-byte swizzle atom)
constexpr int kRaw = 4;        // raw code/trailer stages
constexpr int kOps = 3;        // operand stages
constexpr int kDeqWarps = 8;   // dequant + epilogue warps
constexpr int kThreads = (2 + kDeqWarps) * 32;
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

// Dequantizes 8 codes of one row into one 16-byte chunk of fp16 (q*s' + m').
template <int QT, bool SIGNED>
__device__ __forceinline__ uint4 deq8(uint32_t lo, uint32_t hi, float s, float m) {
    float q[8];
    if (QT == VOXQ_Q8) {
        const uint32_t x = SIGNED ? 0x80808080u : 0u;
        const uint32_t w0 = lo ^ x, w1 = hi ^ x;
        const float off = SIGNED ? 8388736.0f : 8388608.0f;  // 2^23 (+128 for int8)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            q[i] = __uint_as_float(__byte_perm(w0, 0x4B000000u, 0x7440 + i)) - off;
            q[4 + i] = __uint_as_float(__byte_perm(w1, 0x4B000000u, 0x7440 + i)) - off;
        }
    } else {
        // lo holds 4 bytes = 8 codes, byte i = code[2i] << 4 | code[2i+1]
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t b = (lo >> (8 * i)) & 0xffu;
            q[2 * i] = (float)(b >> 4);
            q[2 * i + 1] = (float)(b & 15u);
        }
    }
    uint4 r;
    __half2 h0 = __floats2half2_rn(fmaf(q[0], s, m), fmaf(q[1], s, m));
    __half2 h1 = __floats2half2_rn(fmaf(q[2], s, m), fmaf(q[3], s, m));
    __half2 h2 = __floats2half2_rn(fmaf(q[4], s, m), fmaf(q[5], s, m));
    __half2 h3 = __floats2half2_rn(fmaf(q[6], s, m), fmaf(q[7], s, m));
    r.x = *reinterpret_cast<uint32_t*>(&h0);
    r.y = *reinterpret_cast<uint32_t*>(&h1);
    r.z = *reinterpret_cast<uint32_t*>(&h2);
    r.w = *reinterpret_cast<uint32_t*>(&h3);
    return r;
}

template <int QT, int BN, bool SIGNED>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ GemmArgs g) {
    constexpr int RK = (QT == VOXQ_Q4) ? 2 : 1;  // operand stages per raw stage
    constexpr int kB = BN * kBK * 2;             // fp16 activation operand bytes
    constexpr int TCOLS = BN < 32 ? 32 : BN;     // tensor-memory columns (power of two >= 32)
    constexpr uint32_t IDESC = umma_idesc(BN);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned carve-up: operand stages first (swizzle atoms need it)
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* opA = base;                                  // kOps x 16 KB
    uint8_t* opB = opA + kOps * kA16;                     // kOps x kB
    uint8_t* raw = opB + kOps * kB;                       // kRaw x (codes + trailers)
    __shared__ uint64_t full_raw[kRaw], empty_raw[kRaw], full_a[kOps], full_b[kOps], empty_op[kOps], done_bar;
    __shared__ uint32_t tmem_slot;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BN, n0 = blockIdx.y * kBM;
    const int KU = g.K / kBK;  // operand stages along K

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRaw; i++) {
            mbar_init(&full_raw[i], 1);
            mbar_init(&empty_raw[i], kDeqWarps);
        }
        for (int i = 0; i < kOps; i++) {
            mbar_init(&full_a[i], kDeqWarps);
            mbar_init(&full_b[i], 1);
            mbar_init(&empty_op[i], 1);
        }
        mbar_init(&done_bar, 1);
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            for (int u = 0; u < KU; u++) {
                if (u % RK == 0) {
                    const int r = u / RK, slot = r % kRaw;
                    if (r >= kRaw) mbar_wait_bounded(&empty_raw[slot], ((r / kRaw) & 1) ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
                    mbar_arrive_expect_tx(&full_raw[slot], kRawCodes + kRawTr);
                    uint8_t* rs = raw + slot * (kRawCodes + kRawTr);
                    tma_load_2d(rs, &g.tm_codes, r * 64, n0, &full_raw[slot]);
                    tma_load_2d(rs + kRawCodes, &g.tm_tr, r * 16, n0, &full_raw[slot]);
                }
                const int o = u % kOps;
                if (u >= kOps) mbar_wait_bounded(&empty_op[o], ((u / kOps) & 1) ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
                mbar_arrive_expect_tx(&full_b[o], kB);
                tma_load_2d(opB + o * kB, &g.tm_act, u * kBK, m0, &full_b[o]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            for (int u = 0; u < KU; u++) {
                const int o = u % kOps;
                const uint32_t ph = (u / kOps) & 1;
                mbar_wait_bounded(&full_a[o], ph, VOXQ_DEVERR_WAIT_FULL, g.err);
                mbar_wait_bounded(&full_b[o], ph, VOXQ_DEVERR_WAIT_FULL, g.err);
                tc_fence_after();
                const uint64_t ad = umma_desc(opA + o * kA16);
                const uint64_t bd = umma_desc(opB + o * kB);
#pragma unroll
                for (int kk = 0; kk < kBK / 16; kk++)  // +32 bytes = 16 fp16 along K
                    umma_f16(tmem, ad + 2 * kk, bd + 2 * kk, IDESC, (u > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&empty_op[o]);
            }
            umma_commit(&done_bar);
        }
    } else {
        // ---------------- dequant (then epilogue) ----------------
        const int t = threadIdx.x - 64;  // 0 .. 255
        const int j = t & 7;             // 16-byte chunk (8 codes) within the 64-wide row slice
        float rmul[kBM / 32];
#pragma unroll
        for (int i = 0; i < kBM / 32; i++) {
            const int n = n0 + t / 8 + 32 * i;
            rmul[i] = n < g.N ? g.rowmul[n] : 1.0f;
        }
        for (int u = 0; u < KU; u++) {
            const int r = u / RK, slot = r % kRaw, h = u % RK;
            const int o = u % kOps;
            if (h == 0) mbar_wait_bounded(&full_raw[slot], (r / kRaw) & 1, VOXQ_DEVERR_WAIT_FULL, g.err);
            if (u >= kOps) mbar_wait_bounded(&empty_op[o], ((u / kOps) & 1) ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
            const uint8_t* rc = raw + slot * (kRawCodes + kRawTr);
            const uint8_t* rt = rc + kRawCodes;
            uint8_t* dstA = opA + o * kA16;
#pragma unroll
            for (int i = 0; i < kBM / 32; i++) {
                const int row = t / 8 + 32 * i;
                float s, m;
                uint32_t lo, hi = 0;
                if (QT == VOXQ_Q8) {
                    const uint2 c = *reinterpret_cast<const uint2*>(rc + row * 64 + 8 * j);
                    lo = c.x;
                    hi = c.y;
                    const float2 tr = *reinterpret_cast<const float2*>(rt + row * 16 + 8 * (j >> 2));
                    s = tr.x;
                    m = tr.y;
                } else {
                    lo = *reinterpret_cast<const uint32_t*>(rc + row * 64 + 32 * h + 4 * j);
                    const uint32_t tr = *reinterpret_cast<const uint32_t*>(rt + row * 16 + 4 * (2 * h + (j >> 2)));
                    s = __half2float(__ushort_as_half((unsigned short)(tr & 0xffff)));
                    m = __half2float(__ushort_as_half((unsigned short)(tr >> 16)));
                }
                const uint4 v = deq8<QT, SIGNED>(lo, hi, s * rmul[i], m * rmul[i]);
                // K-major 128-byte swizzle: chunk j of row `row` lands at j ^ (row & 7)
                *reinterpret_cast<uint4*>(dstA + row * 128 + ((j ^ (row & 7)) << 4)) = v;
            }
            // make the generic-proxy writes visible to the tensor core
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&full_a[o]);
                if (h == RK - 1) mbar_arrive(&empty_raw[slot]);
            }
        }

        // ---------------- epilogue ----------------
        mbar_wait_bounded(&done_bar, 0, VOXQ_DEVERR_WAIT_MMA, g.err);
        tc_fence_after();
        const int q = warp & 3;               // tensor-memory lane quarter of this warp
        const int half = (warp - 2) >> 2;     // which half of the columns
        const int nrow = n0 + q * 32 + lane;  // weight row = output column n
        const bool nok = nrow < g.N;
        const float rinv = nok ? 1.0f / g.rowmul[nrow] : 0.0f;
        const float bias = (nok && g.bias) ? g.bias[nrow] : 0.0f;
        constexpr int CH = BN / 2 < 16 ? 16 : BN / 2;  // columns per half
        for (int c0 = half * CH; c0 < (half + 1) * CH && c0 < BN; c0 += 16) {
            uint32_t v[16];
            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
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
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
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
    constexpr int smem = 1024 + kOps * (kA16 + kB) + kRaw * (kRawCodes + kRawTr);
    auto kern = gemm_kernel<QT, BN, SIGNED>;
    static std::once_flag once;
    std::call_once(once, [&] { cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); });
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.M + BN - 1) / BN, (a.N + kBM - 1) / kBM);
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
