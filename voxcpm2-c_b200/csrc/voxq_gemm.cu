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
//   warp 0       raw producer: code (128-byte rows, 128-byte swizzle) + trailer
//                tiles by 2-D TMA into their ring, each raw stage feeding 2 (Q8)
//                or 4 (Q4) operand stages
//   warp 26      activation producer: fp16 activation stages, laid out by the
//                prepass as ready shared-memory images, one bulk copy each
//   warp 1       allocates tensor memory (two accumulators) and issues
//                tcgen05.mma (one thread); tcgen05.commit releases stages and
//                hands a finished accumulator to the epilogue
//   warps 2-17   dequantize codes -> fp16 straight into the UMMA K-major
//                128-byte-swizzled layout (3-deep ring)
//   warps 18-25  epilogue (two per tensor-memory lane quarter, each half of the
//                tile's columns): tcgen05.ld, row/column scaling, bias / residual /
//                SwiGLU, coalesced fp32 stores -- overlapping the next tile's
//                main loop through the second accumulator.
// Every wait is bounded; a wait that gives up records the error word.
#include <cuda.h>

#include <cstdint>
#include <cstdlib>
#include <mutex>

#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

constexpr int kBM = 128;        // weight rows per tile (MMA M)
constexpr int kBK = 64;         // fp16 K per operand stage (one 128-byte swizzle atom)
constexpr int kOpsA = 3;        // fp16 weight operand stages
constexpr int kDeqWarps = 16;   // dequant warps (2 rows x 8 chunks per thread and stage)
constexpr int kEpiWarps = 8;    // epilogue warps: two per tensor-memory lane quarter, each half the columns
constexpr int kEpiParts = kEpiWarps / 4;
constexpr int kThreads = (3 + kDeqWarps + kEpiWarps) * 32;  // + raw producer, MMA, activation producer
constexpr int kBWarp = 2 + kDeqWarps + kEpiWarps;                // the activation producer warp
constexpr int kRawRow = 128;    // code bytes per row and raw stage (Q8: 128 K, Q4: 256 K)
constexpr int kRawTrRow = 32;   // trailer bytes per row and raw stage (Q8: 4 blocks, Q4: 8 blocks)
constexpr int kRawCodes = kBM * kRawRow;
constexpr int kRawStage = kRawCodes + kBM * kRawTrRow;  // 20 KB, a multiple of 1024
constexpr int kA16 = kBM * kBK * 2;  // 16 KB fp16 weight operand
constexpr int kMaxBN = 256;
// Ring depths by activation tile width.  A TMA load takes about a microsecond
// to land, so each ring is as deep (bytes in flight) as shared memory allows:
// fp16 activation operand stages, raw code/trailer stages.
constexpr int ops_b(int bn) { return bn >= 256 ? 3 : bn >= 128 ? 5 : bn >= 64 ? 8 : 16; }
constexpr int raw_stages(int bn) { return bn >= 256 ? 3 : bn >= 128 ? 4 : 5; }

// ---------------------------------------------------------------------------
// Activation prepass: fp32 rows -> fp16 rows scaled by a power of two, written
// as ready-made shared-memory images: for m-tile t (BN rows) and K stage u,
// the BN x 64 fp16 block sits contiguously at ((t * KU + u) * BN) * 128 bytes
// in the UMMA K-major 128-byte-swizzled order (16-byte chunk j of row r at
// chunk j ^ (r & 7)), so the GEMM fetches it with one bulk copy.  Rows M ..
// Mpad-1 are zero; ainv[m] = 2^-a (0 for pad rows).  One warp per row: lane l
// owns the 8-value chunks l, l + 32, ..., so every load of the row is in flight
// before the first shuffle and no block barrier is needed.
// ---------------------------------------------------------------------------
constexpr int kPrepThreads = 256;                  // 8 independent row warps per block
constexpr int kPrepRows = kPrepThreads / 32;
constexpr int kRegIters = 4;                       // chunks per lane held in registers (K <= 1024 read once)
constexpr int kW16Rows = 256;                      // rows per tile of the tiled fp16 weight (covers NT = 1 and 2)

__device__ __forceinline__ uint4 half8(const float4& v0, const float4& v1, float mul) {
    __half2 p0 = __floats2half2_rn(v0.x * mul, v0.y * mul), p1 = __floats2half2_rn(v0.z * mul, v0.w * mul);
    __half2 p2 = __floats2half2_rn(v1.x * mul, v1.y * mul), p3 = __floats2half2_rn(v1.z * mul, v1.w * mul);
    return make_uint4(*reinterpret_cast<uint32_t*>(&p0), *reinterpret_cast<uint32_t*>(&p1),
                      *reinterpret_cast<uint32_t*>(&p2), *reinterpret_cast<uint32_t*>(&p3));
}

__device__ __forceinline__ float absmax8(const float4& v0, const float4& v1) {
    return fmaxf(fmaxf(fmaxf(fabsf(v0.x), fabsf(v0.y)), fmaxf(fabsf(v0.z), fabsf(v0.w))),
                 fmaxf(fmaxf(fabsf(v1.x), fabsf(v1.y)), fmaxf(fabsf(v1.z), fabsf(v1.w))));
}

__device__ __forceinline__ void act_row(const float* __restrict__ a, int M, int K, int64_t lda, int bn,
                                        uint8_t* __restrict__ a16t, float* __restrict__ ainv, int m, int lane) {
    constexpr int RI = kRegIters;
    const int KU = K / kBK, nch = K / 8;
    const bool live = m < M;
    const float* row = a + (int64_t)m * lda;
    float4 v[RI][2];
#pragma unroll
    for (int i = 0; i < RI; i++) {
        const int c = lane + 32 * i;
        v[i][0] = v[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (live && c < nch) {
            v[i][0] = __ldg(reinterpret_cast<const float4*>(row + 8 * c));
            v[i][1] = __ldg(reinterpret_cast<const float4*>(row + 8 * c + 4));
        }
    }
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < RI; i++) mx = fmaxf(mx, absmax8(v[i][0], v[i][1]));
    if (live) {
        for (int c = lane + 32 * RI; c < nch; c += 32)
            mx = fmaxf(mx, absmax8(__ldg(reinterpret_cast<const float4*>(row + 8 * c)),
                                   __ldg(reinterpret_cast<const float4*>(row + 8 * c + 4))));
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int e = 0;
    if (mx > 0.0f && isfinite(mx)) {
        int x;
        frexpf(mx, &x);
        e = min(max(14 - x, -120), 120);
    }
    const float mul = ldexpf(1.0f, e);
    const int t = m / bn, r = m % bn;
    uint8_t* tb = a16t + ((int64_t)t * KU * bn + r) * 128;
    const int64_t ustride = (int64_t)bn * 128;
#pragma unroll
    for (int i = 0; i < RI; i++) {
        const int c = lane + 32 * i;  // K stage c >> 3, 16-byte chunk c & 7
        if (c < nch)
            *reinterpret_cast<uint4*>(tb + (c >> 3) * ustride + (((c & 7) ^ (r & 7)) << 4)) =
                half8(v[i][0], v[i][1], mul);  // zeros for pad rows
    }
    for (int c = lane + 32 * RI; c < nch; c += 32) {
        float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
        if (live) {
            v0 = __ldg(reinterpret_cast<const float4*>(row + 8 * c));
            v1 = __ldg(reinterpret_cast<const float4*>(row + 8 * c + 4));
        }
        *reinterpret_cast<uint4*>(tb + (c >> 3) * ustride + (((c & 7) ^ (r & 7)) << 4)) = half8(v0, v1, mul);
    }
    if (lane == 0) ainv[m] = live ? ldexpf(1.0f, -e) : 0.0f;
}

__global__ void __launch_bounds__(kPrepThreads) act_tile_kernel(const float* __restrict__ a, int M, int K, int64_t lda,
                                                                int bn, uint8_t* __restrict__ a16t,
                                                                float* __restrict__ ainv, int rows) {
    pdl_wait();
    pdl_launch_dependents();
    const int m = blockIdx.x * kPrepRows + (threadIdx.x >> 5);
    if (m < rows) act_row(a, M, K, lda, bn, a16t, ainv, m, threadIdx.x & 31);
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

// Thread-block cluster helpers: every thread of every CTA of the cluster takes
// part in a cluster barrier; shared memory of CTA `rank` is read through its
// shared::cluster address (mapa).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t a) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a)
                 : "memory");
    return v;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

struct GemmArgs {
    CUtensorMap tm_codes;   // u8 [N][rowb], box {128, 128}, 128-byte swizzle
    CUtensorMap tm_tr;      // u8 [N][srow], box {32, 128}
    const uint8_t* w16t;    // two-phase path: tiled fp16 weight images (prep_f16_kernel)
    const uint8_t* a16t;    // tiled fp16 activation images (act_tile_kernel)
    const float* rowmul;    // [N]
    const float* ainv;      // [Mpad]
    float* out;
    const float* bias;
    const float* residual;
    const float* gate;      // SwiGLU: out = silu(gate) * (A W^T)
    float* part;            // split-K partial accumulators [tiles][S][BN][128]
    int64_t ldo, ldr, ldg;
    int M, N, K;
    int S, KUs;             // K splits per tile, operand stages per split
    int cluster;            // S > 1 in one cluster per tile: partials summed in shared memory
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

// Epilogue value for output row m (a tile column) and column n (this lane).
__device__ __forceinline__ float epi_value(const GemmArgs& g, float acc, float scale, float bias, int64_t m, int n) {
    float y = acc * scale;
    if (g.gate) y = silu_f(__ldg(g.gate + m * g.ldg + n)) * y;
    y += bias;
    if (g.residual) y += __ldg(g.residual + m * g.ldr + n);
    return y;
}

// Epilogue role (kEpiWarps warps): tcgen05.ld of a finished accumulator, row /
// column scaling, bias / residual / SwiGLU gate, coalesced fp32 stores -- or,
// for split K, the raw partial sums for the reduction kernel.  Warp e (0 ..
// kEpiWarps-1) reads tensor-memory lane quarter q = warp % 4 and columns part e / 4.
// Tiles are NT x 128 weight rows (sub-tiles, one accumulator each) x BN
// activation rows; NACC accumulator sets alternate between tiles.  Warp e
// serves sub-tile (e / 4) % NT and column part (e / 4) / NT of CP.
template <int BN, int TC, int NT, int NACC, int CP>
__device__ __forceinline__ void epilogue_role(const GemmArgs& g, uint32_t tmem, uint64_t* acc_full, uint64_t* acc_empty,
                                              float* ainv_all, int units, int mt, int S, int e, int q, int lane) {
        pdl_wait();  // row scales of the prepass; residual / gate / output of earlier work
        pdl_launch_dependents();
        // warp e: tensor-memory lane quarter q = warp % 4 (the hardware's access rule),
        // tile columns [cb, ce) = its column part (all of them below CP x 16 columns)
        constexpr int CWID = (BN / CP >= 16) ? BN / CP : BN;
        constexpr int TN = kBM * NT;  // weight rows per tile
        const int sub = (e / 4) % NT, part = (e / 4) / NT;
        const int cb = part * CWID, ce = min(BN, cb + CWID);
        float* ainv_w = ainv_all + e * 2 * (kMaxBN / CP);
        // The tile's activation row scales go to shared memory by cp.async one
        // unit ahead (ainv is padded to whole tiles); column scale and bias one
        // unit ahead in registers.  Nothing the loop needs is fetched after the
        // accumulator wait.
#define VOXQ_EPI_FETCH(W, BUF)                                                                                   \
    do {                                                                                                         \
        const int fw = (W);                                                                                      \
        if (fw < units) {                                                                                        \
            const int ft = fw / S;                                                                               \
            const int fm0 = (ft % mt) * BN, fn = (ft / mt) * TN + sub * kBM + q * 32 + lane;                     \
            for (int c = lane; c < (ce - cb) / 4; c += 32)                                                       \
                cp_async16(ainv_w + (BUF) * (kMaxBN / CP) + 4 * c, g.ainv + fm0 + cb + 4 * c);                   \
            rm_next = fn < g.N ? ldg_ordered(g.rowmul + fn) : 1.0f;                                              \
            b_next = (fn < g.N && g.bias) ? ldg_ordered(g.bias + fn) : 0.0f;                                     \
        }                                                                                                        \
        cp_async_commit();                                                                                       \
    } while (0)
        float rm_next = 1.0f, b_next = 0.0f;
        VOXQ_EPI_FETCH(blockIdx.x, 0);
        int it = 0;
        for (int w = blockIdx.x; w < units; w += gridDim.x, it++) {
            const int t = w / S, sp = w % S;
            const int m0 = (t % mt) * BN, n0 = (t / mt) * TN + sub * kBM;
            const int ab = it & 1;        // row-scale staging buffer
            const int as = it % NACC;     // accumulator set
            const int nrow = n0 + q * 32 + lane;  // weight row = output column n
            const bool nok = nrow < g.N;
            const float rinv = 1.0f / rm_next;
            const float bias = b_next;
            VOXQ_EPI_FETCH(w + gridDim.x, ab ^ 1);
            const int mlim = nok ? min(BN, g.M - m0) : 0;  // valid rows of this tile for this lane
            const float* arow = ainv_w + ab * (kMaxBN / CP) - cb;  // indexed by tile column
            const uint32_t tacc = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((as * NT + sub) * TC);
            mbar_wait_sleepy(&acc_full[as], (it / NACC) & 1, VOXQ_DEVERR_WAIT_MMA, g.err);
            tc_fence_after();
            cp_async_wait<1>();  // this unit's row scales (the next unit's may be in flight)
            __syncwarp();
            if (S == 1) {
                // kept as a loop: a fully unrolled epilogue thrashes the instruction cache
#pragma unroll 1
                for (int c0 = cb; c0 < ce; c0 += 16) {
                    uint32_t v[16];
                    tmem_ld16(tacc + (uint32_t)c0, v);
                    float am[16];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float4 x = *reinterpret_cast<const float4*>(arow + c0 + 4 * i);
                        am[4 * i] = x.x;
                        am[4 * i + 1] = x.y;
                        am[4 * i + 2] = x.z;
                        am[4 * i + 3] = x.w;
                    }
                    float* o = g.out + (int64_t)(m0 + c0) * g.ldo + nrow;
                    if (!g.gate && !g.residual) {
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            if (c0 + i < mlim) o[(int64_t)i * g.ldo] = __uint_as_float(v[i]) * (rinv * am[i]) + bias;
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; i++)
                            if (c0 + i < mlim)
                                o[(int64_t)i * g.ldo] =
                                    epi_value(g, __uint_as_float(v[i]), rinv * am[i], bias, m0 + c0 + i, nrow);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[as]);
            } else {
                // Split K: park the raw partial sum ([BN][128] per unit) for the
                // reduction kernel, which adds the S partials in split order and
                // applies the epilogue.
                float* pp = g.part + ((size_t)(t * S + sp) * BN) * TN + sub * kBM + q * 32 + lane;
#pragma unroll 1
                for (int c0 = cb; c0 < ce; c0 += 16) {
                    uint32_t v[16];
                    tmem_ld16(tacc + (uint32_t)c0, v);
#pragma unroll
                    for (int i = 0; i < 16; i++) pp[(c0 + i) * TN] = __uint_as_float(v[i]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[as]);
            }
        }
        cp_async_wait<0>();
#undef VOXQ_EPI_FETCH
}

// Split K inside one thread-block cluster (the fused kernel with g.cluster):
// the S CTAs of a cluster are the S K-splits of one tile, one unit each, and
// rank r finishes tile columns (activation rows) [r RB, (r+1) RB), RB = BN / S.
//   1. the epilogue warps park the raw accumulator in this CTA's shared memory
//      as P[tile column c][weight row n] (over the operand rings, which the
//      finished MMAs no longer read);
//   2. cluster barrier: every P of the cluster is complete;
//   3. every thread of the CTA pulls, for its items (tile column c of this
//      rank, 4 consecutive weight rows), the S partials from the S CTAs'
//      P through distributed shared memory -- a warp reads 512 contiguous
//      bytes per load, and each thread keeps several items' loads in flight --
//      sums them in rank order (the order of splitk_reduce_kernel, so the bits
//      equal the two-kernel split), applies the epilogue and stores the output;
//   4. cluster barrier: every P stays alive until all ranks have read it.
// No partial touches global memory and no reduction kernel runs.

template <int BN, int TC>
__device__ __forceinline__ void cluster_park_partials(const GemmArgs& g, uint32_t tmem, float* P, int e, int q,
                                                      int lane) {
    constexpr int CWID = (BN / kEpiParts >= 16) ? BN / kEpiParts : BN;
    const int cb = (e / 4) * CWID, ce = min(BN, cb + CWID);
    const uint32_t tacc = tmem + ((uint32_t)(q * 32) << 16);
    float* pc = P + q * 32 + lane;
#pragma unroll 1
    for (int c0 = cb; c0 < ce; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tacc + (uint32_t)c0, v);
#pragma unroll
        for (int i = 0; i < 16; i++) pc[(c0 + i) * kBM] = __uint_as_float(v[i]);
    }
    tc_fence_before();
}

// Values step 3 needs, loaded before the barrier so that no global round trip
// follows it: thread t keeps weight rows n .. n+3 (n = 4 (t % 32), kThreads is a
// multiple of 32) -- their scale and bias -- and the tile's activation row
// scales are staged in shared memory (`am`, RB floats).
struct ReducePrefetch {
    float rinv[4], bias[4];
};

template <int BN>
__device__ __forceinline__ void cluster_reduce_prefetch(const GemmArgs& g, ReducePrefetch& pf, float* am) {
    const int S = g.S, RB = BN / S, mt = (g.M + BN - 1) / BN;
    const int t = blockIdx.x / S, me = (int)cluster_rank();
    const int m0 = (t % mt) * BN + me * RB, n = (t / mt) * kBM + 4 * (threadIdx.x & 31);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        pf.rinv[i] = n + i < g.N ? 1.0f / __ldg(g.rowmul + n + i) : 0.0f;
        pf.bias[i] = (n + i < g.N && g.bias) ? __ldg(g.bias + n + i) : 0.0f;
    }
    if ((int)threadIdx.x < RB) am[threadIdx.x] = m0 + (int)threadIdx.x < g.M ? __ldg(g.ainv + m0 + threadIdx.x) : 0.0f;
}

template <int BN>
__device__ __forceinline__ void cluster_reduce_store(const GemmArgs& g, const float* P, const ReducePrefetch& pf,
                                                     const float* am) {
    const int S = g.S, RB = BN / S, mt = (g.M + BN - 1) / BN;
    const int t = blockIdx.x / S, me = (int)cluster_rank();
    const int m0 = (t % mt) * BN + me * RB, j = threadIdx.x & 31, n = (t / mt) * kBM + 4 * j;
    constexpr int kRowsPerPass = kThreads / 32;  // tile columns the CTA covers per item index
    const uint32_t pbase = smem_u32(P) + 16u * (uint32_t)j;
    uint32_t rbase[8];
#pragma unroll
    for (int sp = 0; sp < 8; sp++) rbase[sp] = sp < S ? dsmem_addr(pbase, (uint32_t)sp) : 0u;
#pragma unroll 1
    for (int c = me * RB + (int)(threadIdx.x >> 5); c < (me + 1) * RB; c += kRowsPerPass) {
        // all S partials of the item in flight before the first add
        const uint32_t off = (uint32_t)(c * kBM) * 4u;
        float4 x[8];
#pragma unroll
        for (int sp = 0; sp < 8; sp++)
            if (sp < S) x[sp] = ld_dsmem_f4(rbase[sp] + off);
        float4 acc = x[0];
#pragma unroll
        for (int sp = 1; sp < 8; sp++)
            if (sp < S) {
                acc.x += x[sp].x;
                acc.y += x[sp].y;
                acc.z += x[sp].z;
                acc.w += x[sp].w;
            }
        const int m = m0 - me * RB + c;
        if (m < g.M) {
            const float a = am[c - me * RB];
            const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
            float* o = g.out + (int64_t)m * g.ldo + n;
#pragma unroll
            for (int i = 0; i < 4; i++)
                if (n + i < g.N) o[i] = epi_value(g, a4[i], a * pf.rinv[i], pf.bias[i], m, n + i);
        }
    }
}

template <int QT, int BN, bool SIGNED>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ GemmArgs g) {
    constexpr int RK = (QT == VOXQ_Q4) ? 4 : 2;  // operand stages per raw stage
    constexpr int OB = ops_b(BN);
    constexpr int kRaw = raw_stages(BN);
    constexpr int kB = BN * kBK * 2;             // fp16 activation operand bytes
    constexpr int TC = BN < 32 ? 32 : BN;        // tensor-memory columns per accumulator
    constexpr uint32_t IDESC = umma_idesc(BN);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte aligned base, derived from the shared array by pointer arithmetic so
    // every access below stays a shared-memory access
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* opA = base;                 // kOpsA x 16 KB (fp16 weights, SW128)
    uint8_t* opB = opA + kOpsA * kA16;   // OB x kB (fp16 activations, SW128)
    uint8_t* raw = opB + OB * kB;        // kRaw x (codes SW128 + trailers)
    __shared__ uint64_t full_raw[kRaw], empty_raw[kRaw], full_a[kOpsA], empty_a[kOpsA], full_b[OB], empty_b[OB],
        acc_full[2], acc_empty[2];
    __shared__ uint32_t tmem_slot;
    __shared__ __align__(16) float ainv_s[kEpiWarps][2][kMaxBN / kEpiParts];  // epilogue: activation row scales

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KU = g.K / kBK;  // operand stages along K
    const int mt = (g.M + BN - 1) / BN, ntl = (g.N + kBM - 1) / kBM;
    const int S = g.S, KUs = g.KUs;
    const int units = mt * ntl * S;  // unit w: tile w / S, K split w % S

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRaw; i++) {
            mbar_init(&full_raw[i], 1);
            mbar_init(&empty_raw[i], kDeqWarps);
        }
        for (int i = 0; i < kOpsA; i++) {
            mbar_init(&full_a[i], kDeqWarps);
            mbar_init(&empty_a[i], 1);
        }
        for (int i = 0; i < OB; i++) {
            mbar_init(&full_b[i], 1);
            mbar_init(&empty_b[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kEpiWarps);
        }
        mbar_fence_init();
        // Weights never depend on earlier kernels: the first raw stages of this
        // CTA's first unit are requested right away, before tensor memory is
        // allocated and the CTA synchronises (the raw producer skips them).
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&g.tm_codes)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&g.tm_tr)) : "memory");
        if ((int)blockIdx.x < units) {
            const int w = blockIdx.x, t = w / S, u0 = (w % S) * KUs, u1 = min(KU, u0 + KUs);
            const int n0 = (t / mt) * kBM;
            int c = 0;
            for (int u = u0; u < u1 && c < kRaw; u += RK, c++) {
                mbar_arrive_expect_tx(&full_raw[c], kRawStage);
                uint8_t* rs = raw + c * kRawStage;
                tma_load_2d(rs, &g.tm_codes, (u / RK) * kRawRow, n0, &full_raw[c]);
                tma_load_2d(rs + kRawCodes, &g.tm_tr, (u / RK) * kRawTrRow, n0, &full_raw[c]);
            }
        }
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

    // The producer and MMA roles run their loops on the whole warp (every lane
    // takes the same waits, lane 0 alone issues), so each warp stays converged
    // and meets the final CTA barrier as one.
    if (warp == 0) {
        // ---------------- raw producer: weight codes + trailers ----------------
        // Weights never depend on the predecessor kernel, so this warp streams from
        // the start.  It has a ring of its own, so it runs ahead of the tensor core
        // by the full raw ring, independently of the activation ring.
        Ring rr;
        int early = 0;  // raw stages thread 0 already requested for the first unit
        if ((int)blockIdx.x < units) {
            const int u0 = (blockIdx.x % S) * KUs, u1 = min(KU, u0 + KUs);
            early = min(kRaw, (u1 - u0 + RK - 1) / RK);
        }
        for (int w = blockIdx.x; w < units; w += gridDim.x) {
            const int t = w / S, u0 = (w % S) * KUs, u1 = min(KU, u0 + KUs);
            const int n0 = (t / mt) * kBM;
            for (int u = u0; u < u1; u += RK) {  // u0 is a multiple of RK
                if ((int)rr.c < early) {
                    rr.c++;
                    continue;
                }
                const int s = rr.slot<kRaw>();
                if (rr.c >= kRaw) mbar_wait_bounded(&empty_raw[s], rr.phase<kRaw>() ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full_raw[s], kRawStage);
                    uint8_t* rs = raw + s * kRawStage;
                    tma_load_2d(rs, &g.tm_codes, (u / RK) * kRawRow, n0, &full_raw[s]);
                    tma_load_2d(rs + kRawCodes, &g.tm_tr, (u / RK) * kRawTrRow, n0, &full_raw[s]);
                }
                __syncwarp();
                rr.c++;
            }
        }
    } else if (warp == kBWarp) {
        // ---------------- activation producer ----------------
        // The fp16 activation images come from the prepass of this call, which
        // let this kernel start early: wait for it before the first load.
        pdl_wait();
        pdl_launch_dependents();
        Ring rb;
        for (int w = blockIdx.x; w < units; w += gridDim.x) {
            const int t = w / S, u0 = (w % S) * KUs, u1 = min(KU, u0 + KUs);
            const int mi = t % mt;
            const uint8_t* bsrc = g.a16t + (size_t)mi * KU * kB;
            for (int u = u0; u < u1; u++) {
                const int s = rb.slot<OB>();
                if (rb.c >= OB) mbar_wait_bounded(&empty_b[s], rb.phase<OB>() ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full_b[s], kB);
                    bulk_g2s(opB + s * kB, bsrc + (size_t)u * kB, kB, &full_b[s]);
                }
                __syncwarp();
                rb.c++;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        Ring ra, rb;
        int it = 0;
        for (int w = blockIdx.x; w < units; w += gridDim.x, it++) {
            const int u0 = (w % S) * KUs, u1 = min(KU, u0 + KUs);
            const int as = it & 1;
            if (it >= 2) mbar_wait_bounded(&acc_empty[as], ((it >> 1) & 1) ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
            tc_fence_after();
            const uint32_t acc = tmem + (uint32_t)(as * TC);
            for (int u = u0; u < u1; u++) {
                const int sa = ra.slot<kOpsA>(), sb = rb.slot<OB>();
                mbar_wait_bounded(&full_a[sa], ra.phase<kOpsA>(), VOXQ_DEVERR_WAIT_FULL, g.err);
                mbar_wait_bounded(&full_b[sb], rb.phase<OB>(), VOXQ_DEVERR_WAIT_FULL, g.err);
                tc_fence_after();
                if (lane == 0) {
                    const uint64_t ad = umma_desc(opA + sa * kA16);
                    const uint64_t bd = umma_desc(opB + sb * kB);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; kk++)  // +32 bytes = 16 fp16 along K
                        umma_f16(acc, ad + 2 * kk, bd + 2 * kk, IDESC, (u > u0 || kk > 0) ? 1u : 0u);
                    umma_commit(&empty_a[sa]);
                    umma_commit(&empty_b[sb]);
                }
                __syncwarp();
                ra.c++;
                rb.c++;
            }
            if (lane == 0) umma_commit(&acc_full[as]);
            __syncwarp();
        }
    } else if (warp < 2 + kDeqWarps) {
        // ---------------- dequant ----------------
        // Raw codes arrive 128-byte swizzled (16-byte chunk c of row r at
        // c ^ (r & 7)).  Thread -> (row, chunk): lane group g = lane / 8 takes row
        // b + {0, 4, 2, 6}[g] (+ 64 i), b = 8 (w / 2) + (w % 2) for dequant warp w.
        // The rows a half-warp reads then differ by 4 in (row & 7) (Q8: disjoint
        // swizzled chunk sets) and the 4 rows of a warp have distinct (row & 7) / 2
        // (Q4), so the shared-memory reads are free of bank conflicts.
        const int dw = warp - 2;
        const int j = lane & 7;  // 16-byte chunk (8 K values) of the 64-wide operand stage
        const int r0 = 8 * (dw >> 1) + (dw & 1) + ((0x6240 >> (4 * (lane >> 3))) & 0xF);
        // reads only weights (rowmul, codes via shared memory): no predecessor wait
        Ring rr, ra;
        constexpr int RPT = kBM * 8 / (kDeqWarps * 32);  // rows per thread and stage
        constexpr int RST = kBM / RPT;                     // row stride between them
        // row multipliers of the next unit's tile are fetched one unit ahead
        float rnext[RPT];
#pragma unroll
        for (int i = 0; i < RPT; i++) {
            const int n = (blockIdx.x / S / mt) * kBM + r0 + RST * i;
            rnext[i] = n < g.N ? ldg_ordered(g.rowmul + n) : 1.0f;
        }
        for (int w = blockIdx.x; w < units; w += gridDim.x) {
            const int u0 = (w % S) * KUs, u1 = min(KU, u0 + KUs);
            float rmul[RPT];
            const int wn = w + gridDim.x;
#pragma unroll
            for (int i = 0; i < RPT; i++) {
                rmul[i] = rnext[i];
                const int n = (wn / S / mt) * kBM + r0 + RST * i;
                rnext[i] = (wn < units && n < g.N) ? ldg_ordered(g.rowmul + n) : 1.0f;
            }
            for (int u = u0; u < u1; u++) {
                const int h = (u - u0) % RK;
                const bool last_use = (h == RK - 1) || (u == u1 - 1);
                const int s = rr.slot<kRaw>();
                if (h == 0) mbar_wait_bounded(&full_raw[s], rr.phase<kRaw>(), VOXQ_DEVERR_WAIT_FULL, g.err);
                const int sa = ra.slot<kOpsA>();
                if (ra.c >= kOpsA) mbar_wait_bounded(&empty_a[sa], ra.phase<kOpsA>() ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
                const uint32_t rc = smem_u32(raw) + s * kRawStage;
                const uint32_t rt = rc + kRawCodes;
                const uint32_t dstA = smem_u32(opA) + sa * kA16;
                const int blk = 2 * h + (j >> 2);  // 32-value block index within the raw stage
#pragma unroll
                for (int i = 0; i < RPT; i++) {
                    const int row = r0 + RST * i;
                    const int sw = row & 7;
                    float sc, mn;
                    uint32_t lo, hi = 0;
                    if (QT == VOXQ_Q8) {
                        // logical bytes 64 h + 8 j .. +8: chunk 4 h + j / 2, half j & 1
                        const uint2 c = lds64(rc + row * kRawRow + (((4 * h + (j >> 1)) ^ sw) << 4) + 8 * (j & 1));
                        lo = c.x;
                        hi = c.y;
                        const uint2 tr = lds64(rt + row * kRawTrRow + 8 * blk);
                        sc = __uint_as_float(tr.x);
                        mn = __uint_as_float(tr.y);
                    } else {
                        // logical bytes 32 h + 4 j .. +4: chunk 2 h + j / 4, word j & 3
                        lo = lds32(rc + row * kRawRow + (((2 * h + (j >> 2)) ^ sw) << 4) + 4 * (j & 3));
                        const uint32_t t = lds32(rt + row * kRawTrRow + 4 * blk);
                        const float2 tr = __half22float2(*reinterpret_cast<const __half2*>(&t));
                        sc = tr.x;
                        mn = tr.y;
                    }
                    const uint4 v = deq8<QT, SIGNED>(lo, hi, sc * rmul[i], mn * rmul[i]);
                    // K-major 128-byte swizzle: chunk j of row `row` lands at j ^ (row & 7)
                    sts128(dstA + row * 128 + ((j ^ sw) << 4), v);
                }
                // make the generic-proxy writes visible to the tensor core
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&full_a[sa]);
                    if (last_use) mbar_arrive(&empty_raw[s]);
                }
                ra.c++;
                if (last_use) rr.c++;
            }
        }
    } else if (warp < 2 + kDeqWarps + kEpiWarps) {
        // ---------------- epilogue ----------------
        if (g.cluster) {
            mbar_wait_sleepy(&acc_full[0], 0, VOXQ_DEVERR_WAIT_MMA, g.err);  // the one unit's accumulator
            tc_fence_after();
        } else {
            epilogue_role<BN, TC, 1, 2, kEpiParts>(g, tmem, acc_full, acc_empty, &ainv_s[0][0][0], units, mt, S,
                                                   warp - (2 + kDeqWarps), warp & 3, lane);
        }
    }
    if (g.cluster) {
        // split K inside the cluster (see cluster_park_partials): every thread
        // of every CTA takes both barriers and reduces
        float* P = reinterpret_cast<float*>(base);  // over the operand rings
        float* am_s = &ainv_s[0][0][0];             // the epilogue role's staging, unused in cluster mode
        if (warp >= 2 + kDeqWarps && warp < 2 + kDeqWarps + kEpiWarps)
            cluster_park_partials<BN, TC>(g, tmem, P, warp - (2 + kDeqWarps), warp & 3, lane);
        pdl_wait();  // the prepass's row scales; residual / gate / output of earlier work
        ReducePrefetch pf;
        cluster_reduce_prefetch<BN>(g, pf, am_s);
        cluster_sync_all();
        pdl_launch_dependents();
        cluster_reduce_store<BN>(g, P, pf, am_s);
        cluster_sync_all();
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
// Two-phase path for large M (the tensor core is the bound).  Phase 1 (one
// launch, one block of 128 threads per unit of work): the activation rows as
// in act_tile_kernel, and the weight dequantized once into fp16 rows
// w16[n][k] = fp16((q s + m) * rowmul[n]) with the same deq8 arithmetic as the
// fused kernel's dequant warps (identical values).  Phase 2: a plain
// TMA -> tcgen05 GEMM on the fp16 operands.  Dequantizing once per call
// instead of once per activation tile removes the dequant warps, their
// shared-memory round trip and proxy fences from the main loop.
// ---------------------------------------------------------------------------
template <int QT, bool SIGNED>
__global__ void __launch_bounds__(kPrepThreads) prep_f16_kernel(const float* __restrict__ a, int M, int K, int64_t lda,
                                                                int bn, uint8_t* __restrict__ a16t,
                                                                float* __restrict__ ainv, int act_rows,
                                                                const uint8_t* __restrict__ codes,
                                                                const uint8_t* __restrict__ scales,
                                                                const float* __restrict__ rowmul, int N,
                                                                __half* __restrict__ w16) {
    pdl_wait();  // activations may come from the previous kernel; w16 may still be read by it
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kPrepRows + (threadIdx.x >> 5);
    if (row < act_rows) {
        act_row(a, M, K, lda, bn, a16t, ainv, row, lane);
        return;
    }
    const int n = row - act_rows;
    if (n >= N) return;
    // Weight row n: lane l dequantizes the 8-weight chunks l, l + 32, ... (one
    // 16-byte fp16 chunk each), all of a group's codes and trailers loaded before
    // the first conversion.  Output layout: the shared-memory image of each
    // (256-row tile, 64-wide K stage) -- rows r of 128 bytes, 16-byte chunk j of
    // row r at j ^ (r & 7) -- contiguous, so the GEMM fetches a stage's weights
    // with one bulk copy.
    constexpr int RI = kRegIters;
    const int cpr = K / 8, KU = K / kBK;
    const int64_t rowb = codes_row_bytes(K, QT), srow = (int64_t)(K / VOXQ_QBLK) * scale_bytes(QT);
    const uint8_t* crow = codes + n * rowb;
    const uint8_t* srow_p = scales + n * srow;
    const float rm = __ldg(rowmul + n);
    const int tp = n / kW16Rows, r = n % kW16Rows;
    uint8_t* tb = reinterpret_cast<uint8_t*>(w16) + ((int64_t)tp * KU * kW16Rows + r) * 128;
    const int64_t ustride = (int64_t)kW16Rows * 128;
    for (int c0 = 0; c0 < cpr; c0 += 32 * RI) {
        uint32_t lo[RI], hi[RI];
        float2 tr[RI];
#pragma unroll
        for (int i = 0; i < RI; i++) {
            const int c = c0 + lane + 32 * i;  // block c / 4 of 32 weights
            lo[i] = hi[i] = 0u;
            tr[i] = make_float2(0.f, 0.f);
            if (c < cpr) {
                if (QT == VOXQ_Q8) {
                    const uint2 cw = __ldg(reinterpret_cast<const uint2*>(crow + 8 * c));
                    lo[i] = cw.x;
                    hi[i] = cw.y;
                    tr[i] = __ldg(reinterpret_cast<const float2*>(srow_p + 8 * (c >> 2)));
                } else {
                    lo[i] = __ldg(reinterpret_cast<const uint32_t*>(crow + 4 * c));
                    tr[i] = __half22float2(*reinterpret_cast<const __half2*>(srow_p + 4 * (c >> 2)));
                }
            }
        }
#pragma unroll
        for (int i = 0; i < RI; i++) {
            const int c = c0 + lane + 32 * i;
            if (c < cpr)
                *reinterpret_cast<uint4*>(tb + (c >> 3) * ustride + (((c & 7) ^ (r & 7)) << 4)) =
                    deq8<QT, SIGNED>(lo[i], hi[i], tr[i].x * rm, tr[i].y * rm);
        }
    }
}

// Two-phase GEMM kernel.  NT = 2: a tile is 256 weight rows (two 128-row
// sub-tiles, one accumulator each, sharing every activation stage) x BN
// activation rows, so a stage carries 64 KB for 8 MMAs (~1024 cycles) and three
// stages in flight cover the ~1.1-1.4 us TMA latency; the two accumulators fill
// tensor memory, so tiles do not overlap their epilogues (16 epilogue warps keep
// it short).  NT = 1: 128-row tiles with double-buffered accumulators.
constexpr int f16_epi_warps(int nt) { return nt == 2 ? 16 : 8; }
constexpr int f16_threads(int nt) { return (2 + f16_epi_warps(nt)) * 32; }
constexpr int f16_stages(int bn, int nt) { return nt == 2 ? 3 : bn >= 256 ? 4 : bn >= 128 ? 6 : 8; }
constexpr int f16_stage_bytes(int bn, int nt) { return nt * kA16 + bn * kBK * 2; }

template <int BN, int NT>
__global__ void __launch_bounds__(f16_threads(NT), 1) gemm_f16_kernel(const __grid_constant__ GemmArgs g) {
    constexpr int R = f16_stages(BN, NT);
    constexpr int kB = BN * kBK * 2;
    constexpr int STG = f16_stage_bytes(BN, NT);
    constexpr int TC = BN < 32 ? 32 : BN;
    constexpr int NACC = NT == 1 ? 2 : 1;
    constexpr int EPIW = f16_epi_warps(NT);
    constexpr int CP = EPIW / (4 * NT);  // column parts per sub-tile
    constexpr uint32_t IDESC = umma_idesc(BN);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // R x (A NT x 16 KB | B kB)
    __shared__ uint64_t full[R], empty[R], acc_full[NACC], acc_empty[NACC];
    __shared__ uint32_t tmem_slot;
    __shared__ __align__(16) float ainv_s[EPIW][2][kMaxBN / CP];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KU = g.K / kBK;
    const int mt = (g.M + BN - 1) / BN, ntl = (g.N + kBM * NT - 1) / (kBM * NT);
    const int S = g.S, KUs = g.KUs;
    const int units = mt * ntl * S;

    if (threadIdx.x == 0) {
        for (int i = 0; i < R; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < NACC; i++) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], EPIW);
        }
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(NACC * NT * TC)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        // ---------------- producer: both operands of a stage, one barrier ----------------
        pdl_wait();  // both operands come from the prepass of this call
        pdl_launch_dependents();
        Ring rr;
        for (int w = blockIdx.x; w < units; w += gridDim.x) {
            const int t = w / S, u0 = (w % S) * KUs, u1 = min(KU, u0 + KUs);
            const int mi = t % mt, n0 = (t / mt) * (kBM * NT);
            const uint8_t* bsrc = g.a16t + (size_t)mi * KU * kB;
            for (int u = u0; u < u1; u++) {
                const int s = rr.slot<R>();
                if (rr.c >= R) mbar_wait_bounded(&empty[s], rr.phase<R>() ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], STG);
                    uint8_t* st = base + s * STG;
                    // weights: rows n0 .. n0 + 128 NT of the tiled fp16 image (256-row tiles)
                    const uint8_t* wsrc = g.w16t + (((size_t)(n0 / kW16Rows) * KU + u) * kW16Rows +
                                                    (n0 % kW16Rows)) * 128;
                    bulk_g2s(st, wsrc, NT * kA16, &full[s]);
                    bulk_g2s(st + NT * kA16, bsrc + (size_t)u * kB, kB, &full[s]);
                }
                __syncwarp();
                rr.c++;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        Ring rr;
        int it = 0;
        for (int w = blockIdx.x; w < units; w += gridDim.x, it++) {
            const int u0 = (w % S) * KUs, u1 = min(KU, u0 + KUs);
            const int as = it % NACC;
            if (it >= NACC) mbar_wait_bounded(&acc_empty[as], ((it / NACC) & 1) ^ 1, VOXQ_DEVERR_WAIT_EMPTY, g.err);
            tc_fence_after();
            for (int u = u0; u < u1; u++) {
                const int s = rr.slot<R>();
                mbar_wait_bounded(&full[s], rr.phase<R>(), VOXQ_DEVERR_WAIT_FULL, g.err);
                tc_fence_after();
                if (lane == 0) {
                    const uint64_t bd = umma_desc(base + s * STG + NT * kA16);
#pragma unroll
                    for (int sub = 0; sub < NT; sub++) {
                        const uint64_t ad = umma_desc(base + s * STG + sub * kA16);
                        const uint32_t acc = tmem + (uint32_t)((as * NT + sub) * TC);
#pragma unroll
                        for (int kk = 0; kk < kBK / 16; kk++)
                            umma_f16(acc, ad + 2 * kk, bd + 2 * kk, IDESC, (u > u0 || kk > 0) ? 1u : 0u);
                    }
                    umma_commit(&empty[s]);
                }
                __syncwarp();
                rr.c++;
            }
            if (lane == 0) umma_commit(&acc_full[as]);
            __syncwarp();
        }
    } else {
        // ---------------- epilogue ----------------
        epilogue_role<BN, TC, NT, NACC, CP>(g, tmem, acc_full, acc_empty, &ainv_s[0][0][0], units, mt, S, warp - 2,
                                            warp & 3, lane);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(NACC * NT * TC)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// Split-K reduction: out[m, n] = epilogue(sum over splits k = 0 .. S-1 of
// part[t][k][m - m0][n - n0]), the splits added in order (deterministic).  One
// thread per 4 consecutive columns of one row; float4 loads of the partials.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const __grid_constant__ GemmArgs g, int bn) {
    pdl_wait();  // the GEMM's partials
    pdl_launch_dependents();
    const int mt = (g.M + bn - 1) / bn;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // over tiles x bn x 32
    const int c4 = (int)(idx & 31);
    const int64_t rt = idx >> 5;
    const int c = (int)(rt % bn);
    const int t = (int)(rt / bn);
    const int m = (t % mt) * bn + c, n = (t / mt) * kBM + 4 * c4;
    if (t >= mt * ((g.N + kBM - 1) / kBM) || m >= g.M || n >= g.N) return;
    const float* p = g.part + ((size_t)t * g.S * bn + c) * kBM + 4 * c4;
    float4 acc = __ldcg(reinterpret_cast<const float4*>(p));
    for (int k = 1; k < g.S; k++) {
        const float4 x = __ldcg(reinterpret_cast<const float4*>(p + (size_t)k * bn * kBM));
        acc.x += x.x;
        acc.y += x.y;
        acc.z += x.z;
        acc.w += x.w;
    }
    const float am = g.ainv[m];
    const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int nn = n + i;
        if (nn < g.N) {
            const float bias = g.bias ? g.bias[nn] : 0.0f;
            g.out[(int64_t)m * g.ldo + nn] = epi_value(g, a4[i], am / g.rowmul[nn], bias, m, nn);
        }
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

static int64_t pad_rows(int M) { return ((int64_t)M + kMaxBN - 1) / kMaxBN * kMaxBN; }

static size_t act_bytes(int M, int K) {
    return align256((size_t)pad_rows(M) * K * 2) + align256((size_t)pad_rows(M) * 4);
}

// Launch plan.  A 128 x N x 16 tcgen05.mma takes the same time for every
// N <= 256 (about 128 cycles), so a tile is as wide as the batch allows (BN =
// 256 once M > 128).  When the tiles cannot fill the SMs, the K range of each
// tile may be split over S CTAs (whole raw stages each); a reduction kernel then
// adds the S partials.  S minimises a simple model: per-CTA operand stages at
// ~0.3 us + pipeline fill, plus for S > 1 the partial traffic at ~4 TB/s and a
// launch.  VOXQ_GEMM_BN / VOXQ_GEMM_SPLIT override (tuning).
struct GemmPlan {
    int bn, S, KUs, tiles;
    bool two_phase;  // dequantize the weight once (prep_f16_kernel), then gemm_f16_kernel
    int nt;          // two-phase: 128-row weight sub-tiles per tile (1 or 2)
    bool cluster;    // fused kernel, the S K-splits of a tile in one cluster (partials in shared memory)
};

static int env_int(const char* name) {
    const char* e = getenv(name);
    return e ? atoi(e) : 0;
}

static int fused_occupancy(int qt, int bn);

static GemmPlan plan_gemm(int M, int N, int K, int qt) {
    static const int forced_bn = env_int("VOXQ_GEMM_BN"), forced_s = env_int("VOXQ_GEMM_SPLIT");
    // VOXQ_GEMM_TWO_PHASE: 1 two-phase at every M, -1 the fused kernel at every M,
    // unset: fused (cluster split K) for M <= 256, two-phase above
    static const int forced_path = env_int("VOXQ_GEMM_TWO_PHASE");
    static const int no_cluster = getenv("VOXQ_GEMM_CLUSTER") && env_int("VOXQ_GEMM_CLUSTER") == 0;
    GemmPlan p;
    p.cluster = false;
    // Batches above 128 rows: dequantizing the weight once per call (about
    // 2.6 B/weight of extra traffic) and running a plain TMA -> tcgen05 GEMM
    // beats the fused kernel's dequant pipeline, which repeats the dequant for
    // every activation tile.  Batches of up to 128 rows fit one activation tile:
    // the fused kernel dequantizes each weight byte exactly once and keeps its
    // K-split partials on chip (cluster), so neither the fp16 weight image nor
    // split-K partials reach HBM.  Measured on the config-3 shapes (CUDA-graph
    // replay, B200): M = 16 / 64 are 0.4 - 1.4 us faster than the two-phase
    // path; at M = 256 the cluster exchange of 128 KB of partials per CTA
    // (distributed shared memory moves ~20 GB/s per SM) makes it slower.
    p.two_phase = forced_path > 0 || (forced_path == 0 && M > 128);
    if (forced_bn == 16 || forced_bn == 32 || forced_bn == 64 || forced_bn == 128 || forced_bn == 256) {
        p.bn = forced_bn;
    } else {
        p.bn = 16;
        while (p.bn < M && p.bn < kMaxBN) p.bn *= 2;
    }
    const int KU = K / kBK, RK = (qt == VOXQ_Q4) ? 4 : 2;
    const int sms = device_sm_count();
    p.nt = 1;
    if (!p.two_phase && M <= p.bn && !no_cluster) {
        // one activation tile: cluster split K over up to 8 CTAs per weight tile,
        // as many as the co-resident CTAs allow
        p.tiles = (N + kBM - 1) / kBM;
        const int cap = sms * fused_occupancy(qt, p.bn);
        const int smax = min(8, KU / RK > 1 ? KU / RK : 1);
        int s = 1;
        if (forced_s > 0) {
            while (2 * s <= min(forced_s, smax)) s *= 2;
        } else {
            while (2 * s <= smax && p.tiles * 2 * s <= cap) s *= 2;
        }
        int kus = (KU + s - 1) / s;
        kus = (kus + RK - 1) / RK * RK;
        p.S = (KU + kus - 1) / kus;
        p.KUs = kus;
        p.cluster = p.S > 1 && p.bn >= p.S;
        if (p.cluster || p.S == 1) return p;
    }
    if (p.two_phase && p.bn == 256) {
        // 256-row tiles when they still cover most SMs (no split K with them)
        const int tiles2 = ((M + p.bn - 1) / p.bn) * ((N + 2 * kBM - 1) / (2 * kBM));
        if (tiles2 * 5 >= sms * 3) {
            p.nt = 2;
            p.tiles = tiles2;
            p.S = 1;
            p.KUs = KU;
            return p;
        }
    }
    p.tiles = ((M + p.bn - 1) / p.bn) * ((N + kBM - 1) / kBM);
    const int smax = KU / RK > 1 ? KU / RK : 1;
    double best = 1e30;
    p.S = 1;
    p.KUs = KU;
    for (int s = 1; s <= smax; s++) {
        if (forced_s > 0 && s != (forced_s < smax ? forced_s : smax)) continue;
        int kus = (KU + s - 1) / s;
        kus = (kus + RK - 1) / RK * RK;
        const int S = (KU + kus - 1) / kus;
        const int64_t units = (int64_t)p.tiles * S;
        const int64_t per_cta = (units + sms - 1) / sms;
        double t = (double)per_cta * kus * 0.3 + 1.5;
        if (S > 1) t += 1.0 + 2.0 * S * p.tiles * p.bn * kBM * 4.0 / 4.0e6;
        if (t < best - 1e-9) {
            best = t;
            p.S = S;
            p.KUs = kus;
        }
    }
    return p;
}

static size_t part_bytes(const GemmPlan& p) {
    return (p.S > 1 && !p.cluster) ? align256((size_t)p.S * p.tiles * p.bn * kBM * 4) : 0;
}

static size_t w16_bytes(const GemmPlan& p, int N, int K) {
    // tiled image: whole 256-row tiles (rows past N are never read: bulk copies
    // stop at the tile's last sub-tile, whose rows past N only feed discarded outputs)
    return p.two_phase ? align256((size_t)(N + kW16Rows - 1) / kW16Rows * kW16Rows * K * 2) : 0;
}

size_t gemm_workspace_bytes(int M, int N, int K, int qtype, bool swiglu) {
    // tiled fp16 activations + row scales, split-K partials, fp16 weight (two-phase)
    // (+ the SwiGLU gate result)
    const GemmPlan p = plan_gemm(M, N, K, qtype);
    return act_bytes(M, K) + part_bytes(p) + w16_bytes(p, N, K) + (swiglu ? align256((size_t)M * N * 4) : 0);
}

template <int QT, int BN, bool SIGNED>
struct FusedKernel {
    static constexpr int kB = BN * kBK * 2;
    static constexpr int smem = 1024 + kOpsA * kA16 + ops_b(BN) * kB + raw_stages(BN) * kRawStage;
    static constexpr int TC = BN < 32 ? 32 : BN;
    // co-resident CTAs per SM (shared memory and tensor memory), set once
    static int occupancy() {
        static int occ = 1;
        static std::once_flag once;
        std::call_once(once, [] {
            auto kern = gemm_kernel<QT, BN, SIGNED>;
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem);
            const int tmem_cap = 512 / (2 * TC);  // co-resident CTAs must fit tensor memory
            if (occ > tmem_cap) occ = tmem_cap;
            if (occ < 1) occ = 1;
        });
        return occ;
    }
};

static int fused_occupancy(int qt, int bn) {
#define VOXQ_OCC(B) \
    case B: return qt == VOXQ_Q4 ? FusedKernel<VOXQ_Q4, B, false>::occupancy() : FusedKernel<VOXQ_Q8, B, false>::occupancy();
    switch (bn) {
        VOXQ_OCC(16)
        VOXQ_OCC(32)
        VOXQ_OCC(64)
        VOXQ_OCC(128)
        default: return qt == VOXQ_Q4 ? FusedKernel<VOXQ_Q4, 256, false>::occupancy()
                                      : FusedKernel<VOXQ_Q8, 256, false>::occupancy();
    }
#undef VOXQ_OCC
}

template <int QT, int BN, bool SIGNED>
static VoxCPMError launch_gemm_t(const GemmArgs& a, cudaStream_t st) {
    using FK = FusedKernel<QT, BN, SIGNED>;
    static_assert(kOpsA * kA16 + ops_b(BN) * FK::kB >= BN * kBM * 4, "cluster partials must fit the operand rings");
    auto kern = gemm_kernel<QT, BN, SIGNED>;
    const int occ = FK::occupancy();
    const int units = ((a.M + BN - 1) / BN) * ((a.N + kBM - 1) / kBM) * a.S;
    const int cap = device_sm_count() * occ;
    cudaLaunchConfig_t cfg = {};
    // cluster split K: exactly one unit per CTA, S consecutive CTAs per cluster
    cfg.gridDim = dim3(a.cluster ? units : (units < cap ? units : cap));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = FK::smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = a.cluster ? (unsigned)a.S : 1u;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.cluster ? 2 : 1;
    VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
    return VOXCPM_SUCCESS;
}

template <int BN, int NT>
static VoxCPMError launch_f16_t(const GemmArgs& a, cudaStream_t st) {
    constexpr int smem = 1024 + f16_stages(BN, NT) * f16_stage_bytes(BN, NT);
    auto kern = gemm_f16_kernel<BN, NT>;
    static std::once_flag once;
    std::call_once(once, [&] { cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); });
    const int units = ((a.M + BN - 1) / BN) * ((a.N + kBM * NT - 1) / (kBM * NT)) * a.S;
    const int cap = device_sm_count();  // one CTA per SM (tensor memory)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(units < cap ? units : cap);
    cfg.blockDim = dim3(f16_threads(NT));
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

static VoxCPMError launch_f16(const GemmArgs& a, int bn, int nt, cudaStream_t st) {
    if (nt == 2) return launch_f16_t<256, 2>(a, st);
    switch (bn) {
        case 16: return launch_f16_t<16, 1>(a, st);
        case 32: return launch_f16_t<32, 1>(a, st);
        case 64: return launch_f16_t<64, 1>(a, st);
        case 128: return launch_f16_t<128, 1>(a, st);
        default: return launch_f16_t<256, 1>(a, st);
    }
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

static void pdl_config(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attr, cudaStream_t st) {
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
}

// One GEMM (+ split-K reduction): out = epilogue(A W^T) with optional gate
// (SwiGLU second half).
static VoxCPMError gemm_one(const GemmPlan& pl, const float* ainv, const uint8_t* a16t, int M, const voxq_qweight* w,
                            float* out, int64_t ldo, const float* bias, const float* residual, int64_t ldr,
                            const float* gate, int64_t ldg, float* part, const __half* w16, cudaStream_t st) {
    const int N = w->N, K = w->K, qt = w->qtype;
    static thread_local GemmArgs ga;
    const uint64_t rowb = (uint64_t)codes_row_bytes(K, qt);
    const uint64_t srow = (uint64_t)(K / VOXQ_QBLK) * scale_bytes(qt);
    ga.w16t = reinterpret_cast<const uint8_t*>(w16);
    if (!pl.two_phase && (!make_map(&ga.tm_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->codes, rowb, (uint64_t)N, rowb, kRawRow, kBM,
                         CU_TENSOR_MAP_SWIZZLE_128B) ||
               !make_map(&ga.tm_tr, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->scales, srow, (uint64_t)N, srow, kRawTrRow, kBM,
                         CU_TENSOR_MAP_SWIZZLE_NONE))) {
        return VOXCPM_ERR_INTERNAL;
    }
    ga.a16t = a16t;
    ga.rowmul = reinterpret_cast<const float*>(static_cast<const uint8_t*>(w->scales) + rowmul_offset(N, K, qt));
    ga.ainv = ainv;
    ga.out = out;
    ga.bias = bias;
    ga.residual = residual;
    ga.gate = gate;
    ga.part = part;
    ga.ldo = ldo;
    ga.ldr = ldr;
    ga.ldg = ldg;
    ga.M = M;
    ga.N = N;
    ga.K = K;
    ga.S = pl.S;
    ga.KUs = pl.KUs;
    ga.cluster = pl.cluster ? 1 : 0;
    ga.q8_signed = w->q8_signed;
    ga.err = device_error_word();
    const int bn = pl.bn;
    VoxCPMError e = pl.two_phase ? launch_f16(ga, bn, pl.nt, st)
                    : qt == VOXQ_Q4 ? launch_bn<VOXQ_Q4>(ga, bn, false, st)
                                    : launch_bn<VOXQ_Q8>(ga, bn, w->q8_signed != 0, st);
    if (e || pl.S == 1 || pl.cluster) return e;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    const int64_t threads = (int64_t)pl.tiles * bn * 32;
    cfg.gridDim = dim3((unsigned)((threads + 255) / 256));
    cfg.blockDim = dim3(256);
    pdl_config(cfg, attr, st);
    VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, splitk_reduce_kernel, ga, bn));
    return VOXCPM_SUCCESS;
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
    if (epi && epi->up && (epi->up->N != N || epi->up->K != K || epi->up->qtype != w->qtype))
        return VOXCPM_ERR_SHAPE_MISMATCH;
    const GemmPlan pl = plan_gemm(M, N, K, w->qtype);
    const int mpad = (M + pl.bn - 1) / pl.bn * pl.bn;
    // workspace: a16t | ainv | split-K partials | SwiGLU gate
    uint8_t* wsb = static_cast<uint8_t*>(ws);
    uint8_t* a16t = wsb;
    float* ainv = reinterpret_cast<float*>(wsb + align256((size_t)pad_rows(M) * K * 2));
    float* part = reinterpret_cast<float*>(wsb + act_bytes(M, K));
    __half* w16 = reinterpret_cast<__half*>(wsb + act_bytes(M, K) + part_bytes(pl));
    float* gbuf = reinterpret_cast<float*>(wsb + act_bytes(M, K) + part_bytes(pl) + w16_bytes(pl, N, K));
    // prepass: activations (+ for the two-phase plan, weight wq -> fp16), one launch
    auto prep = [&](const voxq_qweight* wq, bool act) -> VoxCPMError {
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        cfg.blockDim = dim3(kPrepThreads);
        pdl_config(cfg, attr, st);
        const int act_blocks = act ? mpad : 0;  // activation rows (one warp each)
        if (!pl.two_phase) {
            cfg.gridDim = dim3((unsigned)((mpad + kPrepRows - 1) / kPrepRows));
            VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, act_tile_kernel, a, M, K, lda, pl.bn, a16t, ainv, mpad));
            return VOXCPM_SUCCESS;
        }
        cfg.gridDim = dim3((unsigned)(((int64_t)act_blocks + N + kPrepRows - 1) / kPrepRows));
        const uint8_t* codes = static_cast<const uint8_t*>(wq->codes);
        const uint8_t* sc = static_cast<const uint8_t*>(wq->scales);
        const float* rm = reinterpret_cast<const float*>(sc + rowmul_offset(N, K, wq->qtype));
        if (wq->qtype == VOXQ_Q4)
            VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, prep_f16_kernel<VOXQ_Q4, false>, a, M, K, lda, pl.bn, a16t, ainv,
                                             act_blocks, codes, sc, rm, N, w16));
        else if (wq->q8_signed)
            VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, prep_f16_kernel<VOXQ_Q8, true>, a, M, K, lda, pl.bn, a16t, ainv,
                                             act_blocks, codes, sc, rm, N, w16));
        else
            VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, prep_f16_kernel<VOXQ_Q8, false>, a, M, K, lda, pl.bn, a16t, ainv,
                                             act_blocks, codes, sc, rm, N, w16));
        return VOXCPM_SUCCESS;
    };
    VoxCPMError e = prep(w, true);
    if (e) return e;
    const float* bias = epi ? epi->bias : nullptr;
    const float* res = epi ? epi->residual : nullptr;
    const int64_t ldr = epi ? epi->ldr : 0;
    if (epi && epi->up) {
        // SwiGLU: gate into the workspace, then up with silu(gate) * y fused
        e = gemm_one(pl, ainv, a16t, M, w, gbuf, N, nullptr, nullptr, 0, nullptr, 0, part, w16, st);
        if (e) return e;
        if (pl.two_phase) {  // the up weight replaces the gate weight in w16 once the gate GEMM is done
            e = prep(epi->up, false);
            if (e) return e;
        }
        return gemm_one(pl, ainv, a16t, M, epi->up, out, ldo, bias, res, ldr, gbuf, N, part, w16, st);
    }
    return gemm_one(pl, ainv, a16t, M, w, out, ldo, bias, res, ldr, nullptr, 0, part, w16, st);
}

}  // namespace voxq
