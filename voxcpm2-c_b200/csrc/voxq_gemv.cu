// voxq_gemv.cu -- quantized GEMV (M <= 8 activation rows) for sm_100a.
//
// out[m, n] = sum_k A[m, k] * W[n, k], W in the packed Q4/Q8 layout (voxq.h).
// This is the batch-1 decode regime of the reference's tensor_matmul_nt
// (src/tensor.c:617-678): every weight byte is read once, so the kernel is
// HBM-bound and is built to stream with as few instructions per weight as
// possible.
//
// Exact integer formulation.  Each 16-byte chunk of a weight row holds 32 Q4
// codes (one quantization block) or 16 Q8 codes (half a block).  The matching
// activation chunk x is split once, by a prepass kernel, into three int8
// limbs with per-chunk scales d1, d2 = d1/254, d3 = d2/254:
//     x ~= d1*l1 + d2*l2 + d3*l3,  |l_i| <= 127,  error <= d3/2 (~2^-21 |x|max)
// so the chunk's code dot product is three exact integer dot products, each a
// dp4a per 4 codes on the raw code bytes (Q4 nibbles are split with one LOP3
// per 4 codes; the prepass stores the limbs in the matching even/odd order).
// Per chunk and row:
//     y += scale * (d1*S1 + d2*S2 + d3*S3) + min * sum(x)
// -- the dequantized weight q*scale+min is never formed.
//
// Streaming.  A tile is T consecutive rows of one item (16 KB of codes, one
// contiguous range, plus their contiguous trailers).  One producer warp per
// CTA streams tiles into a 4-deep shared-memory ring with two cp.async.bulk
// copies each; 8 consumer warps each take groups of RG rows x one 512-byte
// K-slab (32 lanes x 16 B), so activation limbs loaded once serve RG rows.
// Rows longer than one slab are split across warps and their partial sums
// combined in shared memory behind one named barrier per tile.  CTAs own
// contiguous tile ranges, so consecutive tiles share an item and its limbs
// stay in L1.  The producer starts streaming before the kernel waits on its
// predecessor: that predecessor is the limb prepass of the same call, or (the
// tensor-path kernel, which splits its activations itself) whatever kernel ran
// before; none of the library's kernels that write packed weights (quantize,
// pack, rowmul) lets a dependent start early, so every weight write before
// the call is complete when the stream reaches it.
#include <mutex>

#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

// Tuning knobs (overridable at build time): consumer warps per CTA (+1
// producer warp) and ring depth.  A stage holds kConsumers groups of 4 rows x
// one 512-byte slab, i.e. kConsumers * 2 KB of codes.
#ifndef VOXQ_GEMV_CONSUMERS
#define VOXQ_GEMV_CONSUMERS 8
#endif
#ifndef VOXQ_GEMV_STAGES
#define VOXQ_GEMV_STAGES 4
#endif
constexpr int kConsumers = VOXQ_GEMV_CONSUMERS;
constexpr int kStages = VOXQ_GEMV_STAGES;
constexpr int kTile = kConsumers * 4 * 512;  // code bytes per stage (all weights of the tile)

// Per-chunk limb record, in 16-byte granules laid out [m][granule][chunk] so a
// warp reading granule g of 32 consecutive chunks issues one coalesced 512-B load.
//   Q4 (32 codes): granules 0..5 = limb L (0..2) x {odd codes, even codes}
//                  words j = 0..3 hold the limbs of elements 8j+1,3,5,7 (odd)
//                  or 8j+0,2,4,6 (even); granule 6 = (d1, d2, d3, sum x)
//   Q8 (16 codes): granules 0..2 = limb L, bytes in element order;
//                  granule 3 = (d1, d2, d3, sum x)
__host__ __device__ constexpr int limb_granules(int qtype) { return qtype == VOXQ_Q4 ? 7 : 4; }

struct LimbJob {
    const float* a;
    uint4* dst;
    int32_t M, lda, chunks;  // chunks per activation row
    int32_t chunk_begin;     // prefix over jobs of M * chunks
};

constexpr int kMaxJobs = VOXQ_MAX_BATCH;
struct LimbParams {
    int32_t count, total, qtype, pad;
    LimbJob job[kMaxJobs];
};

__device__ __forceinline__ int8_t rint_clamp127(float v) {
    float r = rintf(v);
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    return (int8_t)(int)r;
}

// One thread's share of one chunk's limb record: the chunk's TPC threads (Q4
// chunks of 32 values: 4 threads, Q8 chunks of 16 values: 2 threads; `part` =
// this thread's index, 8 consecutive values each) sit in one warp and reduce
// the chunk max / sum by shuffles, so every lane of the warp must call this
// (threads past the end with live = false).  `base` = granule 0 of the chunk,
// granules `gstride` bytes apart.
template <int QT>
__device__ __forceinline__ void limb_part(const float* __restrict__ xrow, int c, int part, bool live, uint8_t* base,
                                          int64_t gstride) {
    constexpr int TPC = QT == VOXQ_Q4 ? 4 : 2;
    constexpr int G = limb_granules(QT);
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (live) {
        const float* x = xrow + (int64_t)c * (8 * TPC) + part * 8;
        const float4 f0 = *reinterpret_cast<const float4*>(x);
        const float4 f1 = *reinterpret_cast<const float4*>(x + 4);
        v[0] = f0.x; v[1] = f0.y; v[2] = f0.z; v[3] = f0.w;
        v[4] = f1.x; v[5] = f1.y; v[6] = f1.z; v[7] = f1.w;
    }
    float amax = 0.0f, sum = 0.0f, asum = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        amax = fmaxf(amax, fabsf(v[i]));
        sum += v[i];
        asum += fabsf(v[i]);
    }
#pragma unroll
    for (int o = 1; o < TPC; o <<= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        sum += __shfl_xor_sync(0xffffffffu, sum, o);
        asum += __shfl_xor_sync(0xffffffffu, asum, o);
    }
    if (!live) return;
    // d1: power of two with amax / d1 <= 127 (exact scaling); d2, d3 refine.
    float d1 = 1.0f;
    if (amax > 0.0f && isfinite(amax)) {
        int e;
        frexpf(amax * (1.0f / 127.0f), &e);
        d1 = ldexpf(1.0f, e);
        if (amax > 127.0f * d1) d1 *= 2.0f;
    }
    const float inv1 = 1.0f / d1;  // exact: power of two
    const float d2 = d1 * (1.0f / 254.0f), d3 = d2 * (1.0f / 254.0f);
    // Two limbs leave an error of at most ~3e-5 * amax per value; a chunk
    // whose magnitude is spread (amax <= 5 * mean |x|) keeps that far below
    // the matmul tolerance, so its third limb is dropped (d3 = 0).
    const bool need3 = amax * (8 * TPC) > 5.0f * asum;
    int8_t l[3][8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float r = v[i];
        const float a = fminf(fmaxf(rintf(r * inv1), -127.0f), 127.0f);
        r = fmaf(-a, d1, r);
        const float b = fminf(fmaxf(rintf(r * (254.0f * inv1)), -127.0f), 127.0f);
        r = fmaf(-b, d2, r);
        const float cc = need3 ? fminf(fmaxf(rintf(r * (64516.0f * inv1)), -127.0f), 127.0f) : 0.0f;
        l[0][i] = (int8_t)(int)a;
        l[1][i] = (int8_t)(int)b;
        l[2][i] = (int8_t)(int)cc;
    }
    auto pack4 = [](int8_t a, int8_t b, int8_t c2, int8_t d) -> uint32_t {
        return (uint32_t)(uint8_t)a | ((uint32_t)(uint8_t)b << 8) | ((uint32_t)(uint8_t)c2 << 16) |
               ((uint32_t)(uint8_t)d << 24);
    };
#pragma unroll
    for (int L = 0; L < 3; L++) {
        if (QT == VOXQ_Q4) {
            // this thread's 8 values are code word `part` of the chunk
            *reinterpret_cast<uint32_t*>(base + (2 * L) * gstride + 4 * part) = pack4(l[L][1], l[L][3], l[L][5], l[L][7]);
            *reinterpret_cast<uint32_t*>(base + (2 * L + 1) * gstride + 4 * part) =
                pack4(l[L][0], l[L][2], l[L][4], l[L][6]);
        } else {
            *reinterpret_cast<uint2*>(base + L * gstride + 8 * part) =
                make_uint2(pack4(l[L][0], l[L][1], l[L][2], l[L][3]), pack4(l[L][4], l[L][5], l[L][6], l[L][7]));
        }
    }
    if (part == 0)
        *reinterpret_cast<uint4*>(base + (G - 1) * gstride) = make_uint4(
            __float_as_uint(d1), __float_as_uint(d2), __float_as_uint(need3 ? d3 : 0.0f), __float_as_uint(sum));
}

// Limb prepass of the dp4a GEMV: one thread per 8 consecutive activation
// values of every job, written to the global limb records.
template <int QT>
__global__ void __launch_bounds__(256) limb_kernel(const __grid_constant__ LimbParams p) {
    pdl_wait();  // the activations may come from the previous kernel
    pdl_launch_dependents();
    constexpr int TPC = QT == VOXQ_Q4 ? 4 : 2;  // threads per chunk
    constexpr int G = limb_granules(QT);
    int j = 0;
    // every chunk's threads sit in one warp (TPC divides 32), and the loop
    // stride is a multiple of 32, so shuffles stay within live groups
    const int total = p.total * TPC;
    const int span = (total + 31) & ~31;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < span; t += gridDim.x * blockDim.x) {
        const bool live = t < total;
        const int cidx = live ? t / TPC : 0;  // global chunk index
        const int part = t % TPC;
        if (j + 1 < p.count && cidx >= p.job[j + 1].chunk_begin) {
            int lo = j + 1, hi = p.count - 1;  // last job with chunk_begin <= cidx
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (p.job[mid].chunk_begin <= cidx) lo = mid; else hi = mid - 1;
            }
            j = lo;
        }
        const LimbJob& jb = p.job[j];
        const int local = cidx - jb.chunk_begin;
        const int m = local / jb.chunks, c = local % jb.chunks;
        limb_part<QT>(jb.a + (int64_t)m * jb.lda, c, part, live,
                      reinterpret_cast<uint8_t*>(jb.dst + (int64_t)m * G * jb.chunks + c), (int64_t)jb.chunks * 16);
    }
}

struct GemvItemDev {
    const uint8_t* codes;
    const uint8_t* scales;
    const uint8_t* up_codes;
    const uint8_t* up_scales;
    const uint4* limbs;  // [M][granule][chunks]
    float* out;
    const float* bias;
    const float* residual;
    int32_t N, K, M, ldo, ldr;
    int32_t rowb;        // code bytes per row
    int32_t srow;        // trailer bytes per row
    int32_t chunks;      // 16-byte code chunks per row
    int32_t slabs;       // ceil(chunks / 32)
    int32_t T;           // rows per tile
    int32_t tile_begin;  // first global tile of this item
    int32_t parts;       // tensor-path kernel: K parts of groups_per_part 4-chunk groups
    int32_t lda;         // tensor-path kernel: activation row stride (elements)
    const float* a;      // tensor-path kernel: the activation row (limbs computed in the kernel)
};

template <int MAXI>
struct GemvParams {
    int32_t count;
    int32_t total_tiles;
    int32_t limb_bytes;  // tensor-path kernel: largest item's limb record (shared-memory buffer)
    int32_t first_weight;  // tensor-path kernel: per-mille share weight of the grid's first half (1000: even)
    int* err;
    GemvItemDev it[MAXI];
};

__device__ __forceinline__ uint32_t dp4a_us(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t dp4a_ss(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory"); }

// Reduces V values per lane across the warp.  Afterwards value v (0 <= v < V)
// is complete in lanes v * (32 / V) .. v * (32 / V) + 32 / V - 1.
template <int V>
__device__ __forceinline__ float transpose_reduce(float (&v)[V], int lane) {
#pragma unroll
    for (int s = 0; s < 5; s++) {
        const int off = 16 >> s;
        const int n = V >> s;  // values still held per lane before this step
        if (n > 1) {
            const bool upper = (lane & off) != 0;
#pragma unroll
            for (int i = 0; i < n / 2; i++) {
                const float send = upper ? v[i] : v[i + n / 2];
                const float keep = upper ? v[i + n / 2] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
        }
    }
    return v[0];
}

template <int MAXI>
__device__ __forceinline__ void fix_item(const GemvParams<MAXI>& p, int tile, int& item) {
    while (item + 1 < p.count && tile >= p.it[item + 1].tile_begin) item++;
}

// Producer (lane 0 of the producer warp): streams the tiles [tb, te) into a
// STAGES-deep ring, two cp.async.bulk copies per weight and stage (codes of
// the tile's T rows, then the 16-byte aligned window of their trailers).
template <int STAGES, int TILE, int TW, int NW, int MAXI>
__device__ __forceinline__ void produce_tiles(const GemvParams<MAXI>& p, int tb, int te, uint64_t* full,
                                              uint64_t* empty, uint8_t* smem) {
    constexpr int CW = TILE / NW;
    constexpr int STAGE = TILE + NW * TW;
    int item = 0;
    for (int t = tb, j = 0; t < te; ++t, ++j) {
        fix_item(p, t, item);
        const GemvItemDev& it = p.it[item];
        const int s = j % STAGES;
        if (j >= STAGES) mbar_wait_bounded(&empty[s], ((j / STAGES) & 1) ^ 1, VOXQ_DEVERR_WAIT_EMPTY, p.err);
        const int row0 = (t - it.tile_begin) * it.T;
        const int rows = min(it.T, it.N - row0);
        const uint32_t cb = (uint32_t)(rows * it.rowb);
        const int64_t so = (int64_t)row0 * it.srow;
        const int64_t sa = so & ~(int64_t)15;
        const uint32_t tbytes = (uint32_t)(((so - sa) + (int64_t)rows * it.srow + 15) & ~(int64_t)15);
        mbar_arrive_expect_tx(&full[s], NW * (cb + tbytes));
        uint8_t* st = smem + s * STAGE;
#pragma unroll
        for (int w = 0; w < NW; w++) {
            const uint8_t* c = w ? it.up_codes : it.codes;
            const uint8_t* sc = w ? it.up_scales : it.scales;
            bulk_g2s(st + w * CW, c + (int64_t)row0 * it.rowb, cb, &full[s]);
            bulk_g2s(st + TILE + w * TW, sc + sa, tbytes, &full[s]);
        }
    }
    // Normally the consumers have waited for every copy.  If a wait gave up,
    // give the copies still in flight a bounded moment to land before the
    // CTA's shared memory is released.
    if (*reinterpret_cast<volatile int*>(p.err) != 0) {
        const int n = te - tb;
        for (int j = (n > STAGES ? n - STAGES : 0); j < n; j++)
            mbar_wait_bounded(&full[j % STAGES], (j / STAGES) & 1, VOXQ_DEVERR_WAIT_FULL, p.err, 20u);
    }
}

// Epilogue of one finished output element.
__device__ __forceinline__ void write_out(const GemvItemDev& it, int n, int m, float v) {
    if (it.bias) v += it.bias[n];
    if (it.residual) v += it.residual[(int64_t)m * it.ldr + n];
    it.out[(int64_t)m * it.ldo + n] = v;
}


// Accumulates one chunk's contribution for RG rows x NW weights of activation
// row m, with NLIMB int8 limbs of the activation (compile-time, so the unused
// third limb costs no instructions).
template <int QT, int NW, int RG, int MT, int NLIMB, bool SIGNED>
__device__ __forceinline__ void chunk_dot(const uint32_t (&ca)[NW][RG][(QT == VOXQ_Q4) ? 8 : 4],
                                          const float (&sc)[NW][RG], const float (&mn)[NW][RG], const uint4* lp,
                                          int chunks, float d1, float d2, float d3, float xs, bool live, int m,
                                          float (&acc)[NW][RG][MT]) {
    constexpr int NL = (QT == VOXQ_Q4) ? 8 : 4;
    uint32_t lw[NLIMB][NL];
#pragma unroll
    for (int L = 0; L < NLIMB; L++) {
        if (QT == VOXQ_Q4) {
            const uint4 o = __ldg(lp + (int64_t)(2 * L) * chunks);
            const uint4 e = __ldg(lp + (int64_t)(2 * L + 1) * chunks);
            lw[L][0] = o.x; lw[L][1] = o.y; lw[L][2] = o.z; lw[L][3] = o.w;
            lw[L][4 % NL] = e.x; lw[L][5 % NL] = e.y; lw[L][6 % NL] = e.z; lw[L][7 % NL] = e.w;
        } else {
            const uint4 o = __ldg(lp + (int64_t)L * chunks);
            lw[L][0] = o.x; lw[L][1] = o.y; lw[L][2] = o.z; lw[L][3] = o.w;
        }
    }
#pragma unroll
    for (int w = 0; w < NW; w++)
#pragma unroll
        for (int r = 0; r < RG; r++) {
            int SL[NLIMB];
#pragma unroll
            for (int L = NLIMB - 1; L >= 0; L--) {
                uint32_t so = 0u, se = 0u;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    if (QT == VOXQ_Q4) {
                        so = dp4a_us(ca[w][r][q], lw[L][q], so);
                        se = dp4a_us(ca[w][r][4 + q % 4], lw[L][4 + q % 4], se);
                    } else {
                        so = SIGNED ? dp4a_ss(ca[w][r][q], lw[L][q], so) : dp4a_us(ca[w][r][q], lw[L][q], so);
                    }
                }
                // Q4: 16 * (odd + even) = 16 * odd + (16 * even)
                const int S = (QT == VOXQ_Q4) ? (int)(se + (so << 4)) : (int)so;
                SL[L] = S;
            }
            // d1 = 254 d2 up to one rounding of d2, so d1 S1 + d2 S2 = d2 (254 S1 + S2);
            // 254 S1 + S2 stays well inside int32 (|S| < 2^20 for a 16-byte chunk)
            float dot = d2 * (float)(SL[0] * 254 + SL[1]);
            if (NLIMB == 3) dot = fmaf(d3, (float)SL[NLIMB - 1], dot);
            const float a2 = fmaf(sc[w][r], dot, fmaf(mn[w][r], xs, acc[w][r][m]));
            acc[w][r][m] = live ? a2 : acc[w][r][m];
        }
}

template <int QT, int MT, int RG, bool SWI, bool SIGNED, int MAXI>
__global__ void __launch_bounds__((kConsumers + 1) * 32) gemv_kernel(const __grid_constant__ GemvParams<MAXI> p) {
    constexpr int NW = SWI ? 2 : 1;  // weights per row (gate, up)
    constexpr int G = limb_granules(QT);
    constexpr int V = RG * MT;
    constexpr int NL = (QT == VOXQ_Q4) ? 8 : 4;   // limb words per chunk and limb
    constexpr int SB = (QT == VOXQ_Q4) ? 4 : 8;   // trailer bytes per block
    constexpr int CW = kTile / NW;                 // code bytes per weight per stage
    constexpr int TW = CW / 4 + 32;                // trailer window bytes per weight
    constexpr int STAGE = kTile + NW * TW;
    constexpr int PART_G = 32;                     // groups per tile when rows span > 1 slab (host-checked)

    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kStages], empty[kStages];
    __shared__ float part[kStages][PART_G][NW][V];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumers);
        }
    }
    mbar_fence_init();
    __syncthreads();

    const int tb = (int)((int64_t)p.total_tiles * blockIdx.x / gridDim.x);
    const int te = (int)((int64_t)p.total_tiles * (blockIdx.x + 1) / gridDim.x);

    if (warp == kConsumers) {
        if (lane == 0) produce_tiles<kStages, kTile, TW, NW>(p, tb, te, full, empty, smem);
        pdl_launch_dependents();
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait();  // limbs come from the prepass launched just before this kernel
    pdl_launch_dependents();
    int item = 0;
    for (int t = tb, j = 0; t < te; ++t, ++j) {
        fix_item(p, t, item);
        const GemvItemDev& it = p.it[item];
        const int s = j % kStages;
        // a wait that gives up records the error and the tile is processed
        // anyway (garbage), so every warp still meets the same barriers
        mbar_wait_bounded(&full[s], (j / kStages) & 1, VOXQ_DEVERR_WAIT_FULL, p.err);
        const uint8_t* st = smem + s * STAGE;
        const int row0 = (t - it.tile_begin) * it.T;
        const int rows = min(it.T, it.N - row0);
        const int delta = (int)(((int64_t)row0 * it.srow) & 15);
        const int SL = it.slabs;
        const int ngroups = ((rows + RG - 1) / RG) * SL;

        // group g = (row group rgi, slab sl), g = warp, warp + kConsumers, ...
        int sl = warp % SL, rgi = warp / SL;
        for (int g = warp; g < ngroups; g += kConsumers) {
            const int chunk0 = sl * 32 + lane;
            const bool live = chunk0 < it.chunks;  // a row's last slab may be partial
            const int chunk = live ? chunk0 : it.chunks - 1;
            float acc[NW][RG][MT];
#pragma unroll
            for (int w = 0; w < NW; w++)
#pragma unroll
                for (int r = 0; r < RG; r++)
#pragma unroll
                    for (int m = 0; m < MT; m++) acc[w][r][m] = 0.0f;
            // codes -> dp4a operands.  Q4 bytes hold (even << 4 | odd): the odd
            // codes are `w & 0x0F..`, the even ones stay in place as 16 * code.
            uint32_t ca[NW][RG][NL];
            float sc[NW][RG], mn[NW][RG];
            const int blk = (QT == VOXQ_Q4) ? chunk : (chunk >> 1);
#pragma unroll
            for (int w = 0; w < NW; w++)
#pragma unroll
                for (int r = 0; r < RG; r++) {
                    const int lr = min(rgi * RG + r, rows - 1);
                    const uint4 c = *reinterpret_cast<const uint4*>(st + w * CW + lr * it.rowb + chunk * 16);
                    const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        if (QT == VOXQ_Q4) {
                            ca[w][r][q] = wd[q] & 0x0F0F0F0Fu;
                            ca[w][r][4 + q % 4] = wd[q] & 0xF0F0F0F0u;
                        } else {
                            ca[w][r][q] = wd[q];
                        }
                    }
                    const uint8_t* tp = st + kTile + w * TW + delta + lr * it.srow + blk * SB;
                    if (QT == VOXQ_Q4) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(tp));
                        sc[w][r] = f.x;
                        mn[w][r] = f.y;
                    } else {
                        const float2 tv = *reinterpret_cast<const float2*>(tp);
                        sc[w][r] = tv.x;
                        mn[w][r] = tv.y;
                    }
                }
#pragma unroll
            for (int m = 0; m < MT; m++) {
                const int mm = m < it.M ? m : it.M - 1;
                const uint4* lp = it.limbs + (int64_t)mm * G * it.chunks + chunk;
                const uint4 dd = __ldg(lp + (int64_t)(G - 1) * it.chunks);
                const float k = (QT == VOXQ_Q4) ? 0.0625f : 1.0f;  // Q4 sums are 16x
                const float d1 = __uint_as_float(dd.x) * k, d2 = __uint_as_float(dd.y) * k;
                const float d3 = __uint_as_float(dd.z) * k, xs = __uint_as_float(dd.w);
                // the third limb only where some lane's chunk needs it
                const bool use3 = __any_sync(0xffffffffu, live && dd.z != 0u);
                if (use3)
                    chunk_dot<QT, NW, RG, MT, 3, SIGNED>(ca, sc, mn, lp, it.chunks, d1, d2, d3, xs, live, m, acc);
                else
                    chunk_dot<QT, NW, RG, MT, 2, SIGNED>(ca, sc, mn, lp, it.chunks, d1, d2, d3, xs, live, m, acc);
            }
            // reduce the group's RG x MT sums across the lanes
            float red[NW];
#pragma unroll
            for (int w = 0; w < NW; w++) {
                float v[V];
#pragma unroll
                for (int r = 0; r < RG; r++)
#pragma unroll
                    for (int m = 0; m < MT; m++) v[r * MT + m] = acc[w][r][m];
                red[w] = transpose_reduce<V>(v, lane);
            }
            constexpr int LPV = 32 / V;
            if ((lane & (LPV - 1)) == 0) {
                const int v = lane / LPV;
                if (SL == 1) {
                    const int n = row0 + rgi * RG + v / MT, m = v % MT;
                    if (rgi * RG + v / MT < rows && m < it.M)
                        write_out(it, n, m, SWI ? silu(red[0]) * red[NW - 1] : red[0]);
                } else {
#pragma unroll
                    for (int w = 0; w < NW; w++) part[s][g][w][v] = red[w];
                }
            }
            sl += kConsumers;
            while (sl >= SL) {
                sl -= SL;
                rgi++;
            }
        }
        if (SL > 1) {
            // rows span several slabs: combine the slab partial sums
            consumer_bar();
            const int nrg = (rows + RG - 1) / RG;
            for (int e = warp * 32 + lane; e < nrg * V; e += kConsumers * 32) {
                const int rgi = e / V, v = e % V;
                float sum[NW];
#pragma unroll
                for (int w = 0; w < NW; w++) {
                    sum[w] = 0.0f;
                    for (int sl = 0; sl < SL; sl++) sum[w] += part[s][rgi * SL + sl][w][v];
                }
                const int r = rgi * RG + v / MT, m = v % MT;
                if (r < rows && m < it.M) write_out(it, row0 + r, m, SWI ? silu(sum[0]) * sum[NW - 1] : sum[0]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

// ---------------------------------------------------------------------------
// Single-row GEMV (M = 1, one weight per item) on the integer tensor path.
//
// The same exact limb formulation, with the integer dot products done by
// mma.sync.m16n8k32 (u8 or s8 codes x s8 limbs, s32 accumulate) instead of
// dp4a.  A tile of the MMA is 16 weight rows x 32 K-slots; lane (g, t) of
// the warp (g = lane / 4, t = lane % 4) supplies the A bytes of rows g and
// g + 8 for slots 4t .. 4t+3 and 16+4t .. 16+4t+3.  Each lane takes ONE
// 16-byte code chunk c = 4 * group + t of those rows, so the four lanes t
// of a group cover four consecutive chunks.  The activation limbs go into B
// block-diagonally: column 2t + L holds limb L of chunk t on the slots of
// lane t and zeros elsewhere, so D[row][2t + L] is exactly chunk t's limb-L
// dot product -- the per-chunk scales and per-block trailers are applied to
// the D fragment that lane t itself holds (c0, c1: row g; c2, c3: row g + 8).
//   Q4 chunk (32 codes): words j, j+1 give one MMA on their odd codes
//     (w & 0x0F0F0F0F) and one on 16 x their even codes (w & 0xF0F0F0F0),
//     into separate accumulators (16 S = 16 D_odd + D_even, exact); the limb
//     record stores the odd / even limbs of each word in the same order.
//     Four MMAs per chunk.
//   Q8 chunk (16 codes): words 2j, 2j+1 are a0, a2 as they are.  Two MMAs.
// The third limb (rare: chunks with a dominant value) is a second block-
// diagonal B in column 2t, issued only when a lane of the warp needs it.
//
// The limbs are computed by the kernel itself: when a CTA's tile range enters
// a new item, its consumer warps split the item's activation row into a
// shared-memory record (chunk-major; the arithmetic of the dp4a kernel's
// prepass, limb_part), so no prepass launch precedes this kernel.
//
// A stage holds T rows (at most 32 KB of codes) in two halves (split_tile);
// two stages per CTA and two CTAs per SM, whose tiles run out of phase.
// K is cut into fixed parts of
// groups_per_part groups (four chunks each); a stage's work is (16-row tile,
// K part) units spread over the 8 consumer warps, and each row's parts are
// summed in part order through shared memory.  The summation order depends
// only on K, not on T, so the launch may pick T (smaller tiles for small
// launches) without changing a single bit of the result.
// ---------------------------------------------------------------------------
#ifndef VOXQ_GEMV_MMA_WARPS
#define VOXQ_GEMV_MMA_WARPS 8
#endif
constexpr int kMmaWarps = VOXQ_GEMV_MMA_WARPS;   // consumer warps (+1 producer)
#ifndef VOXQ_GEMV_MMA_STAGES
#define VOXQ_GEMV_MMA_STAGES 2
#endif
#ifndef VOXQ_GEMV_MMA_MINB
#define VOXQ_GEMV_MMA_MINB 2  // CTAs per SM the register budget is sized for
#endif
constexpr int kMmaStages = VOXQ_GEMV_MMA_STAGES;
constexpr int kMmaTile = 32768;                  // code bytes per stage
constexpr int kMmaTW = kMmaTile / 4 + 32;        // trailer window bytes per stage
// A stage: the code region (two halves of the tile's rows, see split_tile)
// and the trailer region, each with room for the gap between the halves.
constexpr int kMmaCodeRgn = kMmaTile + 256;
constexpr int kMmaTrRgn = kMmaTW + 256;
constexpr int kMmaStage = kMmaCodeRgn + kMmaTrRgn;
constexpr int kMmaSmem = kMmaStages * kMmaStage;
constexpr int kMmaLimbMax = 16384;               // limb record of the largest item (K <= 4096)
// groups (four 16-byte chunks of a row) per K part: 256 bytes of Q4 codes, 128 of Q8
__host__ __device__ constexpr int groups_per_part(int qtype) { return qtype == VOXQ_Q4 ? 4 : 2; }
constexpr int kPartSlots = 256;                 // >= T x parts (T x rowb <= kMmaTile)

template <bool SA>
__device__ __forceinline__ void imma16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    if (SA)
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%0,%1,%2,%3};"
                     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                     : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%0,%1,%2,%3};"
                     : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                     : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The chunk's code dot products with one limb set: D += codes x B, where this
// lane's B words are bw (Q4: 4 odd-code words then 4 even-code words; Q8: 4
// words in element order) or zero.
template <int QT, bool SIGNED>
__device__ __forceinline__ void chunk_mma(int (&d)[4], const uint4& wa, const uint4& wb, const uint32_t (&bw)[8]) {
    const uint32_t xa[4] = {wa.x, wa.y, wa.z, wa.w}, xb[4] = {wb.x, wb.y, wb.z, wb.w};
    if (QT == VOXQ_Q4) {
        int dh[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
            imma16832<false>(d, xa[j] & 0x0F0F0F0Fu, xb[j] & 0x0F0F0F0Fu, xa[j + 1] & 0x0F0F0F0Fu,
                             xb[j + 1] & 0x0F0F0F0Fu, bw[j], bw[j + 1]);
            imma16832<false>(dh, xa[j] & 0xF0F0F0F0u, xb[j] & 0xF0F0F0F0u, xa[j + 1] & 0xF0F0F0F0u,
                             xb[j + 1] & 0xF0F0F0F0u, bw[4 + j], bw[5 + j]);
        }
        // 16 x (odd + even) sums
#pragma unroll
        for (int i = 0; i < 4; i++) d[i] = dh[i] + (d[i] << 4);
    } else {
#pragma unroll
        for (int j = 0; j < 2; j++) imma16832<SIGNED>(d, xa[2 * j], xb[2 * j], xa[2 * j + 1], xb[2 * j + 1], bw[2 * j], bw[2 * j + 1]);
    }
}

// Limb L (0 .. 2) of this lane's chunk from the item's shared-memory limb
// record (chunk address lp, granules gstride bytes apart), or zeros from a
// zero block.
template <int QT>
__device__ __forceinline__ void load_limbs(uint32_t (&bw)[8], uint32_t lp, uint32_t gstride, int L, bool on,
                                           uint32_t zaddr) {
    const uint32_t po = on ? lp + (uint32_t)((QT == VOXQ_Q4) ? 2 * L : L) * gstride : zaddr;
    const uint4 o = lds128(po);
    bw[0] = o.x; bw[1] = o.y; bw[2] = o.z; bw[3] = o.w;
    if (QT == VOXQ_Q4) {
        const uint4 e = lds128(on ? po + gstride : zaddr + 16);
        bw[4] = e.x; bw[5] = e.y; bw[6] = e.z; bw[7] = e.w;
    } else {
        bw[4] = bw[5] = bw[6] = bw[7] = 0u;
    }
}

// How a tile's rows sit in a stage: the first acnt = min(8 nrt, rows) rows
// (half A) and the rest (half B) are copied to regions whose starts differ by
// 64 bytes modulo 128, for the codes and for the trailers.  The consumer gives
// the even lanes of a quad group rows of half A and the odd lanes rows of half
// B, so the two rows one quarter-warp reads sit in different banks (rows of one
// half are a multiple of 128 bytes apart for the usual K).
struct SplitTile {
    int acnt;                  // rows in half A
    int cB;                    // start of half B's codes in the code region
    int tdA, tB;               // trailer region: half A's offset of row 0; start of half B's window
    int tdB;                   // half B's offset of its row 0 in its window
    uint32_t cbA, cbB, tbA, tbB;
    int64_t saA, saB;          // 16-byte aligned trailer sources
};
__device__ __forceinline__ SplitTile split_tile(int row0, int rows, int rowb, int srow) {
    SplitTile x;
    const int nrt = (rows + 15) >> 4;
    x.acnt = min(nrt * 8, rows);
    x.cbA = (uint32_t)(x.acnt * rowb);
    x.cbB = (uint32_t)((rows - x.acnt) * rowb);
    x.cB = (int)((x.cbA + 127) & ~127u) + 64;
    const int64_t soA = (int64_t)row0 * srow, soB = (int64_t)(row0 + x.acnt) * srow;
    x.saA = soA & ~(int64_t)15;
    x.saB = soB & ~(int64_t)15;
    x.tdA = (int)(soA - x.saA);
    x.tdB = (int)(soB - x.saB);
    x.tbA = (uint32_t)((x.tdA + x.acnt * srow + 15) & ~15);
    x.tbB = rows > x.acnt ? (uint32_t)((x.tdB + (rows - x.acnt) * srow + 15) & ~15) : 0u;
    x.tB = (int)((x.tbA + 127) & ~127u) + 64;
    return x;
}

// Producer of the tensor-path kernel (lane 0 of the producer warp): up to
// four bulk copies per tile (codes and trailers of each half).
template <int MAXI>
__device__ __forceinline__ void produce_split(const GemvParams<MAXI>& p, int tb, int te, uint64_t* full,
                                              uint64_t* empty, uint8_t* smem) {
    int item = 0;
    for (int t = tb, j = 0; t < te; ++t, ++j) {
        fix_item(p, t, item);
        const GemvItemDev& it = p.it[item];
        const int s = j % kMmaStages;
        if (j >= kMmaStages) mbar_wait_bounded(&empty[s], ((j / kMmaStages) & 1) ^ 1, VOXQ_DEVERR_WAIT_EMPTY, p.err);
        const int row0 = (t - it.tile_begin) * it.T;
        const int rows = min(it.T, it.N - row0);
        const SplitTile x = split_tile(row0, rows, it.rowb, it.srow);
        mbar_arrive_expect_tx(&full[s], x.cbA + x.cbB + x.tbA + x.tbB);
        uint8_t* st = smem + s * kMmaStage;
        bulk_g2s(st, it.codes + (int64_t)row0 * it.rowb, x.cbA, &full[s]);
        bulk_g2s(st + kMmaCodeRgn, it.scales + x.saA, x.tbA, &full[s]);
        if (x.cbB) {
            bulk_g2s(st + x.cB, it.codes + (int64_t)(row0 + x.acnt) * it.rowb, x.cbB, &full[s]);
            bulk_g2s(st + kMmaCodeRgn + x.tB, it.scales + x.saB, x.tbB, &full[s]);
        }
    }
    // Normally the consumers have waited for every copy.  If a wait gave up,
    // give the copies still in flight a bounded moment to land before the
    // CTA's shared memory is released.
    if (*reinterpret_cast<volatile int*>(p.err) != 0) {
        const int n = te - tb;
        for (int j = (n > kMmaStages ? n - kMmaStages : 0); j < n; j++)
            mbar_wait_bounded(&full[j % kMmaStages], (j / kMmaStages) & 1, VOXQ_DEVERR_WAIT_FULL, p.err, 20u);
    }
}

// TRX (Q4, every item's trailer rows a multiple of 16 bytes): trailers handed
// to the lanes through a per-warp scratch (see the unit loop).
template <int QT, bool SIGNED, bool TRX, int MAXI>
__global__ void __launch_bounds__((kMmaWarps + 1) * 32, VOXQ_GEMV_MMA_MINB) gemv_mma_kernel(const __grid_constant__ GemvParams<MAXI> p) {
    constexpr int G = limb_granules(QT);
    constexpr int SB = (QT == VOXQ_Q4) ? 4 : 8;  // trailer bytes per block
    constexpr int STAGE = kMmaStage;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kMmaStages], empty[kMmaStages];
    // row sums of each (row tile, K part) unit; two sets, alternating between
    // the tiles that combine parts, so a set is rewritten only after every
    // warp has passed the next combining tile's barrier
    __shared__ float part[2][kPartSlots];  // [row][K part] of a stage's rows
    __shared__ __align__(16) uint32_t trx[TRX ? kMmaWarps : 1][2][8 * 20];
    __shared__ __align__(16) uint4 zlimb[2];  // B of the lanes that feed no limb
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kMmaStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kMmaWarps);
        }
        zlimb[0] = zlimb[1] = make_uint4(0u, 0u, 0u, 0u);
    }
    mbar_fence_init();
    __syncthreads();

    // Contiguous tile ranges, the first half of the grid weighted by
    // first_weight / 1000 against the second: with two CTAs per SM the block
    // scheduler gives every SM one CTA of each half, and the SM's first CTA
    // gets more issue slots than its second, so equal ranges would leave the
    // second CTA running alone at the end.
    const int64_t H = gridDim.x / 2, w1 = p.first_weight, w2 = 1000;
    const int64_t wsum = H * w1 + ((int64_t)gridDim.x - H) * w2;
    auto wpos = [&](int64_t b) { return b <= H ? b * w1 : H * w1 + (b - H) * w2; };
    const int tb = (int)((int64_t)p.total_tiles * wpos(blockIdx.x) / wsum);
    const int te = (int)((int64_t)p.total_tiles * wpos(blockIdx.x + 1) / wsum);

    if (warp == kMmaWarps) {
        if (lane == 0) produce_split(p, tb, te, full, empty, smem);
        pdl_launch_dependents();
        return;
    }

    pdl_wait();  // the activations may come from the previous kernel
    pdl_launch_dependents();
    const int g = lane >> 2, tq = lane & 3;
    const int L = g - 2 * tq;  // limb this lane feeds into B (column 2t + L), if 0 or 1
    const bool limb_lane = (unsigned)L < 2u;
    // the current item's limb records, [chunk][granule] (16 bytes each): a chunk's
    // granules in consecutive banks, so the two limb lanes of a quad read theirs
    // without conflict
    const uint32_t limb_s = smem_u32(smem + kMmaStages * STAGE), zaddr = smem_u32(&zlimb[0]);
    int item = -1, pset = 0;
    // per-item constants (refreshed when the tile range enters a new item)
    int P = 1, rt0 = 0, kp0 = 0, ngr = 1, chunks = 1, rowb = 0, srow = 0, T = 1, N = 0, tbeg = 0;
    for (int t = tb, j = 0; t < te; ++t, ++j) {
        int nitem = item < 0 ? 0 : item;
        fix_item(p, t, nitem);
        if (nitem != item) {
            item = nitem;
            const GemvItemDev& it = p.it[item];
            P = it.parts;
            rt0 = warp / P;  // this warp's first unit
            kp0 = warp % P;
            chunks = it.chunks;
            ngr = (chunks + 3) >> 2;
            rowb = it.rowb;
            srow = it.srow;
            T = it.T;
            N = it.N;
            tbeg = it.tile_begin;
            // The item's activation row split into limbs (the prepass arithmetic,
            // limb_part) into the shared buffer, once every consumer warp is done
            // with the previous item's; the producer keeps streaming meanwhile.
            asm volatile("bar.sync 1, %0;" ::"n"(kMmaWarps * 32) : "memory");
            {
                constexpr int TPC = QT == VOXQ_Q4 ? 4 : 2;
                const int total = chunks * TPC, span = (total + 31) & ~31;
                for (int q = warp * 32 + lane; q < span; q += kMmaWarps * 32) {
                    const bool live = q < total;
                    const int c = live ? q / TPC : 0;
                    limb_part<QT>(it.a, c, q % TPC, live, smem + kMmaStages * STAGE + c * (G * 16), 16);
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(kMmaWarps * 32) : "memory");
        }
        const int s = j % kMmaStages;
        // a wait that gives up records the error and the tile is processed
        // anyway (garbage), so every warp still meets the same barriers
        mbar_wait_bounded(&full[s], (j / kMmaStages) & 1, VOXQ_DEVERR_WAIT_FULL, p.err);
        const uint8_t* st = smem + s * STAGE;
        const int row0 = (t - tbeg) * T;
        const int rows = min(T, N - row0);
        const int nrt = (rows + 15) >> 4;  // 16-row tiles
        const SplitTile x = split_tile(row0, rows, rowb, srow);
        // this lane's half: even g -> half A, odd g -> half B (half A when B is empty)
        const int half = g & 1;
        const int hcnt = half ? rows - x.acnt : x.acnt;
        const bool inB = half && hcnt > 0;
        const int hc = inB ? hcnt : x.acnt;
        const uint8_t* hcode = st + (inB ? x.cB : 0);
        const uint8_t* htr = st + kMmaCodeRgn + (inB ? x.tB + x.tdB : x.tdA);
        const int hbase = half ? x.acnt : 0;  // tile row of the half's row 0
        for (int rt = rt0, kp = kp0; rt < nrt;) {
            // MMA rows g and g + 8 = rows i1 and i1 + 4 of this lane's half
            const int i1 = rt * 8 + (g >> 1), i2 = i1 + 4;
            const int c1 = min(i1, hc - 1), c2 = min(i2, hc - 1);
            const uint8_t* pa = hcode + c1 * rowb;
            const uint8_t* pb = hcode + c2 * rowb;
            const uint8_t* ta = htr + c1 * srow;
            const uint8_t* tb2 = htr + c2 * srow;
            float accA = 0.0f, accB = 0.0f;
            constexpr int GPP = groups_per_part(QT);
            if (TRX) {
                // The unit's trailers: lane t reads 16-byte chunk (first group + t) of
                // its two rows (blocks 4k .. 4k+3) and the warp hands element t of
                // chunk i to the lanes t of group i through a scratch with a 20-word
                // row pitch (conflict-free reads).  One wide read per row instead of
                // one narrow read per group, each of which hits the same banks for
                // all eight rows.
                const int k = min(kp * GPP + tq, ngr - 1);
                const uint4 xa = *reinterpret_cast<const uint4*>(ta + 16 * k);
                const uint4 xb = *reinterpret_cast<const uint4*>(tb2 + 16 * k);
                __syncwarp();
                *reinterpret_cast<uint4*>(&trx[warp][0][g * 20 + tq * 4]) = xa;
                *reinterpret_cast<uint4*>(&trx[warp][1][g * 20 + tq * 4]) = xb;
                __syncwarp();
            }
            const int g1 = min(ngr, (kp + 1) * GPP);
#pragma unroll
            for (int gr = kp * GPP; gr < g1; gr++) {
                const int c = gr * 4 + tq;  // this lane's chunk
                const bool cok = c < chunks;
                const int cc = cok ? c : chunks - 1;
                const uint4 wa = *reinterpret_cast<const uint4*>(pa + cc * 16);
                const uint4 wb = *reinterpret_cast<const uint4*>(pb + cc * 16);
                const uint32_t lp = limb_s + (uint32_t)cc * (G * 16);  // this chunk's granule 0
                constexpr uint32_t gs = 16;
                const uint4 rec = lds128(lp + (G - 1) * gs);
                uint32_t bw[8];
                load_limbs<QT>(bw, lp, gs, L, cok && limb_lane, zaddr);
                int d[4] = {0, 0, 0, 0};
                chunk_mma<QT, SIGNED>(d, wa, wb, bw);
                int d3v[4] = {0, 0, 0, 0};
                const bool use3 = __any_sync(0xffffffffu, cok && rec.z != 0u);
                if (use3) {
                    load_limbs<QT>(bw, lp, gs, 2, cok && L == 0, zaddr);
                    chunk_mma<QT, SIGNED>(d3v, wa, wb, bw);
                }
                if (cok) {
                    const float kq = (QT == VOXQ_Q4) ? 0.0625f : 1.0f;  // Q4 sums are 16x
                    const float d2 = __uint_as_float(rec.y) * kq, d3 = __uint_as_float(rec.z) * kq;
                    const float xs = __uint_as_float(rec.w);
                    const int blk = (QT == VOXQ_Q4) ? c : (c >> 1);
                    float sa, ma, sb, mb;
                    if (QT == VOXQ_Q4) {
                        const int ii = gr - kp * GPP;
                        const void* sa_p = TRX ? (const void*)&trx[warp][0][g * 20 + ii * 4 + tq] : (const void*)(ta + blk * SB);
                        const void* sb_p = TRX ? (const void*)&trx[warp][1][g * 20 + ii * 4 + tq] : (const void*)(tb2 + blk * SB);
                        const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(sa_p));
                        const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(sb_p));
                        sa = fa.x; ma = fa.y; sb = fb.x; mb = fb.y;
                    } else {
                        const float2 fa = *reinterpret_cast<const float2*>(ta + blk * SB);
                        const float2 fb = *reinterpret_cast<const float2*>(tb2 + blk * SB);
                        sa = fa.x; ma = fa.y; sb = fb.x; mb = fb.y;
                    }
                    // d1 = 254 d2 up to one rounding of d2: d1 S1 + d2 S2 = d2 (254 S1 + S2)
                    float dotA = d2 * (float)(d[0] * 254 + d[1]);
                    float dotB = d2 * (float)(d[2] * 254 + d[3]);
                    if (use3) {
                        dotA = fmaf(d3, (float)d3v[0], dotA);
                        dotB = fmaf(d3, (float)d3v[2], dotB);
                    }
                    accA = fmaf(sa, dotA, fmaf(ma, xs, accA));
                    accB = fmaf(sb, dotB, fmaf(mb, xs, accB));
                }
            }
            // the four chunk lanes of each row pair
            accA += __shfl_xor_sync(0xffffffffu, accA, 1);
            accB += __shfl_xor_sync(0xffffffffu, accB, 1);
            accA += __shfl_xor_sync(0xffffffffu, accA, 2);
            accB += __shfl_xor_sync(0xffffffffu, accB, 2);
            if (tq == 0) {
                const int ra = hbase + i1, rb = hbase + i2;  // tile rows
                const bool oka = i1 < hcnt, okb = i2 < hcnt;
                if (P == 1) {
                    const GemvItemDev& it = p.it[item];
                    if (oka) write_out(it, row0 + ra, 0, accA);
                    if (okb) write_out(it, row0 + rb, 0, accB);
                } else {
                    if (oka) part[pset][ra * P + kp] = accA;
                    if (okb) part[pset][rb * P + kp] = accB;
                }
            }
            // next unit of this warp: kMmaWarps units further in (row tile, part) order
            kp += kMmaWarps;
            while (kp >= P) {
                kp -= P;
                rt++;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (P > 1) {
            // K parts of each row, summed in part order
            asm volatile("bar.sync 1, %0;" ::"n"(kMmaWarps * 32) : "memory");
            for (int r = warp * 32 + lane; r < rows; r += kMmaWarps * 32) {
                float sum = 0.0f;
                for (int kp = 0; kp < P; kp++) sum += part[pset][r * P + kp];
                write_out(p.it[item], row0 + r, 0, sum);
            }
            pset ^= 1;
        }
    }
}

// Rows per consumer group for each activation-row count.
template <int MT, bool SWI>
struct Shape {
    static constexpr int RG = (MT * (SWI ? 2 : 1) <= 2) ? 4 : 2;
};
static int rows_per_group(int mt, bool swi) { return (mt * (swi ? 2 : 1) <= 2) ? 4 : 2; }

template <int QT, int MT, bool SWI, bool SIGNED, int MAXI>
static VoxCPMError launch_t(const GemvParams<MAXI>& p, cudaStream_t st) {
    constexpr int RG = Shape<MT, SWI>::RG;
    constexpr int NW = SWI ? 2 : 1;
    constexpr int smem = kStages * (kTile + NW * (kTile / NW / 4 + 32));
    auto kern = gemv_kernel<QT, MT, RG, SWI, SIGNED, MAXI>;
    static int occ = 0;
    static std::once_flag once;
    std::call_once(once, [&] {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, (kConsumers + 1) * 32, smem);
    });
    const int cap = device_sm_count() * (occ > 0 ? occ : 1);
    const int blocks = p.total_tiles < cap ? p.total_tiles : cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks < 1 ? 1 : blocks);
    cfg.blockDim = dim3((kConsumers + 1) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
    return VOXCPM_SUCCESS;
}

template <int QT, bool SIGNED, bool TRX, int MAXI>
static VoxCPMError launch_mma_t(GemvParams<MAXI>& p, cudaStream_t st) {
    auto kern = gemv_mma_kernel<QT, SIGNED, TRX, MAXI>;
    // occupancy for each limb-buffer size, in 1 KB steps
    static int occ[kMmaLimbMax / 1024 + 1] = {};
    static std::once_flag once;
    std::call_once(once, [&] {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaSmem + kMmaLimbMax);
    });
    const int lk = (p.limb_bytes + 1023) / 1024;
    const int smem = kMmaSmem + lk * 1024;
    if (occ[lk] == 0) cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ[lk], kern, (kMmaWarps + 1) * 32, smem);
    const int cap = device_sm_count() * (occ[lk] > 0 ? occ[lk] : 1);
    const int blocks = p.total_tiles < cap ? p.total_tiles : cap;
    // Weighted ranges only when the grid is two full CTAs per SM (one CTA of
    // each half on every SM); otherwise even ranges.  1.2 : 1 measured best on
    // a B200 for the config-2 step (1.0: 56.8 us, 1.15: 55.3, 1.2: 54.7, 1.25:
    // 54.3, 1.3: 57.2); VOXQ_GEMV_FIRST_WEIGHT (per mille) overrides.
    static const int weight = [] {
        const char* e = getenv("VOXQ_GEMV_FIRST_WEIGHT");
        const int v = e ? atoi(e) : 1200;
        return v >= 500 && v <= 3000 ? v : 1200;
    }();
    p.first_weight = (occ[lk] == 2 && blocks == cap) ? weight : 1000;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks < 1 ? 1 : blocks);
    cfg.blockDim = dim3((kMmaWarps + 1) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
    return VOXCPM_SUCCESS;
}

static int round_mt(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

// The tensor-path kernel serves single-row launches without SwiGLU
// (VOXQ_GEMV_MMA=0 selects the dp4a kernel instead, for comparison).
static bool mma_path(int mt, bool swi) {
    static const bool on = [] {
        const char* e = getenv("VOXQ_GEMV_MMA");
        return !(e && e[0] == '0');
    }();
    return on && mt == 1 && !swi;
}

// Items the tensor-path kernel takes: single-row, no SwiGLU, and a limb record
// (computed in the kernel) that fits its shared-memory buffer (K <= 4096).
static bool mma_item(const voxq_gemv_item& x) {
    const int64_t rec = (int64_t)codes_row_bytes(x.w.K, x.w.qtype) / 16 * limb_granules(x.w.qtype) * 16;
    return mma_path(round_mt(x.M), x.up_codes != nullptr) && rec <= kMmaLimbMax;
}

template <int MAXI>
static VoxCPMError dispatch(GemvParams<MAXI>& p, int qtype, int mt, bool swi, bool sgn, bool mma,
                            cudaStream_t st) {
    if (mma) {
        if (qtype == VOXQ_Q4) {
            bool trx = true;  // every item's trailer rows in whole 16-byte chunks
            for (int i = 0; i < p.count; i++) trx = trx && (p.it[i].srow & 15) == 0;
            return trx ? launch_mma_t<VOXQ_Q4, false, true, MAXI>(p, st) : launch_mma_t<VOXQ_Q4, false, false, MAXI>(p, st);
        }
        if (qtype == VOXQ_Q8)
            return sgn ? launch_mma_t<VOXQ_Q8, true, false, MAXI>(p, st) : launch_mma_t<VOXQ_Q8, false, false, MAXI>(p, st);
        return VOXCPM_ERR_UNSUPPORTED;
    }
#define VOXQ_GEMV_CASE(QT, MT)                                                                          \
    if (qtype == QT && mt == MT) {                                                                      \
        if (swi) return sgn ? launch_t<QT, MT, true, true, MAXI>(p, st) : launch_t<QT, MT, true, false, MAXI>(p, st); \
        return sgn ? launch_t<QT, MT, false, true, MAXI>(p, st) : launch_t<QT, MT, false, false, MAXI>(p, st);      \
    }
    VOXQ_GEMV_CASE(VOXQ_Q4, 1)
    VOXQ_GEMV_CASE(VOXQ_Q4, 2)
    VOXQ_GEMV_CASE(VOXQ_Q4, 4)
    VOXQ_GEMV_CASE(VOXQ_Q4, 8)
    VOXQ_GEMV_CASE(VOXQ_Q8, 1)
    VOXQ_GEMV_CASE(VOXQ_Q8, 2)
    VOXQ_GEMV_CASE(VOXQ_Q8, 4)
    VOXQ_GEMV_CASE(VOXQ_Q8, 8)
#undef VOXQ_GEMV_CASE
    return VOXCPM_ERR_UNSUPPORTED;
}


VoxCPMError validate_item(const voxq_gemv_item& x) {
    const voxq_qweight& w = x.w;
    if (w.qtype != VOXQ_Q4 && w.qtype != VOXQ_Q8) return VOXCPM_ERR_UNSUPPORTED;
    if (w.N < 0 || w.K < 0 || w.K % VOXQ_QBLK || x.M < 0 || x.M > 8) return VOXCPM_ERR_SHAPE_MISMATCH;
    if (w.N == 0 || x.M == 0) return VOXCPM_SUCCESS;
    if (!x.a || !x.out || (w.K > 0 && (!w.codes || !w.scales))) return VOXCPM_ERR_INTERNAL;
    if (x.lda < w.K || x.ldo < w.N || (x.residual && x.ldr < w.N)) return VOXCPM_ERR_SHAPE_MISMATCH;
    // a row of codes must fit one stage (K <= 16384 for Q8, 32768 for Q4; half that with SwiGLU)
    if (codes_row_bytes(w.K, w.qtype) * (x.up_codes ? 2 : 1) > kTile) return VOXCPM_ERR_UNSUPPORTED;
    // 16-byte activation loads, 16-byte aligned code and trailer arrays
    if ((reinterpret_cast<uintptr_t>(x.a) & 15) || (x.lda & 3)) return VOXCPM_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(w.codes) & 15) || (reinterpret_cast<uintptr_t>(w.scales) & 15))
        return VOXCPM_ERR_UNSUPPORTED;
    if (x.up_codes && ((reinterpret_cast<uintptr_t>(x.up_codes) & 15) ||
                       (reinterpret_cast<uintptr_t>(x.up_scales) & 15) || !x.up_scales))
        return VOXCPM_ERR_UNSUPPORTED;
    return VOXCPM_SUCCESS;
}

// Bytes of the limb workspace for one activation (M rows, K columns).
static size_t limb_bytes(int M, int K, int qtype) {
    const int chunks = (int)(codes_row_bytes(K, qtype) / 16);
    return (size_t)M * limb_granules(qtype) * chunks * 16;
}

// Launches the items that share (qtype, swiglu, signed): one limb prepass for
// their distinct activations, then one GEMV grid.
template <int MAXI>
static VoxCPMError launch_items(const voxq_gemv_item* const* sel, int n, cudaStream_t st, void* ws, size_t ws_bytes,
                                int* err) {
    static thread_local GemvParams<MAXI> p;
    static thread_local LimbParams lp;
    const voxq_gemv_item& f = *sel[0];
    const int qt = f.w.qtype;
    int mt = 1;
    for (int i = 0; i < n; i++) mt = max(mt, round_mt(sel[i]->M));
    const bool swi = f.up_codes != nullptr;
    const int nw = swi ? 2 : 1;
    const bool use_mma = mma_item(f);  // uniform within a group (see gemv_launch_ws)
    int limb_max = 0;

    // distinct activations -> limb jobs (the tensor-path kernel computes its own)
    struct Act { const float* a; int M, lda, K; uint4* dst; };
    Act acts[VOXQ_MAX_BATCH];
    int nact = 0;
    size_t off = 0;
    int c = 0, tiles = 0;
    for (int i = 0; i < n; i++) {
        const voxq_gemv_item& x = *sel[i];
        if (x.w.N == 0 || x.M == 0) continue;
        if (x.w.K == 0) {  // empty reduction: out = epilogue(0)
            VoxCPMError e = gemv_k0(x, st);
            if (e) return e;
            continue;
        }
        int ai = -1;
        for (int k = 0; k < nact; k++)
            if (acts[k].a == x.a && acts[k].M == x.M && acts[k].lda == x.lda && acts[k].K == x.w.K) ai = k;
        if (ai < 0 && !use_mma) {
            const size_t b = limb_bytes(x.M, x.w.K, qt);
            if (off + b > ws_bytes) return VOXCPM_ERR_OOM;
            acts[nact] = {x.a, x.M, x.lda, x.w.K, reinterpret_cast<uint4*>(static_cast<uint8_t*>(ws) + off)};
            off += (b + 255) & ~(size_t)255;
            ai = nact++;
        }
        GemvItemDev& d = p.it[c];
        d.codes = x.w.codes;
        d.scales = reinterpret_cast<const uint8_t*>(x.w.scales);
        d.up_codes = x.up_codes;
        d.up_scales = reinterpret_cast<const uint8_t*>(x.up_scales);
        d.limbs = use_mma ? nullptr : acts[ai].dst;
        d.a = x.a;
        d.lda = x.lda;
        if (use_mma)
            limb_max = max(limb_max, (int)(codes_row_bytes(x.w.K, qt) / 16 * limb_granules(qt) * 16));
        d.out = x.out;
        d.bias = x.bias;
        d.residual = x.residual;
        d.N = x.w.N;
        d.K = x.w.K;
        d.M = x.M;
        d.ldo = x.ldo;
        d.ldr = x.ldr;
        d.rowb = (int32_t)codes_row_bytes(x.w.K, qt);
        d.srow = (x.w.K / VOXQ_QBLK) * scale_bytes(qt);
        d.chunks = d.rowb / 16;
        d.slabs = (d.chunks + 31) / 32;
        // rows per tile: fill the stage; rows spanning several slabs keep the
        // tile a whole number of 512-byte slabs so groups tile it exactly
        int T = (use_mma ? kMmaTile : kTile / nw) / d.rowb;
        if (T > x.w.N) T = x.w.N;
        if (T < 1) T = 1;
        if (d.slabs > 1 && !use_mma) {
            // partial-sum slots per tile: ceil(T / RG) * slabs <= 32
            const int rg = rows_per_group(mt, swi);
            if (T >= rg) T = T / rg * rg;
            while (T > 1 && ((T + rg - 1) / rg) * d.slabs > 32) T--;
        }
        d.parts = ((d.chunks + 3) / 4 + groups_per_part(qt) - 1) / groups_per_part(qt);
        if (use_mma && d.parts > 1 && T * d.parts > kPartSlots) T = kPartSlots / d.parts;
        d.T = T;
        d.tile_begin = tiles;
        tiles += (x.w.N + d.T - 1) / d.T;
        c++;
    }
    if (c == 0) return VOXCPM_SUCCESS;
    p.limb_bytes = limb_max;
    if (use_mma) {
        // Small launches: shorter tiles (down to 16 rows) so every CTA slot gets
        // work.  Results do not depend on T on this path.
        const int want = 4 * device_sm_count();  // two stages of two CTAs per SM
        if (tiles < want) {
            const int f = (want + tiles - 1) / tiles;
            tiles = 0;
            for (int i = 0; i < c; i++) {
                GemvItemDev& d = p.it[i];
                if (d.T > 16) d.T = max(16, d.T / f / 16 * 16);
                d.tile_begin = tiles;
                tiles += (d.N + d.T - 1) / d.T;
            }
        }
    }
    p.count = c;
    p.total_tiles = tiles;
    p.err = err ? err : device_error_word();

    // limb prepass (several launches only if there are more than kMaxJobs activations)
    for (int a0 = 0; a0 < nact; a0 += kMaxJobs) {
        const int na = min(kMaxJobs, nact - a0);
        int total = 0;
        for (int k = 0; k < na; k++) {
            const Act& a = acts[a0 + k];
            LimbJob& j = lp.job[k];
            j.a = a.a;
            j.dst = a.dst;
            j.M = a.M;
            j.lda = a.lda;
            j.chunks = (int32_t)(codes_row_bytes(a.K, qt) / 16);
            j.chunk_begin = total;
            total += a.M * j.chunks;
        }
        lp.count = na;
        lp.total = total;
        lp.qtype = qt;
        cudaLaunchConfig_t cfg = {};
        const int tpc = qt == VOXQ_Q4 ? 4 : 2;
        const int blocks = (total * tpc + 255) / 256;
        cfg.gridDim = dim3(blocks < 1 ? 1 : (blocks > 8 * device_sm_count() ? 8 * device_sm_count() : blocks));
        cfg.blockDim = dim3(256);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (qt == VOXQ_Q4)
            VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, limb_kernel<VOXQ_Q4>, lp));
        else
            VOXQ_CUDA_TRY(cudaLaunchKernelEx(&cfg, limb_kernel<VOXQ_Q8>, lp));
    }
    return dispatch<MAXI>(p, qt, mt, swi, f.w.q8_signed != 0, use_mma, st);
}

// Limb workspace of the items: the tensor-path kernel's items compute their
// limbs in shared memory and need none.
size_t gemv_workspace_bytes(const voxq_gemv_item* items, int count) {
    size_t total = 0;
    for (int i = 0; i < count; i++)
        if (items[i].w.K > 0 && items[i].M > 0 && !mma_item(items[i]))
            total += (limb_bytes(items[i].M, items[i].w.K, items[i].w.qtype) + 255) & ~(size_t)255;
    return total;
}

VoxCPMError gemv_launch_ws(const voxq_gemv_item* items, int count, cudaStream_t st, void* ws, size_t ws_bytes,
                           int* err) {
    if (count < 0 || count > VOXQ_MAX_BATCH) return VOXCPM_ERR_UNSUPPORTED;
    for (int i = 0; i < count; i++) {
        VoxCPMError e = validate_item(items[i]);
        if (e) return e;
    }
    // group by kernel variant, preserving order inside a group; single-row items
    // form their own group (tensor-path kernel), so an item's result does not
    // depend on what it is batched with
    const voxq_gemv_item* sel[VOXQ_MAX_BATCH];
    bool done[VOXQ_MAX_BATCH] = {};
    size_t used = 0;
    auto single = [](const voxq_gemv_item& x) { return mma_item(x); };
    for (int i = 0; i < count; i++) {
        if (done[i]) continue;
        int n = 0;
        const voxq_gemv_item& a = items[i];
        for (int j = i; j < count; j++) {
            const voxq_gemv_item& b = items[j];
            if (!done[j] && b.w.qtype == a.w.qtype && (b.up_codes != nullptr) == (a.up_codes != nullptr) &&
                (b.w.q8_signed != 0) == (a.w.q8_signed != 0) && single(b) == single(a)) {
                sel[n++] = &items[j];
                done[j] = true;
            }
        }
        // each variant group gets its own part of the workspace
        size_t need = 0;
        for (int k = 0; k < n; k++)
            if (sel[k]->w.K > 0 && sel[k]->M > 0 && !mma_item(*sel[k]))
                need += (limb_bytes(sel[k]->M, sel[k]->w.K, sel[k]->w.qtype) + 255) & ~(size_t)255;
        uint8_t* part = static_cast<uint8_t*>(ws) + used;
        VoxCPMError e = (n == 1) ? launch_items<1>(sel, n, st, part, ws_bytes - used, err)
                                 : launch_items<VOXQ_MAX_BATCH>(sel, n, st, part, ws_bytes - used, err);
        if (e) return e;
        used += need;
    }
    return VOXCPM_SUCCESS;
}

VoxCPMError gemv_launch(const voxq_gemv_item* items, int count, cudaStream_t st) {
    if (count < 0 || count > VOXQ_MAX_BATCH) return VOXCPM_ERR_UNSUPPORTED;
    const size_t need = gemv_workspace_bytes(items, count);
    void* ws = gemv_workspace(need);
    if (!ws && need) return VOXCPM_ERR_OOM;
    return gemv_launch_ws(items, count, st, ws, need);
}

// K == 0: the product is an empty sum (silu(0) * 0 == 0 for SwiGLU).
__global__ void gemv_k0_kernel(float* out, int M, int N, int64_t ldo, const float* bias, const float* residual,
                               int64_t ldr) {
    const int64_t total = (int64_t)M * N;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / N), n = (int)(i % N);
        float v = 0.0f;
        if (bias) v += bias[n];
        if (residual) v += residual[m * ldr + n];
        out[m * ldo + n] = v;
    }
}

VoxCPMError gemv_k0(const voxq_gemv_item& x, cudaStream_t st) {
    const int64_t total = (int64_t)x.M * x.w.N;
    const int blocks = (int)((total + 255) / 256 < 1024 ? (total + 255) / 256 : 1024);
    gemv_k0_kernel<<<blocks, 256, 0, st>>>(x.out, x.M, x.w.N, x.ldo, x.bias, x.residual, x.ldr);
    VOXQ_CUDA_TRY(cudaGetLastError());
    return VOXCPM_SUCCESS;
}

}  // namespace voxq

extern "C" VoxCPMError voxq_gemv_batch(const voxq_gemv_item* items, int count, void* stream) {
    if (count == 0) return VOXCPM_SUCCESS;
    if (!items) return VOXCPM_ERR_INTERNAL;
    return voxq::gemv_launch(items, count, (cudaStream_t)stream);
}
