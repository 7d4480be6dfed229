// voxq_gemv.cu -- quantized GEMV (M <= 8 activation rows) for sm_100a.
//
// out[m, n] = sum_k A[m, k] * W[n, k] with W in the packed Q4/Q8 layout
// (voxq.h).  This is the batch-1 decode regime of the reference's
// tensor_matmul_nt (src/tensor.c:617-678): every weight byte is read once and
// the kernel is HBM-bound, so it is built around keeping bytes in flight:
//
//   * Work = "tasks" of RG consecutive weight rows of one item; warps walk one
//     global task list (all items of a grouped launch back to back).
//   * Each row is cut into 16-byte chunks (32 Q4 codes = one block, or 16 Q8
//     codes = half a block); lane l owns chunks l, l+32, ...  A "slab" is the
//     32 chunks the warp's lanes own in one pass over the RG rows.
//   * Every lane streams exactly the chunks (and their block trailers) it will
//     consume into its own slots of a D-deep shared-memory ring with
//     cp.async; the ring runs D slabs ahead of the math, across task and
//     item boundaries.  A lane only ever reads what it copied itself: no
//     barriers.  Launches use programmatic dependent launch, so a following
//     voxq kernel is scheduled while this one drains.
//   * Codes become exact floats without conversion instructions: code bits are
//     OR-ed into the mantissa of 2^23 (byte permute / LOP3) and 2^23 is taken
//     off with packed f32x2 adds; Q4 nibbles stay at their bit position and
//     the matching activation is pre-scaled by 2^-p instead.
//   * Per chunk: y += scale * sum(q*x) + min * sum(x)  (the dequantized weight
//     q*scale+min is never formed; fp32 throughout, packed fma.rn.f32x2).
//   * One transposed butterfly reduces all RG*M row sums of a task at once.
#include <mutex>

#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

struct GemvItemDev {
    const uint8_t* codes;
    const uint8_t* scales;
    const uint8_t* up_codes;
    const uint8_t* up_scales;
    const float* a;
    float* out;
    const float* bias;
    const float* residual;
    int32_t N, K, M, lda, ldo, ldr;
    int32_t chunks;      // 16-byte code chunks per row
    int32_t slabs;       // ceil(chunks / 32)
    int32_t task_begin;  // first global task index of this item
    int32_t pad;
};

template <int MAXI>
struct GemvParams {
    int32_t count;
    int32_t total_tasks;
    int* err;
    GemvItemDev it[MAXI];
};

constexpr int kWarps = 8;  // warps per CTA

// Q4: per position e of the 8 codes in one 32-bit word, the bit offset p(e)
// at which conv_q4 leaves the nibble -> the activation is scaled by 2^-p(e).
__device__ __forceinline__ void q4_prescale(float (&x)[8]) {
    x[0] *= 0.0625f;             // 2^-4
    x[2] *= 0.000244140625f;     // 2^-12
    x[3] *= 0.00390625f;         // 2^-8
    x[4] *= 0.00390625f;         // 2^-8
    x[5] *= 1.52587890625e-05f;  // 2^-16
    x[6] *= 1.52587890625e-05f;  // 2^-16
    x[7] *= 0.000244140625f;     // 2^-12
}

// Q4 word (bytes q0q1 q2q3 q4q5 q6q7, high nibble = even element) -> the eight
// exact floats q_e * 2^p(e) as four f32x2 pairs (e0,e1) .. (e6,e7).
__device__ __forceinline__ void conv_q4(uint32_t w, uint64_t (&v)[4]) {
    const uint32_t w2 = w >> 12;
    const uint32_t E = 0x4B000000u;
    const uint64_t bias = 0xCB000000CB000000ull;  // (-2^23, -2^23)
    float f0 = __uint_as_float((w & 0x000F0u) | E);   // q0 << 4
    float f1 = __uint_as_float((w & 0x0000Fu) | E);   // q1
    float f2 = __uint_as_float((w & 0x0F000u) | E);   // q2 << 12
    float f3 = __uint_as_float((w & 0x00F00u) | E);   // q3 << 8
    float f4 = __uint_as_float((w2 & 0x00F00u) | E);  // q4 << 8
    float f5 = __uint_as_float((w & 0xF0000u) | E);   // q5 << 16
    float f6 = __uint_as_float((w2 & 0xF0000u) | E);  // q6 << 16
    float f7 = __uint_as_float((w2 & 0x0F000u) | E);  // q7 << 12
    v[0] = add2(pk(f0, f1), bias);
    v[1] = add2(pk(f2, f3), bias);
    v[2] = add2(pk(f4, f5), bias);
    v[3] = add2(pk(f6, f7), bias);
}

// Q8 word (4 codes) -> four exact floats as two pairs.  Signed mode reads the
// byte as int8 like scripts/quantize.py:79: (b ^ 0x80) - 128.
template <bool SIGNED>
__device__ __forceinline__ void conv_q8(uint32_t w, uint64_t (&v)[2]) {
    if (SIGNED) w ^= 0x80808080u;
    const uint64_t bias = SIGNED ? 0xCB000080CB000080ull : 0xCB000000CB000000ull;  // -(2^23 [+128])
    float f0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440));
    float f1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441));
    float f2 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442));
    float f3 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443));
    v[0] = add2(pk(f0, f1), bias);
    v[1] = add2(pk(f2, f3), bias);
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// cp.async of 16 / 8 / 4 bytes into this lane's own slot.
__device__ __forceinline__ void cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Position in a warp's stream of (task, slab) stages.
struct Cursor {
    int task;  // global task index (-1: past the end)
    int slab;
    int item;
};

template <int MAXI>
__device__ __forceinline__ void cursor_fix_item(const GemvParams<MAXI>& p, Cursor& c) {
    while (c.item + 1 < p.count && c.task >= p.it[c.item + 1].task_begin) c.item++;
}

template <int MAXI>
__device__ __forceinline__ void cursor_next(const GemvParams<MAXI>& p, Cursor& c, int stride) {
    if (++c.slab >= p.it[c.item].slabs) {
        c.slab = 0;
        c.task += stride;
        if (c.task >= p.total_tasks) {
            c.task = -1;
            return;
        }
        cursor_fix_item(p, c);
    }
}

// Reduces V values per lane across the warp.  Afterwards value v (0 <= v < V)
// is complete in lanes v * (32 / V) .. v * (32 / V) + 32 / V - 1.
template <int V>
__device__ __forceinline__ float transpose_reduce(float (&v)[V], int lane) {
    int n = V;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        if (n > 1) {
            const bool upper = (lane & off) != 0;
            const int h = n / 2;
#pragma unroll
            for (int i = 0; i < V / 2; i++) {
                if (i < h) {
                    float send = upper ? v[i] : v[i + h];
                    float keep = upper ? v[i + h] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
                }
            }
            n = h;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
        }
    }
    return v[0];
}

template <int QT, int MT, int RG, int D, bool SWI, bool SIGNED, int MAXI>
__global__ void __launch_bounds__(kWarps * 32) gemv_kernel(const __grid_constant__ GemvParams<MAXI> p) {
    constexpr int NW = SWI ? 2 : 1;                       // weights per row (gate, up)
    constexpr int SB = (QT == VOXQ_Q4) ? 4 : 8;           // trailer bytes per chunk slot
    constexpr int CPC = (QT == VOXQ_Q4) ? 32 : 16;        // codes per 16-byte chunk
    constexpr int STAGE_CODES = NW * RG * 32 * 16;        // bytes per warp stage
    constexpr int STAGE_SC = NW * RG * 32 * 8;
    constexpr int WARP_BYTES = D * (STAGE_CODES + STAGE_SC);
    constexpr int V = RG * MT;

    extern __shared__ __align__(16) uint8_t smem[];
    const int lane = threadIdx.x & 31;
    const int wib = threadIdx.x >> 5;
    uint8_t* wbase = smem + wib * WARP_BYTES;
    uint8_t* codes_s = wbase;
    uint8_t* sc_s = wbase + D * STAGE_CODES;

    const int stride = gridDim.x * kWarps;
    const int first = blockIdx.x * kWarps + wib;
    if (first >= p.total_tasks) {
        pdl_launch_dependents();
        return;
    }

    // ---- producer side of this lane's ring ----
    Cursor pc = {first, 0, 0};
    cursor_fix_item(p, pc);
    auto issue = [&](int stage) {
        if (pc.task >= 0) {
            const GemvItemDev& it = p.it[pc.item];
            const int chunk = pc.slab * 32 + lane;
            if (chunk < it.chunks) {
                const int n0 = (pc.task - it.task_begin) * RG;
                const int64_t rowb = (int64_t)it.chunks * 16;
                const int nblk = it.K / VOXQ_QBLK;
                const int blk = (QT == VOXQ_Q4) ? chunk : (chunk >> 1);
#pragma unroll
                for (int w = 0; w < NW; w++) {
                    const uint8_t* cb = w ? it.up_codes : it.codes;
                    const uint8_t* sb = w ? it.up_scales : it.scales;
#pragma unroll
                    for (int r = 0; r < RG; r++) {
                        const int row = min(n0 + r, it.N - 1);
                        uint8_t* cd = codes_s + stage * STAGE_CODES + ((w * RG + r) * 32 + lane) * 16;
                        uint8_t* sd = sc_s + stage * STAGE_SC + ((w * RG + r) * 32 + lane) * 8;
                        cp16(cd, cb + row * rowb + (int64_t)chunk * 16);
                        const uint8_t* ss = sb + ((int64_t)row * nblk + blk) * SB;
                        if (SB == 4)
                            cp4(sd, ss);
                        else
                            cp8(sd, ss);
                    }
                }
            }
            cursor_next(p, pc, stride);
        }
        cp_commit();  // empty groups keep the wait_group arithmetic uniform
    };

    // Everything this kernel reads (weights included: a quantize or pack kernel
    // may have just written them) can come from the previous kernel in the
    // stream, so wait for it before the first copy; the next kernel may launch.
    pdl_wait();
    pdl_launch_dependents();
#pragma unroll
    for (int s = 0; s < D; s++) issue(s);

    Cursor cc = {first, 0, 0};
    cursor_fix_item(p, cc);
    float acc[NW][RG][MT];
    int stage = 0;
    while (cc.task >= 0) {
        const GemvItemDev& it = p.it[cc.item];
        if (cc.slab == 0) {
#pragma unroll
            for (int w = 0; w < NW; w++)
#pragma unroll
                for (int r = 0; r < RG; r++)
#pragma unroll
                    for (int m = 0; m < MT; m++) acc[w][r][m] = 0.0f;
        }
        cp_wait<D - 1>();
        const int chunk = cc.slab * 32 + lane;
        if (chunk < it.chunks) {
            // activation chunk: CPC values per row, in 8-element quarters
            uint64_t dot[NW][RG][MT];
#pragma unroll
            for (int w = 0; w < NW; w++)
#pragma unroll
                for (int r = 0; r < RG; r++)
#pragma unroll
                    for (int m = 0; m < MT; m++) dot[w][r][m] = 0ull;
            float xsum[MT];
#pragma unroll
            for (int m = 0; m < MT; m++) xsum[m] = 0.0f;
            uint4 cw[NW][RG];
#pragma unroll
            for (int w = 0; w < NW; w++)
#pragma unroll
                for (int r = 0; r < RG; r++)
                    cw[w][r] = *reinterpret_cast<const uint4*>(codes_s + stage * STAGE_CODES +
                                                               ((w * RG + r) * 32 + lane) * 16);
#pragma unroll
            for (int q = 0; q < CPC / 8; q++) {
                uint64_t xp[MT][4];
#pragma unroll
                for (int m = 0; m < MT; m++) {
                    const int mm = m < it.M ? m : it.M - 1;
                    const float* ap = it.a + (int64_t)mm * it.lda + (int64_t)chunk * CPC + q * 8;
                    float4 a0 = ldg_f4(ap), a1 = ldg_f4(ap + 4);
                    float x[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                    xsum[m] += ((x[0] + x[1]) + (x[2] + x[3])) + ((x[4] + x[5]) + (x[6] + x[7]));
                    if (QT == VOXQ_Q4) q4_prescale(x);
#pragma unroll
                    for (int j = 0; j < 4; j++) xp[m][j] = pk(x[2 * j], x[2 * j + 1]);
                }
#pragma unroll
                for (int w = 0; w < NW; w++)
#pragma unroll
                    for (int r = 0; r < RG; r++) {
                        uint64_t v[4];
                        const uint4 c = cw[w][r];
                        if (QT == VOXQ_Q4) {
                            const uint32_t word = q == 0 ? c.x : q == 1 ? c.y : q == 2 ? c.z : c.w;
                            conv_q4(word, v);
                        } else {
                            uint64_t lo[2], hi[2];
                            conv_q8<SIGNED>(q == 0 ? c.x : c.z, lo);
                            conv_q8<SIGNED>(q == 0 ? c.y : c.w, hi);
                            v[0] = lo[0]; v[1] = lo[1]; v[2] = hi[0]; v[3] = hi[1];
                        }
#pragma unroll
                        for (int m = 0; m < MT; m++)
#pragma unroll
                            for (int j = 0; j < 4; j++) dot[w][r][m] = fma2(v[j], xp[m][j], dot[w][r][m]);
                    }
            }
#pragma unroll
            for (int w = 0; w < NW; w++)
#pragma unroll
                for (int r = 0; r < RG; r++) {
                    float s, mn;
                    const uint8_t* sp = sc_s + stage * STAGE_SC + ((w * RG + r) * 32 + lane) * 8;
                    if (QT == VOXQ_Q4) {
                        const uint32_t t = *reinterpret_cast<const uint32_t*>(sp);
                        s = __half2float(__ushort_as_half((unsigned short)(t & 0xffff)));
                        mn = __half2float(__ushort_as_half((unsigned short)(t >> 16)));
                    } else {
                        const float2 t = *reinterpret_cast<const float2*>(sp);
                        s = t.x;
                        mn = t.y;
                    }
#pragma unroll
                    for (int m = 0; m < MT; m++) {
                        float d0, d1;
                        upk(dot[w][r][m], d0, d1);
                        acc[w][r][m] = fmaf(s, d0 + d1, fmaf(mn, xsum[m], acc[w][r][m]));
                    }
                }
        }
        // refill the slot just consumed with the stage D ahead
        issue(stage);
        stage = stage + 1 == D ? 0 : stage + 1;

        const bool task_done = cc.slab + 1 >= it.slabs;
        if (task_done) {
            const int n0 = (cc.task - it.task_begin) * RG;
            float vg[V];
#pragma unroll
            for (int r = 0; r < RG; r++)
#pragma unroll
                for (int m = 0; m < MT; m++) vg[r * MT + m] = acc[0][r][m];
            float val = transpose_reduce<V>(vg, lane);
            if (SWI) {
                float vu[V];
#pragma unroll
                for (int r = 0; r < RG; r++)
#pragma unroll
                    for (int m = 0; m < MT; m++) vu[r * MT + m] = acc[NW - 1][r][m];
                val = silu(val) * transpose_reduce<V>(vu, lane);
            }
            constexpr int LPV = 32 / V;  // lanes holding each value
            if ((lane & (LPV - 1)) == 0) {
                const int v = lane / LPV;
                const int r = v / MT, m = v % MT;
                const int n = n0 + r;
                if (n < it.N && m < it.M) {
                    if (it.bias) val += it.bias[n];
                    if (it.residual) val += it.residual[(int64_t)m * it.ldr + n];
                    it.out[(int64_t)m * it.ldo + n] = val;
                }
            }
        }
        cursor_next(p, cc, stride);
    }
    cp_wait<0>();
}

// Kernel shape per activation-row count: rows per task and ring depth.
template <int MT, bool SWI>
struct Shape {
    static constexpr int RG0 = MT == 1 ? 4 : MT == 2 ? 4 : MT == 4 ? 2 : 2;
    static constexpr int RG = SWI ? (RG0 > 2 ? RG0 / 2 : RG0) : RG0;
    static constexpr int D = 4;
};

template <int QT, int MT, bool SWI, bool SIGNED, int MAXI>
static VoxCPMError launch_t(const GemvParams<MAXI>& p, cudaStream_t st) {
    constexpr int RG = Shape<MT, SWI>::RG;
    constexpr int D = Shape<MT, SWI>::D;
    constexpr int NW = SWI ? 2 : 1;
    constexpr int smem = kWarps * D * NW * RG * 32 * (16 + 8);
    auto kern = gemv_kernel<QT, MT, RG, D, SWI, SIGNED, MAXI>;
    static int occ = 0;
    static std::once_flag once;
    std::call_once(once, [&] {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kWarps * 32, smem);
    });
    const int sms = device_sm_count();
    const int want = (p.total_tasks + kWarps - 1) / kWarps;
    const int cap = sms * (occ > 0 ? occ : 1);
    const int blocks = want < cap ? (want < 1 ? 1 : want) : cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(kWarps * 32);
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

template <int MAXI>
static VoxCPMError dispatch(const GemvParams<MAXI>& p, int qtype, int mt, bool swi, bool sgn, cudaStream_t st) {
#define VOXQ_GEMV_CASE(QT, MT)                                                                         \
    if (qtype == QT && mt == MT) {                                                                     \
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

static int round_mt(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

static int rows_per_task(int mt, bool swi) {
    switch (mt) {
        case 1: return swi ? Shape<1, true>::RG : Shape<1, false>::RG;
        case 2: return swi ? Shape<2, true>::RG : Shape<2, false>::RG;
        case 4: return swi ? Shape<4, true>::RG : Shape<4, false>::RG;
        default: return swi ? Shape<8, true>::RG : Shape<8, false>::RG;
    }
}

VoxCPMError validate_item(const voxq_gemv_item& x) {
    const voxq_qweight& w = x.w;
    if (w.qtype != VOXQ_Q4 && w.qtype != VOXQ_Q8) return VOXCPM_ERR_UNSUPPORTED;
    if (w.N < 0 || w.K < 0 || w.K % VOXQ_QBLK || x.M < 0 || x.M > 8) return VOXCPM_ERR_SHAPE_MISMATCH;
    if (w.N == 0 || x.M == 0) return VOXCPM_SUCCESS;
    if (!x.a || !x.out || (w.K > 0 && (!w.codes || !w.scales))) return VOXCPM_ERR_INTERNAL;
    if (x.lda < w.K || x.ldo < w.N || (x.residual && x.ldr < w.N)) return VOXCPM_ERR_SHAPE_MISMATCH;
    // 16-byte activation loads, 16-byte code copies, 4/8-byte trailer copies
    if ((reinterpret_cast<uintptr_t>(x.a) & 15) || (x.lda & 3)) return VOXCPM_ERR_UNSUPPORTED;
    const uintptr_t sa = w.qtype == VOXQ_Q4 ? 3 : 7;
    if ((reinterpret_cast<uintptr_t>(w.codes) & 15) || (reinterpret_cast<uintptr_t>(w.scales) & sa))
        return VOXCPM_ERR_UNSUPPORTED;
    if (x.up_codes && ((reinterpret_cast<uintptr_t>(x.up_codes) & 15) ||
                       (reinterpret_cast<uintptr_t>(x.up_scales) & sa) || !x.up_scales))
        return VOXCPM_ERR_UNSUPPORTED;
    return VOXCPM_SUCCESS;
}

static void fill_dev(GemvItemDev& d, const voxq_gemv_item& x, int task_begin) {
    d.codes = x.w.codes;
    d.scales = reinterpret_cast<const uint8_t*>(x.w.scales);
    d.up_codes = x.up_codes;
    d.up_scales = reinterpret_cast<const uint8_t*>(x.up_scales);
    d.a = x.a;
    d.out = x.out;
    d.bias = x.bias;
    d.residual = x.residual;
    d.N = x.w.N;
    d.K = x.w.K;
    d.M = x.M;
    d.lda = x.lda;
    d.ldo = x.ldo;
    d.ldr = x.ldr;
    d.chunks = (int32_t)(codes_row_bytes(x.w.K, x.w.qtype) / 16);
    d.slabs = (d.chunks + 31) / 32;
    d.task_begin = task_begin;
    d.pad = 0;
}

// Launches the items that share (qtype, swiglu, signed) as one grid.
template <int MAXI>
static VoxCPMError launch_items(const voxq_gemv_item* const* sel, int n, cudaStream_t st) {
    static thread_local GemvParams<MAXI> p;
    const voxq_gemv_item& f = *sel[0];
    int mt = 1;
    for (int i = 0; i < n; i++) mt = max(mt, round_mt(sel[i]->M));
    const bool swi = f.up_codes != nullptr;
    const int rg = rows_per_task(mt, swi);
    int tasks = 0, c = 0;
    for (int i = 0; i < n; i++) {
        const voxq_gemv_item& x = *sel[i];
        if (x.w.N == 0 || x.M == 0) continue;
        if (x.w.K == 0) {  // empty reduction: out = epilogue(0)
            VoxCPMError e = gemv_k0(x, st);
            if (e) return e;
            continue;
        }
        fill_dev(p.it[c], x, tasks);
        tasks += (x.w.N + rg - 1) / rg;
        c++;
    }
    if (c == 0) return VOXCPM_SUCCESS;
    p.count = c;
    p.total_tasks = tasks;
    p.err = device_error_word();
    return dispatch<MAXI>(p, f.w.qtype, mt, swi, f.w.q8_signed != 0, st);
}

VoxCPMError gemv_launch(const voxq_gemv_item* items, int count, cudaStream_t st) {
    if (count < 0 || count > VOXQ_MAX_BATCH) return VOXCPM_ERR_UNSUPPORTED;
    for (int i = 0; i < count; i++) {
        VoxCPMError e = validate_item(items[i]);
        if (e) return e;
    }
    // group by kernel variant, preserving order inside a group
    const voxq_gemv_item* sel[VOXQ_MAX_BATCH];
    bool done[VOXQ_MAX_BATCH] = {};
    for (int i = 0; i < count; i++) {
        if (done[i]) continue;
        int n = 0;
        const voxq_gemv_item& a = items[i];
        for (int j = i; j < count; j++) {
            const voxq_gemv_item& b = items[j];
            if (!done[j] && b.w.qtype == a.w.qtype && (b.up_codes != nullptr) == (a.up_codes != nullptr) &&
                (b.w.q8_signed != 0) == (a.w.q8_signed != 0)) {
                sel[n++] = &items[j];
                done[j] = true;
            }
        }
        VoxCPMError e = (n == 1) ? launch_items<1>(sel, n, st) : launch_items<VOXQ_MAX_BATCH>(sel, n, st);
        if (e) return e;
    }
    return VOXCPM_SUCCESS;
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
