// voxq_gemv.cu -- quantized GEMV (M <= 8 activation rows) for sm_100a.
//
// out[m, n] = sum_k A[m, k] * W[n, k] with W in the packed Q4/Q8 layout
// (voxq.h).  This is the batch-1 decode regime of the reference's
// tensor_matmul_nt (src/tensor.c:617-678): every weight byte is read once, so
// the kernel is HBM-bound and built to keep the memory pipe full:
//   * one warp owns RG consecutive weight rows; lane l owns quantization
//     blocks l, l+32, ... of those rows, so a warp-wide 16-byte load per row
//     streams 512 contiguous code bytes (no shared memory, no smem staging);
//   * all RG rows' code loads are issued before any math (deep MLP);
//   * codes become exact floats without conversion instructions: the code
//     bits are OR-ed into the mantissa of 2^23 (byte permute / LOP3) and 2^23
//     is subtracted with packed f32x2 adds; Q4 nibbles are left at their bit
//     position and the matching activation is pre-scaled by 2^-p instead;
//   * per block b: y += scale_b * sum(q*x) + min_b * sum(x), i.e. the
//     dequantized weight q*scale+min is never formed (fp32 throughout);
//   * products accumulate with packed fma.rn.f32x2.
// A grouped launch runs many independent GEMVs (a whole decoder layer stack)
// as one grid: warps walk one global list of row groups, so weight streaming
// never stops at a kernel boundary.
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
    int32_t q8_signed;
    int32_t group_begin;  // first global row-group index of this item
};

template <int MAXI>
struct GemvParams {
    int32_t count;
    int32_t total_groups;
    GemvItemDev it[MAXI];
};

constexpr float kTwo23 = 8388608.0f;

// Q4: per position e of the 8 codes in one 32-bit word, the bit offset p(e)
// at which the nibble is extracted (see conv_q4) -> activation scale 2^-p.
__device__ __forceinline__ void q4_prescale(float (&x)[8]) {
    x[0] *= 0.0625f;           // 2^-4
    x[2] *= 0.000244140625f;   // 2^-12
    x[3] *= 0.00390625f;       // 2^-8
    x[4] *= 0.00390625f;       // 2^-8
    x[5] *= 1.52587890625e-05f;  // 2^-16
    x[6] *= 1.52587890625e-05f;  // 2^-16
    x[7] *= 0.000244140625f;   // 2^-12
}

// Q4 word (bytes q0q1 q2q3 q4q5 q6q7, high nibble = even element) ->
// eight floats q_e * 2^p(e), exact, as four f32x2 pairs (e0,e1)...(e6,e7).
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
// byte as int8: (b ^ 0x80) - 128.
template <bool SIGNED>
__device__ __forceinline__ void conv_q8(uint32_t w, uint64_t (&v)[2]) {
    if (SIGNED) w ^= 0x80808080u;
    const uint64_t bias = SIGNED ? 0xCB000080CB000080ull : 0xCB000000CB000000ull;  // -(2^23[+128])
    float f0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440));
    float f1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441));
    float f2 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442));
    float f3 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443));
    v[0] = add2(pk(f0, f1), bias);
    v[1] = add2(pk(f2, f3), bias);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// Processes rows n0 .. n0+RG-1 of one item.
template <int QT, int MT, int RG, bool SWI, bool SIGNED>
__device__ __forceinline__ void gemv_group(const GemvItemDev& it, int n0, int lane) {
    constexpr int CW = (QT == VOXQ_Q4) ? 4 : 8;  // code words per block
    constexpr int NW = SWI ? 2 : 1;              // weights per row (gate, up)
    const int K = it.K;
    const int nblk = K / VOXQ_QBLK;
    const int64_t rowb = (QT == VOXQ_Q4) ? K / 2 : K;
    const int sb = (QT == VOXQ_Q4) ? 4 : 8;

    float acc[NW][RG][MT];
#pragma unroll
    for (int w = 0; w < NW; w++)
#pragma unroll
        for (int r = 0; r < RG; r++)
#pragma unroll
            for (int m = 0; m < MT; m++) acc[w][r][m] = 0.0f;

    for (int kb = lane; kb < nblk; kb += 32) {
        // ---- issue every code and trailer load of this block first ----
        uint32_t code[NW][RG][CW];
        float s[NW][RG], mn[NW][RG];
#pragma unroll
        for (int w = 0; w < NW; w++) {
            const uint8_t* cbase = w ? it.up_codes : it.codes;
            const uint8_t* sbase = w ? it.up_scales : it.scales;
#pragma unroll
            for (int r = 0; r < RG; r++) {
                const int row = min(n0 + r, it.N - 1);
                const uint8_t* cp = cbase + row * rowb + (int64_t)kb * (CW * 4);
                uint4 c0 = ldg_stream(cp);
                code[w][r][0] = c0.x; code[w][r][1] = c0.y; code[w][r][2] = c0.z; code[w][r][3] = c0.w;
                if (CW == 8) {
                    uint4 c1 = ldg_stream(cp + 16);
                    code[w][r][4 % CW] = c1.x; code[w][r][5 % CW] = c1.y;
                    code[w][r][6 % CW] = c1.z; code[w][r][7 % CW] = c1.w;
                }
                const uint8_t* sp = sbase + ((int64_t)row * nblk + kb) * sb;
                if (QT == VOXQ_Q4) {
                    uint32_t t = __ldg(reinterpret_cast<const unsigned int*>(sp));
                    s[w][r] = __half2float(__ushort_as_half((unsigned short)(t & 0xffff)));
                    mn[w][r] = __half2float(__ushort_as_half((unsigned short)(t >> 16)));
                } else {
                    float2 t = __ldg(reinterpret_cast<const float2*>(sp));
                    s[w][r] = t.x;
                    mn[w][r] = t.y;
                }
            }
        }
        // ---- block dot products, 8 elements at a time ----
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

#pragma unroll
        for (int q = 0; q < 4; q++) {
            uint64_t xp[MT][4];
#pragma unroll
            for (int m = 0; m < MT; m++) {
                const int mm = min(m, it.M - 1);
                const float* ap = it.a + (int64_t)mm * it.lda + kb * VOXQ_QBLK + q * 8;
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
                    if (QT == VOXQ_Q4) {
                        conv_q4(code[w][r][q], v);
                    } else {
                        uint64_t lo[2], hi[2];
                        conv_q8<SIGNED>(code[w][r][2 * q], lo);
                        conv_q8<SIGNED>(code[w][r][2 * q + 1], hi);
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
            for (int r = 0; r < RG; r++)
#pragma unroll
                for (int m = 0; m < MT; m++) {
                    float d0, d1;
                    upk(dot[w][r][m], d0, d1);
                    acc[w][r][m] = fmaf(s[w][r], d0 + d1, fmaf(mn[w][r], xsum[m], acc[w][r][m]));
                }
    }

    // ---- reduce across the warp and write with the epilogue ----
#pragma unroll
    for (int r = 0; r < RG; r++)
#pragma unroll
        for (int m = 0; m < MT; m++) {
            float v = warp_sum(acc[0][r][m]);
            if (SWI) v = silu(v) * warp_sum(acc[NW - 1][r][m]);
            const int n = n0 + r;
            if (lane == ((r * MT + m) & 31) && n < it.N && m < it.M) {
                if (it.bias) v += it.bias[n];
                if (it.residual) v += it.residual[(int64_t)m * it.ldr + n];
                it.out[(int64_t)m * it.ldo + n] = v;
            }
        }
}

template <int QT, int MT, int RG, bool SWI, bool SIGNED, int MAXI>
__global__ void __launch_bounds__(256) gemv_kernel(const __grid_constant__ GemvParams<MAXI> p) {
    const int lane = threadIdx.x & 31;
    const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int nwarps = (int)((gridDim.x * blockDim.x) >> 5);
    pdl_wait();
    int item = 0;
    for (int g = warp; g < p.total_groups; g += nwarps) {
        while (item + 1 < p.count && g >= p.it[item + 1].group_begin) item++;
        const GemvItemDev& it = p.it[item];
        gemv_group<QT, MT, RG, SWI, SIGNED>(it, (g - it.group_begin) * RG, lane);
    }
    pdl_launch_dependents();
}

// Rows per warp group for each activation-row count.
template <int MT, bool SWI>
struct RowsPerGroup {
    static constexpr int base = MT == 1 ? 8 : MT == 2 ? 4 : 2;
    static constexpr int value = SWI ? (base > 2 ? base / 2 : 2) : base;
};

struct LaunchCfg {
    int blocks_per_sm = 0;
};

template <int QT, int MT, bool SWI, bool SIGNED, int MAXI>
static VoxCPMError launch_t(const GemvParams<MAXI>& p, cudaStream_t st) {
    constexpr int RG = RowsPerGroup<MT, SWI>::value;
    auto kern = gemv_kernel<QT, MT, RG, SWI, SIGNED, MAXI>;
    static int occ = 0;
    static std::once_flag once;
    std::call_once(once, [&] { cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, 0); });
    const int sms = device_sm_count();
    int want = (p.total_groups + 7) / 8;
    int cap = sms * (occ > 0 ? occ : 1);
    int blocks = want < cap ? want : cap;
    if (blocks < 1) blocks = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(256);
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
#define VOXQ_GEMV_CASE(QT, MT)                                                                   \
    if (qtype == QT && mt == MT) {                                                               \
        if (swi) return sgn ? launch_t<QT, MT, true, true, MAXI>(p, st)                          \
                            : launch_t<QT, MT, true, false, MAXI>(p, st);                        \
        return sgn ? launch_t<QT, MT, false, true, MAXI>(p, st) : launch_t<QT, MT, false, false, MAXI>(p, st); \
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

static int rows_per_group(int mt, bool swi) {
    switch (mt) {
        case 1: return swi ? RowsPerGroup<1, true>::value : RowsPerGroup<1, false>::value;
        case 2: return swi ? RowsPerGroup<2, true>::value : RowsPerGroup<2, false>::value;
        case 4: return swi ? RowsPerGroup<4, true>::value : RowsPerGroup<4, false>::value;
        default: return swi ? RowsPerGroup<8, true>::value : RowsPerGroup<8, false>::value;
    }
}

VoxCPMError validate_item(const voxq_gemv_item& x) {
    const voxq_qweight& w = x.w;
    if (w.qtype != VOXQ_Q4 && w.qtype != VOXQ_Q8) return VOXCPM_ERR_UNSUPPORTED;
    if (w.N < 0 || w.K < 0 || w.K % VOXQ_QBLK || x.M < 0 || x.M > 8) return VOXCPM_ERR_SHAPE_MISMATCH;
    if (w.N == 0 || x.M == 0) return VOXCPM_SUCCESS;
    if (!x.a || !x.out || (w.K > 0 && (!w.codes || !w.scales))) return VOXCPM_ERR_INTERNAL;
    if (x.lda < w.K || x.ldo < w.N || (x.residual && x.ldr < w.N)) return VOXCPM_ERR_SHAPE_MISMATCH;
    // 16-byte activation loads and code loads
    if ((reinterpret_cast<uintptr_t>(x.a) & 15) || (x.lda & 3)) return VOXCPM_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(w.codes) & 15) || (reinterpret_cast<uintptr_t>(w.scales) & 7))
        return VOXCPM_ERR_UNSUPPORTED;
    if (x.up_codes && ((reinterpret_cast<uintptr_t>(x.up_codes) & 15) ||
                       (reinterpret_cast<uintptr_t>(x.up_scales) & 7) || !x.up_scales))
        return VOXCPM_ERR_UNSUPPORTED;
    return VOXCPM_SUCCESS;
}

static void fill_dev(GemvItemDev& d, const voxq_gemv_item& x, int group_begin) {
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
    d.q8_signed = x.w.q8_signed;
    d.group_begin = group_begin;
}

// Launches the items that share (qtype, swiglu, signed) as one grid.
template <int MAXI>
static VoxCPMError launch_items(const voxq_gemv_item* const* sel, int n, cudaStream_t st) {
    static thread_local GemvParams<MAXI> p;
    const voxq_gemv_item& f = *sel[0];
    int mt = 1;
    for (int i = 0; i < n; i++) mt = max(mt, round_mt(sel[i]->M));
    const bool swi = f.up_codes != nullptr;
    const int rg = rows_per_group(mt, swi);
    int groups = 0, c = 0;
    for (int i = 0; i < n; i++) {
        const voxq_gemv_item& x = *sel[i];
        if (x.w.N == 0 || x.M == 0 || x.w.K == 0) {
            if (x.w.K == 0 && x.w.N > 0 && x.M > 0) {
                // empty reduction: out = epilogue(0)
                VoxCPMError e = gemv_k0(x, st);
                if (e) return e;
            }
            continue;
        }
        fill_dev(p.it[c], x, groups);
        groups += (x.w.N + rg - 1) / rg;
        c++;
    }
    if (c == 0) return VOXCPM_SUCCESS;
    p.count = c;
    p.total_groups = groups;
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

// K == 0: the product is an empty sum.
__global__ void gemv_k0_kernel(float* out, int M, int N, int64_t ldo, const float* bias, const float* residual,
                               int64_t ldr, int swi) {
    const int64_t total = (int64_t)M * N;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / N), n = (int)(i % N);
        float v = 0.0f;
        if (swi) v = 0.0f;  // silu(0) * 0
        if (bias) v += bias[n];
        if (residual) v += residual[m * ldr + n];
        out[m * ldo + n] = v;
    }
}

VoxCPMError gemv_k0(const voxq_gemv_item& x, cudaStream_t st) {
    const int64_t total = (int64_t)x.M * x.w.N;
    const int blocks = (int)((total + 255) / 256 < 1024 ? (total + 255) / 256 : 1024);
    gemv_k0_kernel<<<blocks, 256, 0, st>>>(x.out, x.M, x.w.N, x.ldo, x.bias, x.residual, x.ldr,
                                           x.up_codes != nullptr);
    VOXQ_CUDA_TRY(cudaGetLastError());
    return VOXCPM_SUCCESS;
}

}  // namespace voxq

extern "C" VoxCPMError voxq_gemv_batch(const voxq_gemv_item* items, int count, void* stream) {
    if (count == 0) return VOXCPM_SUCCESS;
    if (!items) return VOXCPM_ERR_INTERNAL;
    return voxq::gemv_launch(items, count, (cudaStream_t)stream);
}
