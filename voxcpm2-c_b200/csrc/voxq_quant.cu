// voxq_quant.cu -- device block quantizer / dequantizer and layout packing.
//
// The quantizer is bit-exact with the reference's offline converter
// (scripts/quantize.py:42-75): the same numpy-2 float32/float64 operation
// sequence, restated with explicitly rounded intrinsics so the compiler can
// neither contract nor reassociate it:
//   w_min, w_max : numpy's float32 reduction order (see block_minmax)
//   scale        : (double(w_max) - double(w_min)) / 15 or / 255 in double,
//                  1.0 when w_max == w_min
//   code         : rint(float(x - w_min) / float(scale)), clipped; NaN -> 0
//   Q4 trailer   : binary16(scale) rounded from the double, binary16(w_min)
//   Q8 trailer   : float(scale), w_min; codes 128..255 stored as their byte
#include <string.h>

#include "voxq_common.cuh"

namespace voxq {

// numpy's float32 min/max over one 32-element block on an AVX-512 host: seed
// r = x[0]; 16 lanes v[i] = op(r, x[1+i]); lanes folded (hi, lo) 16->8->4,
// then (j, j^2), then (0, 1); scalar tail x[17..31].  Each step keeps the
// second operand on a tie, which only decides the sign of a zero result.
__device__ __forceinline__ float sel_min(float a, float x) { return (a < x) ? a : x; }
__device__ __forceinline__ float sel_max(float a, float x) { return (a > x) ? a : x; }

template <bool MAX>
__device__ __forceinline__ float op(float a, float x) {
    return MAX ? sel_max(a, x) : sel_min(a, x);
}

template <bool MAX>
__device__ float block_reduce(const float* b) {
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = op<MAX>(b[0], b[1 + i]);
    float t3[8], t6[4], t8[4];
#pragma unroll
    for (int j = 0; j < 8; j++) t3[j] = op<MAX>(v[8 + j], v[j]);
#pragma unroll
    for (int j = 0; j < 4; j++) t6[j] = op<MAX>(t3[4 + j], t3[j]);
#pragma unroll
    for (int j = 0; j < 4; j++) t8[j] = op<MAX>(t6[j], t6[j ^ 2]);
    float r = op<MAX>(t8[0], t8[1]);
#pragma unroll
    for (int i = 17; i < VOXQ_QBLK; i++) r = op<MAX>(r, b[i]);
    return r;
}

// Quantizes one block (32 floats, already zero-padded) into codes + trailer.
__device__ void quantize_block(const float* b, int qtype, uint8_t* q, float* out_scale_f32,
                               uint16_t* out_scale_h, float* out_min) {
    int nan_at = -1;
#pragma unroll
    for (int i = 0; i < VOXQ_QBLK; i++)
        if (nan_at < 0 && isnan(b[i])) nan_at = i;
    float mn, mx;
    if (nan_at >= 0) {
        mn = mx = b[nan_at];
    } else {
        mn = block_reduce<false>(b);
        mx = block_reduce<true>(b);
    }
    const double levels = (qtype == VOXQ_Q4) ? 15.0 : 255.0;
    const double dmin = (double)mn, dmax = (double)mx;
    const double scale = (dmax != dmin) ? __ddiv_rn(__dsub_rn(dmax, dmin), levels) : 1.0;
    const float fscale = __double2float_rn(scale);
    const float flev = (float)levels;
#pragma unroll
    for (int i = 0; i < VOXQ_QBLK; i++) {
        float t = __fsub_rn(b[i], mn);
        float r = rintf(__fdiv_rn(t, fscale));
        uint8_t c;
        if (isnan(r)) {
            c = 0;
        } else {
            r = r < 0.0f ? 0.0f : r;
            r = r > flev ? flev : r;
            c = (uint8_t)(int)r;
        }
        q[i] = c;
    }
    *out_scale_f32 = fscale;
    *out_scale_h = double_to_half_rn(scale);
    *out_min = mn;
}

// One thread per block.  Writes any of: the quantize.py block stream, the
// packed codes, the packed trailers (scales).
__global__ void quantize_kernel(const float* __restrict__ src, int64_t n, int qtype,
                                uint8_t* __restrict__ blocks, uint8_t* __restrict__ codes,
                                uint8_t* __restrict__ scales) {
    const int64_t nb = (n + VOXQ_QBLK - 1) / VOXQ_QBLK;
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb;
         b += (int64_t)gridDim.x * blockDim.x) {
        float v[VOXQ_QBLK];
        const int64_t base = b * VOXQ_QBLK;
        if (base + VOXQ_QBLK <= n && ((reinterpret_cast<uintptr_t>(src + base) & 15) == 0)) {
#pragma unroll
            for (int i = 0; i < VOXQ_QBLK; i += 4) {
                float4 f = *reinterpret_cast<const float4*>(src + base + i);
                v[i] = f.x; v[i + 1] = f.y; v[i + 2] = f.z; v[i + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < VOXQ_QBLK; i++) v[i] = (base + i < n) ? src[base + i] : 0.0f;
        }
        uint8_t q[VOXQ_QBLK];
        float fscale, mn;
        uint16_t hscale;
        quantize_block(v, qtype, q, &fscale, &hscale, &mn);
        uint32_t w[8];
        int nw;
        if (qtype == VOXQ_Q4) {
            nw = 4;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                uint32_t x = 0;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    uint32_t byte = ((uint32_t)q[8 * i + 2 * j] << 4) | q[8 * i + 2 * j + 1];
                    x |= byte << (8 * j);
                }
                w[i] = x;
            }
        } else {
            nw = 8;
#pragma unroll
            for (int i = 0; i < 8; i++)
                w[i] = q[4 * i] | (q[4 * i + 1] << 8) | (q[4 * i + 2] << 16) | ((uint32_t)q[4 * i + 3] << 24);
        }
        uint32_t tr[2];
        if (qtype == VOXQ_Q4) {
            uint16_t hm = double_to_half_rn((double)mn);
            tr[0] = (uint32_t)hscale | ((uint32_t)hm << 16);
            tr[1] = 0;
        } else {
            tr[0] = __float_as_uint(fscale);
            tr[1] = __float_as_uint(mn);
        }
        const int ntr = (qtype == VOXQ_Q4) ? 1 : 2;
        if (blocks) {
            // 20- or 40-byte records: 4-byte aligned
            uint32_t* dst = reinterpret_cast<uint32_t*>(blocks + b * block_bytes(qtype));
            for (int i = 0; i < nw; i++) dst[i] = w[i];
            for (int i = 0; i < ntr; i++) dst[nw + i] = tr[i];
        }
        if (codes) {
            uint4* dst = reinterpret_cast<uint4*>(codes + b * (nw * 4));
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            if (nw == 8) dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
        if (scales) {
            uint32_t* dst = reinterpret_cast<uint32_t*>(scales + b * scale_bytes(qtype));
            for (int i = 0; i < ntr; i++) dst[i] = tr[i];
        }
    }
}

// NaN encoding of the reference's x86 arithmetic, so NaN results match bit for
// bit: an operation with a NaN operand returns that operand (quieted); an
// invalid operation on non-NaN operands (0 * inf, inf - inf) returns the x86
// default NaN 0xFFC00000.  (The GPU's own default NaN is 0x7FFFFFFF.)
__device__ __forceinline__ float x86_mul(float a, float b) {
    float r = __fmul_rn(a, b);
    if (!isnan(r)) return r;
    if (isnan(a)) return __uint_as_float(__float_as_uint(a) | 0x00400000u);
    if (isnan(b)) return __uint_as_float(__float_as_uint(b) | 0x00400000u);
    return __uint_as_float(0xFFC00000u);
}
__device__ __forceinline__ float x86_add(float a, float b) {
    float r = __fadd_rn(a, b);
    if (!isnan(r)) return r;
    if (isnan(a)) return __uint_as_float(__float_as_uint(a) | 0x00400000u);
    if (isnan(b)) return __uint_as_float(__float_as_uint(b) | 0x00400000u);
    return __uint_as_float(0xFFC00000u);
}

// One thread per element.  Q4: f32(code) * f32(half scale), then + f32(half
// min), each rounded (scripts/quantize.py:67).  Q8: same with f32 trailer.
__global__ void dequantize_kernel(const uint8_t* __restrict__ src, int64_t n, int qtype, int q8_signed,
                                  float* __restrict__ dst) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / VOXQ_QBLK;
        const int j = (int)(i % VOXQ_QBLK);
        float code, s, m;
        if (qtype == VOXQ_Q4) {
            const uint8_t* p = src + b * 20;
            const uint8_t byte = p[j >> 1];
            code = (float)((j & 1) ? (byte & 0xf) : (byte >> 4));
            s = half_bits_to_float((uint16_t)(p[16] | (p[17] << 8)));
            m = half_bits_to_float((uint16_t)(p[18] | (p[19] << 8)));
        } else {
            const uint8_t* p = src + b * 40;
            code = q8_signed ? (float)(int8_t)p[j] : (float)p[j];
            s = __uint_as_float(p[32] | (p[33] << 8) | (p[34] << 16) | ((uint32_t)p[35] << 24));
            m = __uint_as_float(p[36] | (p[37] << 8) | (p[38] << 16) | ((uint32_t)p[39] << 24));
        }
        dst[i] = x86_add(x86_mul(code, s), m);
    }
}

// Block stream <-> packed layout, one thread per block.
__global__ void pack_kernel(const uint8_t* __restrict__ blocks, int64_t nb, int qtype,
                            uint8_t* __restrict__ codes, uint8_t* __restrict__ scales, int unpack) {
    const int cb = (qtype == VOXQ_Q4) ? 16 : 32;
    const int sb = scale_bytes(qtype);
    const int bb = block_bytes(qtype);
    for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nb;
         b += (int64_t)gridDim.x * blockDim.x) {
        uint32_t* rec = reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(blocks) + b * bb);
        uint32_t* c = reinterpret_cast<uint32_t*>(codes + b * cb);
        uint32_t* s = reinterpret_cast<uint32_t*>(scales + b * sb);
        if (!unpack) {
            for (int i = 0; i < cb / 4; i++) c[i] = rec[i];
            for (int i = 0; i < sb / 4; i++) s[i] = rec[cb / 4 + i];
        } else {
            for (int i = 0; i < cb / 4; i++) rec[i] = c[i];
            for (int i = 0; i < sb / 4; i++) rec[cb / 4 + i] = s[i];
        }
    }
}

// Per-row power-of-two multiplier of a packed weight (one warp per row): the
// largest |q*scale+min| a block can produce is at q = 0 or q = max code (or
// -128 when Q8 codes are read signed), so the row maximum comes from the
// trailers alone.  rowmul = 2^e with rowmax * 2^e in [2^13, 2^14).
__global__ void rowmul_kernel(const uint8_t* __restrict__ scales, int N, int K, int qtype, float* __restrict__ rowmul) {
    const int lane = threadIdx.x & 31;
    const int nblk = K / VOXQ_QBLK;
    for (int n = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; n < N; n += (gridDim.x * blockDim.x) >> 5) {
        float mx = 0.0f;
        for (int b = lane; b < nblk; b += 32) {
            float s, m;
            if (qtype == VOXQ_Q4) {
                const uint32_t t = reinterpret_cast<const uint32_t*>(scales)[(int64_t)n * nblk + b];
                s = half_bits_to_float((uint16_t)(t & 0xffff));
                m = half_bits_to_float((uint16_t)(t >> 16));
            } else {
                const float2 t = reinterpret_cast<const float2*>(scales)[(int64_t)n * nblk + b];
                s = t.x;
                m = t.y;
            }
            const float hi = qtype == VOXQ_Q4 ? 15.0f : 255.0f;
            const float v = fmaxf(fmaxf(fabsf(m), fabsf(fmaf(hi, s, m))), qtype == VOXQ_Q8 ? fabsf(fmaf(-128.0f, s, m)) : 0.0f);
            if (isfinite(v)) mx = fmaxf(mx, v);
        }
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) {
            float r = 1.0f;
            if (mx > 0.0f) {
                int e;
                frexpf(mx, &e);  // mx in [2^(e-1), 2^e)
                r = ldexpf(1.0f, min(max(14 - e, -120), 120));
            }
            rowmul[n] = r;
        }
    }
}

static int grid_for(int64_t work, int threads) {
    int64_t g = (work + threads - 1) / threads;
    if (g < 1) g = 1;
    if (g > 148 * 16) g = 148 * 16;
    return (int)g;
}

}  // namespace voxq

using namespace voxq;

extern "C" size_t voxq_quant_bytes(size_t n, int qtype) {
    if (qtype != VOXQ_Q4 && qtype != VOXQ_Q8) return 0;
    return (n + VOXQ_QBLK - 1) / VOXQ_QBLK * (size_t)block_bytes(qtype);
}

extern "C" size_t voxq_codes_bytes(int N, int K, int qtype) {
    if (qtype != VOXQ_Q4 && qtype != VOXQ_Q8) return 0;
    return (size_t)N * (size_t)codes_row_bytes(K, qtype);
}

extern "C" size_t voxq_scales_bytes(int N, int K, int qtype) {
    if (qtype != VOXQ_Q4 && qtype != VOXQ_Q8) return 0;
    return scales_buffer_bytes(N, K, qtype);
}

static VoxCPMError check_qtype(int qtype) {
    return (qtype == VOXQ_Q4 || qtype == VOXQ_Q8) ? VOXCPM_SUCCESS : VOXCPM_ERR_UNSUPPORTED;
}

extern "C" VoxCPMError voxq_quantize(const float* d_src, size_t n, int qtype, uint8_t* d_dst, void* stream) {
    if (check_qtype(qtype)) return VOXCPM_ERR_UNSUPPORTED;
    if (n == 0) return VOXCPM_SUCCESS;
    if (!d_src || !d_dst || (reinterpret_cast<uintptr_t>(d_dst) & 3)) return VOXCPM_ERR_INTERNAL;
    const int64_t nb = (int64_t)((n + VOXQ_QBLK - 1) / VOXQ_QBLK);
    quantize_kernel<<<grid_for(nb, 128), 128, 0, (cudaStream_t)stream>>>(d_src, (int64_t)n, qtype, d_dst,
                                                                          nullptr, nullptr);
    VOXQ_CUDA_TRY(cudaGetLastError());
    return VOXCPM_SUCCESS;
}

extern "C" VoxCPMError voxq_dequantize(const uint8_t* d_src, size_t n, int qtype, int q8_signed, float* d_dst,
                                       void* stream) {
    if (check_qtype(qtype)) return VOXCPM_ERR_UNSUPPORTED;
    if (n == 0) return VOXCPM_SUCCESS;
    if (!d_src || !d_dst) return VOXCPM_ERR_INTERNAL;
    dequantize_kernel<<<grid_for((int64_t)n, 256), 256, 0, (cudaStream_t)stream>>>(d_src, (int64_t)n, qtype,
                                                                                    q8_signed, d_dst);
    VOXQ_CUDA_TRY(cudaGetLastError());
    return VOXCPM_SUCCESS;
}

static VoxCPMError check_packed(int N, int K, int qtype, const void* codes, const void* scales) {
    if (check_qtype(qtype)) return VOXCPM_ERR_UNSUPPORTED;
    if (N < 0 || K < 0 || K % VOXQ_QBLK) return VOXCPM_ERR_SHAPE_MISMATCH;
    if ((N > 0 && K > 0) && (!codes || !scales)) return VOXCPM_ERR_INTERNAL;
    if ((reinterpret_cast<uintptr_t>(codes) & 15) || (reinterpret_cast<uintptr_t>(scales) & 15))
        return VOXCPM_ERR_INTERNAL;
    return VOXCPM_SUCCESS;
}

// Zeroes the gap and padding after the trailers and computes the row multipliers.
static VoxCPMError finish_packed(void* d_scales, int N, int K, int qtype, cudaStream_t st) {
    uint8_t* sc = static_cast<uint8_t*>(d_scales);
    const size_t tb = trailer_bytes(N, K, qtype);
    VOXQ_CUDA_TRY(cudaMemsetAsync(sc + tb, 0, scales_buffer_bytes(N, K, qtype) - tb, st));
    if (N > 0 && K > 0) {
        rowmul_kernel<<<grid_for((int64_t)N * 32, 256), 256, 0, st>>>(
            sc, N, K, qtype, reinterpret_cast<float*>(sc + rowmul_offset(N, K, qtype)));
        VOXQ_CUDA_TRY(cudaGetLastError());
    }
    return VOXCPM_SUCCESS;
}

extern "C" VoxCPMError voxq_quantize_weight(const float* d_w, int N, int K, int qtype, uint8_t* d_codes,
                                            void* d_scales, uint8_t* d_blocks, void* stream) {
    VoxCPMError e = check_packed(N, K, qtype, d_codes, d_scales);
    if (e) return e;
    const int64_t n = (int64_t)N * K;
    if (n == 0) return VOXCPM_SUCCESS;
    if (d_blocks && (reinterpret_cast<uintptr_t>(d_blocks) & 3)) return VOXCPM_ERR_INTERNAL;
    const int64_t nb = n / VOXQ_QBLK;
    quantize_kernel<<<grid_for(nb, 128), 128, 0, (cudaStream_t)stream>>>(
        d_w, n, qtype, d_blocks, d_codes, reinterpret_cast<uint8_t*>(d_scales));
    VOXQ_CUDA_TRY(cudaGetLastError());
    return finish_packed(d_scales, N, K, qtype, (cudaStream_t)stream);
}

extern "C" VoxCPMError voxq_pack_blocks(const uint8_t* d_blocks, int N, int K, int qtype, uint8_t* d_codes,
                                        void* d_scales, void* stream) {
    VoxCPMError e = check_packed(N, K, qtype, d_codes, d_scales);
    if (e) return e;
    const int64_t nb = (int64_t)N * K / VOXQ_QBLK;
    if (nb == 0) return VOXCPM_SUCCESS;
    if (!d_blocks || (reinterpret_cast<uintptr_t>(d_blocks) & 3)) return VOXCPM_ERR_INTERNAL;
    pack_kernel<<<grid_for(nb, 256), 256, 0, (cudaStream_t)stream>>>(d_blocks, nb, qtype, d_codes,
                                                                      reinterpret_cast<uint8_t*>(d_scales), 0);
    VOXQ_CUDA_TRY(cudaGetLastError());
    return finish_packed(d_scales, N, K, qtype, (cudaStream_t)stream);
}

extern "C" VoxCPMError voxq_unpack_blocks(const uint8_t* d_codes, const void* d_scales, int N, int K, int qtype,
                                          uint8_t* d_blocks, void* stream) {
    VoxCPMError e = check_packed(N, K, qtype, d_codes, d_scales);
    if (e) return e;
    const int64_t nb = (int64_t)N * K / VOXQ_QBLK;
    if (nb == 0) return VOXCPM_SUCCESS;
    if (!d_blocks || (reinterpret_cast<uintptr_t>(d_blocks) & 3)) return VOXCPM_ERR_INTERNAL;
    pack_kernel<<<grid_for(nb, 256), 256, 0, (cudaStream_t)stream>>>(
        d_blocks, nb, qtype, const_cast<uint8_t*>(d_codes),
        reinterpret_cast<uint8_t*>(const_cast<void*>(d_scales)), 1);
    VOXQ_CUDA_TRY(cudaGetLastError());
    return VOXCPM_SUCCESS;
}
