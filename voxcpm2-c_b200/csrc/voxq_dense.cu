// voxq_dense.cu -- unquantized fp32 / fp16 weights (the reference's default
// path, src/tensor_cuda.cu:192-333, cuBLAS SGEMM with TF32 off there).
//
// Full fp32 arithmetic on CUDA cores: a warp-per-row GEMV for M <= 8 and a
// register-tiled SIMT GEMM otherwise.  This path serves weights that are not
// quantized (VOXCPM_QUANT unset, or K % 32 != 0); the quantized kernels are
// the hot path.
#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

template <bool F16>
__device__ __forceinline__ float wload(const void* w, int64_t i) {
    if (F16) return __half2float(reinterpret_cast<const __half*>(w)[i]);
    return reinterpret_cast<const float*>(w)[i];
}

// One warp per weight row, all M (<= 8) activation rows at once.
template <bool F16>
__global__ void __launch_bounds__(256) dense_gemv_kernel(const float* __restrict__ a, int M, int64_t lda,
                                                         const void* __restrict__ w, int N, int K,
                                                         float* __restrict__ out, int64_t ldo) {
    const int lane = threadIdx.x & 31;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int n = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; n < N; n += nwarps) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const int64_t wrow = (int64_t)n * K;
        for (int k = lane; k < K; k += 32) {
            const float wv = wload<F16>(w, wrow + k);
#pragma unroll
            for (int m = 0; m < 8; m++)
                if (m < M) acc[m] = fmaf(a[m * lda + k], wv, acc[m]);
        }
#pragma unroll
        for (int m = 0; m < 8; m++) {
            float v = acc[m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && m < M) out[m * ldo + n] = v;
        }
    }
}

// 64x64 output tile, BK = 16, 256 threads, 4x4 outputs per thread.
template <bool F16>
__global__ void __launch_bounds__(256) dense_gemm_kernel(const float* __restrict__ a, int M, int64_t lda,
                                                         const void* __restrict__ w, int N, int K,
                                                         float* __restrict__ out, int64_t ldo) {
    __shared__ float As[16][64 + 4];
    __shared__ float Ws[16][64 + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int i = threadIdx.x; i < 64 * 16; i += 256) {
            const int r = i >> 4, c = i & 15;
            const int m = m0 + r, n = n0 + r, k = k0 + c;
            As[c][r] = (m < M && k < K) ? a[m * lda + k] : 0.0f;
            Ws[c][r] = (n < N && k < K) ? wload<F16>(w, (int64_t)n * K + k) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int c = 0; c < 16; c++) {
            float av[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) av[i] = As[c][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; j++) wv[j] = Ws[c][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
            if (m < M && n < N) out[m * ldo + n] = acc[i][j];
        }
}

__global__ void widen_kernel(const uint16_t* __restrict__ src, float* __restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __half2float(__ushort_as_half(src[i]));
}

VoxCPMError widen_fp16(const uint16_t* src, float* dst, size_t n, cudaStream_t st) {
    if (n == 0) return VOXCPM_SUCCESS;
    int blocks = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
    widen_kernel<<<blocks, 256, 0, st>>>(src, dst, (int64_t)n);
    VOXQ_CUDA_TRY(cudaGetLastError());
    return VOXCPM_SUCCESS;
}

VoxCPMError dense_launch(const float* a, int M, int64_t lda, const void* w, int w_is_fp16, int N, int K,
                         float* out, int64_t ldo, cudaStream_t st) {
    if (M == 0 || N == 0) return VOXCPM_SUCCESS;
    if (!a || !w || !out) return VOXCPM_ERR_INTERNAL;
    if (M <= 8) {
        int blocks = (N + 7) / 8;
        if (blocks > device_sm_count() * 8) blocks = device_sm_count() * 8;
        if (w_is_fp16)
            dense_gemv_kernel<true><<<blocks, 256, 0, st>>>(a, M, lda, w, N, K, out, ldo);
        else
            dense_gemv_kernel<false><<<blocks, 256, 0, st>>>(a, M, lda, w, N, K, out, ldo);
    } else {
        dim3 grid((N + 63) / 64, (M + 63) / 64);
        if (w_is_fp16)
            dense_gemm_kernel<true><<<grid, 256, 0, st>>>(a, M, lda, w, N, K, out, ldo);
        else
            dense_gemm_kernel<false><<<grid, 256, 0, st>>>(a, M, lda, w, N, K, out, ldo);
    }
    VOXQ_CUDA_TRY(cudaGetLastError());
    return VOXCPM_SUCCESS;
}

}  // namespace voxq
