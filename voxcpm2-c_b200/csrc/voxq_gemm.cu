// voxq_gemm.cu -- quantized matmul for M > 8 activation rows.
//
// Interim path: the M rows run through the GEMV kernel in groups of eight.
// The tcgen05 tensor-core kernel replaces it.
#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

size_t gemm_workspace_bytes(int M, int K) { return 256; }

VoxCPMError gemm_launch(const float* a, int M, int64_t lda, const voxq_qweight* w, float* out, int64_t ldo,
                        const voxq_epilogue* epi, void* ws, cudaStream_t st) {
    (void)ws;
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

}  // namespace voxq
