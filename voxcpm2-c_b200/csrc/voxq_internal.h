// voxq_internal.h -- declarations shared between the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "voxq.h"

namespace voxq {

// Device facts cached per device.
int device_sm_count();
int current_device();

// Programmatic dependent launch on the voxq kernels (VOXQ_PDL=0 disables).
bool pdl_enabled();

// Largest activation-row count the quantized matmul runs as GEMVs (groups of
// 8 rows in one launch) instead of the tensor-core GEMM (VOXQ_GEMV_ROWS_MAX).
int gemv_rows_max();

// Grouped / single GEMV (voxq_gemv.cu).
VoxCPMError validate_item(const voxq_gemv_item& x);
VoxCPMError gemv_launch(const voxq_gemv_item* items, int count, cudaStream_t st);
// Same with a caller-provided limb workspace of gemv_workspace_bytes() bytes
// and, optionally, a caller-provided device error word (default: the
// library's per-device word).
size_t gemv_workspace_bytes(const voxq_gemv_item* items, int count);
VoxCPMError gemv_launch_ws(const voxq_gemv_item* items, int count, cudaStream_t st, void* ws, size_t ws_bytes,
                           int* err = nullptr);
VoxCPMError gemv_k0(const voxq_gemv_item& x, cudaStream_t st);

// Tensor-core GEMM for M > 8 (voxq_gemm.cu).  `ws` is a device workspace of
// at least gemm_workspace_bytes(M, N, K, qtype, swiglu) bytes, 256-byte aligned.
size_t gemm_workspace_bytes(int M, int N, int K, int qtype, bool swiglu);
VoxCPMError gemm_launch(const float* a, int M, int64_t lda, const voxq_qweight* w, float* out, int64_t ldo,
                        const voxq_epilogue* epi, void* ws, cudaStream_t st);

// Dense fp32 / fp16 weights (voxq_dense.cu).
VoxCPMError dense_launch(const float* a, int M, int64_t lda, const void* w, int w_is_fp16, int N, int K,
                         float* out, int64_t ldo, cudaStream_t st);

// fp16 -> fp32, exact (voxq_dense.cu).
VoxCPMError widen_fp16(const uint16_t* src, float* dst, size_t n, cudaStream_t st);

// Per-device device-side error word (allocated on first use, zeroed).
int* device_error_word();

// Error word of voxq_matmul_nt_q_noalloc on the current device (a static
// device variable; reading it allocates nothing).  -1 if it cannot be read.
int noalloc_error(bool clear);

// The current device's library stream (tensor_cuda_init), or nullptr when the
// library is not initialised on it.
void* library_stream();

// Drops the AudioVAE convolutions' cached device weights and staging
// (voxq_conv.cu); called by tensor_cuda_shutdown.
void conv_cache_clear();

// The packed layout of a weight that tensor_to_cuda quantized (looked up by
// its device pointer); false for any other tensor (voxq_runtime.cu).
bool device_qweight(const Tensor* w, voxq_qweight* out);

// Adds to the counters voxq_matmul_traffic reports (projections the library
// runs on behalf of an engine call other than tensor_matmul_nt_cuda).
void count_matmul_traffic(uint64_t calls, uint64_t weight_bytes);

// binary16 -> binary32 on the host, as include/tensor.h:350-371 (voxq_container.cu).
float half_to_float(uint16_t h);

// Drops the transformer blocks' device cache mirrors, norm weights and
// staging (voxq_block.cu); called by tensor_cuda_shutdown.
void block_cache_clear();

// Per-device workspace arena (voxq_runtime.cu): grows on demand, never
// shrinks, ordered on the stream that uses it.
void* workspace(size_t bytes);
void* gemv_workspace(size_t bytes);

}  // namespace voxq
