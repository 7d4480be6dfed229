// voxq_selftest.cu -- failure-detection self-test for the bounded waits.
//
// One kernel waits, with the library's mbar_wait_bounded, on an mbarrier that
// no thread ever arrives on.  The wait gives up after `polls` suspended polls,
// records VOXQ_DEVERR_WAIT_FULL in the device error word and the kernel
// returns normally: this is how every pipeline kernel fails (no trap, no hang).
#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

__global__ void wait_timeout_kernel(int* err, uint32_t polls) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait_bounded(&bar, 0, VOXQ_DEVERR_WAIT_FULL, err, polls);
}

}  // namespace voxq

extern "C" int voxq_selftest_wait_timeout(int polls) {
    int* err = voxq::device_error_word();
    if (!err) return VOXCPM_ERR_CUDA_NOT_FOUND;
    if (polls < 1) polls = 1;
    if (polls > 100) polls = 100;
    voxq::wait_timeout_kernel<<<1, 32>>>(err, (uint32_t)polls);
    if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) return VOXCPM_ERR_INTERNAL;
    return voxq_device_error(1);
}
