// voxq_noalloc.cu -- the quantized GEMV entry point that allocates nothing.
//
// Some callers cannot let a library allocate device memory on their behalf:
// engines that reserve their whole device-memory budget up front (weights,
// KV caches, activation arenas) and run streaming synthesis against that fixed
// budget, or hosts whose policy forbids device allocation once set-up is done
// because cudaMalloc / cudaFree can synchronise the whole device and stall a
// real-time audio stream at an unpredictable moment.  voxq_matmul_nt_q gets
// its activation-limb scratch from a growable per-device arena (cudaMalloc on
// first use or growth); this variant instead uses one fixed array that the
// library image itself carries in device memory.
//
// The scratch is a file-scope static __device__ array of
// VOXQ_NOALLOC_SCRATCH_BYTES bytes (896 KiB).  The activation limbs take
// M * 7 * K / 2 bytes for Q4 and M * 4 * K bytes for Q8, so the array covers
// every GEMV shape the kernel accepts: M <= 8 rows, K <= 32768 for Q4
// (917,504 bytes at the limit) and K <= 16384 for Q8 (524,288 bytes).  Every
// GPU that loads the library holds it until the process exits.  Host code
// cannot hand the array's name to a kernel (on the host it is only a
// stand-in, not a device address), so the device address is looked up with
// cudaGetSymbolAddress once per device, on that device's first call.
//
// Kernels launched here record a bounded wait that gave up in this file's own
// error word, g_noalloc_error.  voxq_noalloc_device_error reads it without
// allocating anything; voxq_device_error reports it too.
#include <mutex>

#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

static __device__ __align__(256) uint8_t g_noalloc_scratch[VOXQ_NOALLOC_SCRATCH_BYTES];
static __device__ int g_noalloc_error;  // this entry point's device error word

namespace {
constexpr int kMaxDevices = 16;
struct NoallocDev {
    bool ready = false;
    void* scratch = nullptr;
    int* err = nullptr;
};
NoallocDev g_na[kMaxDevices];
std::mutex g_na_mu;

// Resolves (once per device, with that device current) the device addresses
// of the static scratch array and error word, and clears the error word on the
// caller's stream (waiting for it, so the clear is done before any launch on
// any stream).
VoxCPMError noalloc_setup(int dev, cudaStream_t st, NoallocDev** out) {
    std::lock_guard<std::mutex> lk(g_na_mu);
    NoallocDev& d = g_na[dev];
    if (!d.ready) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            fprintf(stderr, "[voxq] noalloc: cudaGetSymbolAddress(scratch) failed on device %d: %s\n", dev,
                    cudaGetErrorString(e));
            return VOXCPM_ERR_INTERNAL;
        }
        void* q = nullptr;
        e = cudaGetSymbolAddress(&q, g_noalloc_error);
        if (e != cudaSuccess) {
            fprintf(stderr, "[voxq] noalloc: cudaGetSymbolAddress(error word) failed on device %d: %s\n", dev,
                    cudaGetErrorString(e));
            return VOXCPM_ERR_INTERNAL;
        }
        e = cudaMemsetAsync(q, 0, sizeof(int), st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) {
            fprintf(stderr, "[voxq] noalloc: clearing the error word failed on device %d: %s\n", dev,
                    cudaGetErrorString(e));
            return VOXCPM_ERR_INTERNAL;
        }
        d.scratch = p;
        d.err = static_cast<int*>(q);
        d.ready = true;
    }
    *out = &d;
    return VOXCPM_SUCCESS;
}
}  // namespace

int noalloc_error(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_noalloc_error, sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    if (clear && v) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_noalloc_error, &zero, sizeof(int)) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
    }
    return v;
}

}  // namespace voxq

using namespace voxq;

extern "C" VoxCPMError voxq_matmul_nt_q_noalloc(const float* d_a, int M, int64_t lda, const voxq_qweight* w,
                                                float* d_out, int64_t ldo, const voxq_epilogue* epi, void* stream) {
    if (!w) return VOXCPM_ERR_INTERNAL;
    if (M < 0 || w->N < 0 || w->K < 0) return VOXCPM_ERR_SHAPE_MISMATCH;
    if (M == 0 || w->N == 0) return VOXCPM_SUCCESS;
    if (M > 8) {
        fprintf(stderr, "[voxq] voxq_matmul_nt_q_noalloc: M = %d, at most 8 activation rows\n", M);
        return VOXCPM_ERR_UNSUPPORTED;
    }
    const voxq_qweight* up = epi ? epi->up : nullptr;
    if (up && (up->N != w->N || up->K != w->K || up->qtype != w->qtype || up->q8_signed != w->q8_signed))
        return VOXCPM_ERR_SHAPE_MISMATCH;
    voxq_gemv_item it = {};
    it.w = *w;
    it.a = d_a;
    it.out = d_out;
    it.M = M;
    it.lda = (int32_t)lda;
    it.ldo = (int32_t)ldo;
    if (epi) {
        it.bias = epi->bias;
        it.residual = epi->residual;
        it.ldr = (int32_t)epi->ldr;
        if (up) {
            it.up_codes = up->codes;
            it.up_scales = up->scales;
        }
    }
    VoxCPMError e = validate_item(it);
    if (e) return e;
    const size_t need = gemv_workspace_bytes(&it, 1);
    if (need > VOXQ_NOALLOC_SCRATCH_BYTES) {
        fprintf(stderr, "[voxq] voxq_matmul_nt_q_noalloc: needs %zu scratch bytes, the fixed array holds %d\n", need,
                (int)VOXQ_NOALLOC_SCRATCH_BYTES);
        return VOXCPM_ERR_OOM;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return VOXCPM_ERR_CUDA_NOT_FOUND;
    NoallocDev* d = nullptr;
    e = noalloc_setup(dev, (cudaStream_t)stream, &d);
    if (e) return e;
    return gemv_launch_ws(&it, 1, (cudaStream_t)stream, d->scratch, VOXQ_NOALLOC_SCRATCH_BYTES, d->err);
}

extern "C" int voxq_noalloc_device_error(int clear) { return noalloc_error(clear != 0); }
