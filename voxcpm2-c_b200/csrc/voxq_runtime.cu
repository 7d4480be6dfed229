// voxq_runtime.cu -- device state, workspace arena and the reference ABI.
//
// Implements the CUDA block of the reference's include/tensor.h (316-342)
// with the semantics of src/tensor_cuda.cu, re-designed for a resident,
// quantized weight set:
//   * no per-call cudaMalloc/cudaFree: per-device arenas for the activation
//     and output staging and the GEMM workspace, pinned host staging buffers;
//   * one non-blocking stream per device; a call synchronises only when its
//     output lives on the host (the reference syncs the whole device twice);
//   * under VOXCPM_QUANT=q8|q4, tensor_to_cuda quantizes 2-D weights on the
//     device (bit-exact with scripts/quantize.py) and keeps only the packed
//     blocks; a side table maps the tensor's device pointer to its layout.
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

static constexpr int kMaxDev = 16;
static constexpr int kSlots = 5;  // 0: activation, 1: output, 2: temp weight, 3: GEMM workspace, 4: GEMV limbs

struct QRec {
    void* base;      // one allocation: codes, then scales
    uint8_t* codes;
    void* scales;
    int N, K, qtype;
    bool from_fp16;
};

struct DevState {
    int* err = nullptr;  // device-side error word of the bounded waits
    bool init = false;
    int quant = VOXQ_F32;  // format tensor_to_cuda gives 2-D weights
    int sms = 0;
    cudaStream_t stream = nullptr;
    void* slot[kSlots] = {};
    size_t slot_bytes[kSlots] = {};
    void* h_in = nullptr;  // pinned staging
    size_t h_in_bytes = 0;
    void* h_out = nullptr;
    size_t h_out_bytes = 0;
    std::vector<void*> retired;  // outgrown workspace buffers, freed at shutdown
};

// Blocks of a pre-quantized weight waiting for tensor_to_cuda
// (voxq_tensor_attach_blocks), keyed by the host tensor; `data` is the
// tensor's host buffer at attach time, so a tensor later allocated at the
// same address does not inherit them.
struct Pending {
    int qtype;
    void* blocks;
    size_t nbytes;
    const void* data;
};

static DevState g_dev[kMaxDev];
static std::mutex g_mu;  // guards g_dev growth and the side tables
static std::unordered_map<const void*, QRec> g_qtab;
static std::unordered_map<const Tensor*, Pending> g_pending;
static std::atomic<int> g_pending_n{0};
static thread_local int t_dev = -1;

int current_device() {
    if (t_dev >= 0) return t_dev;
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) d = 0;
    return d;
}

int device_sm_count() {
    int d = 0;
    cudaGetDevice(&d);
    if (d < 0 || d >= kMaxDev) return 148;
    if (g_dev[d].sms == 0) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
        g_dev[d].sms = v > 0 ? v : 148;
    }
    return g_dev[d].sms;
}

int gemv_rows_max() {
    static const int v = [] {
        const char* e = getenv("VOXQ_GEMV_ROWS_MAX");
        const int r = e ? atoi(e) : 8;
        return r >= 8 && r <= 64 ? r / 8 * 8 : 8;
    }();
    return v;
}

bool pdl_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("VOXQ_PDL");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

// Grows slot k to at least `bytes`.  The old buffer may still be read by work
// queued on any stream, so it is not freed here (that would need a device-wide
// synchronisation in the middle of a call): it is retired and freed at
// tensor_cuda_shutdown.  Growth is geometric, so the retired buffers total less
// than the live one.
static void* slot_get(DevState& s, int k, size_t bytes) {
    if (bytes == 0) bytes = 256;
    if (s.slot_bytes[k] >= bytes) return s.slot[k];
    size_t want = 1 << 20;
    while (want < bytes) want <<= 1;
    void* p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (s.slot[k]) s.retired.push_back(s.slot[k]);
    s.slot[k] = p;
    s.slot_bytes[k] = want;
    return p;
}

int* device_error_word() {
    int d = 0;
    cudaGetDevice(&d);
    if (d < 0 || d >= kMaxDev) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    DevState& s = g_dev[d];
    if (!s.err) {
        if (cudaMalloc(&s.err, sizeof(int)) != cudaSuccess) {
            s.err = nullptr;
            return nullptr;
        }
        cudaMemset(s.err, 0, sizeof(int));
    }
    return s.err;
}

void* workspace(size_t bytes) {
    int d = 0;
    cudaGetDevice(&d);
    std::lock_guard<std::mutex> lk(g_mu);
    return slot_get(g_dev[d], 3, bytes);
}

void* gemv_workspace(size_t bytes) {
    int d = 0;
    cudaGetDevice(&d);
    std::lock_guard<std::mutex> lk(g_mu);
    return slot_get(g_dev[d], 4, bytes);
}

static bool pinned_get(void** p, size_t* have, size_t bytes) {
    if (*have >= bytes) return true;
    size_t want = 1 << 16;
    while (want < bytes) want <<= 1;
    if (*p) cudaFreeHost(*p);
    *p = nullptr;
    *have = 0;
    if (cudaMallocHost(p, want) != cudaSuccess) {
        *p = nullptr;
        return false;
    }
    *have = want;
    return true;
}

static int parse_quant_env() {
    const char* e = getenv("VOXCPM_QUANT");
    if (!e || !*e) return VOXQ_F32;
    if (!strcmp(e, "q8") || !strcmp(e, "Q8")) return VOXQ_Q8;
    if (!strcmp(e, "q4") || !strcmp(e, "Q4")) return VOXQ_Q4;
    return VOXQ_F32;
}

static DevState* state() {
    int d = current_device();
    if (d < 0 || d >= kMaxDev) return nullptr;
    return &g_dev[d];
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

bool device_qweight(const Tensor* w, voxq_qweight* out) {
    if (!w || !w->is_cuda || !w->data) return false;
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_qtab.find(w->data);
    if (it == g_qtab.end()) return false;
    const QRec& q = it->second;
    *out = voxq_qweight{q.codes, q.scales, q.N, q.K, q.qtype, 0};
    return true;
}

void* library_stream() {
    DevState* s = state();
    return (s && s->init) ? (void*)s->stream : nullptr;
}

}  // namespace voxq

using namespace voxq;

// ===========================================================================
// Additive entry points
// ===========================================================================

extern "C" const char* voxq_version(void) { return "voxq-b200 0.1 (sm_100a)"; }

// tensor_matmul_nt_cuda's work counters (voxq_matmul_traffic)
static std::atomic<uint64_t> g_mm_calls{0}, g_mm_wbytes{0};

void voxq::count_matmul_traffic(uint64_t calls, uint64_t weight_bytes) {
    g_mm_calls.fetch_add(calls, std::memory_order_relaxed);
    g_mm_wbytes.fetch_add(weight_bytes, std::memory_order_relaxed);
}

extern "C" void voxq_matmul_traffic(uint64_t* calls, uint64_t* weight_bytes, int reset) {
    const uint64_t c = reset ? g_mm_calls.exchange(0) : g_mm_calls.load();
    const uint64_t b = reset ? g_mm_wbytes.exchange(0) : g_mm_wbytes.load();
    if (calls) *calls = c;
    if (weight_bytes) *weight_bytes = b;
}

extern "C" int voxq_device_error(int clear) {
    int* e = device_error_word();
    if (!e) return -1;
    int v = 0;
    if (cudaMemcpy(&v, e, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (clear && v && cudaMemset(e, 0, sizeof(int)) != cudaSuccess) return -1;
    const int na = noalloc_error(clear != 0);
    if (na < 0) return -1;
    return v ? v : na;
}

extern "C" VoxCPMError voxq_tensor_attach_blocks(const Tensor* t, int qtype, void* blocks, size_t nbytes) {
    if (!t || !blocks) return VOXCPM_ERR_INTERNAL;
    if (qtype != VOXQ_Q4 && qtype != VOXQ_Q8) return VOXCPM_ERR_UNSUPPORTED;
    if (t->is_cuda || t->ndim != 2 || !t->shape || t->shape[0] <= 0 || t->shape[1] <= 0 ||
        t->shape[1] % VOXQ_QBLK != 0)
        return VOXCPM_ERR_SHAPE_MISMATCH;
    if (nbytes != voxq_quant_bytes((size_t)t->shape[0] * t->shape[1], qtype)) return VOXCPM_ERR_SHAPE_MISMATCH;
    const void* data = t->is_fp16 ? (const void*)t->data_fp16 : (const void*)t->data;
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_pending.find(t);
    if (it != g_pending.end()) {
        free(it->second.blocks);
        it->second = Pending{qtype, blocks, nbytes, data};
    } else {
        g_pending.emplace(t, Pending{qtype, blocks, nbytes, data});
        g_pending_n.fetch_add(1);
    }
    return VOXCPM_SUCCESS;
}

// Removes t's pending blocks from the table into *out (true) or reports none.
static bool take_pending(const Tensor* t, Pending* out) {
    if (g_pending_n.load() == 0) return false;
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_pending.find(t);
    if (it == g_pending.end()) return false;
    *out = it->second;
    g_pending.erase(it);
    g_pending_n.fetch_sub(1);
    return true;
}

extern "C" int voxq_tensor_detach_blocks(const Tensor* t) {
    Pending p;
    if (!take_pending(t, &p)) return 0;
    free(p.blocks);
    return 1;
}

extern "C" VoxCPMError voxq_set_device(int device) {
    if (device < 0 || device >= kMaxDev) return VOXCPM_ERR_CUDA_NOT_FOUND;
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        return VOXCPM_ERR_CUDA_NOT_FOUND;
    }
    t_dev = device;
    return VOXCPM_SUCCESS;
}

extern "C" VoxCPMError voxq_matmul_nt_q(const float* d_a, int M, int64_t lda, const voxq_qweight* w, float* d_out,
                                        int64_t ldo, const voxq_epilogue* epi, void* stream) {
    if (!w) return VOXCPM_ERR_INTERNAL;
    if (M < 0 || w->N < 0 || w->K < 0) return VOXCPM_ERR_SHAPE_MISMATCH;
    if (M == 0 || w->N == 0) return VOXCPM_SUCCESS;
    const voxq_qweight* up = epi ? epi->up : nullptr;
    if (up && (up->N != w->N || up->K != w->K || up->qtype != w->qtype || up->q8_signed != w->q8_signed))
        return VOXCPM_ERR_SHAPE_MISMATCH;
    cudaStream_t st = (cudaStream_t)stream;
    if (M <= gemv_rows_max()) {
        // groups of up to 8 activation rows, one GEMV item each, in one launch
        voxq_gemv_item its[VOXQ_MAX_BATCH / 2];
        const int groups = (M + 7) / 8;
        for (int g = 0; g < groups; g++) {
            voxq_gemv_item& it = its[g];
            it = voxq_gemv_item{};
            const int m0 = 8 * g;
            it.w = *w;
            it.a = d_a + (int64_t)m0 * lda;
            it.out = d_out + (int64_t)m0 * ldo;
            it.M = M - m0 < 8 ? M - m0 : 8;
            it.lda = (int32_t)lda;
            it.ldo = (int32_t)ldo;
            if (epi) {
                it.bias = epi->bias;
                it.residual = epi->residual ? epi->residual + (int64_t)m0 * epi->ldr : nullptr;
                it.ldr = (int32_t)epi->ldr;
                if (up) {
                    it.up_codes = up->codes;
                    it.up_scales = up->scales;
                }
            }
        }
        return gemv_launch(its, groups, st);
    }
    void* ws = workspace(gemm_workspace_bytes(M, w->N, w->K, w->qtype, up != nullptr));
    if (!ws) return VOXCPM_ERR_OOM;
    return gemm_launch(d_a, M, lda, w, d_out, ldo, epi, ws, st);
}

extern "C" VoxCPMError voxq_matmul_nt_dense(const float* d_a, int M, int64_t lda, const void* d_w, int w_is_fp16,
                                            int N, int K, float* d_out, int64_t ldo, void* stream) {
    if (M < 0 || N < 0 || K < 0) return VOXCPM_ERR_SHAPE_MISMATCH;
    if (M == 0 || N == 0) return VOXCPM_SUCCESS;
    if (lda < K || ldo < N) return VOXCPM_ERR_SHAPE_MISMATCH;
    return dense_launch(d_a, M, lda, d_w, w_is_fp16, N, K, d_out, ldo, (cudaStream_t)stream);
}

// ===========================================================================
// Reference ABI: include/tensor.h:316-342 (src/tensor_cuda.cu)
// ===========================================================================

extern "C" VoxCPMError tensor_cuda_init(void) {
    DevState* s = state();
    if (!s) return VOXCPM_ERR_CUDA_NOT_FOUND;
    if (s->init) return VOXCPM_SUCCESS;
    const int d = current_device();
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || d >= n) {
        cudaGetLastError();
        fprintf(stderr, "[voxq] no CUDA device %d available\n", d);
        return VOXCPM_ERR_CUDA_NOT_FOUND;
    }
    if (cudaSetDevice(d) != cudaSuccess || cudaFree(0) != cudaSuccess) {
        cudaGetLastError();
        return VOXCPM_ERR_CUDA_NOT_FOUND;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, d) == cudaSuccess && prop.major < 10) {
        fprintf(stderr, "[voxq] device %d is sm_%d%d; this library is built for sm_100a only\n", d, prop.major,
                prop.minor);
        return VOXCPM_ERR_CUDA_NOT_FOUND;
    }
    VOXQ_CUDA_TRY(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
    s->quant = parse_quant_env();
    s->init = true;
    return VOXCPM_SUCCESS;
}

extern "C" void tensor_cuda_shutdown(void) {
    DevState* s = state();
    if (!s || !s->init) return;
    cudaStreamSynchronize(s->stream);
    cudaDeviceSynchronize();  // the workspaces may also serve voxq_* calls on other streams
    conv_cache_clear();
    block_cache_clear();
    for (int k = 0; k < kSlots; k++) {
        if (s->slot[k]) cudaFree(s->slot[k]);
        s->slot[k] = nullptr;
        s->slot_bytes[k] = 0;
    }
    for (void* p : s->retired) cudaFree(p);
    s->retired.clear();
    if (s->h_in) cudaFreeHost(s->h_in);
    if (s->h_out) cudaFreeHost(s->h_out);
    s->h_in = s->h_out = nullptr;
    s->h_in_bytes = s->h_out_bytes = 0;
    cudaStreamDestroy(s->stream);
    s->stream = nullptr;
    s->init = false;
}

static bool lookup_q(const void* p, QRec* out) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_qtab.find(p);
    if (it == g_qtab.end()) return false;
    *out = it->second;
    return true;
}

// tensor_to_cuda for a weight with attached pre-quantized blocks: the blocks
// go to the packed device layout as they are (voxq_pack_blocks), the host
// buffers are freed, and the tensor becomes the same opaque device weight the
// quantizing upload makes.
static VoxCPMError upload_attached(DevState* s, Tensor* t, const Pending& pb) {
    const int N = t->shape[0], K = t->shape[1], qt = pb.qtype;
    const size_t cb = voxq_codes_bytes(N, K, qt), sb = voxq_scales_bytes(N, K, qt);
    uint8_t* d_blocks = nullptr;
    void* base = nullptr;
    auto fail = [&](VoxCPMError e, cudaError_t ce, const char* what) {
        if (ce != cudaSuccess)
            fprintf(stderr, "[voxq] tensor_to_cuda (attached blocks): %s failed: %s\n", what, cudaGetErrorString(ce));
        cudaStreamSynchronize(s->stream);
        cudaGetLastError();
        if (d_blocks) cudaFree(d_blocks);
        if (base) cudaFree(base);
        free(pb.blocks);
        return e;
    };
    cudaError_t ce;
    if ((ce = cudaMalloc(&d_blocks, pb.nbytes)) != cudaSuccess) {
        d_blocks = nullptr;
        return fail(VOXCPM_ERR_OOM, ce, "cudaMalloc");
    }
    if ((ce = cudaMalloc(&base, align256(cb) + sb)) != cudaSuccess) {
        base = nullptr;
        return fail(VOXCPM_ERR_OOM, ce, "cudaMalloc");
    }
    if ((ce = cudaMemcpyAsync(d_blocks, pb.blocks, pb.nbytes, cudaMemcpyHostToDevice, s->stream)) != cudaSuccess)
        return fail(VOXCPM_ERR_INTERNAL, ce, "cudaMemcpy");
    uint8_t* codes = (uint8_t*)base;
    void* scales = (uint8_t*)base + align256(cb);
    VoxCPMError e = voxq_pack_blocks(d_blocks, N, K, qt, codes, scales, s->stream);
    if (e) return fail(e, cudaSuccess, "");
    if ((ce = cudaStreamSynchronize(s->stream)) != cudaSuccess)
        return fail(VOXCPM_ERR_INTERNAL, ce, "cudaStreamSynchronize");
    cudaFree(d_blocks);
    free(pb.blocks);
    {
        std::lock_guard<std::mutex> lk(g_mu);
        g_qtab[base] = QRec{base, codes, scales, N, K, qt, false};
    }
    if (t->is_fp16) {
        free(t->data_fp16);
        t->data_fp16 = nullptr;
        t->is_fp16 = false;
    } else {
        free(t->data);
    }
    t->data = (float*)base;
    t->is_cuda = true;
    return VOXCPM_SUCCESS;
}

extern "C" VoxCPMError tensor_to_cuda(Tensor* t) {
    if (!t) return VOXCPM_ERR_INTERNAL;
    if (t->is_cuda) return VOXCPM_SUCCESS;
    if (t->size == 0) return VOXCPM_SUCCESS;
    DevState* s = state();
    if (!s || !s->init) return VOXCPM_ERR_CUDA_NOT_FOUND;
    {
        Pending pb;
        if (take_pending(t, &pb)) {
            const void* data = t->is_fp16 ? (const void*)t->data_fp16 : (const void*)t->data;
            // blocks attached to an earlier tensor at this address: dropped
            if (data == pb.data && t->ndim == 2 &&
                pb.nbytes == voxq_quant_bytes((size_t)t->shape[0] * t->shape[1], pb.qtype))
                return upload_attached(s, t, pb);
            free(pb.blocks);
        }
    }
    const bool quantize = s->quant != VOXQ_F32 && t->ndim == 2 && t->shape[1] > 0 &&
                          t->shape[1] % VOXQ_QBLK == 0 && (t->is_fp16 ? t->data_fp16 != nullptr : t->data != nullptr);
    if (quantize) {
        const int N = t->shape[0], K = t->shape[1], qt = s->quant;
        const size_t n = (size_t)N * K;
        const size_t cb = voxq_codes_bytes(N, K, qt), sb = voxq_scales_bytes(N, K, qt);
        // every temporary is released on every exit; `base` is kept only on success
        float* d_f32 = nullptr;
        uint16_t* d_h = nullptr;
        void* base = nullptr;
        auto fail = [&](VoxCPMError e, cudaError_t ce, const char* what) {
            if (ce != cudaSuccess)
                fprintf(stderr, "[voxq] tensor_to_cuda: %s failed: %s\n", what, cudaGetErrorString(ce));
            cudaStreamSynchronize(s->stream);
            cudaGetLastError();
            if (d_h) cudaFree(d_h);
            if (d_f32) cudaFree(d_f32);
            if (base) cudaFree(base);
            return e;
        };
        cudaError_t ce;
        if ((ce = cudaMalloc(&d_f32, n * sizeof(float))) != cudaSuccess) {
            d_f32 = nullptr;
            return fail(VOXCPM_ERR_OOM, ce, "cudaMalloc");
        }
        if ((ce = cudaMalloc(&base, align256(cb) + sb)) != cudaSuccess) {
            base = nullptr;
            return fail(VOXCPM_ERR_OOM, ce, "cudaMalloc");
        }
        if (t->is_fp16) {
            if ((ce = cudaMalloc(&d_h, n * 2)) != cudaSuccess) {
                d_h = nullptr;
                return fail(VOXCPM_ERR_OOM, ce, "cudaMalloc");
            }
            // on the library stream: the kernels below read d_h there (a synchronous copy
            // from pageable memory may return before its DMA lands, and the library's
            // non-blocking stream is not ordered behind the legacy stream)
            if ((ce = cudaMemcpyAsync(d_h, t->data_fp16, n * 2, cudaMemcpyHostToDevice, s->stream)) != cudaSuccess)
                return fail(VOXCPM_ERR_INTERNAL, ce, "cudaMemcpy");
            // exact widening, then the quantizer sees the same floats quantize.py would
            VoxCPMError e = widen_fp16(d_h, d_f32, n, s->stream);
            if (e) return fail(e, cudaSuccess, "");
        } else if ((ce = cudaMemcpyAsync(d_f32, t->data, n * sizeof(float), cudaMemcpyHostToDevice, s->stream)) !=
                   cudaSuccess) {
            return fail(VOXCPM_ERR_INTERNAL, ce, "cudaMemcpy");
        }
        uint8_t* codes = (uint8_t*)base;
        void* scales = (uint8_t*)base + align256(cb);
        VoxCPMError e = voxq_quantize_weight(d_f32, N, K, qt, codes, scales, nullptr, s->stream);
        if (e) return fail(e, cudaSuccess, "");
        if ((ce = cudaStreamSynchronize(s->stream)) != cudaSuccess)
            return fail(VOXCPM_ERR_INTERNAL, ce, "cudaStreamSynchronize");
        if (d_h) cudaFree(d_h);
        cudaFree(d_f32);
        {
            std::lock_guard<std::mutex> lk(g_mu);
            g_qtab[base] = QRec{base, codes, scales, N, K, qt, t->is_fp16};
        }
        if (t->is_fp16) {
            free(t->data_fp16);
            t->data_fp16 = nullptr;
            t->is_fp16 = false;
        } else {
            free(t->data);
        }
        t->data = (float*)base;  // opaque packed weight; only tensor_* calls read it
        t->is_cuda = true;
        return VOXCPM_SUCCESS;
    }
    if (t->is_fp16) {
        if (!t->data_fp16) return VOXCPM_ERR_INTERNAL;
        const size_t bytes = t->size * sizeof(uint16_t);
        uint16_t* d = nullptr;
        VOXQ_CUDA_TRY(cudaMalloc(&d, bytes));
        VOXQ_CUDA_TRY(cudaMemcpyAsync(d, t->data_fp16, bytes, cudaMemcpyHostToDevice, s->stream));
        VOXQ_CUDA_TRY(cudaStreamSynchronize(s->stream));  // before the host buffer is freed
        free(t->data_fp16);
        t->data_fp16 = d;
        t->is_cuda = true;
        return VOXCPM_SUCCESS;
    }
    if (!t->data) return VOXCPM_SUCCESS;
    float* d = nullptr;
    VOXQ_CUDA_TRY(cudaMalloc(&d, t->size * sizeof(float)));
    VOXQ_CUDA_TRY(cudaMemcpyAsync(d, t->data, t->size * sizeof(float), cudaMemcpyHostToDevice, s->stream));
    VOXQ_CUDA_TRY(cudaStreamSynchronize(s->stream));  // before the host buffer is freed
    free(t->data);
    t->data = d;
    t->is_cuda = true;
    return VOXCPM_SUCCESS;
}

extern "C" VoxCPMError tensor_to_cpu(Tensor* t) {
    if (!t) return VOXCPM_ERR_INTERNAL;
    if (!t->is_cuda) return VOXCPM_SUCCESS;
    if (t->size == 0) return VOXCPM_SUCCESS;
    DevState* s = state();
    if (s && s->init) VOXQ_CUDA_TRY(cudaStreamSynchronize(s->stream));
    QRec q;
    if (t->data && lookup_q(t->data, &q)) {
        const size_t n = (size_t)q.N * q.K;
        uint8_t* d_blocks = nullptr;
        float* d_f = nullptr;
        VOXQ_CUDA_TRY(cudaMalloc(&d_blocks, voxq_quant_bytes(n, q.qtype)));
        VOXQ_CUDA_TRY(cudaMalloc(&d_f, n * sizeof(float)));
        cudaStream_t st = s ? s->stream : nullptr;
        VoxCPMError e = voxq_unpack_blocks(q.codes, q.scales, q.N, q.K, q.qtype, d_blocks, st);
        if (!e) e = voxq_dequantize(d_blocks, n, q.qtype, 0, d_f, st);
        if (e) return e;
        float* h = (float*)malloc(n * sizeof(float));
        if (!h) return VOXCPM_ERR_OOM;
        VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
        VOXQ_CUDA_TRY(cudaMemcpy(h, d_f, n * sizeof(float), cudaMemcpyDeviceToHost));
        cudaFree(d_blocks);
        cudaFree(d_f);
        cudaFree(q.base);
        {
            std::lock_guard<std::mutex> lk(g_mu);
            g_qtab.erase(q.base);
        }
        t->data = h;
        t->is_cuda = false;
        return VOXCPM_SUCCESS;
    }
    if (t->is_fp16) {
        if (!t->data_fp16) return VOXCPM_ERR_INTERNAL;
        const size_t bytes = t->size * sizeof(uint16_t);
        uint16_t* h = (uint16_t*)malloc(bytes);
        if (!h) return VOXCPM_ERR_OOM;
        VOXQ_CUDA_TRY(cudaMemcpy(h, t->data_fp16, bytes, cudaMemcpyDeviceToHost));
        VOXQ_CUDA_TRY(cudaFree(t->data_fp16));
        t->data_fp16 = h;
        t->is_cuda = false;
        return VOXCPM_SUCCESS;
    }
    if (!t->data) return VOXCPM_SUCCESS;
    float* h = (float*)malloc(t->size * sizeof(float));
    if (!h) return VOXCPM_ERR_OOM;
    VOXQ_CUDA_TRY(cudaMemcpy(h, t->data, t->size * sizeof(float), cudaMemcpyDeviceToHost));
    VOXQ_CUDA_TRY(cudaFree(t->data));
    t->data = h;
    t->is_cuda = false;
    return VOXCPM_SUCCESS;
}

extern "C" VoxCPMError tensor_cuda_free(Tensor* t) {
    if (!t) return VOXCPM_ERR_INTERNAL;
    if (t->is_cuda) {
        DevState* s = state();
        if (s && s->init) cudaStreamSynchronize(s->stream);
        QRec q;
        if (t->data && lookup_q(t->data, &q)) {
            VOXQ_CUDA_TRY(cudaFree(q.base));
            std::lock_guard<std::mutex> lk(g_mu);
            g_qtab.erase(q.base);
            t->data = nullptr;
        } else if (t->is_fp16 && t->data_fp16) {
            VOXQ_CUDA_TRY(cudaFree(t->data_fp16));
            t->data_fp16 = nullptr;
        } else if (t->data) {
            VOXQ_CUDA_TRY(cudaFree(t->data));
            t->data = nullptr;
        }
        t->is_cuda = false;
    }
    return VOXCPM_SUCCESS;
}

extern "C" VoxCPMError tensor_cuda_upload_weight(Tensor** t_ptr) {
    if (!t_ptr || !*t_ptr) return VOXCPM_SUCCESS;
    return tensor_to_cuda(*t_ptr);
}

extern "C" VoxCPMError tensor_matmul_nt_cuda(const Tensor* a, const Tensor* b, Tensor* out) {
    if (!a || !b || !out) return VOXCPM_ERR_INTERNAL;
    if (a->ndim != 2 || b->ndim != 2) return VOXCPM_ERR_SHAPE_MISMATCH;
    const int M = a->shape[0], K = a->shape[1], N = b->shape[0];
    if (b->shape[1] != K) return VOXCPM_ERR_SHAPE_MISMATCH;
    if (out->ndim != 2 || out->shape[0] != M || out->shape[1] != N) return VOXCPM_ERR_SHAPE_MISMATCH;
    DevState* s = state();
    if (!s || !s->init) return VOXCPM_ERR_CUDA_NOT_FOUND;
    if (M == 0 || N == 0) return VOXCPM_SUCCESS;
    cudaStream_t st = s->stream;
    std::unique_lock<std::mutex> lk(g_mu);

    // activation
    const float* d_a = a->data;
    const size_t a_bytes = (size_t)M * K * sizeof(float);
    if (!a->is_cuda) {
        float* da = (float*)slot_get(*s, 0, a_bytes);
        if (!da || !pinned_get(&s->h_in, &s->h_in_bytes, a_bytes)) return VOXCPM_ERR_OOM;
        memcpy(s->h_in, a->data, a_bytes);
        VOXQ_CUDA_TRY(cudaMemcpyAsync(da, s->h_in, a_bytes, cudaMemcpyHostToDevice, st));
        d_a = da;
    }
    // output.  A host `out` of the quantized GEMV (M <= 8) is written by the
    // kernel straight into the mapped pinned staging buffer (its epilogue uses
    // plain stores), which saves the device -> host copy and its API call;
    // every other host output goes through a device slot and one copy.
    const size_t o_bytes = (size_t)M * N * sizeof(float);
    float* d_o = out->data;
    auto qit = b->is_cuda && b->data ? g_qtab.find(b->data) : g_qtab.end();
    const bool direct_out = !out->is_cuda && qit != g_qtab.end() && M <= gemv_rows_max();
    if (direct_out) {
        if (!pinned_get(&s->h_out, &s->h_out_bytes, o_bytes)) return VOXCPM_ERR_OOM;
        d_o = (float*)s->h_out;
    } else if (!out->is_cuda) {
        d_o = (float*)slot_get(*s, 1, o_bytes);
        if (!d_o) return VOXCPM_ERR_OOM;
    }
    // weight
    VoxCPMError e;
    g_mm_calls.fetch_add(1, std::memory_order_relaxed);
    if (qit != g_qtab.end()) {
        const QRec& q = qit->second;
        voxq_qweight w = {q.codes, q.scales, q.N, q.K, q.qtype, 0};
        g_mm_wbytes.fetch_add(voxq_codes_bytes(q.N, q.K, q.qtype) + voxq_scales_bytes(q.N, q.K, q.qtype),
                              std::memory_order_relaxed);
        if (M > gemv_rows_max()) {
            void* ws = slot_get(*s, 3, gemm_workspace_bytes(M, N, K, q.qtype, false));
            if (!ws) return VOXCPM_ERR_OOM;
            lk.unlock();
            e = gemm_launch(d_a, M, K, &w, d_o, N, nullptr, ws, st);
        } else {
            lk.unlock();
            e = voxq_matmul_nt_q(d_a, M, K, &w, d_o, N, nullptr, st);
        }
    } else {
        const void* d_w = b->is_fp16 ? (const void*)b->data_fp16 : (const void*)b->data;
        g_mm_wbytes.fetch_add((uint64_t)N * K * (b->is_fp16 ? 2 : 4), std::memory_order_relaxed);
        if (!b->is_cuda) {
            const size_t wb = (size_t)N * K * (b->is_fp16 ? 2 : 4);
            void* dw = slot_get(*s, 2, wb);
            if (!dw) return VOXCPM_ERR_OOM;
            VOXQ_CUDA_TRY(cudaMemcpyAsync(dw, d_w, wb, cudaMemcpyHostToDevice, st));
            d_w = dw;
        }
        lk.unlock();
        e = dense_launch(d_a, M, K, d_w, b->is_fp16 ? 1 : 0, N, K, d_o, N, st);
    }
    if (e) return e;
    if (direct_out) {
        VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
        memcpy(out->data, s->h_out, o_bytes);
    } else if (!out->is_cuda) {
        lk.lock();
        if (!pinned_get(&s->h_out, &s->h_out_bytes, o_bytes)) return VOXCPM_ERR_OOM;
        VOXQ_CUDA_TRY(cudaMemcpyAsync(s->h_out, d_o, o_bytes, cudaMemcpyDeviceToHost, st));
        VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
        memcpy(out->data, s->h_out, o_bytes);
    } else if (!a->is_cuda) {
        // the staged activation slot may be reused by the next call: order it
        VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
    }
    return VOXCPM_SUCCESS;
}
