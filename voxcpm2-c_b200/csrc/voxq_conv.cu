// voxq_conv.cu -- the AudioVAE's 1-D convolutions on the device.
//
// The reference decodes audio on the host even in its GPU build (src/model.c:
// 554-556 keeps every AudioVAE weight on the CPU); its decoder is a chain of
// weight-normalised 1-D convolutions -- depthwise k = 7, pointwise k = 1, the
// 64 -> 2048 projection and six transposed upsampling convolutions -- computed by
// conv1d_forward and conv1d_transpose_forward (src/nn.c:765-931).  These entry
// points compute the same functions on the device, in fp32 like the reference:
//
//   conv1d:      out[n,o,t] = b[o] + sum_{c in group(o)} sum_k
//                             w[o, c - c0, k] * x[n, c, t*stride + k - pad]
//   transposed:  out[n,o,t] = b[o] + sum_c sum_{k, s: s*stride + k - pad = t}
//                             w[c, o, k] * x[n, c, s]
//
// One thread computes kTPT consecutive time steps of one output channel; a
// warp covers 32 * kTPT consecutive steps of that channel (coalesced loads of x
// and stores of out, one broadcast weight per tap).  Host tensors are staged
// through the library stream; host weights are uploaded once per pointer and
// kept (the AudioVAE's effective weights are fixed for the model's lifetime),
// keyed by pointer, size and a content fingerprint.
#include <algorithm>
#include <mutex>
#include <unordered_map>
#include <utility>

#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

constexpr int kTPT = 4;           // time steps per thread
constexpr int kConvThreads = 256;  // 8 output channels per block

__global__ void __launch_bounds__(kConvThreads) conv1d_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                              const float* __restrict__ b, float* __restrict__ out,
                                                              int Cin, int Tin, int Cout, int Tout, int Kw, int stride,
                                                              int pad, int groups, int splits) {
    // blockIdx.z = n * splits + part: with splits > 1 the CTA sums one slice of
    // its group's input channels and writes a partial ([part][n][o][t], no
    // bias) for split_sum_kernel; with one split it writes out directly
    const int o = blockIdx.y * (kConvThreads / 32) + (threadIdx.x >> 5);
    const int n = blockIdx.z / splits, sp = blockIdx.z % splits;
    const int t0 = (blockIdx.x * 32 + (threadIdx.x & 31)) * kTPT;
    if (o >= Cout || t0 >= Tout) return;
    const int ipg = Cin / groups, opg = Cout / groups;
    const int c0 = (o / opg) * ipg;
    const int per = (ipg + splits - 1) / splits, cb = sp * per, ce = min(ipg, cb + per);
    const float* xn = x + (int64_t)n * Cin * Tin;
    const float* wo = w + (int64_t)o * ipg * Kw;
    float acc[kTPT];
#pragma unroll
    for (int j = 0; j < kTPT; j++) acc[j] = (b && splits == 1) ? b[o] : 0.0f;
    for (int c = cb; c < ce; c++) {
        const float* xc = xn + (int64_t)(c0 + c) * Tin;
        const float* wc = wo + c * Kw;
        for (int k = 0; k < Kw; k++) {
            const float wv = __ldg(wc + k);
#pragma unroll
            for (int j = 0; j < kTPT; j++) {
                const int ti = (t0 + j) * stride + k - pad;
                if (ti >= 0 && ti < Tin) acc[j] = fmaf(wv, __ldg(xc + ti), acc[j]);
            }
        }
    }
    const int B = gridDim.z / splits;
    float* on = out + (((int64_t)sp * B + n) * Cout + o) * Tout;
#pragma unroll
    for (int j = 0; j < kTPT; j++)
        if (t0 + j < Tout) on[t0 + j] = acc[j];
}

__global__ void __launch_bounds__(kConvThreads) convt1d_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ w,
                                                               const float* __restrict__ b, float* __restrict__ out,
                                                               int Cin, int Tin, int Cout, int Tout, int Kw,
                                                               int stride, int pad, int splits) {
    // blockIdx.z = n * splits + part, as in conv1d_kernel
    const int o = blockIdx.y * (kConvThreads / 32) + (threadIdx.x >> 5);
    const int n = blockIdx.z / splits, sp = blockIdx.z % splits;
    const int t0 = (blockIdx.x * 32 + (threadIdx.x & 31)) * kTPT;
    if (o >= Cout || t0 >= Tout) return;
    const int per = (Cin + splits - 1) / splits, cb = sp * per, ce = min(Cin, cb + per);
    const float* xn = x + (int64_t)n * Cin * Tin;
    float acc[kTPT];
#pragma unroll
    for (int j = 0; j < kTPT; j++) acc[j] = 0.0f;
    for (int c = cb; c < ce; c++) {
        const float* xc = xn + (int64_t)c * Tin;
        const float* wc = w + ((int64_t)c * Cout + o) * Kw;
#pragma unroll
        for (int j = 0; j < kTPT; j++) {
            // taps k with (t + pad - k) a non-negative multiple of stride below Tin * stride
            const int tp = t0 + j + pad;
            for (int k = tp % stride; k < Kw && k <= tp; k += stride) {
                const int s = (tp - k) / stride;
                if (s < Tin) acc[j] = fmaf(__ldg(wc + k), __ldg(xc + s), acc[j]);
            }
        }
    }
    const int B = gridDim.z / splits;
    float* on = out + (((int64_t)sp * B + n) * Cout + o) * Tout;
#pragma unroll
    for (int j = 0; j < kTPT; j++)
        if (t0 + j < Tout) on[t0 + j] = acc[j] + ((b && splits == 1) ? b[o] : 0.0f);
}

// out[n][o][t] = (bias[o] + part[0][n][o][t]) + part[1][n][o][t] + ... (fixed order)
__global__ void split_sum_kernel(const float* __restrict__ part, const float* __restrict__ b, float* __restrict__ out,
                                 int Cout, int Tout, int splits, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float r = b ? b[(int)((i / Tout) % Cout)] : 0.0f;
        for (int sp = 0; sp < splits; sp++) r += part[(int64_t)sp * n + i];
        out[i] = r;
    }
}

// h = h + sin(alpha[c] h)^2 / beta over [B][C][T] (snake_forward).
__global__ void snake_kernel(float* __restrict__ h, const float* __restrict__ alpha, int C, int T, float beta,
                             int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)((i / T) % C);
        const float v = h[i];
        const float sn = sinf(alpha[c] * v);
        h[i] = v + (sn * sn) / beta;
    }
}

__global__ void add_kernel(float* __restrict__ h, const float* __restrict__ r, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        h[i] = h[i] + r[i];
}

__global__ void tanh_kernel(float* __restrict__ h, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        h[i] = tanhf(h[i]);
}

// [B][T][D] -> [B][D][T]
__global__ void btd_to_bdt_kernel(const float* __restrict__ x, float* __restrict__ y, int T, int D, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i % T);
        const int64_t r = i / T;
        const int d = (int)(r % D);
        const int64_t b = r / D;
        y[i] = x[(b * T + t) * D + d];
    }
}

static int ew_grid(int64_t n) {
    const int64_t g = (n + 255) / 256;
    return (int)(g < 4096 ? (g > 0 ? g : 1) : 4096);
}

namespace {

struct DevBuf {
    float* p;
    size_t n;
    uint64_t fp;  // fingerprint of the host contents uploaded
};

// FNV-1a over the size and 64 evenly spaced values (first and last included):
// a host buffer freed and reallocated at the same address with other contents
// is uploaded again.  Constant cost per call; a weight changed in place at
// unsampled positions is not detected (voxq_conv_cache_clear drops the cache).
uint64_t fingerprint(const float* h, size_t n) {
    uint64_t f = 0xcbf29ce484222325ull ^ n;
    const size_t samples = n < 64 ? n : 64;
    for (size_t i = 0; i < samples; i++) {
        const size_t j = samples > 1 ? i * (n - 1) / (samples - 1) : 0;
        uint32_t bits;
        memcpy(&bits, h + j, 4);
        f = (f ^ bits) * 0x100000001b3ull;
    }
    return f;
}
std::mutex g_conv_mu;
std::unordered_map<const void*, DevBuf> g_conv_w;  // host weight / bias pointer -> device copy
float* g_conv_io[2] = {nullptr, nullptr};          // device staging of x and out
size_t g_conv_io_n[2] = {0, 0};

// Device pointer of a Tensor's fp32 payload: its own for device tensors, a
// cached upload for host tensors (weights and biases).
VoxCPMError weight_ptr(const Tensor* t, cudaStream_t st, const float** out) {
    *out = nullptr;
    if (!t) return VOXCPM_SUCCESS;
    if (t->is_fp16 || !t->data) return VOXCPM_ERR_UNSUPPORTED;
    if (t->is_cuda) {
        *out = t->data;
        return VOXCPM_SUCCESS;
    }
    std::lock_guard<std::mutex> lk(g_conv_mu);
    const uint64_t fp = fingerprint(t->data, t->size);
    auto it = g_conv_w.find(t->data);
    if (it != g_conv_w.end() && it->second.n == t->size && it->second.fp == fp) {
        *out = it->second.p;
        return VOXCPM_SUCCESS;
    }
    float* d = nullptr;
    VOXQ_CUDA_TRY(cudaMalloc(&d, t->size * sizeof(float)));
    VOXQ_CUDA_TRY(cudaMemcpyAsync(d, t->data, t->size * sizeof(float), cudaMemcpyHostToDevice, st));
    VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
    if (it != g_conv_w.end()) cudaFree(it->second.p);
    g_conv_w[t->data] = DevBuf{d, t->size, fp};
    *out = d;
    return VOXCPM_SUCCESS;
}

// Input-channel splits for a convolution whose outputs alone give too few
// warps to keep the SMs' memory pipes busy (the decoder's first blocks: 1024
// output channels x 32 steps, each warp walking 2048 channels): enough splits
// for ~64 warps per SM, each split at least 16 channels, partials within 64 MB.
float* g_conv_part = nullptr;
size_t g_conv_part_n = 0;

int conv_splits(int B, int Cout, int Tout, int chans) {
    const int64_t warps = (int64_t)B * Cout * ((Tout + 32 * kTPT - 1) / (32 * kTPT));
    const int64_t target = (int64_t)device_sm_count() * 64;
    int64_t sp = (target + warps - 1) / warps;
    sp = std::min<int64_t>(sp, std::max(1, chans / 16));
    sp = std::min<int64_t>(sp, 64);
    while (sp > 1 && sp * B * Cout * Tout > ((int64_t)16 << 20)) sp--;
    return (int)std::max<int64_t>(sp, 1);
}

// The partials buffer (held under g_conv_mu); grows, draining the stream first.
float* part_buf(size_t n, cudaStream_t st) {
    if (g_conv_part_n >= n) return g_conv_part;
    cudaStreamSynchronize(st);
    if (g_conv_part) cudaFree(g_conv_part);
    g_conv_part = nullptr;
    g_conv_part_n = 0;
    if (cudaMalloc(&g_conv_part, n * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    g_conv_part_n = n;
    return g_conv_part;
}

float* io_buf(int k, size_t n) {
    if (g_conv_io_n[k] >= n) return g_conv_io[k];
    size_t want = 1 << 18;
    while (want < n) want <<= 1;
    float* p = nullptr;
    if (cudaMalloc(&p, want * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (g_conv_io[k]) {
        cudaDeviceSynchronize();  // the old buffer may still be read by queued work
        cudaFree(g_conv_io[k]);
    }
    g_conv_io[k] = p;
    g_conv_io_n[k] = want;
    return p;
}

// Runs one convolution with host or device x / out (x [B, Cin, Tin], out
// [B, Cout, Tout] fp32, contiguous).
template <typename Launch>
VoxCPMError run_conv(const Tensor* x, Tensor* out, cudaStream_t st, Launch launch) {
    const float* d_x = x->data;
    float* d_o = out->data;
    std::unique_lock<std::mutex> lk(g_conv_mu);
    if (!x->is_cuda) {
        float* b = io_buf(0, x->size);
        if (!b) return VOXCPM_ERR_OOM;
        VOXQ_CUDA_TRY(cudaMemcpyAsync(b, x->data, x->size * sizeof(float), cudaMemcpyHostToDevice, st));
        d_x = b;
    }
    if (!out->is_cuda) {
        d_o = io_buf(1, out->size);
        if (!d_o) return VOXCPM_ERR_OOM;
    }
    if (!launch(d_x, d_o)) return VOXCPM_ERR_OOM;
    VOXQ_CUDA_TRY(cudaGetLastError());
    if (!out->is_cuda) {
        VOXQ_CUDA_TRY(cudaMemcpyAsync(out->data, d_o, out->size * sizeof(float), cudaMemcpyDeviceToHost, st));
    }
    // host outputs are valid on return; staged inputs are free for the next call
    if (!out->is_cuda || !x->is_cuda) VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
    return VOXCPM_SUCCESS;
}

// The decoder's resident activations: current, next, and a residual
// sub-block's saved input (each as large as the largest activation).
float* g_vae_buf[3] = {nullptr, nullptr, nullptr};
size_t g_vae_n = 0;

}  // namespace

void conv_cache_clear() {
    std::lock_guard<std::mutex> lk(g_conv_mu);
    for (int k = 0; k < 3; k++) {
        if (g_vae_buf[k]) cudaFree(g_vae_buf[k]);
        g_vae_buf[k] = nullptr;
    }
    g_vae_n = 0;
    if (g_conv_part) cudaFree(g_conv_part);
    g_conv_part = nullptr;
    g_conv_part_n = 0;
    for (auto& kv : g_conv_w) cudaFree(kv.second.p);
    g_conv_w.clear();
    for (int k = 0; k < 2; k++) {
        if (g_conv_io[k]) cudaFree(g_conv_io[k]);
        g_conv_io[k] = nullptr;
        g_conv_io_n[k] = 0;
    }
}

}  // namespace voxq

using namespace voxq;

extern "C" void voxq_conv_cache_clear(void) { conv_cache_clear(); }

extern "C" VoxCPMError voxq_conv1d_forward(const voxq_conv1d_desc* conv, const Tensor* x, Tensor* out) {
    if (!conv || !x || !out || !conv->weight) return VOXCPM_ERR_INTERNAL;
    cudaStream_t st = (cudaStream_t)library_stream();
    if (!st) return VOXCPM_ERR_CUDA_NOT_FOUND;
    if (x->ndim != 3 || out->ndim != 3 || x->is_fp16 || out->is_fp16) return VOXCPM_ERR_SHAPE_MISMATCH;
    const int B = x->shape[0], Cin = x->shape[1], Tin = x->shape[2];
    const int Cout = conv->out_channels, Kw = conv->kernel_size, stride = conv->stride, pad = conv->padding;
    const int groups = conv->groups > 0 ? conv->groups : 1;
    if (Cin != conv->in_channels || Cin % groups || Cout % groups || stride < 1 || Kw < 1)
        return VOXCPM_ERR_SHAPE_MISMATCH;
    const int Tout = (Tin + 2 * pad - Kw) / stride + 1;
    if (Tout <= 0 || out->shape[0] != B || out->shape[1] != Cout || out->shape[2] != Tout)
        return VOXCPM_ERR_SHAPE_MISMATCH;
    if (conv->weight->size != (size_t)Cout * (Cin / groups) * Kw || (conv->bias && conv->bias->size < (size_t)Cout))
        return VOXCPM_ERR_SHAPE_MISMATCH;
    const float *d_w = nullptr, *d_b = nullptr;
    VoxCPMError e = weight_ptr(conv->weight, st, &d_w);
    if (!e) e = weight_ptr(conv->bias, st, &d_b);
    if (e) return e;
    const int splits = conv_splits(B, Cout, Tout, Cin / groups);
    return run_conv(x, out, st, [&](const float* d_x, float* d_o) -> bool {
        const size_t n = (size_t)B * Cout * Tout;
        float* part = splits > 1 ? part_buf((size_t)splits * n, st) : nullptr;
        if (splits > 1 && !part) return false;
        const dim3 grid((unsigned)((Tout + 32 * kTPT - 1) / (32 * kTPT)),
                        (unsigned)((Cout + kConvThreads / 32 - 1) / (kConvThreads / 32)), (unsigned)(B * splits));
        conv1d_kernel<<<grid, kConvThreads, 0, st>>>(d_x, d_w, d_b, splits > 1 ? part : d_o, Cin, Tin, Cout, Tout, Kw,
                                                      stride, pad, groups, splits);
        if (splits > 1) split_sum_kernel<<<ew_grid((int64_t)n), 256, 0, st>>>(part, d_b, d_o, Cout, Tout, splits, (int64_t)n);
        return true;
    });
}

extern "C" VoxCPMError voxq_conv1d_transpose_forward(const voxq_conv1d_transpose_desc* conv, const Tensor* x,
                                                     Tensor* out) {
    if (!conv || !x || !out || !conv->weight) return VOXCPM_ERR_INTERNAL;
    cudaStream_t st = (cudaStream_t)library_stream();
    if (!st) return VOXCPM_ERR_CUDA_NOT_FOUND;
    if (x->ndim != 3 || out->ndim != 3 || x->is_fp16 || out->is_fp16) return VOXCPM_ERR_SHAPE_MISMATCH;
    const int B = x->shape[0], Cin = x->shape[1], Tin = x->shape[2];
    const int Cout = conv->out_channels, Kw = conv->kernel_size, stride = conv->stride, pad = conv->padding;
    if (Cin != conv->in_channels || stride < 1 || Kw < 1 || pad < 0) return VOXCPM_ERR_SHAPE_MISMATCH;
    const int Tout = (Tin - 1) * stride - 2 * pad + Kw;
    if (Tout <= 0 || out->shape[0] != B || out->shape[1] != Cout || out->shape[2] != Tout)
        return VOXCPM_ERR_SHAPE_MISMATCH;
    if (conv->weight->size != (size_t)Cin * Cout * Kw || (conv->bias && conv->bias->size < (size_t)Cout))
        return VOXCPM_ERR_SHAPE_MISMATCH;
    const float *d_w = nullptr, *d_b = nullptr;
    VoxCPMError e = weight_ptr(conv->weight, st, &d_w);
    if (!e) e = weight_ptr(conv->bias, st, &d_b);
    if (e) return e;
    const int splits = conv_splits(B, Cout, Tout, Cin);
    return run_conv(x, out, st, [&](const float* d_x, float* d_o) -> bool {
        const size_t n = (size_t)B * Cout * Tout;
        float* part = splits > 1 ? part_buf((size_t)splits * n, st) : nullptr;
        if (splits > 1 && !part) return false;
        const dim3 grid((unsigned)((Tout + 32 * kTPT - 1) / (32 * kTPT)),
                        (unsigned)((Cout + kConvThreads / 32 - 1) / (kConvThreads / 32)), (unsigned)(B * splits));
        convt1d_kernel<<<grid, kConvThreads, 0, st>>>(d_x, d_w, d_b, splits > 1 ? part : d_o, Cin, Tin, Cout, Tout, Kw,
                                                       stride, pad, splits);
        if (splits > 1) split_sum_kernel<<<ew_grid((int64_t)n), 256, 0, st>>>(part, d_b, d_o, Cout, Tout, splits, (int64_t)n);
        return true;
    });
}

extern "C" VoxCPMError voxq_vae_decode(const voxq_vae_op* ops, int n_ops, float snake_beta, const Tensor* latent,
                                       Tensor* waveform) {
    if (!ops || n_ops < 0 || !latent || !waveform) return VOXCPM_ERR_INTERNAL;
    cudaStream_t st = (cudaStream_t)library_stream();
    if (!st) return VOXCPM_ERR_CUDA_NOT_FOUND;
    if (latent->ndim != 3 || latent->is_cuda || latent->is_fp16 || !latent->data) return VOXCPM_ERR_SHAPE_MISMATCH;
    if (waveform->is_cuda || waveform->is_fp16 || !waveform->data) return VOXCPM_ERR_SHAPE_MISMATCH;
    const int B = latent->shape[0], T0 = latent->shape[1], D0 = latent->shape[2];
    // shapes of every step first (the checks of conv1d_forward / conv1d_transpose_forward / snake_forward)
    int C = D0, T = T0;
    size_t most = (size_t)B * C * T;
    for (int i = 0; i < n_ops; i++) {
        const voxq_vae_op& op = ops[i];
        if (op.kind == VOXQ_VAE_CONV) {
            const voxq_conv1d_desc* c = op.conv;
            if (!c || !c->weight || c->in_channels != C || c->stride < 1 || c->kernel_size < 1)
                return VOXCPM_ERR_SHAPE_MISMATCH;
            T = (T + 2 * c->padding - c->kernel_size) / c->stride + 1;
            C = c->out_channels;
        } else if (op.kind == VOXQ_VAE_CONVT) {
            const voxq_conv1d_transpose_desc* c = op.convt;
            if (!c || !c->weight || c->in_channels != C || c->stride < 1 || c->kernel_size < 1)
                return VOXCPM_ERR_SHAPE_MISMATCH;
            T = (T - 1) * c->stride - 2 * c->padding + c->kernel_size;
            C = c->out_channels;
        } else if (op.kind == VOXQ_VAE_SNAKE) {
            if (!op.alpha || op.alpha->is_fp16 || op.alpha->size < (size_t)C) return VOXCPM_ERR_SHAPE_MISMATCH;
        } else if (op.kind < VOXQ_VAE_SAVE || op.kind > VOXQ_VAE_TANH) {
            return VOXCPM_ERR_INTERNAL;
        }
        if (T <= 0 || C <= 0) return VOXCPM_ERR_SHAPE_MISMATCH;
        const size_t n = (size_t)B * C * T;
        if (n > most) most = n;
    }
    if (C != 1) return VOXCPM_ERR_SHAPE_MISMATCH;
    const int samples = T;
    if (waveform->ndim == 2) {
        if (waveform->shape[0] != B || waveform->shape[1] != samples) return VOXCPM_ERR_SHAPE_MISMATCH;
    } else if (waveform->ndim == 1) {
        if (B != 1 || waveform->size < (size_t)samples) return VOXCPM_ERR_SHAPE_MISMATCH;
    } else {
        return VOXCPM_ERR_SHAPE_MISMATCH;
    }
    {
        std::lock_guard<std::mutex> lk(g_conv_mu);
        if (g_vae_n < most) {
            cudaStreamSynchronize(st);
            for (int k = 0; k < 3; k++) {
                if (g_vae_buf[k]) cudaFree(g_vae_buf[k]);
                g_vae_buf[k] = nullptr;
            }
            g_vae_n = 0;
            for (int k = 0; k < 3; k++) VOXQ_CUDA_TRY(cudaMalloc(&g_vae_buf[k], most * sizeof(float)));
            g_vae_n = most;
        }
    }
    float *cur = g_vae_buf[0], *nxt = g_vae_buf[1], *saved = g_vae_buf[2];
    // latent [B][T][D] -> h [B][D][T] (staged through `nxt`)
    const int64_t n0 = (int64_t)B * T0 * D0;
    VOXQ_CUDA_TRY(cudaMemcpyAsync(nxt, latent->data, (size_t)n0 * sizeof(float), cudaMemcpyHostToDevice, st));
    btd_to_bdt_kernel<<<ew_grid(n0), 256, 0, st>>>(nxt, cur, T0, D0, n0);
    VOXQ_CUDA_TRY(cudaGetLastError());
    C = D0;
    T = T0;
    int saved_c = -1, saved_t = -1;
    for (int i = 0; i < n_ops; i++) {
        const voxq_vae_op& op = ops[i];
        const int64_t n = (int64_t)B * C * T;
        if (op.kind == VOXQ_VAE_CONV || op.kind == VOXQ_VAE_CONVT) {
            const int Cout = op.kind == VOXQ_VAE_CONV ? op.conv->out_channels : op.convt->out_channels;
            const int Tout = op.kind == VOXQ_VAE_CONV
                                 ? (T + 2 * op.conv->padding - op.conv->kernel_size) / op.conv->stride + 1
                                 : (T - 1) * op.convt->stride - 2 * op.convt->padding + op.convt->kernel_size;
            int sx[3] = {B, C, T}, so[3] = {B, Cout, Tout};
            Tensor tx = {}, to = {};
            tx.data = cur;
            tx.shape = sx;
            tx.ndim = 3;
            tx.size = (size_t)n;
            tx.is_cuda = true;
            to.data = nxt;
            to.shape = so;
            to.ndim = 3;
            to.size = (size_t)B * Cout * Tout;
            to.is_cuda = true;
            const VoxCPMError e = op.kind == VOXQ_VAE_CONV ? voxq_conv1d_forward(op.conv, &tx, &to)
                                                           : voxq_conv1d_transpose_forward(op.convt, &tx, &to);
            if (e) return e;
            std::swap(cur, nxt);  // the saved input is a third buffer, never written here
            C = Cout;
            T = Tout;
        } else if (op.kind == VOXQ_VAE_SNAKE) {
            const float* a = nullptr;
            const VoxCPMError e = weight_ptr(op.alpha, st, &a);  // host alpha, uploaded once
            if (e) return e;
            snake_kernel<<<ew_grid(n), 256, 0, st>>>(cur, a, C, T, snake_beta, n);
        } else if (op.kind == VOXQ_VAE_SAVE) {
            VOXQ_CUDA_TRY(cudaMemcpyAsync(saved, cur, (size_t)n * sizeof(float), cudaMemcpyDeviceToDevice, st));
            saved_c = C;
            saved_t = T;
        } else if (op.kind == VOXQ_VAE_ADD_SAVED) {
            if (saved_c != C || saved_t != T) return VOXCPM_ERR_SHAPE_MISMATCH;
            add_kernel<<<ew_grid(n), 256, 0, st>>>(cur, saved, n);
        } else if (op.kind == VOXQ_VAE_TANH) {
            tanh_kernel<<<ew_grid(n), 256, 0, st>>>(cur, n);
        }
        VOXQ_CUDA_TRY(cudaGetLastError());
    }
    VOXQ_CUDA_TRY(cudaMemcpyAsync(waveform->data, cur, (size_t)B * samples * sizeof(float), cudaMemcpyDeviceToHost,
                                  st));
    VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
    return VOXCPM_SUCCESS;
}
