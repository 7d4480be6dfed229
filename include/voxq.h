/*
 * voxq.h -- C ABI of libvoxq, the sm_100a (B200) quantized-matmul library that
 * replaces the voxcpm2-c reference's GPU offload (src/tensor_cuda.cu).
 *
 * Two groups of entry points:
 *
 *  1. The reference's CUDA block of include/tensor.h (tensor.h:316-342), same
 *     names, arguments, ownership rules and error codes, so the reference
 *     engine (src/model.c, src/nn.c, ...) links against libvoxq unchanged.
 *
 *  2. Additive voxq_* entry points on plain device pointers: the block
 *     quantizer of scripts/quantize.py (bit-exact), dequantizers, the packed
 *     device weight layout, the fused matmul with epilogues, and a grouped
 *     launch for many independent GEMVs.  The reference has no quantized GPU
 *     path at all; these are the calls its engine would make for one.
 *
 * All sizes are element counts unless named *_bytes.  Functions return
 * VOXCPM_SUCCESS (0) or a negative VoxCPMError.  `stream` is a cudaStream_t
 * passed as void* (NULL = the legacy default stream).
 */
#ifndef VOXQ_H
#define VOXQ_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Exported from libvoxq.so (the library builds with hidden visibility). */
#if defined(__GNUC__)
#define VOXQ_API __attribute__((visibility("default")))
#else
#define VOXQ_API
#endif

/* ------------------------------------------------------------------------ */
/* Reference ABI types.  Layout- and value-compatible with the reference's   */
/* include/voxcpm.h:45-58 (VoxCPMError) and include/tensor.h:45-56 (Tensor). */
/* When the reference headers are already included they are used instead.   */
/* ------------------------------------------------------------------------ */
#ifndef TENSOR_H
#ifndef VOXCPM_H
typedef enum {
    VOXCPM_SUCCESS = 0,
    VOXCPM_ERR_FILE_NOT_FOUND = -1,
    VOXCPM_ERR_INVALID_MODEL = -2,
    VOXCPM_ERR_INVALID_TEXT = -3,
    VOXCPM_ERR_INVALID_AUDIO = -4,
    VOXCPM_ERR_SHAPE_MISMATCH = -5,
    VOXCPM_ERR_OOM = -6,
    VOXCPM_ERR_GPU = -7,
    VOXCPM_ERR_INTERNAL = -8,
    VOXCPM_ERR_UNSUPPORTED = -9,
    VOXCPM_ERR_TIMEOUT = -10,
    VOXCPM_ERR_CUDA_NOT_FOUND = -11,
} VoxCPMError;
#endif

typedef struct {
    float* data;          /* fp32 data (host or device) */
    int* shape;           /* [ndim], heap-owned */
    int ndim;
    int64_t strides[5];   /* in elements */
    size_t size;          /* element count */
    bool is_cuda;
    bool is_owned;
    uint16_t* data_fp16;  /* fp16 payload when is_fp16 */
    bool is_fp16;
    char name[64];
} Tensor;
#endif

/* ======================================================================== */
/* 1. Drop-in replacements for the reference's tensor.h CUDA block           */
/* ======================================================================== */

/* src/tensor_cuda.cu:47-82.  Selects the device (voxq_set_device, default 0),
 * creates the library stream and reads VOXCPM_QUANT (f32 | q8 | q4; default
 * f32), the format that tensor_to_cuda gives 2-D weights.  Returns
 * VOXCPM_ERR_CUDA_NOT_FOUND when no device is usable. */
VOXQ_API VoxCPMError tensor_cuda_init(void);

/* src/tensor_cuda.cu:84-90. */
VOXQ_API void tensor_cuda_shutdown(void);

/* src/tensor_cuda.cu:96-126.  Moves t to the device and frees the host buffer
 * (also for non-owned tensors, as the reference does).  Under VOXCPM_QUANT=q8
 * or q4 a 2-D tensor with shape[1] % 32 == 0 is quantized on the device,
 * bit-exactly as scripts/quantize.py:42-75 would, and kept only in the packed
 * device layout; t->data then points at that opaque buffer. */
VOXQ_API VoxCPMError tensor_to_cuda(Tensor* t);

/* src/tensor_cuda.cu:128-159.  A quantized tensor comes back dequantized. */
VOXQ_API VoxCPMError tensor_to_cpu(Tensor* t);

/* src/tensor_cuda.cu:161-174. */
VOXQ_API VoxCPMError tensor_cuda_free(Tensor* t);

/* src/tensor_cuda.cu:192-333: out[M,N] = a[M,K] . b[N,K]^T, fp32 rows.
 * a and out may live on the host or the device; b is a device weight (fp32,
 * fp16 or quantized) or a host fp32/fp16 tensor (uploaded for this call).
 * A host `out` is valid on return; a device `out` is complete in the order of
 * the library stream (every later voxq call and tensor_to_cpu sees it).
 * Shape errors -> VOXCPM_ERR_SHAPE_MISMATCH; not initialised ->
 * VOXCPM_ERR_CUDA_NOT_FOUND (the caller then uses its CPU path). */
VOXQ_API VoxCPMError tensor_matmul_nt_cuda(const Tensor* a, const Tensor* b, Tensor* out);

/* src/tensor_cuda.cu:352-355 (defined there, not declared in tensor.h). */
VOXQ_API VoxCPMError tensor_cuda_upload_weight(Tensor** t_ptr);

/* ======================================================================== */
/* 2. Additive voxq_* entry points                                          */
/* ======================================================================== */

/* Block formats: the codes of scripts/quantize.py:28 (QUANT_TYPES). */
enum { VOXQ_F32 = 0, VOXQ_F16 = 1, VOXQ_Q4 = 2, VOXQ_Q8 = 3 };
#define VOXQ_BLOCK 32

/* Library version string. */
VOXQ_API const char* voxq_version(void);

/* Selects the CUDA device for the calling thread's later calls (multi-GPU
 * runners use one host thread or process per GPU).  No counterpart in the
 * reference, which hard-codes device 0 (src/tensor_cuda.cu:50).  Limitation:
 * the kernels that need more than 48 KB of shared memory get their opt-in on
 * the first device that launches them in a process, so one process drives one
 * GPU (a launch on a second device returns VOXCPM_ERR_INTERNAL); run one
 * process per GPU, as bench.py and the serving workers do. */
VOXQ_API VoxCPMError voxq_set_device(int device);

/* Device-side status of the current device's kernels: 0, or the code of the
 * first bounded wait that gave up (1 full-stage, 2 empty-stage, 3 MMA
 * completion, 4 tensor-memory allocation).  A kernel that gives up returns
 * early instead of hanging; its outputs are then undefined.  Covers the
 * library's kernels and those of voxq_matmul_nt_q_noalloc (the library's
 * word is reported first).  clear != 0 resets both words.  Returns -1 if a
 * word cannot be read. */
VOXQ_API int voxq_device_error(int clear);

/* Projections run in this process, all devices -- tensor_matmul_nt_cuda
 * calls and the seven of every voxq_transformer_block_forward call -- and the
 * weight bytes they streamed (packed codes + scales of a quantized weight, 4
 * or 2 bytes per element of a dense one).  reset != 0 zeroes both counters
 * after reading them.  Either pointer may be NULL. */
VOXQ_API void voxq_matmul_traffic(uint64_t* calls, uint64_t* weight_bytes, int reset);

/* Failure-detection self-test (no counterpart in the reference): launches one
 * kernel that waits, through the same bounded wait the GEMV/GEMM kernels use,
 * on a barrier that nothing ever completes, giving up after `polls` suspended
 * polls of at most 1 ms.  Returns the device error code the kernel recorded
 * (expected: 1, full-stage wait) and clears it, or a negative VoxCPMError if
 * the launch failed.  The context stays usable; no fault is raised. */
VOXQ_API int voxq_selftest_wait_timeout(int polls);

/* Bytes of the quantize.py block stream for n elements: ceil(n/32) blocks of
 * 20 (Q4) or 40 (Q8) bytes (scripts/quantize.py:88-104 without its 20-byte
 * tensor header). */
VOXQ_API size_t voxq_quant_bytes(size_t n, int qtype);

/* Quantizes n fp32 values (flattened, last block zero-padded,
 * scripts/quantize.py:239-260) into the quantize.py block stream, bit-exact
 * with quantize_q4_block / quantize_q8_block (scripts/quantize.py:42-75).
 * voxq_quantize runs on the device (d_src, d_dst device pointers). */
VOXQ_API VoxCPMError voxq_quantize(const float* d_src, size_t n, int qtype, uint8_t* d_dst, void* stream);

/* Inverse of the above, bit-exact with dequantize_q4_block /
 * dequantize_q8_block (scripts/quantize.py:56-82).  q8_signed = 1 reads Q8
 * codes as int8 like scripts/quantize.py:79; q8_signed = 0 reads them as the
 * unsigned codes the quantizer wrote (the default everywhere else). */
VOXQ_API VoxCPMError voxq_dequantize(const uint8_t* d_src, size_t n, int qtype, int q8_signed, float* d_dst,
                            void* stream);

/* ---- Packed device weight layout ----------------------------------------
 * A weight W[N,K] with K % 32 == 0 is stored as two arrays:
 *   codes   Q8: uint8 [N][K]     (code of W[n][k] at n*K + k)
 *           Q4: uint8 [N][K/2]   (byte i of a row = code[2i] << 4 | code[2i+1])
 *   scales  Q8: float2 [N][K/32] (scale, min)   Q4: half2 [N][K/32] (scale, min)
 *           then, at the next 16-byte boundary, float rowmul[N] = 2^e with
 *           max_k |W[n][k]| * 2^e in [2^13, 2^14) (exact row scaling for the
 *           fp16 tensor-core path; written by voxq_quantize_weight and
 *           voxq_pack_blocks), then 16 bytes of padding
 * i.e. each quantize.py block split into its code bytes and its trailer.
 * Same bytes per weight as the block stream (1.25 / 0.625).  Both arrays must
 * be 16-byte aligned; allocate them with voxq_codes_bytes / voxq_scales_bytes. */
typedef struct {
    const uint8_t* codes;  /* device */
    const void* scales;    /* device */
    int32_t N, K;
    int32_t qtype;         /* VOXQ_Q4 or VOXQ_Q8 */
    int32_t q8_signed;     /* Q8 codes read as int8 (scripts/quantize.py:79) */
} voxq_qweight;

VOXQ_API size_t voxq_codes_bytes(int N, int K, int qtype);
VOXQ_API size_t voxq_scales_bytes(int N, int K, int qtype);

/* Quantizes a device fp32 weight W[N,K] straight into the packed layout and,
 * when d_blocks is non-NULL, also into the quantize.py block stream. */
VOXQ_API VoxCPMError voxq_quantize_weight(const float* d_w, int N, int K, int qtype, uint8_t* d_codes,
                                 void* d_scales, uint8_t* d_blocks, void* stream);

/* Block stream (e.g. read from a quantize.py file) -> packed layout, and back. */
VOXQ_API VoxCPMError voxq_pack_blocks(const uint8_t* d_blocks, int N, int K, int qtype, uint8_t* d_codes,
                             void* d_scales, void* stream);
VOXQ_API VoxCPMError voxq_unpack_blocks(const uint8_t* d_codes, const void* d_scales, int N, int K, int qtype,
                               uint8_t* d_blocks, void* stream);

/* ---- Matmul -------------------------------------------------------------
 * out[M,N] = epilogue(A[M,K] . W[N,K]^T), A and out fp32 row-major on the
 * device (row strides lda / ldo in elements).  Epilogue, applied in order:
 *   up != NULL  : out = silu(A.W^T) * (A.Up^T)     (src/nn.c:148-169)
 *   bias != NULL: out += bias[n]                   (src/loc_dit.c:52-66)
 *   residual    : out += residual[m*ldr + n]       (src/nn.c:655, 685)
 * residual may alias out.  M <= 8 runs the HBM-streaming GEMV kernel; larger
 * M runs the tcgen05 tensor-core GEMM (fp16 operands, fp32 accumulation in
 * tensor memory), which needs a workspace from the library's device arena. */
typedef struct {
    const float* bias;         /* [N] or NULL */
    const float* residual;     /* [M][ldr] or NULL */
    int64_t ldr;
    const voxq_qweight* up;    /* SwiGLU up-projection, or NULL */
} voxq_epilogue;

VOXQ_API VoxCPMError voxq_matmul_nt_q(const float* d_a, int M, int64_t lda, const voxq_qweight* w, float* d_out,
                             int64_t ldo, const voxq_epilogue* epi, void* stream);

/* voxq_matmul_nt_q for M <= 8 activation rows that allocates no device memory.
 * No counterpart in the reference.  For callers that cannot let the library
 * allocate: engines that reserve their whole device-memory budget up front, or
 * hosts that forbid device allocation after set-up because cudaMalloc /
 * cudaFree can synchronise the device and stall a real-time audio stream.
 * Its scratch is a fixed array of VOXQ_NOALLOC_SCRATCH_BYTES (896 KiB) inside
 * the library's own device image (every GPU that loads the library holds it
 * until exit).  The activation limbs it holds take M * 3.5 * K bytes for Q4 and
 * M * 4 * K bytes for Q8, so it covers every shape the GEMV accepts: M <= 8,
 * K <= 32768 for Q4 and K <= 16384 for Q8 (half those K with the SwiGLU `up`
 * weight).  Larger K -> VOXCPM_ERR_UNSUPPORTED (the GEMV's own limit); a
 * scratch need above the array -> VOXCPM_ERR_OOM; M > 8 ->
 * VOXCPM_ERR_UNSUPPORTED.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) and clears its error word on `stream`,
 * waiting for that stream, so make that first call before any stream capture.
 * All calls share the one array and keep no state in it between calls: calls
 * that overlap on the GPU (other streams, other host threads) race. */
#define VOXQ_NOALLOC_SCRATCH_BYTES (896 * 1024)
VOXQ_API VoxCPMError voxq_matmul_nt_q_noalloc(const float* d_a, int M, int64_t lda, const voxq_qweight* w,
                                              float* d_out, int64_t ldo, const voxq_epilogue* epi, void* stream);

/* Device-side status of voxq_matmul_nt_q_noalloc's kernels on the current
 * device, read without allocating: 0, or the code of the first bounded wait
 * that gave up (same codes as voxq_device_error, which reports this word too).
 * clear != 0 resets it.  Returns -1 if the word cannot be read.  No
 * counterpart in the reference. */
VOXQ_API int voxq_noalloc_device_error(int clear);

/* Dense fp32 / fp16 weights (the reference's unquantized path,
 * src/tensor_cuda.cu:192-333), full fp32 arithmetic. */
VOXQ_API VoxCPMError voxq_matmul_nt_dense(const float* d_a, int M, int64_t lda, const void* d_w, int w_is_fp16,
                                 int N, int K, float* d_out, int64_t ldo, void* stream);

/* ---- Grouped GEMV ------------------------------------------------------
 * Runs `count` independent quantized GEMVs (M <= 8 each) in ONE launch that
 * streams all their weights back to back: the QKV or gate/up group of a
 * decoder layer, or a whole stack of layers whose inputs are ready.  Each
 * item is an independent voxq_matmul_nt_q call.  count <= VOXQ_MAX_BATCH. */
#define VOXQ_MAX_BATCH 192
typedef struct {
    voxq_qweight w;
    const float* a;            /* [M][lda] */
    float* out;                /* [M][ldo] */
    const float* bias;         /* or NULL */
    const float* residual;     /* or NULL */
    const uint8_t* up_codes;   /* SwiGLU up weight (same N, K, qtype), or NULL */
    const void* up_scales;
    int32_t M;
    int32_t lda, ldo, ldr;
} voxq_gemv_item;

VOXQ_API VoxCPMError voxq_gemv_batch(const voxq_gemv_item* items, int count, void* stream);

/* ---- AudioVAE convolutions ---------------------------------------------
 * The reference decodes audio on the host even in its GPU build: every
 * AudioVAE weight stays on the CPU (src/model.c:554-556) and the decoder's
 * 1-D convolutions run in src/nn.c:765-931.  These compute the same two
 * functions on the device, in fp32, with the engine's own descriptors (the
 * layouts of Conv1D and Conv1DTranspose, include/nn.h:198-229), so an engine
 * can route conv1d_forward / conv1d_transpose_forward here:
 *   conv1d:     out[n,o,t] = b[o] + sum over c in o's group, k of
 *               w[o][c - group start][k] * x[n][c][t*stride + k - padding]
 *   transposed: out[n,o,t] = b[o] + sum over c, k, s with s*stride + k - padding = t
 *               of w[c][o][k] * x[n][c][s]
 * x [batch, in_channels, time] and out [batch, out_channels, out_time] are
 * fp32, host or device (a host out is valid on return).  A host weight or
 * bias is uploaded on its first use and kept, keyed by its pointer, size and a
 * fingerprint of 64 sampled values (so a buffer freed and reallocated at the
 * same address is uploaded again), until voxq_conv_cache_clear or
 * tensor_cuda_shutdown; a cached host weight must not be changed in place
 * (the AudioVAE's effective weights never are).  Same shape checks and error
 * codes as nn.c; not initialised -> VOXCPM_ERR_CUDA_NOT_FOUND (the caller then
 * uses its CPU loop). */
typedef struct {
    Tensor* weight;  /* [out_channels, in_channels / groups, kernel_size] */
    Tensor* bias;    /* [out_channels] or NULL */
    int in_channels, out_channels, kernel_size, stride, padding, groups;
} voxq_conv1d_desc;
typedef struct {
    Tensor* weight;  /* [in_channels, out_channels, kernel_size] */
    Tensor* bias;    /* [out_channels] or NULL */
    int in_channels, out_channels, kernel_size, stride, padding;
} voxq_conv1d_transpose_desc;

/* src/nn.c:765-834 (conv1d_forward). */
VOXQ_API VoxCPMError voxq_conv1d_forward(const voxq_conv1d_desc* conv, const Tensor* x, Tensor* out);
/* src/nn.c:864-931 (conv1d_transpose_forward). */
VOXQ_API VoxCPMError voxq_conv1d_transpose_forward(const voxq_conv1d_transpose_desc* conv, const Tensor* x,
                                                   Tensor* out);
/* Drops the convolutions' cached device copies of host weights (no
 * counterpart in the reference). */
VOXQ_API void voxq_conv_cache_clear(void);

/* The AudioVAE decoder (audio_vae_decode, src/audio_vae.c:941-1116) as a
 * list of steps run on the device with the activation resident: the latent
 * [batch, time, latent_dim] (host) is permuted to [batch, latent_dim, time]
 * and uploaded once, each step transforms the current activation h, and the
 * final h [batch, 1, samples] is copied to waveform ([batch, samples], or
 * [samples] for batch 1) with audio_vae_decode's shape rules.  Steps:
 *   VOXQ_VAE_CONV / VOXQ_VAE_CONVT  h = conv(h) (conv1d_forward /
 *                                   conv1d_transpose_forward, as above)
 *   VOXQ_VAE_SNAKE      h = h + sin(alpha[c] h)^2 / beta per channel c
 *                       (snake_forward, src/audio_vae.c:310-351; alpha a
 *                       host tensor of >= channels values)
 *   VOXQ_VAE_SAVE       remember h (a residual sub-block's input)
 *   VOXQ_VAE_ADD_SAVED  h = h + the remembered tensor
 *                       (residual_sub_block_forward, src/audio_vae.c:354-421)
 *   VOXQ_VAE_TANH       h = tanh(h) (tensor_tanh)
 * An engine builds the list from its AudioVAEDecoder (include/model.h:
 * 352-417).  Shape errors -> VOXCPM_ERR_SHAPE_MISMATCH; not initialised ->
 * VOXCPM_ERR_CUDA_NOT_FOUND. */
enum { VOXQ_VAE_CONV = 1, VOXQ_VAE_CONVT = 2, VOXQ_VAE_SNAKE = 3, VOXQ_VAE_SAVE = 4, VOXQ_VAE_ADD_SAVED = 5,
       VOXQ_VAE_TANH = 6 };
typedef struct {
    int kind;
    const voxq_conv1d_desc* conv;             /* VOXQ_VAE_CONV */
    const voxq_conv1d_transpose_desc* convt;  /* VOXQ_VAE_CONVT */
    const Tensor* alpha;                      /* VOXQ_VAE_SNAKE */
} voxq_vae_op;
VOXQ_API VoxCPMError voxq_vae_decode(const voxq_vae_op* ops, int n_ops, float snake_beta, const Tensor* latent,
                                     Tensor* waveform);

/* ---- Transformer block on the device -------------------------------------
 * transformer_block_forward (src/nn.c:579-700) with every step on the device:
 *   h   = x + Attention(RMSNorm_attn(x))
 *   out = h + SwiGLU(RMSNorm_ffn(h))
 * where RMSNorm (src/tensor.c:811-849) is x / sqrt(mean(x^2) + eps) * weight
 * (sum of squares in double, NaN counted as 0), Attention is
 * attention_forward (src/nn.c:208-530: Q/K/V projections, RoPE
 * tensor_rotary_emb (src/tensor.c:883-950) at positions pos.. when freqs_cis
 * is given, K/V written into the cache at [pos, pos + seq), scores
 * q.k / sqrt(head_dim) + mask[s][t], softmax with 1 / (sum + 1e-10)
 * (src/tensor.c:710-752), GQA head h reading kv head h / (n_heads /
 * n_kv_heads), output projection) and SwiGLU is swiglu_forward
 * (src/nn.c:100-170: silu(x W1^T) * (x W3^T), then W2).  The residual adds
 * and SiLU-gating are fused into the projections' epilogues.
 *
 * Descriptors have the layouts of the engine's TransformerBlock, RmsNorm,
 * Attention and SwiGLU (include/nn.h:26-29, 58-64, 79-89, 136-141).  x, out
 * [batch, seq, d_model], the caches [batch, n_kv_heads, max_seq, head_dim],
 * mask [rows, cols] and freqs_cis [positions, head_dim / 2, 2] are host
 * tensors; the projection weights must be device weights quantized by
 * tensor_to_cuda (VOXCPM_QUANT=q8|q4) and the norm weights host tensors
 * (uploaded on first use and kept, keyed by pointer and a fingerprint).  The
 * caches are mirrored on the device per cache pointer (rows [0, pos) are
 * re-read from the host when the mirror cannot vouch for them: first use,
 * pos == 0 restarts, or a host row that no longer matches) and the new rows
 * are also written back to the host cache, so the engine's own state stays
 * exact.  out is valid on return.  Returns VOXCPM_ERR_CUDA_NOT_FOUND (the
 * caller then runs its host code) when the library is not initialised, a
 * weight is not a quantized device weight, an operand is already on the
 * device, or a shape is outside what the kernels take (head_dim a multiple
 * of 4 up to 256, cache positions up to 32768); the reference's own shape
 * errors are left to that host path. */
typedef struct {
    Tensor* weight;  /* [d_model] */
    float eps;
} voxq_rmsnorm_desc;
typedef struct {
    Tensor* wq;  /* [n_heads * head_dim, d_model] */
    Tensor* wk;  /* [n_kv_heads * head_dim, d_model] */
    Tensor* wv;
    Tensor* wo;  /* [d_model, n_heads * head_dim] */
    int d_model, n_heads, n_kv_heads, head_dim;
} voxq_attention_desc;
typedef struct {
    Tensor* w1;  /* gate [d_ff, d_model] */
    Tensor* w2;  /* down [d_model, d_ff] */
    Tensor* w3;  /* up   [d_ff, d_model] */
    int d_model, d_ff;
} voxq_swiglu_desc;
typedef struct {
    voxq_rmsnorm_desc* rms_attn;
    voxq_attention_desc* attn;
    voxq_rmsnorm_desc* rms_ffn;
    voxq_swiglu_desc* ffn;
} voxq_block_desc;

/* src/nn.c:579-700 (transformer_block_forward). */
VOXQ_API VoxCPMError voxq_transformer_block_forward(const voxq_block_desc* block, const Tensor* x, Tensor* cache_k,
                                                    Tensor* cache_v, const Tensor* mask, const Tensor* freqs_cis,
                                                    int pos, Tensor* out);
/* Drops the blocks' device cache mirrors, norm weights and staging. */
VOXQ_API void voxq_block_cache_clear(void);

/* ---- LocDiT sampler on the device ------------------------------------------
 * loc_dit_sample (src/loc_dit.c:437-593) with loc_dit_forward
 * (src/loc_dit.c:95-435) inside, the sequence resident on the device for the
 * whole sampler: per Euler step t = 1 - i dt (dt = (1 - 1e-6) / n_timesteps),
 * the time and delta embeddings (sinusoidal, interleaved sin / cos, then
 * Linear-SiLU-Linear), the input projection of x_t, the sequence
 * [mu; x_proj; cond_proj] + (time + delta), the n_layers transformer blocks
 * (bidirectional, no RoPE), the output RMSNorm of the x rows and the output
 * projection, then x_t -= dt * v.  With classifier-free guidance
 * (cfg_value > 1 and a non-empty cond) the conditional and unconditional
 * branches (cond replaced by zeros, so its projection is the bias) run as one
 * batch of two sequences through every block and are combined as
 * v = v_uncond + cfg (v_cond - v_uncond) -- the reference runs them as two
 * forwards.  x_init [1, feat_dim, patch] is the starting noise (the reference
 * draws it with tensor_rand_normal, seed 42); out [1, feat_dim, patch] (host)
 * receives x after the last step.  The descriptor has the layout of the
 * engine's LocDiT (include/model.h); its projection weights must be
 * quantized device weights (VOXCPM_QUANT), biases and norm weights host
 * tensors.  Returns VOXCPM_ERR_CUDA_NOT_FOUND (the caller then runs its host
 * sampler) for anything else (batch other than 1, unquantized weights, ...). */
typedef struct {
    Tensor* in_proj_weight;  /* [d_model, feat_dim] */
    Tensor* in_proj_bias;
    Tensor* cond_proj_weight;  /* [d_model, feat_dim] */
    Tensor* cond_proj_bias;
    Tensor* out_proj_weight;  /* [feat_dim, d_model] */
    Tensor* out_proj_bias;
    Tensor* time_mlp_1_weight;  /* [d_model, d_model] */
    Tensor* time_mlp_1_bias;
    Tensor* time_mlp_2_weight;
    Tensor* time_mlp_2_bias;
    Tensor* delta_mlp_1_weight;
    Tensor* delta_mlp_1_bias;
    Tensor* delta_mlp_2_weight;
    Tensor* delta_mlp_2_bias;
    voxq_block_desc* layers;  /* n_layers blocks */
    int n_layers;
    voxq_rmsnorm_desc* output_norm;
    int d_model;
    int feat_dim;
} voxq_locdit_desc;
VOXQ_API VoxCPMError voxq_locdit_sample(const voxq_locdit_desc* dit, const Tensor* mu, const Tensor* cond,
                                        int n_timesteps, float cfg_value, const Tensor* x_init, Tensor* out);

/* loc_enc_forward (src/loc_enc.c:19-190) on the device, the hidden state
 * resident across all layers: audio_feats [B, T, P, F] (host) -> in_proj
 * (+ bias) -> per time step [special token; P projected patches] -> the
 * n_layers blocks (bidirectional attention over all T (P + 1) tokens, no RoPE,
 * scratch K/V as the reference's single-use per-call cache) -> each step's
 * first token -> output RMSNorm -> out [B, T, D] (host).  The descriptor has
 * the field layout of the engine's LocEnc (include/model.h:141-150).  Returns
 * VOXCPM_ERR_CUDA_NOT_FOUND (the caller then runs its own code) for host
 * weights, device operands, shapes the kernels do not take, or before
 * tensor_cuda_init. */
typedef struct {
    const Tensor* in_proj_weight;   /* [D, F], quantized by tensor_to_cuda */
    const Tensor* in_proj_bias;     /* [D] host, or NULL */
    const Tensor* special_token;    /* [1, 1, 1, D] host */
    const voxq_block_desc* layers;  /* n_layers blocks */
    int n_layers;
    const voxq_rmsnorm_desc* output_norm;
    int d_model;
    int patch_size;
} voxq_locenc_desc;
VOXQ_API VoxCPMError voxq_locenc_forward(const voxq_locenc_desc* enc, const Tensor* audio_feats, Tensor* out);

/* ---- quantize.py weight containers (VXCPM2) ---------------------------
 * Reads the container written by the reference's quantizer
 * (scripts/quantize.py:110-312): a 256-byte header, the layer-group offset
 * table, and tensors stored as (name_hash, ndim, dims[3]) + data in the file's
 * quant type (f32, f16, 20-byte Q4 or 40-byte Q8 blocks over the flattened
 * tensor).  The reference's C loader cannot read these files (it knows only
 * the VXCP format, src/model.c:1715-1727, 1815-1858); this reader takes 2-D
 * Q4 / Q8 tensors straight to the packed device layout, bytes unchanged.
 * Host calls; the file stays mapped until voxq_vxcpm2_close. */
typedef struct voxq_vxcpm2 voxq_vxcpm2;  /* opaque */
typedef struct {
    uint32_t version, n_layers, n_layers_enc, n_ralm_layers, n_dit_layers;
    uint32_t d_model, d_ff, n_heads, n_kv_heads, head_dim, max_seq_len, vocab_size;
    uint32_t quant;            /* 0 f32, 1 f16, 2 q4, 3 q8 (VOXQ_F32 .. VOXQ_Q8) */
    uint32_t sample_rate, audio_vae_dim;
    float rope_theta;
    uint64_t checksum;         /* as stored at byte 72 */
    uint32_t n_groups;
} voxq_vxcpm2_header;
typedef struct {
    uint32_t name_hash, ndim, dims[3];
    int32_t dtype;             /* the file's quant type */
    int32_t group;             /* layer group */
    uint64_t elements;         /* prod(dims[:ndim]) */
    uint64_t offset, bytes;    /* data (after the 20-byte tensor header) in the file */
} voxq_vxcpm2_tensor;

/* VOXCPM_ERR_FILE_NOT_FOUND, _INVALID_MODEL (magic, bounds, truncated tensor)
 * or _UNSUPPORTED (unknown quant type). */
VOXQ_API VoxCPMError voxq_vxcpm2_open(const char* path, voxq_vxcpm2** out);
VOXQ_API void voxq_vxcpm2_close(voxq_vxcpm2* f);
VOXQ_API VoxCPMError voxq_vxcpm2_info(const voxq_vxcpm2* f, voxq_vxcpm2_header* hdr, int* n_tensors);
VOXQ_API VoxCPMError voxq_vxcpm2_tensor_info(const voxq_vxcpm2* f, int i, voxq_vxcpm2_tensor* t);
/* Host pointer to tensor i's data inside the mapped file. */
VOXQ_API const uint8_t* voxq_vxcpm2_data(const voxq_vxcpm2* f, int i);
/* SHA-256 checksum of scripts/quantize.py:309-315; VOXCPM_ERR_INVALID_MODEL on
 * mismatch, VOXCPM_ERR_UNSUPPORTED when the stored value is 0 (the reference
 * quantizer leaves it 0: it raises before writing it, scripts/quantize.py:308-310). */
VOXQ_API VoxCPMError voxq_vxcpm2_verify(const voxq_vxcpm2* f);
/* Tensor i as fp32 on the host (dequantize_q4_block / dequantize_q8_block of
 * scripts/quantize.py:56-82; q8_signed selects the signed Q8 reading). */
VOXQ_API VoxCPMError voxq_vxcpm2_dequantize(const voxq_vxcpm2* f, int i, int q8_signed, float* h_out);
/* 2-D Q4 / Q8 tensor i ([N][K], K % 32 == 0) -> packed device weight
 * (arrays sized by voxq_codes_bytes / voxq_scales_bytes).  Returns after the
 * copy is complete. */
VOXQ_API VoxCPMError voxq_vxcpm2_upload_qweight(const voxq_vxcpm2* f, int i, uint8_t* d_codes, void* d_scales,
                                              void* stream);

/* ======================================================================== */
/* Pre-quantized weights in the engine's own VXCP container                 */
/* ======================================================================== */
/*
 * The VXCP format (docs/WEIGHT_FORMAT.md §2, §5; read by weight_index_build /
 * weight_load_tensor, src/model.c:1628-1877) names dtype 3 (Q4_0) and 4 (Q4_1)
 * but its loader sizes both as 0 bytes and rejects them (src/model.c:1715-1727,
 * 1855-1858), and it has no Q8 code.  voxq's VXCP quantized dtypes:
 *
 *   4  Q4_1  20-byte blocks of 32 values, fields in docs/WEIGHT_FORMAT.md §5
 *            order: fp16 d, fp16 m, uint8 q[16] with byte i = q[2i] << 4 |
 *            q[2i+1] (the nibble order of scripts/quantize.py:48-50);
 *            value = q * d + m in fp32.  d, m, q are quantize_q4_block's
 *            scale, min and codes (scripts/quantize.py:42-54).
 *   5  Q8    40-byte blocks: fp32 d, fp32 m, uint8 q[32]; value = q * d + m
 *            (q unsigned); quantize_q8_block's scale, min and codes
 *            (scripts/quantize.py:69-75), header first like Q4_1.
 *
 * Blocks run over the flattened tensor, the last one zero-padded, as in
 * scripts/quantize.py:239-260.  Q4_0 (3, 18-byte blocks per §5) has no
 * producer and no defined dequantization; readers size it and reject it.
 */
enum { VOXQ_VXCP_FP32 = 0, VOXQ_VXCP_BF16 = 1, VOXQ_VXCP_FP16 = 2, VOXQ_VXCP_Q4_0 = 3, VOXQ_VXCP_Q4_1 = 4,
       VOXQ_VXCP_Q8 = 5 };

typedef struct {
    uint32_t tensors;    /* tensors in the file */
    uint32_t quantized;  /* tensors written as Q4_1 / Q8 */
    uint64_t bytes_in, bytes_out;  /* file sizes */
} voxq_vxcp_stats;

/* Rewrites the VXCP model file src_path as dst_path with every 2-D fp32 /
 * fp16 / bf16 tensor whose row length is a multiple of 32 quantized to
 * qtype (VOXQ_Q4 -> dtype 4, VOXQ_Q8 -> dtype 5) on the current device,
 * bit-exact with scripts/quantize.py's blocks; other tensors, and those whose
 * name contains one of the n_keep strings in keep (e.g. "embed_tokens", a
 * table the engine reads on the host, src/tslm.c:415), are copied unchanged.
 * Header, metadata order, string table and both CRC32C checksums are written
 * as make_model / convert_weights.py write them.  Host call; returns after the
 * file is closed.  VOXCPM_ERR_FILE_NOT_FOUND, _INVALID_MODEL (magic, version,
 * bounds), _UNSUPPORTED (a Q4_0 or unknown dtype, qtype not Q4 / Q8),
 * _OOM, _INTERNAL (write failure; the partial file is removed). */
VOXQ_API VoxCPMError voxq_vxcp_quantize(const char* src_path, const char* dst_path, int qtype,
                                        const char* const* keep, int n_keep, voxq_vxcp_stats* stats);

/* Hands tensor_to_cuda the quantize.py block stream (block fields in
 * scripts/quantize.py order: codes, then scale and min) of a 2-D host weight
 * loaded from a pre-quantized file.  Ownership of `blocks` (malloc'd,
 * voxq_quant_bytes(N*K, qtype) bytes) passes to the library.  The tensor's own
 * host data (the dequantized values, for any host-side reader) is left as it
 * is; the next tensor_to_cuda(t) uploads the blocks to the packed device
 * layout instead of quantizing t's values (whatever VOXCPM_QUANT says) and
 * frees both.  Needs no device and no tensor_cuda_init.
 * VOXCPM_ERR_SHAPE_MISMATCH (not 2-D, K % 32 != 0, wrong byte count, device
 * tensor) or _UNSUPPORTED (qtype); on error ownership stays with the caller. */
VOXQ_API VoxCPMError voxq_tensor_attach_blocks(const Tensor* t, int qtype, void* blocks, size_t nbytes);

/* Frees the blocks attached to t, if any (call before freeing a tensor that
 * was never uploaded).  Returns 1 if blocks were attached, else 0. */
VOXQ_API int voxq_tensor_detach_blocks(const Tensor* t);

#ifdef __cplusplus
}
#endif

#endif /* VOXQ_H */
