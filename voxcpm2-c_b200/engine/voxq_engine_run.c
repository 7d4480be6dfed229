/*
 * voxq_engine_run.c -- runs the unchanged voxcpm2-c engine (src/model.c
 * voxcpm_create -> [voxcpm_to_cuda] -> voxcpm_generate, the flow of
 * examples/tts_minimal.c and src/main.c) on a model file and reports what a
 * synthesis run needs to be checked and measured: the latent of every patch,
 * the time spent per stage and the real-time factor.
 *
 *   voxq_engine_run --model M.vxcpm [--patches N] [--tokens T] [--token-seed S]
 *                   [--gpu] [--latents OUT.f32] [--audio OUT.f32] [--ralm-max-seq L]
 *   prints one JSON line.
 *
 *   voxq_engine_run --model M.vxcpm --serve [--gpu] [--ralm-max-seq L] [--latents-dir D]
 *   serving worker: loads the model once, prints {"ready": ...}, then runs one
 *   utterance per line read from standard input ("INDEX TOKENS TOKEN_SEED
 *   PATCHES"), printing one JSON line per utterance (its time, the hash of its
 *   latents, and with D the latents in D/utt<INDEX>.f32) until "quit" or end
 *   of input.  voxcpm_generate re-creates its caches on every call
 *   (src/model.c:706-730), so utterances are independent.
 *
 * The engine's sources are compiled as they are.  The run is observed at the
 * engine's own function boundaries, which the linker redirects here
 * (-Wl,--wrap=NAME sends model.c's calls of NAME, defined in another object,
 * to __wrap_NAME; each wrapper calls __real_NAME):
 *   loc_dit_sample     copies each patch's latent [1, 64, 4] (the sampler's
 *                      output, src/loc_dit.c:437) and times the stage;
 *   tslm_forward, ralm_forward, loc_enc_forward, audio_vae_decode,
 *   tensor_matmul_nt   time per stage (tensor_matmul_nt: every projection of
 *                      every stage; in a VOXCPM_CUDA build it is the call
 *                      into tensor_matmul_nt_cuda, src/tensor.c:629-640);
 *   tokenizer_create_from_weights, tokenizer_encode
 *                      the input: no tokenizer ships with a random-init
 *                      model, so the run's text is T token ids drawn
 *                      uniformly from the 73448-entry vocabulary with a
 *                      seeded xorshift64 (a vocabulary of placeholder
 *                      strings is built with tokenizer_create_bpe so the
 *                      engine holds a real tokenizer object);
 *   conv1d_forward, conv1d_transpose_forward (the libvoxq build only)
 *                      the AudioVAE decoder's convolutions (src/nn.c:765-931),
 *                      which the reference runs on the host even in its GPU
 *                      build, go to voxq_conv1d_forward /
 *                      voxq_conv1d_transpose_forward on the device (same
 *                      functions, fp32); VOXQ_ENGINE_VAE=cpu keeps them on the
 *                      host;
 *   ralm_setup_cache   with --ralm-max-seq L, sets the RALM cache length to
 *                      L before the cache is allocated.  voxcpm_generate fixes
 *                      it at 2048 positions (src/model.c:709), which holds
 *                      63 patches of a 64-token text; longer runs need more.
 *                      Without the flag the engine's value stands.
 */
#define _POSIX_C_SOURCE 200809L
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "model.h"
#include "nn.h"
#include "tensor.h"
#include "tokenizer.h"
#include "voxcpm.h"
#ifdef VOXQ_ENGINE_LIBVOXQ
#include "voxq.h"
#endif

static double now(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
}

/* ---- run options and observations ---- */
static int g_tokens = 64;
static uint64_t g_token_seed = 1;
static int g_ralm_max_seq = 0;
static float* g_latents = NULL;
static int g_latent_cap = 0, g_latent_n = 0;

enum { ST_TSLM, ST_RALM, ST_DIT, ST_LOCENC, ST_VAE, ST_MATMUL, ST_N };
static const char* k_stage[ST_N] = {"tslm_forward", "ralm_forward", "loc_dit_sample", "loc_enc_forward",
                                   "audio_vae_decode", "tensor_matmul_nt"};
static double g_stage_s[ST_N];
static long g_stage_calls[ST_N];
static int g_in_stage = -1;  /* the outermost stage in progress (matmul time is also split per stage) */
static double g_matmul_in[ST_N];

#define TIMED(stage, call)                                        \
    do {                                                          \
        const int outer = g_in_stage;                             \
        if (outer < 0) g_in_stage = (stage);                      \
        const double t0_ = now();                                 \
        r = (call);                                               \
        g_stage_s[stage] += now() - t0_;                          \
        g_stage_calls[stage]++;                                   \
        g_in_stage = outer;                                       \
    } while (0)

VoxCPMError __real_tslm_forward(TSLM* tslm, const Tensor* x, const Tensor* freqs_cis, Tensor* out);
VoxCPMError __wrap_tslm_forward(TSLM* tslm, const Tensor* x, const Tensor* freqs_cis, Tensor* out) {
    VoxCPMError r;
    TIMED(ST_TSLM, __real_tslm_forward(tslm, x, freqs_cis, out));
    return r;
}

VoxCPMError __real_ralm_forward(RALM* ralm, const Tensor* x, const Tensor* freqs_cis, Tensor* out);
VoxCPMError __wrap_ralm_forward(RALM* ralm, const Tensor* x, const Tensor* freqs_cis, Tensor* out) {
    VoxCPMError r;
    TIMED(ST_RALM, __real_ralm_forward(ralm, x, freqs_cis, out));
    return r;
}

VoxCPMError __real_loc_enc_forward(const LocEnc* enc, const Tensor* feats, Tensor* out);
/* loc_enc_forward: in the libvoxq build the whole encoder runs on the device
 * (voxq_locenc_forward: the hidden state resident across the 12 layers, one
 * upload of the features, one download of the step embeddings) instead of a
 * host round trip per layer; VOXQ_ENGINE_LOCENC=cpu keeps the engine's own
 * loop (its blocks still go to the device one by one). */
static int g_enc_gpu = 1;
static VoxCPMError enc_forward(const LocEnc* enc, const Tensor* feats, Tensor* out) {
#ifdef VOXQ_ENGINE_LIBVOXQ
    if (g_enc_gpu) {
        const VoxCPMError r = voxq_locenc_forward((const voxq_locenc_desc*)enc, feats, out);
        if (r != VOXCPM_ERR_CUDA_NOT_FOUND) return r;
    }
#endif
    return __real_loc_enc_forward(enc, feats, out);
}
VoxCPMError __wrap_loc_enc_forward(const LocEnc* enc, const Tensor* feats, Tensor* out) {
    VoxCPMError r;
    TIMED(ST_LOCENC, enc_forward(enc, feats, out));
    return r;
}

VoxCPMError __real_audio_vae_decode(const AudioVAE* vae, const Tensor* z, Tensor* out);
static VoxCPMError vae_decode(const AudioVAE* vae, const Tensor* z, Tensor* out);
VoxCPMError __wrap_audio_vae_decode(const AudioVAE* vae, const Tensor* z, Tensor* out) {
    VoxCPMError r;
    TIMED(ST_VAE, vae_decode(vae, z, out));
    return r;
}

/* VOXQ_ENGINE_MATMUL_LOG=path: one line per tensor_matmul_nt call (shape,
 * where the operands live, and sums of the host output), so two builds of the
 * engine can be compared call by call. */
static FILE* g_mm_log = NULL;
static const char* g_dump_calls = NULL;  /* comma-separated call indices */
static const char* g_dump_dir = NULL;
static int dump_wanted(long i) {
    for (const char* p = g_dump_calls; p && *p;) {
        if (atol(p) == i) return 1;
        p = strchr(p, ',');
        if (p) p++;
    }
    return 0;
}

VoxCPMError __real_tensor_matmul_nt(const Tensor* a, const Tensor* b, Tensor* out);
VoxCPMError __wrap_tensor_matmul_nt(const Tensor* a, const Tensor* b, Tensor* out) {
    const double t0 = now();
    VoxCPMError r = __real_tensor_matmul_nt(a, b, out);
    const double dt = now() - t0;
    g_stage_s[ST_MATMUL] += dt;
    if (g_mm_log && out && !out->is_cuda && out->data) {
        double sum = 0, asum = 0;
        for (size_t i = 0; i < out->size; i++) {
            sum += out->data[i];
            asum += out->data[i] < 0 ? -out->data[i] : out->data[i];
        }
        fprintf(g_mm_log, "%ld %d %d %d stage=%d a_cuda=%d b_cuda=%d b_fp16=%d r=%d sum=%.9g asum=%.9g v0=%.9g v1=%.9g\n",
                g_stage_calls[ST_MATMUL], a->shape[0], b->shape[0], a->shape[1], g_in_stage, (int)a->is_cuda,
                (int)b->is_cuda, (int)b->is_fp16, (int)r, sum, asum, out->size > 0 ? out->data[0] : 0.0,
                out->size > 1 ? out->data[out->size - 1] : 0.0);
    }
    if (g_dump_dir && dump_wanted(g_stage_calls[ST_MATMUL])) {
        /* VOXQ_ENGINE_DUMP_CALL=i,j,... with VOXQ_ENGINE_DUMP_DIR: the host
         * activation and output of those calls, as raw float32 */
        char path[1024];
        snprintf(path, sizeof path, "%s/call%ld_a.f32", g_dump_dir, g_stage_calls[ST_MATMUL]);
        FILE* f = fopen(path, "wb");
        if (f && !a->is_cuda) fwrite(a->data, sizeof(float), a->size, f);
        if (f) fclose(f);
        snprintf(path, sizeof path, "%s/call%ld_out.f32", g_dump_dir, g_stage_calls[ST_MATMUL]);
        f = fopen(path, "wb");
        if (f && !out->is_cuda) fwrite(out->data, sizeof(float), out->size, f);
        if (f) fclose(f);
    }
    g_stage_calls[ST_MATMUL]++;
    if (g_in_stage >= 0) g_matmul_in[g_in_stage] += dt;
    return r;
}

VoxCPMError __real_loc_dit_sample(const LocDiT* dit, const Tensor* mu, const Tensor* cond, int n_timesteps,
                                  float cfg_value, Tensor* out);
/* loc_dit_sample: in the libvoxq build the whole sampler runs on the device
 * (voxq_locdit_sample: the sequence resident, the CFG branches batched) with
 * the starting noise drawn here exactly as loc_dit_sample draws it
 * (src/loc_dit.c:471-474: tensor_rand_normal, seed 42); VOXQ_ENGINE_DIT=cpu
 * keeps the engine's own sampler (its blocks still go to the device). */
static int g_dit_gpu = 1;
static VoxCPMError dit_sample(const LocDiT* dit, const Tensor* mu, const Tensor* cond, int n_timesteps,
                              float cfg_value, Tensor* out) {
#ifdef VOXQ_ENGINE_LIBVOXQ
    if (g_dit_gpu && dit && mu && out && out->ndim == 3) {
        Tensor* x0 = tensor_create(3, (int[]){out->shape[0], out->shape[1], out->shape[2]});
        if (x0) {
            uint64_t seed = 42;
            tensor_rand_normal(x0, &seed);
            const VoxCPMError r = voxq_locdit_sample((const voxq_locdit_desc*)dit, mu, cond, n_timesteps, cfg_value,
                                                     x0, out);
            tensor_free(x0);
            if (r != VOXCPM_ERR_CUDA_NOT_FOUND) return r;
        }
    }
#endif
    return __real_loc_dit_sample(dit, mu, cond, n_timesteps, cfg_value, out);
}

VoxCPMError __wrap_loc_dit_sample(const LocDiT* dit, const Tensor* mu, const Tensor* cond, int n_timesteps,
                                  float cfg_value, Tensor* out) {
    VoxCPMError r;
    TIMED(ST_DIT, dit_sample(dit, mu, cond, n_timesteps, cfg_value, out));
    if (r == VOXCPM_SUCCESS && out && out->data && !out->is_cuda) {
        const int n = (int)out->size;
        if (g_latent_n + n > g_latent_cap) {
            g_latent_cap = 2 * (g_latent_n + n);
            g_latents = (float*)realloc(g_latents, (size_t)g_latent_cap * sizeof(float));
            if (!g_latents) return VOXCPM_ERR_OOM;
        }
        memcpy(g_latents + g_latent_n, out->data, (size_t)n * sizeof(float));
        g_latent_n += n;
    }
    return r;
}

#ifdef VOXQ_ENGINE_LIBVOXQ
/* AudioVAE decode.  VOXQ_ENGINE_VAE = device (default): the whole decoder on
 * the device with its activation resident (voxq_vae_decode, steps listed from
 * the engine's AudioVAEDecoder in the order audio_vae_decode runs them,
 * src/audio_vae.c:941-1116); convs: the engine's own decoder with only its
 * convolutions on the device (conv1d_forward / conv1d_transpose_forward
 * below); cpu: all on the host. */
static int g_vae_gpu = 1;     /* convolutions go to the device */
static int g_vae_whole = 1;   /* the whole decoder goes to the device */
static const float kSnakeBeta = 1.0f;  /* AUDIOVAE_SNAKE_BETA, src/audio_vae.c:39 */

static int wn_desc(const WNConv* wn, voxq_vae_op* op, voxq_conv1d_desc* c, voxq_conv1d_transpose_desc* t) {
    /* wnconv_forward (src/audio_vae.c:279-305): the effective weight and the bias */
    if (!wn || !wn->effective_weight) return 0;
    memset(op, 0, sizeof(*op));
    if (wn->is_transpose) {
        *t = (voxq_conv1d_transpose_desc){wn->effective_weight, wn->bias, wn->in_channels, wn->out_channels,
                                          wn->kernel_size, wn->stride, wn->padding};
        op->kind = VOXQ_VAE_CONVT;
        op->convt = t;
    } else {
        *c = (voxq_conv1d_desc){wn->effective_weight, wn->bias, wn->in_channels, wn->out_channels,
                                wn->kernel_size, wn->stride, wn->padding, wn->groups};
        op->kind = VOXQ_VAE_CONV;
        op->conv = c;
    }
    return 1;
}

static VoxCPMError vae_decode_device(const AudioVAE* vae, const Tensor* z, Tensor* out) {
    enum { kMaxOps = 256, kMaxConvs = 128 };
    voxq_vae_op ops[kMaxOps];
    voxq_conv1d_desc cd[kMaxConvs];
    voxq_conv1d_transpose_desc td[kMaxConvs];
    int n = 0, nc = 0;
    const AudioVAEDecoder* d = vae ? vae->decoder : NULL;
    if (!d || !z || z->ndim != 3 || z->shape[2] != vae->latent_dim) return VOXCPM_ERR_CUDA_NOT_FOUND;
#define CONV(wn)                                                                     \
    do {                                                                             \
        if (n >= kMaxOps || nc >= kMaxConvs || !wn_desc((wn), &ops[n], &cd[nc], &td[nc])) \
            return VOXCPM_ERR_CUDA_NOT_FOUND;                                        \
        n++;                                                                         \
        nc++;                                                                        \
    } while (0)
#define STEP(k, a)                                                                   \
    do {                                                                             \
        if (n >= kMaxOps) return VOXCPM_ERR_CUDA_NOT_FOUND;                          \
        memset(&ops[n], 0, sizeof(ops[n]));                                          \
        ops[n].kind = (k);                                                           \
        ops[n].alpha = (a);                                                          \
        n++;                                                                         \
    } while (0)
    CONV(d->conv_in);
    CONV(d->proj_up);
    for (int i = 0; i < AUDIOVAE_NUM_DECODER_BLOCKS; i++) {  /* decoder_block_forward */
        const AudioVAEDecoderBlock* b = &d->decoder_blocks[i];
        if (b->snake_alpha) STEP(VOXQ_VAE_SNAKE, b->snake_alpha);
        CONV(b->convtr);
        for (int j = 0; j < b->num_res_blocks && j < AUDIOVAE_RES_BLOCKS_PER_BLOCK; j++) {  /* residual_sub_block_forward */
            const AudioVAEResBlock* rb = &b->res_blocks[j];
            STEP(VOXQ_VAE_SAVE, NULL);
            if (rb->snake_alpha1) STEP(VOXQ_VAE_SNAKE, rb->snake_alpha1);
            CONV(rb->conv_depthwise);
            if (rb->snake_alpha2) STEP(VOXQ_VAE_SNAKE, rb->snake_alpha2);
            CONV(rb->conv_pointwise);
            STEP(VOXQ_VAE_ADD_SAVED, NULL);
        }
    }
    if (d->final_snake_alpha) STEP(VOXQ_VAE_SNAKE, d->final_snake_alpha);
    CONV(d->conv_out);
    STEP(VOXQ_VAE_TANH, NULL);
#undef CONV
#undef STEP
    return voxq_vae_decode(ops, n, kSnakeBeta, z, out);
}
#endif

static VoxCPMError vae_decode(const AudioVAE* vae, const Tensor* z, Tensor* out) {
#ifdef VOXQ_ENGINE_LIBVOXQ
    if (g_vae_whole) {
        const VoxCPMError r = vae_decode_device(vae, z, out);
        if (r != VOXCPM_ERR_CUDA_NOT_FOUND) return r;
    }
#endif
    return __real_audio_vae_decode(vae, z, out);
}

#ifdef VOXQ_ENGINE_LIBVOXQ
/* Conv1D / Conv1DTranspose (include/nn.h:198-229) and voxq's descriptors have
 * the same layout. */
VoxCPMError __real_conv1d_forward(const Conv1D* conv, const Tensor* x, Tensor* out);
VoxCPMError __wrap_conv1d_forward(const Conv1D* conv, const Tensor* x, Tensor* out) {
    if (g_vae_gpu) {
        const VoxCPMError r = voxq_conv1d_forward((const voxq_conv1d_desc*)conv, x, out);
        if (r != VOXCPM_ERR_CUDA_NOT_FOUND) return r;
    }
    return __real_conv1d_forward(conv, x, out);
}
/* transformer_block_forward (src/nn.c:579-700), called from tslm.c, ralm.c,
 * loc_dit.c and loc_enc.c, goes to voxq_transformer_block_forward: the whole
 * block on the device (TransformerBlock, RmsNorm, Attention and SwiGLU have
 * voxq's descriptor layouts).  VOXQ_ENGINE_BLOCK=cpu keeps the host code. */
static int g_block_gpu = 1;
static long g_block_dev = 0, g_block_host = 0;
VoxCPMError __real_transformer_block_forward(const TransformerBlock* block, const Tensor* x, Tensor* cache_k,
                                             Tensor* cache_v, const Tensor* mask, const Tensor* freqs_cis, int pos,
                                             Tensor* out);
VoxCPMError __wrap_transformer_block_forward(const TransformerBlock* block, const Tensor* x, Tensor* cache_k,
                                             Tensor* cache_v, const Tensor* mask, const Tensor* freqs_cis, int pos,
                                             Tensor* out) {
    if (g_block_gpu) {
        const VoxCPMError r = voxq_transformer_block_forward((const voxq_block_desc*)block, x, cache_k, cache_v, mask,
                                                             freqs_cis, pos, out);
        if (r != VOXCPM_ERR_CUDA_NOT_FOUND) {
            g_block_dev++;
            return r;
        }
    }
    g_block_host++;
    return __real_transformer_block_forward(block, x, cache_k, cache_v, mask, freqs_cis, pos, out);
}

VoxCPMError __real_conv1d_transpose_forward(const Conv1DTranspose* conv, const Tensor* x, Tensor* out);
VoxCPMError __wrap_conv1d_transpose_forward(const Conv1DTranspose* conv, const Tensor* x, Tensor* out) {
    if (g_vae_gpu) {
        const VoxCPMError r = voxq_conv1d_transpose_forward((const voxq_conv1d_transpose_desc*)conv, x, out);
        if (r != VOXCPM_ERR_CUDA_NOT_FOUND) return r;
    }
    return __real_conv1d_transpose_forward(conv, x, out);
}
#endif

VoxCPMError __real_ralm_setup_cache(RALM* ralm, int batch_size);
VoxCPMError __wrap_ralm_setup_cache(RALM* ralm, int batch_size) {
    if (ralm && g_ralm_max_seq > 0) ralm->max_seq_len = g_ralm_max_seq;
    return __real_ralm_setup_cache(ralm, batch_size);
}

#define VOCAB 73448
Tokenizer* __real_tokenizer_create_from_weights(const uint8_t* mmap_data, const WeightIndex* idx);
Tokenizer* __wrap_tokenizer_create_from_weights(const uint8_t* mmap_data, const WeightIndex* idx) {
    Tokenizer* t = __real_tokenizer_create_from_weights(mmap_data, idx);
    if (t) return t;
    static char store[VOCAB][12];
    static const char* vocab[VOCAB];
    for (int i = 0; i < VOCAB; i++) {
        snprintf(store[i], sizeof store[i], "<%d>", i);
        vocab[i] = store[i];
    }
    return tokenizer_create_bpe(vocab, VOCAB, 11);
}

int __real_tokenizer_encode(const Tokenizer* tok, const char* text, int32_t* out_tokens, int max_tokens);
int __wrap_tokenizer_encode(const Tokenizer* tok, const char* text, int32_t* out_tokens, int max_tokens) {
    (void)tok;
    (void)text;
    if (!out_tokens) return g_tokens;
    if (max_tokens < g_tokens) return -VOXCPM_ERR_INTERNAL;
    uint64_t s = g_token_seed ? g_token_seed : 1;  /* xorshift64 (src/tensor.c:339-345); 0 would stay 0 */
    for (int i = 0; i < g_tokens; i++) {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        out_tokens[i] = (int32_t)(((unsigned __int128)s * VOCAB) >> 64);
    }
    return g_tokens;
}

/* FNV-1a 64 of the bytes of the latents gathered so far */
static unsigned long long latents_fnv(void) {
    unsigned long long h = 1469598103934665603ull;
    const unsigned char* b = (const unsigned char*)g_latents;
    for (size_t i = 0; i < (size_t)g_latent_n * sizeof(float); i++) {
        h ^= b[i];
        h *= 1099511628211ull;
    }
    return h;
}

static void print_stages(void) {
#ifdef VOXQ_ENGINE_LIBVOXQ
    printf("\"blocks\": {\"device\": %ld, \"host\": %ld}, ", g_block_dev, g_block_host);
#endif
    printf("\"stages\": {");
    for (int s = 0; s < ST_N; s++) {
        printf("%s\"%s\": {\"s\": %.5f, \"calls\": %ld", s ? ", " : "", k_stage[s], g_stage_s[s], g_stage_calls[s]);
        if (s != ST_MATMUL) printf(", \"matmul_s\": %.5f", g_matmul_in[s]);  /* tensor_matmul_nt time inside */
        printf("}");
    }
    printf("}");
}

/* Serving worker: one utterance per input line, until "quit" or end of input. */
static int serve(VoxCPMModel* model, const char* latents_dir) {
    char line[256];
    while (fgets(line, sizeof line, stdin)) {
        if (!strncmp(line, "quit", 4)) break;
        long idx = -1;
        int tokens = 0, patches = 0;
        unsigned long long seed = 0;
        if (sscanf(line, "%ld %d %llu %d", &idx, &tokens, &seed, &patches) != 4 || idx < 0 || tokens < 1 ||
            patches < 1) {
            printf("{\"error\": \"bad request\"}\n");
            fflush(stdout);
            continue;
        }
        g_tokens = tokens;
        g_token_seed = seed;
        g_latent_n = 0;
        memset(g_stage_s, 0, sizeof(g_stage_s));
        memset(g_stage_calls, 0, sizeof(g_stage_calls));
        memset(g_matmul_in, 0, sizeof(g_matmul_in));
#ifdef VOXQ_ENGINE_LIBVOXQ
        voxq_matmul_traffic(NULL, NULL, 1);
        g_block_dev = g_block_host = 0;
#endif
        VoxCPMGenConfig gen = voxcpm_gen_config_default();
        gen.text = "synthetic token ids";
        gen.cfg_value = 2.0f;
        gen.inference_timesteps = 10;
        gen.max_new_tokens = 4 * patches;
        VoxCPMAudio audio;
        memset(&audio, 0, sizeof(audio));
        const double t0 = now();
        const VoxCPMError err = voxcpm_generate(model, &gen, &audio);
        const double gen_s = now() - t0;
        unsigned long long calls = 0, wbytes = 0;
#ifdef VOXQ_ENGINE_LIBVOXQ
        uint64_t c64 = 0, b64 = 0;
        voxq_matmul_traffic(&c64, &b64, 1);
        calls = c64;
        wbytes = b64;
#endif
        if (err != VOXCPM_SUCCESS) {
            printf("{\"utt\": %ld, \"error\": \"%s\"}\n", idx, voxcpm_error_string(err));
            fflush(stdout);
            continue;
        }
        if (latents_dir) {
            char path[1024];
            snprintf(path, sizeof path, "%s/utt%ld.f32", latents_dir, idx);
            FILE* f = fopen(path, "wb");
            if (f) {
                fwrite(g_latents, sizeof(float), (size_t)g_latent_n, f);
                fclose(f);
            }
        }
        const double audio_s = audio.sample_rate > 0 ? (double)audio.num_samples / audio.sample_rate : 0.0;
        printf("{\"utt\": %ld, \"tokens\": %d, \"token_seed\": %llu, \"patches\": %d, \"latent_floats\": %d, "
               "\"latents_fnv\": \"%016llx\", \"samples\": %d, \"audio_s\": %.6f, \"generate_s\": %.4f, "
               "\"matmul_calls\": %llu, \"weight_bytes\": %llu, ",
               idx, tokens, seed, g_latent_n / 256, g_latent_n, latents_fnv(), audio.num_samples, audio_s, gen_s,
               calls, wbytes);
        print_stages();
        printf("}\n");
        fflush(stdout);
        voxcpm_audio_free(&audio);
    }
    return 0;
}

int main(int argc, char** argv) {
    const char* model_path = NULL;
    const char* latents_dir = NULL;
    int serve_mode = 0;
    const char* latents_path = NULL;
    const char* audio_path = NULL;
    int patches = 4, gpu = 0;
    for (int i = 1; i < argc; i++) {
        const char* a = argv[i];
        const char* v = i + 1 < argc ? argv[i + 1] : NULL;
        if (!strcmp(a, "--model") && v) { model_path = v; i++; }
        else if (!strcmp(a, "--patches") && v) { patches = atoi(v); i++; }
        else if (!strcmp(a, "--tokens") && v) { g_tokens = atoi(v); i++; }
        else if (!strcmp(a, "--token-seed") && v) { g_token_seed = strtoull(v, NULL, 10); i++; }
        else if (!strcmp(a, "--latents") && v) { latents_path = v; i++; }
        else if (!strcmp(a, "--audio") && v) { audio_path = v; i++; }
        else if (!strcmp(a, "--ralm-max-seq") && v) { g_ralm_max_seq = atoi(v); i++; }
        else if (!strcmp(a, "--latents-dir") && v) { latents_dir = v; i++; }
        else if (!strcmp(a, "--serve")) serve_mode = 1;
        else if (!strcmp(a, "--gpu")) gpu = 1;
        else {
            fprintf(stderr, "usage: %s --model M.vxcpm [--patches N] [--tokens T] [--token-seed S] [--gpu] "
                            "[--latents OUT.f32] [--audio OUT.f32] [--ralm-max-seq L] [--serve [--latents-dir D]]\n",
                    argv[0]);
            return 2;
        }
    }
    if (!model_path || patches < 1 || g_tokens < 1) return 2;
    const char* mm_log = getenv("VOXQ_ENGINE_MATMUL_LOG");
    if (mm_log && *mm_log) g_mm_log = fopen(mm_log, "w");
    g_dump_calls = getenv("VOXQ_ENGINE_DUMP_CALL");
#ifdef VOXQ_ENGINE_LIBVOXQ
    {
        const char* v = getenv("VOXQ_ENGINE_VAE");
        if (v && !strcmp(v, "cpu")) g_vae_gpu = g_vae_whole = 0;
        if (v && !strcmp(v, "convs")) g_vae_whole = 0;
    }
    if (getenv("VOXQ_ENGINE_BLOCK") && !strcmp(getenv("VOXQ_ENGINE_BLOCK"), "cpu")) g_block_gpu = 0;
    if (getenv("VOXQ_ENGINE_DIT") && !strcmp(getenv("VOXQ_ENGINE_DIT"), "cpu")) g_dit_gpu = 0;
    if (getenv("VOXQ_ENGINE_LOCENC") && !strcmp(getenv("VOXQ_ENGINE_LOCENC"), "cpu")) g_enc_gpu = 0;
#endif
    g_dump_dir = getenv("VOXQ_ENGINE_DUMP_DIR");

    const double t_create = now();
    VoxCPMModelConfig cfg = voxcpm_model_config_default();
    cfg.model_path = model_path;
    cfg.n_threads = 1;
    cfg.use_gpu = gpu != 0;
    VoxCPMError err = VOXCPM_SUCCESS;
    VoxCPMModel* model = voxcpm_create(&cfg, &err);
    if (!model) {
        fprintf(stderr, "voxcpm_create failed: %s\n", voxcpm_error_string(err));
        return 1;
    }
    const double create_s = now() - t_create;
    double upload_s = 0;
    if (gpu) {
        const double t0 = now();
        err = voxcpm_to_cuda(model);
        upload_s = now() - t0;
        if (err != VOXCPM_SUCCESS) {
            fprintf(stderr, "voxcpm_to_cuda failed: %s\n", voxcpm_error_string(err));
            voxcpm_free(model);
            return 1;
        }
    }

    if (serve_mode) {
        printf("{\"ready\": true, \"build\": \"%s\", \"create_s\": %.3f, \"upload_s\": %.3f, \"ralm_max_seq\": %d}\n",
#ifdef VOXCPM_CUDA
               "gpu",
#else
               "cpu",
#endif
               create_s, upload_s, g_ralm_max_seq);
        fflush(stdout);
        const int rc = serve(model, latents_dir);
        voxcpm_free(model);
        free(g_latents);
        if (g_mm_log) fclose(g_mm_log);
        return rc;
    }

    VoxCPMGenConfig gen = voxcpm_gen_config_default();
    gen.text = "synthetic token ids";
    gen.cfg_value = 2.0f;
    gen.inference_timesteps = 10;
    gen.max_new_tokens = 4 * patches;
    VoxCPMAudio audio;
    memset(&audio, 0, sizeof(audio));
    memset(g_stage_s, 0, sizeof(g_stage_s));
    memset(g_stage_calls, 0, sizeof(g_stage_calls));
    memset(g_matmul_in, 0, sizeof(g_matmul_in));
    const double t0 = now();
    err = voxcpm_generate(model, &gen, &audio);
    const double gen_s = now() - t0;
    if (err != VOXCPM_SUCCESS) {
        fprintf(stderr, "voxcpm_generate failed: %s\n", voxcpm_error_string(err));
        voxcpm_free(model);
        return 1;
    }
    const double audio_s = audio.sample_rate > 0 ? (double)audio.num_samples / audio.sample_rate : 0.0;
    double asum = 0;
    for (int i = 0; i < audio.num_samples; i++) asum += audio.samples[i] < 0 ? -audio.samples[i] : audio.samples[i];

    if (latents_path) {
        FILE* f = fopen(latents_path, "wb");
        if (!f || fwrite(g_latents, sizeof(float), (size_t)g_latent_n, f) != (size_t)g_latent_n || fclose(f)) {
            fprintf(stderr, "cannot write %s\n", latents_path);
            return 1;
        }
    }
    if (audio_path) {
        FILE* f = fopen(audio_path, "wb");
        const size_t n = (size_t)audio.num_samples;
        if (!f || fwrite(audio.samples, sizeof(float), n, f) != n || fclose(f)) {
            fprintf(stderr, "cannot write %s\n", audio_path);
            return 1;
        }
    }
    printf("{\"build\": \"%s\", \"vae\": \"%s\", \"patches\": %d, \"tokens\": %d, \"token_seed\": %llu, \"latent_floats\": %d, "
           "\"samples\": %d, \"sample_rate\": %d, \"audio_s\": %.6f, \"generate_s\": %.4f, \"rtf\": %.5f, "
           "\"create_s\": %.3f, \"upload_s\": %.3f, \"audio_abs_mean\": %.9g, \"ralm_max_seq\": %d, ",
#ifdef VOXCPM_CUDA
           "gpu",
#else
           "cpu",
#endif
#ifdef VOXQ_ENGINE_LIBVOXQ
           g_vae_whole ? "device" : g_vae_gpu ? "convs" : "cpu",
#else
           "cpu",
#endif
           patches, g_tokens, (unsigned long long)g_token_seed, g_latent_n, audio.num_samples, audio.sample_rate,
           audio_s, gen_s, audio_s > 0 ? gen_s / audio_s : 0.0, create_s, upload_s,
           audio.num_samples ? asum / audio.num_samples : 0.0, g_ralm_max_seq);
    print_stages();
    printf("}\n");
    voxcpm_audio_free(&audio);
    voxcpm_free(model);
    free(g_latents);
    if (g_mm_log) fclose(g_mm_log);
    return 0;
}
