/*
 * make_model.c -- writes a random-init VoxCPM2 model in the engine's VXCP
 * format (the main file and its "_audiovae" companion), so the unchanged
 * reference engine can load and run it where no real checkpoint exists.
 *
 *   make_model OUT_PREFIX [--seed S] [--threads T]
 *     -> OUT_PREFIX.vxcpm, OUT_PREFIX_audiovae.vxcpm
 *   prints one JSON line: file sizes, tensor counts and the CRC32C of each
 *   file's metadata + data (the header's data_checksum), which pins that two
 *   machines wrote the same bytes.
 *
 * Format (the reader is weight_index_build / weight_load_tensor,
 * src/model.c:1622-1877; layout documented in docs/WEIGHT_FORMAT.md):
 *   64-byte header: magic "VXCP", version 1, num_tensors, reserved zeros,
 *     CRC32C of bytes 0-55 at 56 (computed with bytes 56-63 zero), CRC32C of
 *     metadata + string table + data at 60;
 *   num_tensors 32-byte entries: name_offset, name_length, dtype, ndim,
 *     shape[4] (unused dims 1);
 *   the string table (NUL-terminated names, no padding);
 *   tensor data in entry order, back to back, starting right after the last
 *     NUL (the reader derives every offset from the sizes; no alignment).
 * Tensor names and shapes are the ones the engine's loaders ask for
 * (src/model.c:1129-1560, src/audio_vae.c:579-860) at the architecture of
 * voxcpm_config_default (src/model.c:1129-1166), which the engine hard-codes.
 *
 * Values (seeded, deterministic on any x86-64 with the same libm):
 *   - every 2-D weight the engine multiplies through tensor_matmul_nt is
 *     "Q8-exact": each 32-element block holds w = (q - 128) * 2^-11 with
 *     q = clip(rint(128 + 41 z), 0, 255), z ~ N(0,1) (std ~0.02), and one
 *     element at q = 0 and one at q = 255.  The block's min/max are then
 *     -128 * 2^-11 and 127 * 2^-11, quantize.py's Q8 scale is exactly 2^-11
 *     and its codes are exactly q, so quantize -> dequantize returns the same
 *     floats: a GPU run that quantizes these weights on upload and a CPU run
 *     on the stored floats multiply by identical weights.  The values are
 *     exact in fp16, which is how they are stored (dtype 2);
 *   - the token embedding: 0.02 z in fp16 (read on the host by the engine);
 *   - 1-D norm weights 1.0, biases and the LocEnc special token 0.02 z, fp32;
 *   - AudioVAE (fp32; its convolutions read the floats directly): weight_v
 *     0.02 z, weight_g 1.0 (unit-norm filters), biases 0, snake alphas 1.0.
 * z comes from a splitmix64 stream per tensor (seeded by the tensor's index)
 * through the Box-Muller transform.
 */
#define _POSIX_C_SOURCE 200809L
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

enum { DT_F32 = 0, DT_F16 = 2 };
enum { V_Q8EXACT, V_NORMAL, V_ONES, V_ZEROS };

typedef struct {
    char name[128];
    int ndim;
    uint32_t shape[4];
    int dtype;
    int values;
    float scale;  /* V_NORMAL: standard deviation */
} TensorSpec;

typedef struct {
    TensorSpec* t;
    int n, cap;
} SpecList;

static void add(SpecList* L, const char* name, int ndim, const uint32_t* shape, int dtype, int values, float scale) {
    if (L->n == L->cap) {
        L->cap = L->cap ? 2 * L->cap : 256;
        L->t = (TensorSpec*)realloc(L->t, (size_t)L->cap * sizeof(TensorSpec));
        if (!L->t) { perror("realloc"); exit(1); }
    }
    TensorSpec* s = &L->t[L->n++];
    memset(s, 0, sizeof(*s));
    snprintf(s->name, sizeof(s->name), "%s", name);
    s->ndim = ndim;
    for (int i = 0; i < 4; i++) s->shape[i] = i < ndim ? shape[i] : 1;
    s->dtype = dtype;
    s->values = values;
    s->scale = scale;
}

static void w2(SpecList* L, const char* name, uint32_t n, uint32_t k) {
    uint32_t sh[2] = {n, k};
    add(L, name, 2, sh, DT_F16, V_Q8EXACT, 0.f);
}
static void vec(SpecList* L, const char* name, uint32_t n, int values) {
    uint32_t sh[1] = {n};
    add(L, name, 1, sh, DT_F32, values, 0.02f);
}

/* One MiniCPM transformer layer (model.c transformer_block_from_weights /
 * enc_block_from_weights): hidden D, 16 query heads and 2 KV heads of 128, FFN F. */
static void layer(SpecList* L, const char* prefix, uint32_t D, uint32_t F) {
    char k[160];
    const uint32_t Q = 16 * 128, KV = 2 * 128;
    snprintf(k, sizeof k, "%s.input_layernorm.weight", prefix); vec(L, k, D, V_ONES);
    snprintf(k, sizeof k, "%s.self_attn.q_proj.weight", prefix); w2(L, k, Q, D);
    snprintf(k, sizeof k, "%s.self_attn.k_proj.weight", prefix); w2(L, k, KV, D);
    snprintf(k, sizeof k, "%s.self_attn.v_proj.weight", prefix); w2(L, k, KV, D);
    snprintf(k, sizeof k, "%s.self_attn.o_proj.weight", prefix); w2(L, k, D, Q);
    snprintf(k, sizeof k, "%s.mlp.gate_proj.weight", prefix); w2(L, k, F, D);
    snprintf(k, sizeof k, "%s.mlp.up_proj.weight", prefix); w2(L, k, F, D);
    snprintf(k, sizeof k, "%s.mlp.down_proj.weight", prefix); w2(L, k, D, F);
    snprintf(k, sizeof k, "%s.post_attention_layernorm.weight", prefix); vec(L, k, D, V_ONES);
}

static void main_model(SpecList* L) {
    const uint32_t D = 2048, FF = 6144, DH = 1024, FH = 4096, LAT = 64, VOCAB = 73448;
    char k[160];
    uint32_t emb[2] = {VOCAB, D};
    add(L, "base_lm.embed_tokens.weight", 2, emb, DT_F16, V_NORMAL, 0.02f);
    vec(L, "base_lm.norm.weight", D, V_ONES);
    for (int i = 0; i < 28; i++) { snprintf(k, sizeof k, "base_lm.layers.%d", i); layer(L, k, D, FF); }
    vec(L, "residual_lm.norm.weight", D, V_ONES);
    for (int i = 0; i < 8; i++) { snprintf(k, sizeof k, "residual_lm.layers.%d", i); layer(L, k, D, FF); }
    w2(L, "enc_to_lm_proj.weight", D, DH);      vec(L, "enc_to_lm_proj.bias", D, V_NORMAL);
    w2(L, "lm_to_dit_proj.weight", DH, D);      vec(L, "lm_to_dit_proj.bias", DH, V_NORMAL);
    w2(L, "res_to_dit_proj.weight", DH, D);     vec(L, "res_to_dit_proj.bias", DH, V_NORMAL);
    w2(L, "fusion_concat_proj.weight", D, 2 * D); vec(L, "fusion_concat_proj.bias", D, V_NORMAL);
    w2(L, "fsq_layer.in_proj.weight", LAT, D);  vec(L, "fsq_layer.in_proj.bias", LAT, V_NORMAL);
    w2(L, "fsq_layer.out_proj.weight", D, LAT); vec(L, "fsq_layer.out_proj.bias", D, V_NORMAL);
    w2(L, "stop_proj.weight", D, D);            vec(L, "stop_proj.bias", D, V_NORMAL);
    w2(L, "stop_head.weight", 2, D);
    uint32_t st[4] = {1, 1, 1, DH};
    add(L, "feat_encoder.special_token", 4, st, DT_F32, V_NORMAL, 0.02f);
    w2(L, "feat_encoder.in_proj.weight", DH, LAT); vec(L, "feat_encoder.in_proj.bias", DH, V_NORMAL);
    vec(L, "feat_encoder.encoder.norm.weight", DH, V_ONES);
    for (int i = 0; i < 12; i++) { snprintf(k, sizeof k, "feat_encoder.encoder.layers.%d", i); layer(L, k, DH, FH); }
    const char* e = "feat_decoder.estimator";
    snprintf(k, sizeof k, "%s.in_proj.weight", e); w2(L, k, DH, LAT);
    snprintf(k, sizeof k, "%s.in_proj.bias", e); vec(L, k, DH, V_NORMAL);
    snprintf(k, sizeof k, "%s.cond_proj.weight", e); w2(L, k, DH, LAT);
    snprintf(k, sizeof k, "%s.cond_proj.bias", e); vec(L, k, DH, V_NORMAL);
    snprintf(k, sizeof k, "%s.out_proj.weight", e); w2(L, k, LAT, DH);
    snprintf(k, sizeof k, "%s.out_proj.bias", e); vec(L, k, LAT, V_NORMAL);
    const char* mlps[2] = {"time_mlp", "delta_time_mlp"};
    for (int m = 0; m < 2; m++)
        for (int j = 1; j <= 2; j++) {
            snprintf(k, sizeof k, "%s.%s.linear_%d.weight", e, mlps[m], j); w2(L, k, DH, DH);
            snprintf(k, sizeof k, "%s.%s.linear_%d.bias", e, mlps[m], j); vec(L, k, DH, V_NORMAL);
        }
    snprintf(k, sizeof k, "%s.decoder.norm.weight", e); vec(L, k, DH, V_ONES);
    for (int i = 0; i < 12; i++) { snprintf(k, sizeof k, "%s.decoder.layers.%d", e, i); layer(L, k, DH, FH); }
}

/* Weight-normalised conv (audio_vae.c wnconv_create_and_load): weight_v with
 * the given shape, weight_g over `gdim` channels, bias over `bdim`. */
static void wnconv(SpecList* L, const char* prefix, uint32_t a, uint32_t b, uint32_t kk, uint32_t gdim, uint32_t bdim) {
    char k[192];
    uint32_t v[3] = {a, b, kk}, g[3] = {gdim, 1, 1};
    snprintf(k, sizeof k, "%s.weight_v", prefix); add(L, k, 3, v, DT_F32, V_NORMAL, 0.02f);
    snprintf(k, sizeof k, "%s.weight_g", prefix); add(L, k, 3, g, DT_F32, V_ONES, 0.f);
    snprintf(k, sizeof k, "%s.bias", prefix); vec(L, k, bdim, V_ZEROS);
}
static void alpha(SpecList* L, const char* name, uint32_t c) {
    uint32_t sh[3] = {1, c, 1};
    add(L, name, 3, sh, DT_F32, V_ONES, 0.f);
}

/* AudioVAE V2: decoder 64 -> 2048 -> ... -> 32 -> 1 (strides 8, 6, 5, 2, 2, 2,
 * audio_vae.c:43-44), encoder 1 -> 128 -> ... -> 2048 -> 64 (rates 2, 5, 8, 8).
 * Transposed-conv kernels are 2 * stride (the strides and paddings are the
 * engine's; the kernel size is a choice, recorded here). */
static void audio_vae(SpecList* L) {
    static const uint32_t dstride[6] = {8, 6, 5, 2, 2, 2}, erate[4] = {2, 5, 8, 8};
    char k[192];
    wnconv(L, "audio_vae.decoder.conv_in", 64, 1, 7, 64, 64);
    wnconv(L, "audio_vae.decoder.proj_up", 2048, 64, 1, 2048, 2048);
    for (int i = 0; i < 6; i++) {
        const uint32_t ci = 2048u >> i, co = ci / 2;
        snprintf(k, sizeof k, "audio_vae.decoder.decoder_blocks.%d.snake_alpha", i); alpha(L, k, ci);
        snprintf(k, sizeof k, "audio_vae.decoder.decoder_blocks.%d.convtr", i);
        wnconv(L, k, ci, co, 2 * dstride[i], ci, co);
        for (int j = 0; j < 3; j++) {
            snprintf(k, sizeof k, "audio_vae.decoder.decoder_blocks.%d.res_blocks.%d.snake_alpha1", i, j); alpha(L, k, co);
            snprintf(k, sizeof k, "audio_vae.decoder.decoder_blocks.%d.res_blocks.%d.conv_depthwise", i, j);
            wnconv(L, k, co, 1, 7, co, co);
            snprintf(k, sizeof k, "audio_vae.decoder.decoder_blocks.%d.res_blocks.%d.snake_alpha2", i, j); alpha(L, k, co);
            snprintf(k, sizeof k, "audio_vae.decoder.decoder_blocks.%d.res_blocks.%d.conv_pointwise", i, j);
            wnconv(L, k, co, co, 1, co, co);
        }
    }
    alpha(L, "audio_vae.decoder.final_snake_alpha", 32);
    wnconv(L, "audio_vae.decoder.conv_out", 1, 32, 7, 1, 1);
    wnconv(L, "audio_vae.encoder.block.0", 128, 1, 7, 128, 128);
    for (int i = 0; i < 4; i++) {
        const uint32_t ci = 128u << i, co = 2 * ci;
        for (int j = 0; j < 3; j++) {
            snprintf(k, sizeof k, "audio_vae.encoder.block.%d.block.%d.block.0.alpha", i + 1, j); alpha(L, k, ci);
            snprintf(k, sizeof k, "audio_vae.encoder.block.%d.block.%d.block.1", i + 1, j); wnconv(L, k, ci, 1, 7, ci, ci);
            snprintf(k, sizeof k, "audio_vae.encoder.block.%d.block.%d.block.2.alpha", i + 1, j); alpha(L, k, ci);
            snprintf(k, sizeof k, "audio_vae.encoder.block.%d.block.%d.block.3", i + 1, j); wnconv(L, k, ci, ci, 1, ci, ci);
        }
        snprintf(k, sizeof k, "audio_vae.encoder.block.%d.block.3.alpha", i + 1); alpha(L, k, ci);
        snprintf(k, sizeof k, "audio_vae.encoder.block.%d.block.4", i + 1); wnconv(L, k, co, ci, 2 * erate[i], co, co);
    }
    wnconv(L, "audio_vae.encoder.fc_mu", 64, 2048, 3, 64, 64);
    wnconv(L, "audio_vae.encoder.fc_logvar", 64, 2048, 3, 64, 64);
}

/* ---- CRC32C (Castagnoli, reflected polynomial 0x82F63B78), slice-by-8 ---- */
static uint32_t crc_tab[8][256];
static void crc_init(void) {
    for (uint32_t i = 0; i < 256; i++) {
        uint32_t c = i;
        for (int j = 0; j < 8; j++) c = (c >> 1) ^ (0x82F63B78u & (0u - (c & 1u)));
        crc_tab[0][i] = c;
    }
    for (uint32_t i = 0; i < 256; i++)
        for (int t = 1; t < 8; t++) crc_tab[t][i] = (crc_tab[t - 1][i] >> 8) ^ crc_tab[0][crc_tab[t - 1][i] & 0xFF];
}
/* running CRC: state is the inverted register (start 0xFFFFFFFF, finish ~) */
static uint32_t crc_update(uint32_t c, const uint8_t* p, size_t n) {
    while (n && ((uintptr_t)p & 7)) { c = (c >> 8) ^ crc_tab[0][(c ^ *p++) & 0xFF]; n--; }
    while (n >= 8) {
        uint64_t v;
        memcpy(&v, p, 8);
        v ^= c;
        c = crc_tab[7][v & 0xFF] ^ crc_tab[6][(v >> 8) & 0xFF] ^ crc_tab[5][(v >> 16) & 0xFF] ^
            crc_tab[4][(v >> 24) & 0xFF] ^ crc_tab[3][(v >> 32) & 0xFF] ^ crc_tab[2][(v >> 40) & 0xFF] ^
            crc_tab[1][(v >> 48) & 0xFF] ^ crc_tab[0][v >> 56];
        p += 8;
        n -= 8;
    }
    while (n--) c = (c >> 8) ^ crc_tab[0][(c ^ *p++) & 0xFF];
    return c;
}

/* ---- values ---- */
static uint64_t splitmix(uint64_t* s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
/* Box-Muller pair from two 53-bit uniforms in (0, 1]. */
static void normal2(uint64_t* s, double* a, double* b) {
    const double u1 = ((splitmix(s) >> 11) + 1) * 0x1.0p-53, u2 = (splitmix(s) >> 11) * 0x1.0p-53;
    const double r = sqrt(-2.0 * log(u1)), th = 6.283185307179586 * u2;
    *a = r * cos(th);
    *b = r * sin(th);
}

/* float -> binary16, round to nearest even (finite inputs far from overflow). */
static uint16_t f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xFF) - 127 + 15;
    uint32_t m = x & 0x7FFFFFu;
    if (((x >> 23) & 0xFF) == 0) return (uint16_t)sign;  /* f32 subnormals and zero -> signed zero */
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {  /* half subnormal */
        if (e < -10) return (uint16_t)sign;
        m |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (h & 1))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t h = ((uint32_t)e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1))) h++;
    return (uint16_t)(sign | h);
}

static size_t elems(const TensorSpec* t) {
    size_t n = 1;
    for (int i = 0; i < t->ndim; i++) n *= t->shape[i];
    return n;
}
static size_t nbytes(const TensorSpec* t) { return elems(t) * (t->dtype == DT_F16 ? 2 : 4); }

/* Fills tensor i's bytes. */
static void fill(const TensorSpec* t, int index, uint64_t seed, uint8_t* dst) {
    uint64_t s = seed * 0x9E3779B97F4A7C15ull + (uint64_t)index * 0xD1B54A32D192ED03ull + 1;
    const size_t n = elems(t);
    float* f32 = (float*)dst;
    uint16_t* f16 = (uint16_t*)dst;
    double za, zb;
    if (t->values == V_Q8EXACT) {
        const size_t K = t->shape[1];
        for (size_t base = 0; base < n; base += 32) {
            int q[32];
            for (int j = 0; j < 32; j += 2) {
                normal2(&s, &za, &zb);
                double v0 = rint(128.0 + 41.0 * za), v1 = rint(128.0 + 41.0 * zb);
                q[j] = v0 < 0 ? 0 : v0 > 255 ? 255 : (int)v0;
                q[j + 1] = v1 < 0 ? 0 : v1 > 255 ? 255 : (int)v1;
            }
            const uint64_t r = splitmix(&s);
            const int p0 = (int)(r & 31), p1 = (p0 + 1 + (int)((r >> 8) % 31)) & 31;
            q[p0] = 0;
            q[p1] = 255;
            for (int j = 0; j < 32; j++) {
                const float w = (float)(q[j] - 128) * 0x1.0p-11f;
                if (t->dtype == DT_F16) f16[base + j] = f2h(w); else f32[base + j] = w;
            }
        }
        (void)K;
        return;
    }
    for (size_t i = 0; i < n; i += 2) {
        float v0 = 0.f, v1 = 0.f;
        if (t->values == V_NORMAL) {
            normal2(&s, &za, &zb);
            v0 = (float)(za * t->scale);
            v1 = (float)(zb * t->scale);
        } else if (t->values == V_ONES) {
            v0 = v1 = 1.0f;
        }
        if (t->dtype == DT_F16) {
            f16[i] = f2h(v0);
            if (i + 1 < n) f16[i + 1] = f2h(v1);
        } else {
            f32[i] = v0;
            if (i + 1 < n) f32[i + 1] = v1;
        }
    }
}

typedef struct {
    const SpecList* L;
    uint64_t seed;
    uint8_t** bufs;
    int next;
    pthread_mutex_t mu;
} Pool;

static void* worker(void* arg) {
    Pool* P = (Pool*)arg;
    for (;;) {
        pthread_mutex_lock(&P->mu);
        const int i = P->next++;
        pthread_mutex_unlock(&P->mu);
        if (i >= P->L->n) return NULL;
        fill(&P->L->t[i], i, P->seed, P->bufs[i]);
    }
}

static void put32(uint8_t* p, uint32_t v) { memcpy(p, &v, 4); }

/* Writes one VXCP file; returns 0 and the data checksum, or -1. */
static int write_file(const char* path, const SpecList* L, uint64_t seed, int threads, uint32_t* data_crc,
                      uint64_t* file_bytes) {
    const uint32_t nt = (uint32_t)L->n;
    size_t str_bytes = 0;
    for (int i = 0; i < L->n; i++) str_bytes += strlen(L->t[i].name) + 1;
    const size_t meta_bytes = (size_t)nt * 32;
    uint8_t* meta = (uint8_t*)calloc(1, meta_bytes + str_bytes);
    if (!meta) return -1;
    uint32_t off = 0;
    for (int i = 0; i < L->n; i++) {
        const TensorSpec* t = &L->t[i];
        uint8_t* m = meta + (size_t)i * 32;
        const uint32_t len = (uint32_t)strlen(t->name);
        put32(m + 0, off);
        put32(m + 4, len);
        put32(m + 8, (uint32_t)t->dtype);
        put32(m + 12, (uint32_t)t->ndim);
        for (int d = 0; d < 4; d++) put32(m + 16 + 4 * d, t->shape[d]);
        memcpy(meta + meta_bytes + off, t->name, len + 1);
        off += len + 1;
    }
    /* tensor data, generated in parallel per tensor */
    if (L->n <= 0) { fprintf(stderr, "make_model: empty tensor list\n"); return -1; }
    uint8_t** bufs = (uint8_t**)calloc((size_t)L->n, sizeof(uint8_t*));
    if (!bufs) { fprintf(stderr, "make_model: out of memory\n"); return -1; }
    for (int i = 0; i < L->n; i++) {
        bufs[i] = (uint8_t*)malloc(nbytes(&L->t[i]));
        if (!bufs[i]) { fprintf(stderr, "make_model: out of memory\n"); return -1; }
    }
    Pool P = {L, seed, bufs, 0, PTHREAD_MUTEX_INITIALIZER};
    pthread_t th[64];
    if (threads < 1) threads = 1;
    if (threads > 64) threads = 64;
    for (int i = 0; i < threads; i++) pthread_create(&th[i], NULL, worker, &P);
    for (int i = 0; i < threads; i++) pthread_join(th[i], NULL);

    uint32_t c = 0xFFFFFFFFu;
    c = crc_update(c, meta, meta_bytes + str_bytes);
    for (int i = 0; i < L->n; i++) c = crc_update(c, bufs[i], nbytes(&L->t[i]));
    *data_crc = ~c;

    uint8_t hdr[64] = {0};
    put32(hdr + 0, 0x56435850u);  /* "VXCP" */
    put32(hdr + 4, 1);
    put32(hdr + 8, nt);
    put32(hdr + 56, ~crc_update(0xFFFFFFFFu, hdr, 64));  /* bytes 56..63 still zero */
    put32(hdr + 60, *data_crc);

    FILE* f = fopen(path, "wb");
    if (!f) { perror(path); return -1; }
    size_t total = fwrite(hdr, 1, 64, f) + fwrite(meta, 1, meta_bytes + str_bytes, f);
    for (int i = 0; i < L->n; i++) {
        total += fwrite(bufs[i], 1, nbytes(&L->t[i]), f);
        free(bufs[i]);
    }
    if (fclose(f) != 0) { perror(path); return -1; }
    free(bufs);
    free(meta);
    *file_bytes = total;
    return 0;
}

int main(int argc, char** argv) {
    if (argc < 2) {
        fprintf(stderr, "usage: %s OUT_PREFIX [--seed S] [--threads T]\n", argv[0]);
        return 2;
    }
    const char* prefix = argv[1];
    uint64_t seed = 1;
    int threads = 8;
    for (int i = 2; i + 1 < argc; i += 2) {
        if (!strcmp(argv[i], "--seed")) seed = strtoull(argv[i + 1], NULL, 10);
        else if (!strcmp(argv[i], "--threads")) threads = atoi(argv[i + 1]);
    }
    crc_init();
    SpecList M = {0}, V = {0};
    main_model(&M);
    audio_vae(&V);
    char p1[4096], p2[4096];
    snprintf(p1, sizeof p1, "%s.vxcpm", prefix);
    snprintf(p2, sizeof p2, "%s_audiovae.vxcpm", prefix);
    uint32_t c1 = 0, c2 = 0;
    uint64_t b1 = 0, b2 = 0;
    if (write_file(p1, &M, seed, threads, &c1, &b1) || write_file(p2, &V, seed + 1000003, threads, &c2, &b2)) return 1;
    printf("{\"model\": \"%s\", \"model_bytes\": %llu, \"model_tensors\": %d, \"model_data_crc32c\": %u, "
           "\"audiovae\": \"%s\", \"audiovae_bytes\": %llu, \"audiovae_tensors\": %d, \"audiovae_data_crc32c\": %u, "
           "\"seed\": %llu}\n",
           p1, (unsigned long long)b1, M.n, c1, p2, (unsigned long long)b2, V.n, c2, (unsigned long long)seed);
    return 0;
}
