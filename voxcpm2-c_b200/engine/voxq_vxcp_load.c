/*
 * voxq_vxcp_load.c -- the engine's VXCP weight loader with the quantized
 * dtypes: weight_index_build and weight_load_tensor (include/model.h:516-532)
 * as the engine declares them, reading every dtype the engine reads plus
 * voxq's Q4_1 (4) and Q8 (5) blocks (layouts in include/voxq.h).
 *
 * The engine's own loader (src/model.c:1628-1877) sizes Q4_0 / Q4_1 as 0
 * bytes, which shifts every later tensor's offset, and rejects them on load.
 * Linked in place of those two functions (the harness build weakens the
 * engine's definitions in its model.o, so every caller -- model.c itself,
 * audio_vae.c -- reaches these), the unchanged engine starts from a file
 * written by voxq_vxcp_quantize:
 *   - index: data offsets from the sizes of each dtype (fp32 4, bf16 / fp16 2
 *     bytes per value; Q4_0 18, Q4_1 20, Q8 40 bytes per 32-value block),
 *     from the byte after the string table's last NUL, entries sorted by name
 *     for weight_index_find's binary search (src/model.c:1733, 1773-1786);
 *     header CRC32C checked and a mismatch only reported, as the engine does;
 *     bounds checked against the mapping and shapes against the file size
 *     (the engine does neither), and a load never reads past its entry;
 *   - fp32 / fp16 / bf16 tensors load exactly as the engine loads them
 *     (src/model.c:1811-1858: fp16 kept as fp16 except 1-D, bf16 widened,
 *     NaN set to 0 in fp32 data);
 *   - Q4_1 / Q8 tensors become fp32 host data, value = q * d + m computed in
 *     fp32 (quantize.py's dequantize_q4_block / dequantize_q8_block with
 *     unsigned Q8 codes, scripts/quantize.py:56-82), so any host-side reader
 *     sees the quantized weights; in the libvoxq build a 2-D one with rows a
 *     multiple of 32 also gets its blocks attached (voxq_tensor_attach_blocks,
 *     quantize.py field order), and tensor_to_cuda then puts exactly those
 *     blocks on the device instead of quantizing again;
 *   - Q4_0 (no dequantization defined) and unknown dtypes: VOXCPM_ERR_UNSUPPORTED.
 * Build with -ffp-contract=off so q * d + m rounds twice, as numpy does.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "model.h"
#include "tensor.h"

#ifdef VOXQ_LOADER_ATTACH
VoxCPMError voxq_tensor_attach_blocks(const Tensor* t, int qtype, void* blocks, size_t nbytes);
int voxq_tensor_detach_blocks(const Tensor* t);
#define VOXQ_ATTACH_Q4 2 /* VOXQ_Q4 */
#define VOXQ_ATTACH_Q8 3 /* VOXQ_Q8 */

/* Linked with --wrap=tensor_free: a weight freed without ever being uploaded
 * (one the engine keeps on the host) releases its attached blocks too. */
void __real_tensor_free(Tensor* t);
void __wrap_tensor_free(Tensor* t) {
    if (t) voxq_tensor_detach_blocks(t);
    __real_tensor_free(t);
}
#endif

enum { QL_FP32 = 0, QL_BF16 = 1, QL_FP16 = 2, QL_Q4_0 = 3, QL_Q4_1 = 4, QL_Q8 = 5 };

static uint32_t ql_rd32(const uint8_t* p) {
    uint32_t v;
    memcpy(&v, p, 4);
    return v;
}

static uint32_t ql_crc32c(const uint8_t* p, size_t n) {
    static uint32_t tab[256];
    static int ready = 0;
    if (!ready) {
        for (uint32_t i = 0; i < 256; i++) {
            uint32_t c = i;
            for (int k = 0; k < 8; k++) c = (c & 1) ? (c >> 1) ^ 0x82F63B78u : c >> 1;
            tab[i] = c;
        }
        ready = 1;
    }
    uint32_t c = 0xFFFFFFFFu;
    while (n--) c = (c >> 8) ^ tab[(c ^ *p++) & 0xFF];
    return ~c;
}

/* Bytes of n values of a dtype; 0 and *ok = 0 for an unknown one. */
static uint64_t ql_bytes(uint32_t dtype, uint64_t n, int* ok) {
    const uint64_t blocks = (n + 31) / 32;
    *ok = 1;
    switch (dtype) {
        case QL_FP32: return 4 * n;
        case QL_BF16:
        case QL_FP16: return 2 * n;
        case QL_Q4_0: return 18 * blocks;
        case QL_Q4_1: return 20 * blocks;
        case QL_Q8: return 40 * blocks;
        default: *ok = 0; return 0;
    }
}

static int ql_name_cmp(const void* a, const void* b) {
    return strcmp(((const WeightEntry*)a)->name, ((const WeightEntry*)b)->name);
}

static void ql_index_free(WeightIndex* idx) {
    if (!idx) return;
    for (int i = 0; i < idx->count; i++) free(idx->entries[i].name);
    free(idx->entries);
    free(idx);
}

/* The mapping's size, for weight_load_tensor's bounds (the engine's
 * signature carries none): recorded per mapping by weight_index_build. */
#define QL_MAPS 8
static struct { const uint8_t* base; size_t size; } ql_maps[QL_MAPS];

static size_t ql_map_size(const uint8_t* base) {
    for (int i = 0; i < QL_MAPS; i++)
        if (ql_maps[i].base == base) return ql_maps[i].size;
    return 0;
}

WeightIndex* weight_index_build(const uint8_t* data, size_t data_size) {
    if (!data || data_size < VXCPM_HEADER_SIZE) return NULL;
    if (ql_rd32(data) != VXCPM_MAGIC) {
        fprintf(stderr, "[voxq loader] not a VXCP file (magic 0x%08X)\n", ql_rd32(data));
        return NULL;
    }
    if (ql_rd32(data + 4) != VXCPM_VERSION) {
        fprintf(stderr, "[voxq loader] unsupported VXCP version %u\n", ql_rd32(data + 4));
        return NULL;
    }
    uint8_t hdr[VXCPM_HEADER_SIZE];
    memcpy(hdr, data, VXCPM_HEADER_SIZE);
    memset(hdr + 56, 0, 8);
    if (ql_crc32c(hdr, VXCPM_HEADER_SIZE) != ql_rd32(data + 56))
        fprintf(stderr, "[voxq loader] header CRC mismatch (non-fatal)\n");
    const uint32_t nt = ql_rd32(data + 8);
    const size_t st_off = VXCPM_HEADER_SIZE + (size_t)nt * VXCPM_META_ENTRY_SIZE;
    if (nt == 0 || st_off > data_size) return NULL;
    size_t name_end = 0;
    for (uint32_t i = 0; i < nt; i++) {
        const uint8_t* m = data + VXCPM_HEADER_SIZE + (size_t)i * VXCPM_META_ENTRY_SIZE;
        const size_t e = (size_t)ql_rd32(m) + ql_rd32(m + 4);
        if (e > name_end) name_end = e;
    }
    if (st_off + name_end + 1 > data_size) return NULL;

    WeightIndex* idx = (WeightIndex*)calloc(1, sizeof(WeightIndex));
    if (!idx) return NULL;
    idx->entries = (WeightEntry*)calloc(nt, sizeof(WeightEntry));
    idx->capacity = (int)nt;
    if (!idx->entries) {
        free(idx);
        return NULL;
    }
    uint64_t pos = st_off + name_end + 1;
    for (uint32_t i = 0; i < nt; i++) {
        const uint8_t* m = data + VXCPM_HEADER_SIZE + (size_t)i * VXCPM_META_ENTRY_SIZE;
        WeightEntry* e = &idx->entries[idx->count];
        const uint32_t len = ql_rd32(m + 4);
        e->name = (char*)malloc((size_t)len + 1);
        if (!e->name) goto fail;
        memcpy(e->name, data + st_off + ql_rd32(m), len);
        e->name[len] = '\0';
        idx->count++;
        e->dtype = ql_rd32(m + 8);
        e->ndim = ql_rd32(m + 12);
        /* no tensor inside the file holds more values than twice its bytes (the
         * smallest encoding, Q4_0, takes 18 bytes per 32 values): a shape past
         * that is corrupt, and checking before each product keeps n from wrapping */
        const uint64_t cap = 2 * (uint64_t)data_size;
        uint64_t n = 1;
        for (int d = 0; d < 4; d++) {
            e->shape[d] = ql_rd32(m + 16 + 4 * d);
            if (d < (int)e->ndim) {
                const uint64_t s = e->shape[d];
                if (s && n > cap / s) {
                    fprintf(stderr, "[voxq loader] tensor '%s' has an impossible shape\n", e->name);
                    goto fail;
                }
                n *= s;
            }
        }
        int ok;
        /* an unknown dtype is sized as fp32, as the engine does */
        uint64_t b = ql_bytes(e->dtype, n, &ok);
        if (!ok) b = 4 * n;
        e->data_offset = pos;
        e->data_size = b;
        pos += b;
        if (pos > data_size) {
            fprintf(stderr, "[voxq loader] tensor '%s' ends past the file (%llu > %zu)\n", e->name,
                    (unsigned long long)pos, data_size);
            goto fail;
        }
    }
    qsort(idx->entries, (size_t)idx->count, sizeof(WeightEntry), ql_name_cmp);
    for (int i = 0; i < QL_MAPS; i++)
        if (ql_maps[i].base == NULL || ql_maps[i].base == data) {
            ql_maps[i].base = data;
            ql_maps[i].size = data_size;
            break;
        }
    return idx;
fail:
    ql_index_free(idx);
    return NULL;
}

/* One 32-value block of Q4_1 / Q8 (VXCP order) -> fp32, numpy's arithmetic. */
static void ql_dequant_block(const uint8_t* b, uint32_t dtype, float* out, int count) {
    if (dtype == QL_Q4_1) {
        uint16_t hd, hm;
        memcpy(&hd, b, 2);
        memcpy(&hm, b + 2, 2);
        const float d = fp16_to_fp32(hd), mn = fp16_to_fp32(hm);
        for (int j = 0; j < count; j++) {
            const uint8_t byte = b[4 + j / 2];
            const float q = (float)((j & 1) ? (byte & 0xF) : (byte >> 4));
            out[j] = q * d + mn;
        }
    } else {
        float d, mn;
        memcpy(&d, b, 4);
        memcpy(&mn, b + 4, 4);
        for (int j = 0; j < count; j++) out[j] = (float)b[8 + j] * d + mn;
    }
}

VoxCPMError weight_load_tensor(const uint8_t* data, const WeightEntry* entry, Tensor** out_tensor) {
    if (!data || !entry || !out_tensor) return VOXCPM_ERR_INTERNAL;
    int ndim = (int)entry->ndim;
    if (ndim < 1 || ndim > 4) ndim = 1;
    int shape[4];
    int64_t n = 1;
    for (int i = 0; i < ndim; i++) {
        shape[i] = (int)entry->shape[i];
        if (shape[i] < 0) return VOXCPM_ERR_INVALID_MODEL;
        n *= shape[i];
    }
    const size_t map = ql_map_size(data);
    if (map && entry->data_offset + entry->data_size > map) return VOXCPM_ERR_INVALID_MODEL;
    /* the values this load reads must lie inside the entry (an ndim outside
     * 1..4 is read as one dimension, as the engine reads it, while the index
     * sized it from the stored ndim) */
    int ok_dtype;
    if (n < 0 || ql_bytes(entry->dtype, (uint64_t)n, &ok_dtype) > entry->data_size) return VOXCPM_ERR_INVALID_MODEL;
    const uint8_t* src = data + entry->data_offset;
    if (entry->dtype != QL_FP32 && entry->dtype != QL_BF16 && entry->dtype != QL_FP16 &&
        entry->dtype != QL_Q4_1 && entry->dtype != QL_Q8)
        return VOXCPM_ERR_UNSUPPORTED;
    Tensor* t = tensor_create(ndim, shape);
    if (!t) return VOXCPM_ERR_OOM;
    switch (entry->dtype) {
        case QL_FP32:
            memcpy(t->data, src, (size_t)n * sizeof(float));
            break;
        case QL_FP16:
            if (ndim == 1) {
                for (int64_t i = 0; i < n; i++) {
                    uint16_t h;
                    memcpy(&h, src + 2 * i, 2);
                    t->data[i] = fp16_to_fp32(h);
                }
            } else {
                free(t->data);
                t->data = NULL;
                t->data_fp16 = (uint16_t*)malloc((size_t)n * 2);
                if (!t->data_fp16) {
                    tensor_free(t);
                    return VOXCPM_ERR_OOM;
                }
                memcpy(t->data_fp16, src, (size_t)n * 2);
                t->is_fp16 = true;
            }
            break;
        case QL_BF16:
            for (int64_t i = 0; i < n; i++) {
                uint16_t h;
                memcpy(&h, src + 2 * i, 2);
                const uint32_t u = (uint32_t)h << 16;
                memcpy(&t->data[i], &u, 4);
            }
            break;
        default: {  /* Q4_1, Q8 */
            const size_t bb = entry->dtype == QL_Q4_1 ? 20 : 40;
            for (int64_t i = 0; i < n; i += 32) {
                const int cnt = n - i < 32 ? (int)(n - i) : 32;
                ql_dequant_block(src + (size_t)(i / 32) * bb, entry->dtype, t->data + i, cnt);
            }
#ifdef VOXQ_LOADER_ATTACH
            if (ndim == 2 && shape[1] % 32 == 0) {
                /* quantize.py field order: codes, then the two scalars */
                const size_t blocks = (size_t)(n / 32), hb = bb == 20 ? 4 : 8, cb = bb - hb;
                uint8_t* q = (uint8_t*)malloc(blocks * bb);
                if (!q) {
                    tensor_free(t);
                    return VOXCPM_ERR_OOM;
                }
                for (size_t k = 0; k < blocks; k++) {
                    memcpy(q + k * bb, src + k * bb + hb, cb);
                    memcpy(q + k * bb + cb, src + k * bb, hb);
                }
                if (voxq_tensor_attach_blocks(t, bb == 20 ? VOXQ_ATTACH_Q4 : VOXQ_ATTACH_Q8, q, blocks * bb) !=
                    VOXCPM_SUCCESS)
                    free(q);
            }
#endif
            break;
        }
    }
    if (!t->is_fp16) {
        int64_t nan = 0;
        for (int64_t i = 0; i < n; i++)
            if (isnan(t->data[i])) {
                t->data[i] = 0.0f;
                nan++;
            }
        if (nan) fprintf(stderr, "[voxq loader] '%s': %lld NaN set to 0\n", entry->name, (long long)nan);
    }
    *out_tensor = t;
    return VOXCPM_SUCCESS;
}
