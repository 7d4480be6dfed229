/*
 * vxcp_load_check.c -- runs voxq_vxcp_load.c's weight_index_build /
 * weight_load_tensor on a VXCP file and prints one JSON line per tensor, so
 * the loader can be checked on the host against values computed elsewhere.
 *
 *   vxcp_load_check FILE
 *     {"name": ..., "dtype": d, "shape": [...], "offset": o, "bytes": b,
 *      "fp16": 0|1, "fnv": FNV-1a 64 of the loaded host data (fp32, or fp16
 *      when kept as fp16), "attached": qtype or 0, "blocks_fnv": FNV-1a 64 of
 *      the blocks handed to voxq_tensor_attach_blocks}
 *   then {"tensors": n, "status": 0}; a failed load prints its error code.
 *
 * voxq_tensor_attach_blocks / voxq_tensor_detach_blocks are this program's
 * own recorders here (no device library is linked).
 */
#include <fcntl.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "model.h"
#include "tensor.h"

static const Tensor* g_att_t;
static int g_att_q;
static uint64_t g_att_fnv;

static uint64_t fnv(const void* p, size_t n) {
    const uint8_t* b = (const uint8_t*)p;
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < n; i++) h = (h ^ b[i]) * 1099511628211ull;
    return h;
}

VoxCPMError voxq_tensor_attach_blocks(const Tensor* t, int qtype, void* blocks, size_t nbytes) {
    g_att_t = t;
    g_att_q = qtype;
    g_att_fnv = fnv(blocks, nbytes);
    free(blocks);
    return VOXCPM_SUCCESS;
}

int voxq_tensor_detach_blocks(const Tensor* t) { return t == g_att_t; }

void __real_tensor_free(Tensor* t) { tensor_free(t); }

int main(int argc, char** argv) {
    if (argc != 2) {
        fprintf(stderr, "usage: %s FILE\n", argv[0]);
        return 2;
    }
    const int fd = open(argv[1], O_RDONLY);
    struct stat sb;
    if (fd < 0 || fstat(fd, &sb) != 0) {
        perror(argv[1]);
        return 1;
    }
    const uint8_t* data = (const uint8_t*)mmap(NULL, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (data == MAP_FAILED) return 1;
    WeightIndex* idx = weight_index_build(data, (size_t)sb.st_size);
    if (!idx) {
        printf("{\"tensors\": 0, \"status\": %d}\n", (int)VOXCPM_ERR_INVALID_MODEL);
        return 0;
    }
    int status = 0;
    for (int i = 0; i < idx->count; i++) {
        const WeightEntry* e = &idx->entries[i];
        Tensor* t = NULL;
        g_att_t = NULL;
        g_att_q = 0;
        const VoxCPMError r = weight_load_tensor(data, e, &t);
        printf("{\"name\": \"%s\", \"dtype\": %u, \"shape\": [", e->name, e->dtype);
        for (uint32_t d = 0; d < e->ndim; d++) printf("%s%u", d ? ", " : "", e->shape[d]);
        printf("], \"offset\": %llu, \"bytes\": %llu, \"load\": %d", (unsigned long long)e->data_offset,
               (unsigned long long)e->data_size, (int)r);
        if (r == VOXCPM_SUCCESS) {
            const int f16 = t->is_fp16 ? 1 : 0;
            const uint64_t h = f16 ? fnv(t->data_fp16, t->size * 2) : fnv(t->data, t->size * 4);
            printf(", \"fp16\": %d, \"fnv\": \"%016llx\", \"attached\": %d, \"blocks_fnv\": \"%016llx\"", f16,
                   (unsigned long long)h, g_att_t == t ? g_att_q : 0,
                   (unsigned long long)(g_att_t == t ? g_att_fnv : 0));
            tensor_free(t);
        } else {
            status = (int)r;
        }
        printf("}\n");
    }
    printf("{\"tensors\": %d, \"status\": %d}\n", idx->count, status);
    weight_index_free(idx);
    return 0;
}
