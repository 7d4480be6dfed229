// voxq_vxcp.cu -- quantizes a model file in the engine's VXCP container on
// the device (voxq_vxcp_quantize).
//
// VXCP (docs/WEIGHT_FORMAT.md; read by src/model.c:1628-1877):
//   64-byte header: u32 magic "VXCP", u32 version 1, u32 num_tensors, ten
//     reserved u32, CRC32C of bytes 0-55 (computed with 56-63 zero) at 56,
//     CRC32C of metadata + string table + data at 60;
//   num_tensors 32-byte entries: u32 name_offset, name_length, dtype, ndim,
//     shape[4];
//   the string table (NUL-terminated names); tensor data in entry order, back
//   to back from the byte after the string table's last NUL (the reader
//   derives every offset from the sizes, src/model.c:1693-1731).
// Sizes per dtype: fp32 4, bf16 / fp16 2 bytes per value; Q4_0 18, Q4_1 20,
// Q8 40 bytes per 32-value block (the block layouts are in include/voxq.h).
//
// The quantized tensors' blocks come from voxq_quantize (bit-exact with
// scripts/quantize.py:42-75) and are rewritten field by field into the VXCP
// block order; nothing else in the file changes except those tensors' dtype
// and the two checksums.
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {
namespace {

constexpr uint32_t kMagic = 0x56435850u;  // "VXCP"
constexpr size_t kHeader = 64, kMeta = 32;

uint32_t rd32(const uint8_t* p) {
    uint32_t v;
    memcpy(&v, p, 4);
    return v;
}
void wr32(uint8_t* p, uint32_t v) { memcpy(p, &v, 4); }

// CRC32C (Castagnoli, reflected polynomial 0x82F63B78), slicing by 8.
struct Crc32c {
    uint32_t tab[8][256];
    Crc32c() {
        for (uint32_t i = 0; i < 256; i++) {
            uint32_t c = i;
            for (int k = 0; k < 8; k++) c = (c & 1) ? (c >> 1) ^ 0x82F63B78u : c >> 1;
            tab[0][i] = c;
        }
        for (uint32_t i = 0; i < 256; i++)
            for (int t = 1; t < 8; t++) tab[t][i] = (tab[t - 1][i] >> 8) ^ tab[0][tab[t - 1][i] & 0xFF];
    }
    uint32_t update(uint32_t c, const uint8_t* p, size_t n) const {
        while (n >= 8) {
            uint64_t v;
            memcpy(&v, p, 8);
            v ^= c;
            c = tab[7][v & 0xFF] ^ tab[6][(v >> 8) & 0xFF] ^ tab[5][(v >> 16) & 0xFF] ^ tab[4][(v >> 24) & 0xFF] ^
                tab[3][(v >> 32) & 0xFF] ^ tab[2][(v >> 40) & 0xFF] ^ tab[1][(v >> 48) & 0xFF] ^ tab[0][v >> 56];
            p += 8;
            n -= 8;
        }
        while (n--) c = (c >> 8) ^ tab[0][(c ^ *p++) & 0xFF];
        return c;
    }
};

const Crc32c& crc() {
    static const Crc32c c;
    return c;
}

// Bytes of n values of a VXCP dtype; false for an unknown dtype.
bool vxcp_bytes(uint32_t dtype, uint64_t n, uint64_t* out) {
    const uint64_t blocks = (n + 31) / 32;
    switch (dtype) {
        case VOXQ_VXCP_FP32: *out = 4 * n; return true;
        case VOXQ_VXCP_BF16:
        case VOXQ_VXCP_FP16: *out = 2 * n; return true;
        case VOXQ_VXCP_Q4_0: *out = 18 * blocks; return true;
        case VOXQ_VXCP_Q4_1: *out = 20 * blocks; return true;
        case VOXQ_VXCP_Q8: *out = 40 * blocks; return true;
        default: return false;
    }
}

__global__ void bf16_widen_kernel(const uint16_t* __restrict__ src, float* __restrict__ dst, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __uint_as_float((uint32_t)src[i] << 16);
}

// quantize.py block stream -> VXCP block order (header fields first).
void to_vxcp_order(const uint8_t* src, uint8_t* dst, size_t blocks, int qtype) {
    if (qtype == VOXQ_Q4) {
        for (size_t b = 0; b < blocks; b++, src += 20, dst += 20) {
            memcpy(dst, src + 16, 4);  // fp16 scale, fp16 min
            memcpy(dst + 4, src, 16);  // codes
        }
    } else {
        for (size_t b = 0; b < blocks; b++, src += 40, dst += 40) {
            memcpy(dst, src + 32, 8);  // fp32 scale, fp32 min
            memcpy(dst + 8, src, 32);  // codes
        }
    }
}

struct Mapped {
    const uint8_t* p = nullptr;
    size_t n = 0;
    int fd = -1;
    ~Mapped() {
        if (p) munmap((void*)p, n);
        if (fd >= 0) close(fd);
    }
};

struct DevBufs {
    void* raw = nullptr;    // the tensor's stored values
    float* f32 = nullptr;   // widened
    uint8_t* blk = nullptr;  // quantize.py blocks
    uint8_t* h_blk = nullptr;  // pinned copy of the blocks
    size_t cap = 0;         // elements
    cudaStream_t st = nullptr;
    ~DevBufs() { release(); if (st) cudaStreamDestroy(st); }
    void release() {
        if (raw) cudaFree(raw);
        if (f32) cudaFree(f32);
        if (blk) cudaFree(blk);
        if (h_blk) cudaFreeHost(h_blk);
        raw = f32 = nullptr;
        blk = h_blk = nullptr;
        cap = 0;
    }
    bool reserve(size_t n) {
        if (n <= cap) return true;
        release();
        const size_t qb = voxq_quant_bytes(n, VOXQ_Q8);  // >= the Q4 stream
        if (cudaMalloc(&raw, n * 4) != cudaSuccess || cudaMalloc((void**)&f32, n * 4) != cudaSuccess ||
            cudaMalloc((void**)&blk, qb) != cudaSuccess || cudaMallocHost((void**)&h_blk, qb) != cudaSuccess) {
            cudaGetLastError();
            release();
            return false;
        }
        cap = n;
        return true;
    }
};

}  // namespace
}  // namespace voxq

using namespace voxq;

extern "C" VoxCPMError voxq_vxcp_quantize(const char* src_path, const char* dst_path, int qtype,
                                          const char* const* keep, int n_keep, voxq_vxcp_stats* stats) {
    if (!src_path || !dst_path || n_keep < 0 || (n_keep > 0 && !keep)) return VOXCPM_ERR_INTERNAL;
    if (qtype != VOXQ_Q4 && qtype != VOXQ_Q8) return VOXCPM_ERR_UNSUPPORTED;
    Mapped in;
    in.fd = open(src_path, O_RDONLY);
    if (in.fd < 0) return VOXCPM_ERR_FILE_NOT_FOUND;
    struct stat sb;
    if (fstat(in.fd, &sb) != 0 || sb.st_size < (off_t)kHeader) return VOXCPM_ERR_INVALID_MODEL;
    in.n = (size_t)sb.st_size;
    void* mp = mmap(nullptr, in.n, PROT_READ, MAP_PRIVATE, in.fd, 0);
    if (mp == MAP_FAILED) return VOXCPM_ERR_INVALID_MODEL;
    in.p = (const uint8_t*)mp;
    const uint8_t* f = in.p;
    if (rd32(f) != kMagic || rd32(f + 4) != 1) return VOXCPM_ERR_INVALID_MODEL;
    const uint32_t nt = rd32(f + 8);
    if (nt == 0 || kHeader + (size_t)nt * kMeta > in.n) return VOXCPM_ERR_INVALID_MODEL;
    const size_t st_off = kHeader + (size_t)nt * kMeta;

    // metadata, names, data offsets (src/model.c:1680-1731's rule)
    std::vector<uint8_t> meta(f + kHeader, f + st_off);
    size_t name_end = 0;
    for (uint32_t i = 0; i < nt; i++) {
        const uint8_t* m = &meta[(size_t)i * kMeta];
        const size_t e = (size_t)rd32(m) + rd32(m + 4);
        if (e > name_end) name_end = e;
    }
    const size_t data_start = st_off + name_end + 1;
    if (data_start > in.n) return VOXCPM_ERR_INVALID_MODEL;
    std::vector<uint64_t> off(nt), bytes(nt), elems(nt);
    uint64_t pos = data_start;
    for (uint32_t i = 0; i < nt; i++) {
        const uint8_t* m = &meta[(size_t)i * kMeta];
        const uint32_t ndim = rd32(m + 12);
        if (rd32(m) + (uint64_t)rd32(m + 4) > name_end || ndim < 1 || ndim > 4) return VOXCPM_ERR_INVALID_MODEL;
        uint64_t n = 1;
        for (uint32_t d = 0; d < ndim; d++) n *= rd32(m + 16 + 4 * d);
        if (!vxcp_bytes(rd32(m + 8), n, &bytes[i])) return VOXCPM_ERR_UNSUPPORTED;
        if (rd32(m + 8) == VOXQ_VXCP_Q4_0) return VOXCPM_ERR_UNSUPPORTED;
        elems[i] = n;
        off[i] = pos;
        pos += bytes[i];
    }
    if (pos > in.n) return VOXCPM_ERR_INVALID_MODEL;

    // which tensors to quantize
    std::vector<char> quant(nt, 0);
    uint32_t n_quant = 0;
    size_t max_elems = 0;
    for (uint32_t i = 0; i < nt; i++) {
        uint8_t* m = &meta[(size_t)i * kMeta];
        const uint32_t dt = rd32(m + 8), ndim = rd32(m + 12), K = rd32(m + 20);
        if (!(dt == VOXQ_VXCP_FP32 || dt == VOXQ_VXCP_FP16 || dt == VOXQ_VXCP_BF16) || ndim != 2 || K == 0 ||
            K % 32 != 0 || elems[i] == 0)
            continue;
        const std::string name((const char*)f + st_off + rd32(m), rd32(m + 4));
        bool kept = false;
        for (int k = 0; k < n_keep && !kept; k++) kept = keep[k] && *keep[k] && name.find(keep[k]) != std::string::npos;
        if (kept) continue;
        quant[i] = 1;
        n_quant++;
        if (elems[i] > max_elems) max_elems = (size_t)elems[i];
        wr32(m + 8, qtype == VOXQ_Q4 ? VOXQ_VXCP_Q4_1 : VOXQ_VXCP_Q8);
    }

    DevBufs dev;
    if (n_quant) {
        if (cudaStreamCreateWithFlags(&dev.st, cudaStreamNonBlocking) != cudaSuccess) {
            cudaGetLastError();
            dev.st = nullptr;
            return VOXCPM_ERR_CUDA_NOT_FOUND;
        }
        if (!dev.reserve(max_elems)) return VOXCPM_ERR_OOM;
    }

    FILE* out = fopen(dst_path, "wb");
    if (!out) return VOXCPM_ERR_FILE_NOT_FOUND;
    auto abort_write = [&](VoxCPMError e) {
        fclose(out);
        remove(dst_path);
        return e;
    };
    const Crc32c& C = crc();
    uint8_t hdr[kHeader];
    memcpy(hdr, f, kHeader);
    wr32(hdr + 56, 0);
    wr32(hdr + 60, 0);
    // header, metadata and names now; the data checksum is patched in at the end
    const size_t str_bytes = data_start - st_off;
    if (fwrite(hdr, 1, kHeader, out) != kHeader || fwrite(meta.data(), 1, meta.size(), out) != meta.size() ||
        fwrite(f + st_off, 1, str_bytes, out) != str_bytes)
        return abort_write(VOXCPM_ERR_INTERNAL);
    uint32_t dc = C.update(0xFFFFFFFFu, meta.data(), meta.size());
    dc = C.update(dc, f + st_off, str_bytes);
    std::vector<uint8_t> obuf;
    uint64_t written = kHeader + meta.size() + str_bytes;
    for (uint32_t i = 0; i < nt; i++) {
        const uint8_t* src = f + off[i];
        if (!quant[i]) {
            if (fwrite(src, 1, bytes[i], out) != bytes[i]) return abort_write(VOXCPM_ERR_INTERNAL);
            dc = C.update(dc, src, bytes[i]);
            written += bytes[i];
            continue;
        }
        const size_t n = (size_t)elems[i];
        const uint32_t dt = rd32(f + kHeader + (size_t)i * kMeta + 8);
        cudaError_t ce = cudaMemcpyAsync(dt == VOXQ_VXCP_FP32 ? (void*)dev.f32 : dev.raw, src, bytes[i],
                                         cudaMemcpyHostToDevice, dev.st);
        if (ce != cudaSuccess) return abort_write(VOXCPM_ERR_INTERNAL);
        if (dt == VOXQ_VXCP_FP16) {
            // exact widening: the quantizer sees the floats quantize.py would
            if (VoxCPMError e = widen_fp16((const uint16_t*)dev.raw, dev.f32, n, dev.st)) return abort_write(e);
        } else if (dt == VOXQ_VXCP_BF16) {
            const int grid = (int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
            bf16_widen_kernel<<<grid, 256, 0, dev.st>>>((const uint16_t*)dev.raw, dev.f32, n);
            if (cudaGetLastError() != cudaSuccess) return abort_write(VOXCPM_ERR_INTERNAL);
        }
        if (VoxCPMError e = voxq_quantize(dev.f32, n, qtype, dev.blk, dev.st)) return abort_write(e);
        const size_t qb = voxq_quant_bytes(n, qtype);
        if (cudaMemcpyAsync(dev.h_blk, dev.blk, qb, cudaMemcpyDeviceToHost, dev.st) != cudaSuccess ||
            cudaStreamSynchronize(dev.st) != cudaSuccess)
            return abort_write(VOXCPM_ERR_INTERNAL);
        obuf.resize(qb);
        to_vxcp_order(dev.h_blk, obuf.data(), (n + 31) / 32, qtype);
        if (fwrite(obuf.data(), 1, qb, out) != qb) return abort_write(VOXCPM_ERR_INTERNAL);
        dc = C.update(dc, obuf.data(), qb);
        written += qb;
    }
    dc = ~dc;
    wr32(hdr + 56, ~C.update(0xFFFFFFFFu, hdr, kHeader));  // bytes 56..63 still zero
    wr32(hdr + 60, dc);
    if (fseek(out, 0, SEEK_SET) != 0 || fwrite(hdr, 1, kHeader, out) != kHeader) return abort_write(VOXCPM_ERR_INTERNAL);
    if (fclose(out) != 0) {
        remove(dst_path);
        return VOXCPM_ERR_INTERNAL;
    }
    if (stats) *stats = voxq_vxcp_stats{nt, n_quant, (uint64_t)in.n, written};
    return VOXCPM_SUCCESS;
}
