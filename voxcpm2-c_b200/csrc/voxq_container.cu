// voxq_container.cu -- reader for the weight container that the reference's
// quantizer writes (scripts/quantize.py:110-312, convert_quant):
//
//   [0, 256)     header: magic "VXCPM2\0\0", u32 version, n_layers,
//                n_layers_enc, n_ralm_layers, n_dit_layers, d_model, d_ff,
//                n_heads, n_kv_heads, head_dim, max_seq_len, vocab_size,
//                quant (0 f32, 1 f16, 2 q4, 3 q8), sample_rate,
//                audio_vae_dim, f32 rope_theta @68, u64 checksum @72,
//                u32 n_layer_groups @80              (scripts/quantize.py:119-139, 283-300)
//   [256, ...)   (n_layer_groups + 1) u64 file offsets of the groups  (:146-151, 304-307)
//   groups       tensors back to back: u32 name_hash, u32 ndim, u32 dims[3],
//                then the data of prod(dims[:ndim]) elements in the file's
//                quant type: f32, f16, or 20-byte Q4 / 40-byte Q8 blocks over
//                the flattened tensor, last block zero-padded  (:178-276, 88-104)
//   checksum     first 8 bytes (little endian) of SHA-256 over the file with
//                bytes [72, 80) zeroed                              (:309-315)
//
// The reference's C engine cannot read this container (its loader only knows
// the VXCP format, src/model.c:1715-1727, 1815-1858); this reader is how
// quantize.py output reaches the device: 2-D Q4 / Q8 tensors are packed into
// the voxq_qweight layout (voxq_pack_blocks) without requantizing.
// Host code only; the file is mapped read-only.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "voxq_common.cuh"
#include "voxq_internal.h"

struct voxq_vxcpm2 {
    const uint8_t* base = nullptr;
    size_t size = 0;
    voxq_vxcpm2_header hdr{};
    std::vector<voxq_vxcpm2_tensor> tensors;
};

namespace voxq {
namespace {

constexpr size_t kHeaderBytes = 256;
constexpr int kBlockElems = 32;

template <typename T>
T rd(const uint8_t* p) {
    T v;
    memcpy(&v, p, sizeof(T));  // little-endian host (x86-64 / aarch64)
    return v;
}

// Bytes of a tensor's data (without its 20-byte header), scripts/quantize.py:88-104.
bool data_bytes(uint64_t n, uint32_t quant, uint64_t* out) {
    const uint64_t blocks = (n + kBlockElems - 1) / kBlockElems;
    switch (quant) {
        case 0: *out = n * 4; return true;
        case 1: *out = n * 2; return true;
        case 2: *out = blocks * 20; return true;
        case 3: *out = blocks * 40; return true;
        default: return false;
    }
}

// ---- SHA-256 (FIPS 180-4).  The round constants and the initial hash are
// the first 32 fractional bits of the cube / square roots of the first
// primes, computed here from that definition.
struct Sha256 {
    uint32_t k[64], h[8];
    uint8_t buf[64];
    uint64_t total = 0;
    int fill = 0;

    static uint32_t frac32(double x) { return (uint32_t)(uint64_t)((x - std::floor(x)) * 4294967296.0); }
    static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

    Sha256() {
        int primes[64], np = 0;
        for (int c = 2; np < 64; c++) {
            bool pr = true;
            for (int i = 0; i < np && primes[i] * primes[i] <= c; i++)
                if (c % primes[i] == 0) pr = false;
            if (pr) primes[np++] = c;
        }
        for (int i = 0; i < 64; i++) k[i] = frac32(std::cbrt((double)primes[i]));
        for (int i = 0; i < 8; i++) h[i] = frac32(std::sqrt((double)primes[i]));
    }
    void block(const uint8_t* p) {
        uint32_t w[64];
        for (int i = 0; i < 16; i++)
            w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
        for (int i = 16; i < 64; i++) {
            const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
            const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
            w[i] = w[i - 16] + s0 + w[i - 7] + s1;
        }
        uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
        for (int i = 0; i < 64; i++) {
            const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[i] + w[i];
            const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
            hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
        }
        h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
    }
    void update(const uint8_t* p, size_t n) {
        total += n;
        while (n > 0) {
            if (fill == 0 && n >= 64) {
                block(p);
                p += 64;
                n -= 64;
                continue;
            }
            const size_t take = n < (size_t)(64 - fill) ? n : (size_t)(64 - fill);
            memcpy(buf + fill, p, take);
            fill += (int)take;
            p += take;
            n -= take;
            if (fill == 64) {
                block(buf);
                fill = 0;
            }
        }
    }
    void final(uint8_t out[32]) {
        const uint64_t bits = total * 8;
        const uint8_t one = 0x80, zero = 0;
        update(&one, 1);
        while (fill != 56) update(&zero, 1);
        uint8_t len[8];
        for (int i = 0; i < 8; i++) len[i] = (uint8_t)(bits >> (56 - 8 * i));
        update(len, 8);
        for (int i = 0; i < 8; i++)
            for (int j = 0; j < 4; j++) out[4 * i + j] = (uint8_t)(h[i] >> (24 - 8 * j));
    }
};


VoxCPMError parse(voxq_vxcpm2* f) {
    const uint8_t* b = f->base;
    if (f->size < kHeaderBytes) return VOXCPM_ERR_INVALID_MODEL;
    static const uint8_t magic[8] = {'V', 'X', 'C', 'P', 'M', '2', 0, 0};
    if (memcmp(b, magic, 8) != 0) return VOXCPM_ERR_INVALID_MODEL;
    voxq_vxcpm2_header& h = f->hdr;
    uint32_t* fields[] = {&h.version, &h.n_layers, &h.n_layers_enc, &h.n_ralm_layers, &h.n_dit_layers, &h.d_model,
                          &h.d_ff, &h.n_heads, &h.n_kv_heads, &h.head_dim, &h.max_seq_len, &h.vocab_size,
                          &h.quant, &h.sample_rate, &h.audio_vae_dim};
    for (int i = 0; i < 15; i++) *fields[i] = rd<uint32_t>(b + 8 + 4 * i);
    h.rope_theta = rd<float>(b + 68);
    h.checksum = rd<uint64_t>(b + 72);
    h.n_groups = rd<uint32_t>(b + 80);
    if (h.quant > 3) return VOXCPM_ERR_UNSUPPORTED;
    const uint64_t index_end = kHeaderBytes + ((uint64_t)h.n_groups + 1) * 8;
    if (h.n_groups > (1u << 24) || index_end > f->size) return VOXCPM_ERR_INVALID_MODEL;
    for (uint32_t g = 0; g < h.n_groups; g++) {
        const uint64_t start = rd<uint64_t>(b + kHeaderBytes + 8 * g);
        const uint64_t end = rd<uint64_t>(b + kHeaderBytes + 8 * (g + 1));
        if (end <= start) continue;  // empty group (scripts/quantize.py:178-179)
        if (start < index_end || end > f->size) return VOXCPM_ERR_INVALID_MODEL;
        uint64_t pos = start;
        while (pos < end) {
            if (pos + 20 > end) return VOXCPM_ERR_INVALID_MODEL;
            voxq_vxcpm2_tensor t{};
            t.name_hash = rd<uint32_t>(b + pos);
            t.ndim = rd<uint32_t>(b + pos + 4);
            for (int d = 0; d < 3; d++) t.dims[d] = rd<uint32_t>(b + pos + 8 + 4 * d);
            if (t.ndim > 3) return VOXCPM_ERR_INVALID_MODEL;
            uint64_t n = 1;
            for (uint32_t d = 0; d < t.ndim; d++) {
                if (t.dims[d] != 0 && n > (1ull << 40) / t.dims[d]) return VOXCPM_ERR_INVALID_MODEL;
                n *= t.dims[d];
            }
            uint64_t bytes = 0;
            data_bytes(n, h.quant, &bytes);
            if (pos + 20 + bytes > end) return VOXCPM_ERR_INVALID_MODEL;  // truncated tensor
            t.dtype = (int32_t)h.quant;
            t.group = (int32_t)g;
            t.elements = n;
            t.offset = pos + 20;
            t.bytes = bytes;
            f->tensors.push_back(t);
            pos += 20 + bytes;
        }
    }
    return VOXCPM_SUCCESS;
}

}  // namespace

float half_to_float(uint16_t h) {
    // IEEE binary16 -> binary32, exact (include/tensor.h:350-371 decodes the same way)
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else {  // subnormal: renormalise
            int sh = 0;
            uint32_t mm = m;
            while (!(mm & 1024)) {
                mm <<= 1;
                sh++;
            }
            bits = s | (uint32_t)(127 - 15 + 1 - sh) << 23 | (mm & 1023) << 13;
        }
    } else if (e == 31) {
        bits = s | 0x7F800000u | m << 13;
    } else {
        bits = s | (e - 15 + 127) << 23 | m << 13;
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

}  // namespace voxq

extern "C" {

VoxCPMError voxq_vxcpm2_open(const char* path, voxq_vxcpm2** out) {
    if (!path || !out) return VOXCPM_ERR_INTERNAL;
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return VOXCPM_ERR_FILE_NOT_FOUND;
    struct stat sb;
    if (fstat(fd, &sb) != 0 || sb.st_size <= 0) {
        close(fd);
        return VOXCPM_ERR_INVALID_MODEL;
    }
    void* m = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) return VOXCPM_ERR_OOM;
    voxq_vxcpm2* f = new voxq_vxcpm2;
    f->base = static_cast<const uint8_t*>(m);
    f->size = (size_t)sb.st_size;
    const VoxCPMError e = voxq::parse(f);
    if (e != VOXCPM_SUCCESS) {
        voxq_vxcpm2_close(f);
        return e;
    }
    *out = f;
    return VOXCPM_SUCCESS;
}

void voxq_vxcpm2_close(voxq_vxcpm2* f) {
    if (!f) return;
    if (f->base) munmap(const_cast<uint8_t*>(f->base), f->size);
    delete f;
}

VoxCPMError voxq_vxcpm2_info(const voxq_vxcpm2* f, voxq_vxcpm2_header* hdr, int* n_tensors) {
    if (!f) return VOXCPM_ERR_INTERNAL;
    if (hdr) *hdr = f->hdr;
    if (n_tensors) *n_tensors = (int)f->tensors.size();
    return VOXCPM_SUCCESS;
}

VoxCPMError voxq_vxcpm2_tensor_info(const voxq_vxcpm2* f, int i, voxq_vxcpm2_tensor* t) {
    if (!f || !t) return VOXCPM_ERR_INTERNAL;
    if (i < 0 || i >= (int)f->tensors.size()) return VOXCPM_ERR_SHAPE_MISMATCH;
    *t = f->tensors[(size_t)i];
    return VOXCPM_SUCCESS;
}

const uint8_t* voxq_vxcpm2_data(const voxq_vxcpm2* f, int i) {
    if (!f || i < 0 || i >= (int)f->tensors.size()) return nullptr;
    return f->base + f->tensors[(size_t)i].offset;
}

VoxCPMError voxq_vxcpm2_verify(const voxq_vxcpm2* f) {
    if (!f) return VOXCPM_ERR_INTERNAL;
    // The reference quantizer never fills the field (it raises while reading
    // back its write-only output, scripts/quantize.py:308-310): 0 = no checksum.
    if (f->hdr.checksum == 0) return VOXCPM_ERR_UNSUPPORTED;
    voxq::Sha256 sh;
    static const uint8_t zero8[8] = {};
    sh.update(f->base, 72);
    sh.update(zero8, 8);
    sh.update(f->base + 80, f->size - 80);
    uint8_t dig[32];
    sh.final(dig);
    uint64_t v = 0;
    for (int i = 7; i >= 0; i--) v = v << 8 | dig[i];
    return v == f->hdr.checksum ? VOXCPM_SUCCESS : VOXCPM_ERR_INVALID_MODEL;
}

VoxCPMError voxq_vxcpm2_dequantize(const voxq_vxcpm2* f, int i, int q8_signed, float* out) {
    if (!f || !out) return VOXCPM_ERR_INTERNAL;
    if (i < 0 || i >= (int)f->tensors.size()) return VOXCPM_ERR_SHAPE_MISMATCH;
    const voxq_vxcpm2_tensor& t = f->tensors[(size_t)i];
    const uint8_t* p = f->base + t.offset;
    const uint64_t n = t.elements;
    switch (t.dtype) {
        case 0:
            memcpy(out, p, n * 4);
            break;
        case 1:
            for (uint64_t k = 0; k < n; k++) out[k] = voxq::half_to_float(voxq::rd<uint16_t>(p + 2 * k));
            break;
        case 2:  // scripts/quantize.py:56-67: f32(q) * f32(f16 scale) + f32(f16 min)
            for (uint64_t k = 0; k < n; k++) {
                const uint8_t* blk = p + (k / 32) * 20;
                const int j = (int)(k % 32);
                const uint8_t byte = blk[j / 2];
                const float q = (float)((j & 1) ? (byte & 15) : (byte >> 4));
                const float sc = voxq::half_to_float(voxq::rd<uint16_t>(blk + 16));
                const float mn = voxq::half_to_float(voxq::rd<uint16_t>(blk + 18));
                out[k] = q * sc + mn;
            }
            break;
        case 3:  // scripts/quantize.py:77-82 (q8_signed) or the unsigned reading of the codes
            for (uint64_t k = 0; k < n; k++) {
                const uint8_t* blk = p + (k / 32) * 40;
                const uint8_t byte = blk[k % 32];
                const float q = q8_signed ? (float)(int8_t)byte : (float)byte;
                out[k] = q * voxq::rd<float>(blk + 32) + voxq::rd<float>(blk + 36);
            }
            break;
        default:
            return VOXCPM_ERR_UNSUPPORTED;
    }
    return VOXCPM_SUCCESS;
}

VoxCPMError voxq_vxcpm2_upload_qweight(const voxq_vxcpm2* f, int i, uint8_t* d_codes, void* d_scales, void* stream) {
    if (!f || !d_codes || !d_scales) return VOXCPM_ERR_INTERNAL;
    if (i < 0 || i >= (int)f->tensors.size()) return VOXCPM_ERR_SHAPE_MISMATCH;
    const voxq_vxcpm2_tensor& t = f->tensors[(size_t)i];
    if (t.dtype != VOXQ_Q4 && t.dtype != VOXQ_Q8) return VOXCPM_ERR_UNSUPPORTED;
    if (t.ndim != 2 || t.dims[1] % 32 != 0 || t.dims[0] == 0 || t.dims[0] > (1u << 30) || t.dims[1] > (1u << 30))
        return VOXCPM_ERR_SHAPE_MISMATCH;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* d_blocks = nullptr;
    VOXQ_CUDA_TRY(cudaMalloc(&d_blocks, t.bytes));
    VoxCPMError e = VOXCPM_SUCCESS;
    if (cudaMemcpyAsync(d_blocks, f->base + t.offset, t.bytes, cudaMemcpyHostToDevice, st) != cudaSuccess)
        e = VOXCPM_ERR_GPU;
    if (!e) e = voxq_pack_blocks(d_blocks, (int)t.dims[0], (int)t.dims[1], t.dtype, d_codes, d_scales, stream);
    if (cudaStreamSynchronize(st) != cudaSuccess && !e) e = VOXCPM_ERR_GPU;
    cudaFree(d_blocks);
    return e;
}

}  // extern "C"
