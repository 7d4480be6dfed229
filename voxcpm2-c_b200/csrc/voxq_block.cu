// voxq_block.cu -- the engine's transformer block (src/nn.c:579-700) on the device.
//
// The reference runs everything of a block but its projections on one host
// thread: RMSNorm, the attention (per-head permutes, RoPE, the KV-cache copy,
// scores, softmax, the weighted sum), SiLU gating and the residual adds, with
// a synchronous host <-> device round trip per projection.  Here one call
// uploads the block input once, runs
//
//   n   = RMSNorm(x)                      rmsnorm_kernel
//   q, k, v = n Wq^T, n Wk^T, n Wv^T      one grouped GEMV launch (M <= 8) or three GEMMs
//   RoPE(q, k); k, v -> cache[pos ..]     rope_cache_kernel
//   a   = softmax(q k^T / sqrt(d) + mask) v   attn_kernel (one CTA per query row and head), or
//                                         for many query rows attn_mma_kernel (tensor cores)
//   h   = x + a Wo^T                      projection with the residual epilogue
//   n2  = RMSNorm(h)
//   g   = silu(n2 W1^T) * (n2 W3^T)       projection with the SwiGLU epilogue
//   out = h + g W2^T                      projection with the residual epilogue
//
// and downloads the output and the new cache rows once, with one wait.  The
// KV cache is mirrored on the device per host cache pointer; the host cache is
// kept identical (new rows written back), so a call that falls back to the
// host code, or any other reader of the cache, sees the reference's state.
#include <math.h>

#include <algorithm>
#include <string.h>

#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "voxq_common.cuh"
#include "voxq_internal.h"

namespace voxq {

constexpr int kBlockThreads = 256;
constexpr int kAttnThreads = 128;
constexpr int kMaxCacheLen = 32768;  // score row in shared memory (128 KB)
constexpr int kMaxHeadDim = 256;

// RMSNorm of one row per CTA: sum of squares in double (NaN counted as 0),
// rms = sqrt(sum / D + eps) in double, out = (float)(x * (1 / rms)) * w.
// The LocDiT and LocEnc paths normalise in place (out == x): every read of the
// sum pass is done before the barriers that end the reduction, and in the
// output pass each thread writes only the elements it reads itself.
__global__ void __launch_bounds__(kBlockThreads) rmsnorm_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ w, float eps,
                                                                float* __restrict__ out, int D) {
    __shared__ double red[kBlockThreads / 32];
    const float* xr = x + (int64_t)blockIdx.x * D;
    double s = 0.0;
    for (int d = threadIdx.x; d < D; d += kBlockThreads) {
        float v = xr[d];
        if (isnan(v)) v = 0.0f;
        s += (double)v * (double)v;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < kBlockThreads / 32 ? red[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const double inv = 1.0 / sqrt(red[0] / (double)D + (double)eps);
    float* orow = out + (int64_t)blockIdx.x * D;
    for (int d = threadIdx.x; d < D; d += kBlockThreads) {
        const float n = (float)((double)xr[d] * inv);
        orow[d] = w ? n * w[d] : n;
    }
}

// RoPE and the cache write.  blockIdx.x = token m = b * seq + s; blockIdx.y =
// head slot: [0, H) query heads, [H, H + KVH) key heads, [H + KVH, H + 2 KVH)
// value heads.  Pair (i, i + half): (x0 c - x1 s, x0 s + x1 c) with (c, s) =
// freqs[s][i] (freqs holds the call's rows only, [seq][half][2]).
// q_out [B][H][seq][hd]; cache [B][KVH][max_seq][hd] at row pos + s; knew /
// vnew [B][KVH][seq][hd] (the rows written back to the host cache).
__global__ void rope_cache_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                  const float* __restrict__ v, const float* __restrict__ freqs,
                                  float* __restrict__ q_out, float* __restrict__ ck, float* __restrict__ cv,
                                  float* __restrict__ knew, float* __restrict__ vnew, int seq, int H, int KVH,
                                  int hd, int max_seq, int pos) {
    const int m = blockIdx.x, slot = blockIdx.y;
    const int b = m / seq, s = m % seq;
    const int half = hd / 2;
    const float* src;
    float* dst;
    float* dst2 = nullptr;
    bool rope = freqs != nullptr;
    if (slot < H) {
        src = q + ((int64_t)m * H + slot) * hd;
        dst = q_out + (((int64_t)b * H + slot) * seq + s) * hd;
    } else if (slot < H + KVH) {
        const int h = slot - H;
        src = k + ((int64_t)m * KVH + h) * hd;
        dst = ck + (((int64_t)b * KVH + h) * max_seq + pos + s) * hd;
        if (knew) dst2 = knew + (((int64_t)b * KVH + h) * seq + s) * hd;
    } else {
        const int h = slot - H - KVH;
        src = v + ((int64_t)m * KVH + h) * hd;
        dst = cv + (((int64_t)b * KVH + h) * max_seq + pos + s) * hd;
        if (vnew) dst2 = vnew + (((int64_t)b * KVH + h) * seq + s) * hd;
        rope = false;
    }
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        float x0 = src[i], x1 = src[i + half];
        if (rope) {
            const float c = freqs[((int64_t)s * half + i) * 2], sn = freqs[((int64_t)s * half + i) * 2 + 1];
            const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
            const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
            x0 = y0;
            x1 = y1;
        }
        dst[i] = x0;
        dst[i + half] = x1;
        if (dst2) {
            dst2[i] = x0;
            dst2[i + half] = x1;
        }
    }
}

// One query row of one head per CTA: scores over the cache's first L
// positions, softmax, weighted sum of the value rows.  blockIdx = (s, h, b).
// out [B][seq][H][hd] (the [M][H*hd] input of the output projection).
// mask: [mrows][mcols] rows of the call's queries (host mask rows 0 .. seq),
// added where s < mrows and t < mcols.
__global__ void __launch_bounds__(kAttnThreads) attn_kernel(const float* __restrict__ q, const float* __restrict__ ck,
                                                            const float* __restrict__ cv,
                                                            const float* __restrict__ mask, int mrows, int mcols,
                                                            float* __restrict__ out, int seq, int H, int KVH, int hd,
                                                            int max_seq, int L, float inv_scale) {
    extern __shared__ float sh[];
    float* qs = sh;              // [hd]
    float* sc = sh + kMaxHeadDim;  // [L]
    __shared__ float red[kAttnThreads / 32];
    const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int kh = h / (H / KVH);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float* qr = q + (((int64_t)b * H + h) * seq + s) * hd;
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) qs[d] = qr[d];
    __syncthreads();
    const float* kb = ck + ((int64_t)b * KVH + kh) * max_seq * hd;
    const float* vb = cv + ((int64_t)b * KVH + kh) * max_seq * hd;
    // scores: one warp per key row, lanes over head_dim
    for (int t = warp; t < L; t += kAttnThreads / 32) {
        const float* kr = kb + (int64_t)t * hd;
        float acc = 0.0f;
        for (int d = lane; d < hd; d += 32) acc = fmaf(qs[d], kr[d], acc);
#pragma unroll
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) {
            float v = acc * inv_scale;
            if (mask && s < mrows && t < mcols) v += mask[(int64_t)s * mcols + t];
            sc[t] = v;
        }
    }
    __syncthreads();
    // softmax over [0, L): max, exp(x - max), 1 / (sum + 1e-10)
    float mx = -INFINITY;
    for (int t = threadIdx.x; t < L; t += kAttnThreads) mx = fmaxf(mx, sc[t]);
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < kAttnThreads / 32; w++) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float sum = 0.0f;
    for (int t = threadIdx.x; t < L; t += kAttnThreads) {
        const float e = expf(sc[t] - mx);
        sc[t] = e;
        sum += e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    sum = 0.0f;
    for (int w = 0; w < kAttnThreads / 32; w++) sum += red[w];
    const float inv = 1.0f / (sum + 1e-10f);
    for (int t = threadIdx.x; t < L; t += kAttnThreads) sc[t] *= inv;
    __syncthreads();
    // out[d] = sum over t in order of p[t] v[t][d]
    float* orow = out + (((int64_t)b * seq + s) * H + h) * hd;
    for (int d = threadIdx.x; d < hd; d += kAttnThreads) {
        float acc = 0.0f;
        for (int t = 0; t < L; t++) acc = fmaf(sc[t], vb[(int64_t)t * hd + d], acc);
        orow[d] = acc;
    }
}

// Attention for many query rows (prefill, the LocDiT's sequences): the same
// function as attn_kernel, tiled so a key / value tile in shared memory serves
// 64 query vectors -- the query rows of a CTA times the G = H / KVH query heads
// that read one kv head -- instead of every CTA re-reading the whole cache.
// Four threads per query vector, each holding head_dim / 4 interleaved
// dimensions (d = part + 4 j, conflict-free shared reads); an online softmax
// (running max m and sum l, accumulator rescaled by exp(m_old - m_new)) over
// key tiles of kFK; out = acc / (l + 1e-10).  grid = (ceil(seq / (64 / G)),
// KVH, B).
constexpr int kFK = 32;
constexpr int kFThreads = 256;
template <int HD>
__global__ void __launch_bounds__(kFThreads) attn_tiled_kernel(const float* __restrict__ q, const float* __restrict__ ck,
                                                               const float* __restrict__ cv,
                                                               const float* __restrict__ mask, int mrows, int mcols,
                                                               float* __restrict__ out, int seq, int H, int KVH,
                                                               int max_seq, int L, float inv_scale, int nsplit,
                                                               float* __restrict__ partial) {
    constexpr int DPT = HD / 4;
    __shared__ __align__(16) float Ks[kFK][HD];
    __shared__ __align__(16) float Vs[kFK][HD];
    const int G = H / KVH, QR = 64 / G;
    const int kh = blockIdx.y, b = blockIdx.z;
    // blockIdx.x = query tile * nsplit + key split; split sp takes whole key
    // tiles [sp * tps, (sp + 1) * tps)
    const int qt = blockIdx.x / nsplit, sp = blockIdx.x % nsplit;
    const int ntiles = (L + kFK - 1) / kFK, tps = (ntiles + nsplit - 1) / nsplit;
    const int t_beg = sp * tps * kFK, t_end = min(L, (sp + 1) * tps * kFK);
    const int r = threadIdx.x >> 2, part = threadIdx.x & 3;
    const int h = kh * G + r % G, s = qt * QR + r / G;
    const bool valid = s < seq;
    float qv[DPT], acc[DPT];
    const float* qr = q + (((int64_t)b * H + h) * seq + (valid ? s : 0)) * HD;
#pragma unroll
    for (int j = 0; j < DPT; j++) {
        qv[j] = valid ? qr[part + 4 * j] : 0.0f;
        acc[j] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    const float* kb = ck + ((int64_t)b * KVH + kh) * max_seq * HD;
    const float* vb = cv + ((int64_t)b * KVH + kh) * max_seq * HD;
    for (int t0 = t_beg; t0 < t_end; t0 += kFK) {
        __syncthreads();  // the previous tile is consumed
        const int nt = min(kFK, t_end - t0);
        for (int i = threadIdx.x; i < kFK * HD / 4; i += kFThreads) {
            const int row = (i * 4) / HD, col = (i * 4) % HD;
            float4 kk = make_float4(0.f, 0.f, 0.f, 0.f), vv = kk;
            if (row < nt) {
                kk = *reinterpret_cast<const float4*>(kb + (int64_t)(t0 + row) * HD + col);
                vv = *reinterpret_cast<const float4*>(vb + (int64_t)(t0 + row) * HD + col);
            }
            *reinterpret_cast<float4*>(&Ks[row][col]) = kk;
            *reinterpret_cast<float4*>(&Vs[row][col]) = vv;
        }
        __syncthreads();
        float sc[kFK];
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < kFK; k++) {
            float pd = 0.0f;
#pragma unroll
            for (int j = 0; j < DPT; j++) pd = fmaf(qv[j], Ks[k][part + 4 * j], pd);
            pd += __shfl_xor_sync(0xffffffffu, pd, 1);
            pd += __shfl_xor_sync(0xffffffffu, pd, 2);
            float v = pd * inv_scale;
            const int t = t0 + k;
            if (mask && s < mrows && t < mcols) v += mask[(int64_t)s * mcols + t];
            if (k >= nt) v = -INFINITY;
            sc[k] = v;
            mx = fmaxf(mx, v);
        }
        const float mn = fmaxf(m, mx);
        if (mn == -INFINITY) continue;  // every key so far masked
        const float f = expf(m - mn);   // 0 on the first visible tile (m = -inf)
        l *= f;
#pragma unroll
        for (int j = 0; j < DPT; j++) acc[j] *= f;
#pragma unroll
        for (int k = 0; k < kFK; k++) {
            const float p = expf(sc[k] - mn);
            l += p;
#pragma unroll
            for (int j = 0; j < DPT; j++) acc[j] = fmaf(p, Vs[k][part + 4 * j], acc[j]);
        }
        m = mn;
    }
    if (nsplit > 1) {
        // this split's running max, sum and unnormalised accumulator, combined by attn_combine_kernel
        const int nqt = gridDim.x / nsplit;
        float* rec = partial + (((((int64_t)b * KVH + kh) * nqt + qt) * nsplit + sp) * 64 + r) * (HD + 2);
        if (part == 0) {
            rec[0] = m;
            rec[1] = l;
        }
#pragma unroll
        for (int j = 0; j < DPT; j++) rec[2 + part + 4 * j] = acc[j];
        return;
    }
    if (!valid) return;
    const float inv = 1.0f / (l + 1e-10f);
    float* orow = out + (((int64_t)b * seq + s) * H + h) * HD;
#pragma unroll
    for (int j = 0; j < DPT; j++) orow[part + 4 * j] = acc[j] * inv;
}

// ---------------------------------------------------------------------------
// attn_tiled_kernel's function with both products on the tensor cores.
//
// Same grid, same 64 query vectors per CTA (the query rows of a CTA times the
// G heads that read one kv head), same key tiles of kFK, same key splits and
// partial records (so attn_combine_kernel merges them).  Four warps, each
// owning 16 of the vectors as the M = 16 side of mma.sync m16n8k8 TF32 tiles:
//
//   S = Q K^T   (16 x 32 per warp per key tile: 4 n-blocks of 8 keys,
//               HD / 8 k-steps over the head dims)
//   online softmax on S in registers (the tiled kernel's m / l recurrence)
//   O += P V    (16 x HD per warp: HD / 8 n-blocks, 4 k-steps of 8 keys)
//
// Every operand is split into a TF32 high part and a TF32 low part (the
// rounding remainder), and each product is a_lo b_hi + a_hi b_lo + a_hi b_hi
// accumulated in fp32: the dropped a_lo b_lo term is ~2^-22 relative, so the
// result matches the fp32 CUDA-core kernel to within fp32 rounding.
//
// The P operand comes straight from the S accumulators: a lane holds keys
// 2t and 2t + 1 of each 8-key block (C layout), while the A operand wants
// columns t and t + 4; reading the block's keys in the order
// (0, 2, 4, 6, 1, 3, 5, 7) -- A column t is key 2t, column t + 4 is key
// 2t + 1 -- makes the two layouts coincide, and the V operand is read in the
// same key order.  Shared-memory rows have a pitch of HD + 4 floats, which
// puts the 32 lanes of every fragment load in 32 different banks.
constexpr int kMThreads = 128;
constexpr int kMPitchPad = 4;
constexpr int kMPvGroup = 8;  // head-dim blocks whose P V products are interleaved

__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(x));
    const float r = x - __uint_as_float(hi);
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(r));
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d[i] += a b[i] for NG accumulators with both operands split: three TF32
// products per accumulator, small ones first (a_lo b_hi, a_hi b_lo, a_hi b_hi).
// Each product is issued for all NG accumulators before the next one, so
// consecutive MMAs are independent and overlap in the pipe; every accumulator
// still receives its three products in the same order.
template <int NG>
__device__ __forceinline__ void mma_tf32x3_group(float (*d)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                                 const uint32_t (&bh)[NG][2], const uint32_t (&bl)[NG][2]) {
#pragma unroll
    for (int i = 0; i < NG; i++) mma_tf32(d[i], al, bh[i][0], bh[i][1]);
#pragma unroll
    for (int i = 0; i < NG; i++) mma_tf32(d[i], ah, bl[i][0], bl[i][1]);
#pragma unroll
    for (int i = 0; i < NG; i++) mma_tf32(d[i], ah, bh[i][0], bh[i][1]);
}

template <int HD>
constexpr int attn_mma_smem_bytes() {
    return (64 + 2 * kFK) * (HD + kMPitchPad) * (int)sizeof(float);
}

template <int HD>
__global__ void __launch_bounds__(kMThreads) attn_mma_kernel(const float* __restrict__ q, const float* __restrict__ ck,
                                                             const float* __restrict__ cv,
                                                             const float* __restrict__ mask, int mrows, int mcols,
                                                             float* __restrict__ out, int seq, int H, int KVH,
                                                             int max_seq, int L, float inv_scale, int nsplit,
                                                             float* __restrict__ partial) {
    constexpr int P = HD + kMPitchPad;  // shared row pitch (floats)
    constexpr int NB = HD / 8;          // 8-wide blocks of the head dims
    extern __shared__ __align__(16) float asm_sh[];
    float* Qs = asm_sh;          // [64][P]   the CTA's query vectors
    float* Ks = Qs + 64 * P;     // [kFK][P]  key tile
    float* Vs = Ks + kFK * P;    // [kFK][P]  value tile
    const int G = H / KVH, QR = 64 / G;
    const int kh = blockIdx.y, b = blockIdx.z;
    const int qt = blockIdx.x / nsplit, sp = blockIdx.x % nsplit;
    const int ntiles = (L + kFK - 1) / kFK, tps = (ntiles + nsplit - 1) / nsplit;
    const int t_beg = sp * tps * kFK, t_end = min(L, (sp + 1) * tps * kFK);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;

    // the 64 query vectors (zeros past the sequence)
    for (int i = threadIdx.x; i < 64 * HD / 4; i += kMThreads) {
        const int r = (i * 4) / HD, col = (i * 4) % HD;
        const int h = kh * G + r % G, s = qt * QR + r / G;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (s < seq) v = *reinterpret_cast<const float4*>(q + (((int64_t)b * H + h) * seq + s) * HD + col);
        *reinterpret_cast<float4*>(Qs + r * P + col) = v;
    }

    // this lane's two query vectors (MMA rows g and g + 8 of the warp's 16)
    const int r0 = warp * 16 + g, r1 = r0 + 8;
    const int s0 = qt * QR + r0 / G, s1 = qt * QR + r1 / G;
    float o[NB][4];
#pragma unroll
    for (int j = 0; j < NB; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // l: this lane's share of the row sums
    const float* kb = ck + ((int64_t)b * KVH + kh) * max_seq * HD;
    const float* vb = cv + ((int64_t)b * KVH + kh) * max_seq * HD;
    const float* qa = Qs + r0 * P + t;
    const float* qb = Qs + r1 * P + t;

    for (int t0 = t_beg; t0 < t_end; t0 += kFK) {
        __syncthreads();  // the previous tile is consumed (and, at first, Qs is written)
        const int nt = min(kFK, t_end - t0);
        for (int i = threadIdx.x; i < kFK * HD / 4; i += kMThreads) {
            const int row = (i * 4) / HD, col = (i * 4) % HD;
            float4 kk = make_float4(0.f, 0.f, 0.f, 0.f), vv = kk;
            if (row < nt) {
                kk = *reinterpret_cast<const float4*>(kb + (int64_t)(t0 + row) * HD + col);
                vv = *reinterpret_cast<const float4*>(vb + (int64_t)(t0 + row) * HD + col);
            }
            *reinterpret_cast<float4*>(Ks + row * P + col) = kk;
            *reinterpret_cast<float4*>(Vs + row * P + col) = vv;
        }
        __syncthreads();

        // S = Q K^T for the tile's 4 blocks of 8 keys
        float sc[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll 4
        for (int kk = 0; kk < NB; kk++) {
            uint32_t ah[4], al[4];
            tf32_split(qa[kk * 8], ah[0], al[0]);
            tf32_split(qb[kk * 8], ah[1], al[1]);
            tf32_split(qa[kk * 8 + 4], ah[2], al[2]);
            tf32_split(qb[kk * 8 + 4], ah[3], al[3]);
            uint32_t bh[4][2], bl[4][2];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float* kr = Ks + (j * 8 + g) * P + kk * 8 + t;
                tf32_split(kr[0], bh[j][0], bl[j][0]);
                tf32_split(kr[4], bh[j][1], bl[j][1]);
            }
            mma_tf32x3_group<4>(sc, ah, al, bh, bl);
        }

        // scale, mask, keys past the tile's end; row maxima over the quad
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int key = j * 8 + 2 * t + (c & 1), tk = t0 + key;
                const int srow = c < 2 ? s0 : s1;
                float v = sc[j][c] * inv_scale;
                if (mask && srow < mrows && tk < mcols) v += mask[(int64_t)srow * mcols + tk];
                if (key >= nt) v = -INFINITY;
                sc[j][c] = v;
                if (c < 2)
                    mx0 = fmaxf(mx0, v);
                else
                    mx1 = fmaxf(mx1, v);
            }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        // a row whose keys so far are all masked keeps zero weights (and m = -inf)
        const bool live0 = mn0 != -INFINITY, live1 = mn1 != -INFINITY;
        const float f0 = live0 ? expf(m0 - mn0) : 1.0f, f1 = live1 ? expf(m1 - mn1) : 1.0f;
        float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; j++)
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const bool r1c = c >= 2;
                const float p = (r1c ? live1 : live0) ? expf(sc[j][c] - (r1c ? mn1 : mn0)) : 0.0f;
                sc[j][c] = p;
                if (r1c)
                    ps1 += p;
                else
                    ps0 += p;
            }
        l0 = fmaf(l0, f0, ps0);
        l1 = fmaf(l1, f1, ps1);
        m0 = live0 ? mn0 : m0;
        m1 = live1 ? mn1 : m1;
#pragma unroll
        for (int j = 0; j < NB; j++) {
            o[j][0] *= f0;
            o[j][1] *= f0;
            o[j][2] *= f1;
            o[j][3] *= f1;
        }

        // O += P V, keys of block j read in the order (0, 2, 4, 6, 1, 3, 5, 7)
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t ah[4], al[4];
            tf32_split(sc[j][0], ah[0], al[0]);  // row g,     key 2t
            tf32_split(sc[j][2], ah[1], al[1]);  // row g + 8, key 2t
            tf32_split(sc[j][1], ah[2], al[2]);  // row g,     key 2t + 1
            tf32_split(sc[j][3], ah[3], al[3]);  // row g + 8, key 2t + 1
            const float* v0 = Vs + (j * 8 + 2 * t) * P + g;
            const float* v1 = v0 + P;
            constexpr int NG = kMPvGroup < NB ? kMPvGroup : NB;
#pragma unroll
            for (int n0 = 0; n0 < NB; n0 += NG) {
                uint32_t bh[NG][2], bl[NG][2];
#pragma unroll
                for (int i = 0; i < NG; i++) {
                    tf32_split(v0[(n0 + i) * 8], bh[i][0], bl[i][0]);
                    tf32_split(v1[(n0 + i) * 8], bh[i][1], bl[i][1]);
                }
                mma_tf32x3_group<NG>(o + n0, ah, al, bh, bl);
            }
        }
    }

    // the row sums over the quad
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    if (nsplit > 1) {
        // this split's running max, sum and unnormalised accumulator, combined by attn_combine_kernel
        const int nqt = gridDim.x / nsplit;
        float* rec = partial + ((((int64_t)b * KVH + kh) * nqt + qt) * nsplit + sp) * 64 * (HD + 2);
        float* ra = rec + (int64_t)r0 * (HD + 2);
        float* rb = rec + (int64_t)r1 * (HD + 2);
        if (t == 0) {
            ra[0] = m0;
            ra[1] = l0;
            rb[0] = m1;
            rb[1] = l1;
        }
#pragma unroll
        for (int n = 0; n < NB; n++) {
            ra[2 + n * 8 + 2 * t] = o[n][0];
            ra[3 + n * 8 + 2 * t] = o[n][1];
            rb[2 + n * 8 + 2 * t] = o[n][2];
            rb[3 + n * 8 + 2 * t] = o[n][3];
        }
        return;
    }
    const float inv0 = 1.0f / (l0 + 1e-10f), inv1 = 1.0f / (l1 + 1e-10f);
    if (s0 < seq) {
        float* orow = out + (((int64_t)b * seq + s0) * H + kh * G + r0 % G) * HD + 2 * t;
#pragma unroll
        for (int n = 0; n < NB; n++)
            *reinterpret_cast<float2*>(orow + n * 8) = make_float2(o[n][0] * inv0, o[n][1] * inv0);
    }
    if (s1 < seq) {
        float* orow = out + (((int64_t)b * seq + s1) * H + kh * G + r1 % G) * HD + 2 * t;
#pragma unroll
        for (int n = 0; n < NB; n++)
            *reinterpret_cast<float2*>(orow + n * 8) = make_float2(o[n][2] * inv1, o[n][3] * inv1);
    }
}

// Combines the key splits of attn_tiled_kernel: one warp per query vector,
// M = max m_sp, l = sum l_sp e^(m_sp - M), acc = sum acc_sp e^(m_sp - M),
// out = acc / (l + 1e-10) -- the single pass's result up to fp32 rounding;
// a vector whose keys were all masked gets zeros, as in the single pass.
template <int HD>
__global__ void attn_combine_kernel(const float* __restrict__ partial, float* __restrict__ out, int seq, int H,
                                    int KVH, int B, int nqt, int nsplit) {
    const int G = H / KVH, QR = 64 / G;
    const int64_t gw = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= (int64_t)B * KVH * nqt * 64) return;
    const int r = (int)(gw % 64);
    const int64_t tile = gw / 64;  // ((b * KVH + kh) * nqt + qt)
    const int qt = (int)(tile % nqt), kh = (int)((tile / nqt) % KVH), b = (int)(tile / ((int64_t)nqt * KVH));
    const int h = kh * G + r % G, s = qt * QR + r / G;
    if (s >= seq) return;
    const float* rec0 = partial + (tile * nsplit * 64 + r) * (HD + 2);
    const int64_t step = (int64_t)64 * (HD + 2);
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; sp++) M = fmaxf(M, rec0[sp * step]);
    constexpr int DPL = HD / 32;
    float acc[DPL];
#pragma unroll
    for (int j = 0; j < DPL; j++) acc[j] = 0.0f;
    float l = 0.0f;
    if (M != -INFINITY) {
        for (int sp = 0; sp < nsplit; sp++) {
            const float* rec = rec0 + sp * step;
            const float ms = rec[0];
            if (ms == -INFINITY) continue;
            const float f = expf(ms - M);
            l = fmaf(rec[1], f, l);
#pragma unroll
            for (int j = 0; j < DPL; j++) acc[j] = fmaf(rec[2 + lane + 32 * j], f, acc[j]);
        }
    }
    const float inv = 1.0f / (l + 1e-10f);
    float* orow = out + (((int64_t)b * seq + s) * H + h) * HD;
#pragma unroll
    for (int j = 0; j < DPL; j++) orow[lane + 32 * j] = acc[j] * inv;
}

// Gathers cache rows [r0, r1) of every (b, kv head) from a contiguous host
// staging block [B][KVH][r1 - r0][hd] into the device cache.
__global__ void cache_fill_kernel(const float* __restrict__ src, float* __restrict__ dst, int BK, int rows, int hd,
                                  int max_seq, int r0) {
    const int64_t n = (int64_t)BK * rows * hd;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int d = (int)(i % hd);
        const int64_t rr = i / hd;
        const int r = (int)(rr % rows), bk = (int)(rr / rows);
        dst[((int64_t)bk * max_seq + r0 + r) * hd + d] = src[i];
    }
}

// ---- LocDiT sampler kernels ----

__global__ void silu_inplace_kernel(float* __restrict__ x, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float v = x[i];
        x[i] = v / (1.0f + expf(-v));
    }
}

__global__ void add_vec_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ c,
                               int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) c[i] = a[i] + b[i];
}

// [rows][cols] -> [cols][rows]
__global__ void transpose_kernel(const float* __restrict__ x, float* __restrict__ y, int rows, int cols) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < rows * cols) {
        const int r = i / cols, c = i % cols;
        y[(int64_t)c * rows + r] = x[i];
    }
}

// The sequences of the nb branches, [nb][S][D] with S = 1 + P + Tc: row 0 mu,
// rows 1..P the input projection, then the condition projection (branch 0)
// or its bias alone (branch 1: the zero condition), each plus gc.
__global__ void dit_seq_kernel(float* __restrict__ seq, const float* __restrict__ mu,
                               const float* __restrict__ xproj, const float* __restrict__ crows,
                               const float* __restrict__ cbias, const float* __restrict__ gc, int nb, int P, int Tc,
                               int D) {
    const int S = 1 + P + Tc;
    const int64_t n = (int64_t)nb * S * D;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int r = (int)((i / D) % S), j = (int)(i / ((int64_t)S * D));
        float v;
        if (r == 0) v = mu[d];
        else if (r <= P) v = xproj[(int64_t)(r - 1) * D + d];
        else v = j == 0 ? crows[(int64_t)(r - 1 - P) * D + d] : (cbias ? cbias[d] : 0.0f);
        seq[i] = v + gc[d];
    }
}

// x rows 1..P of every branch: [nb][S][D] -> [nb * P][D]
__global__ void dit_slice_kernel(const float* __restrict__ seq, float* __restrict__ xs, int nb, int P, int S, int D) {
    const int64_t n = (int64_t)nb * P * D;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int p = (int)((i / D) % P), j = (int)(i / ((int64_t)P * D));
        xs[i] = seq[((int64_t)j * S + 1 + p) * D + d];
    }
}

// LocEnc input sequence (src/loc_enc.c:104-122): per (b, t) the special
// token, then the step's P projected patches; x [B][T (P + 1)][D].
__global__ void enc_seq_kernel(float* __restrict__ x, const float* __restrict__ proj,
                               const float* __restrict__ special, int B, int T, int P, int D) {
    const int64_t n = (int64_t)B * T * (P + 1) * D;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int64_t r = i / D;  // (b, t, j) row
        const int j = (int)(r % (P + 1));
        const int64_t bt = r / (P + 1);
        x[i] = j == 0 ? special[d] : proj[(bt * P + (j - 1)) * D + d];
    }
}

// Each step's first token (src/loc_enc.c:168-177): cls [B T][D].
__global__ void enc_cls_kernel(const float* __restrict__ x, float* __restrict__ cls, int BT, int P, int D) {
    const int64_t n = (int64_t)BT * D;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int d = (int)(i % D);
        const int64_t bt = i / D;
        cls[i] = x[bt * (P + 1) * D + d];
    }
}

// Euler step with guidance: v rows [nb * P][F] (branch 0 conditional);
// x [F][P] -= dt * (v_u + cfg (v_c - v_u)) (or v_c alone).
__global__ void dit_step_kernel(float* __restrict__ x, const float* __restrict__ v, int nb, int P, int F, float cfg,
                                float dt) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= F * P) return;
    const int f = i / P, p = i % P;
    const float vc = v[(int64_t)p * F + f];
    float pred = vc;
    if (nb == 2) {
        const float vu = v[(int64_t)(P + p) * F + f];
        pred = vu + cfg * (vc - vu);
    }
    x[i] = x[i] - dt * pred;
}

namespace {

// Device mirror of one host KV cache (K and V of one layer).
struct Mirror {
    float* k = nullptr;
    float* v = nullptr;
    size_t floats = 0;           // per buffer
    int BK = 0, max_seq = 0, hd = 0;
    int valid = 0;               // leading positions equal to the host cache
    std::vector<float> last_row;  // host K row valid - 1 of (b 0, kv head 0), as last written
    uint64_t used = 0;
};

struct NormW {
    float* p = nullptr;
    size_t n = 0;
    uint64_t fp = 0;
};

struct BlockDev {
    std::unordered_map<const void*, Mirror> mirrors;  // host cache_k data pointer -> mirror
    Mirror scratch;                                   // a cache filled whole by one call (pos 0, seq = max_seq)
    std::vector<std::pair<size_t, float*>> spare;     // evicted mirror buffers, reused by size
    std::unordered_map<const void*, NormW> norms;     // host norm weight pointer -> device copy
    float* arena = nullptr;
    size_t arena_floats = 0;
    float* dit_arena = nullptr;  // the LocDiT sampler's resident buffers
    size_t dit_arena_floats = 0;
    float* h_stage = nullptr;  // pinned
    size_t h_stage_floats = 0;
    float* attn_part = nullptr;  // key-split partials of the tiled attention
    size_t attn_part_floats = 0;
    // the last mask uploaded by a non-graph call, kept on the device while the
    // host rows stay equal (the engine builds one mask per forward and passes it
    // to every layer)
    float* mask_dev = nullptr;
    size_t mask_dev_floats = 0;
    std::vector<float> mask_host;
    int mask_rows = 0, mask_cols = 0;
    uint64_t clock = 0;
    // CUDA graphs of repeated fill calls (pos 0, seq = cache length: the LocDiT's
    // per-forward blocks), keyed by every pointer and size the launches bake in;
    // a key is captured the second time it is seen
    std::map<std::vector<uint64_t>, cudaGraphExec_t> graphs;
    std::map<std::vector<uint64_t>, int> seen;
};
constexpr size_t kMaxGraphs = 96;

constexpr int kMaxMirrors = 192;
std::mutex g_blk_mu;
BlockDev g_blk[16];

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

void spare_put(BlockDev& bd, size_t floats, float* p) {
    bd.spare.push_back({floats, p});
    if (bd.spare.size() > 64) {  // keep the spare list short
        cudaFree(bd.spare.front().second);
        bd.spare.erase(bd.spare.begin());
    }
}

float* dev_alloc(BlockDev& bd, size_t floats) {
    for (size_t i = 0; i < bd.spare.size(); i++) {
        if (bd.spare[i].first == floats) {
            float* p = bd.spare[i].second;
            bd.spare.erase(bd.spare.begin() + (long)i);
            return p;
        }
    }
    float* p = nullptr;
    if (cudaMalloc(&p, floats * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return p;
}

// Grows a device or pinned buffer (old contents dropped).  The stream is
// drained first: queued work may still use the old buffer.
bool grow(float** p, size_t* have, size_t want, bool pinned, cudaStream_t st) {
    if (*have >= want) return true;
    size_t n = 1 << 16;
    while (n < want) n <<= 1;
    cudaStreamSynchronize(st);
    if (*p) pinned ? cudaFreeHost(*p) : cudaFree(*p);
    *p = nullptr;
    *have = 0;
    const cudaError_t e = pinned ? cudaMallocHost(p, n * sizeof(float)) : cudaMalloc(p, n * sizeof(float));
    if (e != cudaSuccess) {
        cudaGetLastError();
        *p = nullptr;
        return false;
    }
    *have = n;
    return true;
}

// Device copy of a host norm weight (fp32 or fp16), cached by pointer and fingerprint.
VoxCPMError norm_weight(BlockDev& bd, const Tensor* t, cudaStream_t st, const float** out) {
    *out = nullptr;
    if (!t) return VOXCPM_SUCCESS;
    if (t->is_cuda) return VOXCPM_ERR_CUDA_NOT_FOUND;
    const void* key = t->is_fp16 ? (const void*)t->data_fp16 : (const void*)t->data;
    if (!key) return VOXCPM_ERR_CUDA_NOT_FOUND;
    std::vector<float> host(t->size);
    for (size_t i = 0; i < t->size; i++) host[i] = t->is_fp16 ? half_to_float(t->data_fp16[i]) : t->data[i];
    const uint64_t fp = fingerprint(host.data(), host.size());
    auto it = bd.norms.find(key);
    if (it != bd.norms.end() && it->second.n == t->size && it->second.fp == fp) {
        *out = it->second.p;
        return VOXCPM_SUCCESS;
    }
    float* d = nullptr;
    VOXQ_CUDA_TRY(cudaMalloc(&d, t->size * sizeof(float)));
    VOXQ_CUDA_TRY(cudaMemcpyAsync(d, host.data(), t->size * sizeof(float), cudaMemcpyHostToDevice, st));
    VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
    if (it != bd.norms.end()) cudaFree(it->second.p);
    bd.norms[key] = NormW{d, t->size, fp};
    *out = d;
    return VOXCPM_SUCCESS;
}

// The mirror of a host cache, made valid for rows [0, pos).
VoxCPMError mirror_for(BlockDev& bd, Tensor* ck, Tensor* cv, int BK, int max_seq, int hd, int pos, bool seq_fills,
                       cudaStream_t st, Mirror** out) {
    *out = nullptr;
    const size_t floats = (size_t)BK * max_seq * hd;
    if (pos == 0 && seq_fills) {  // the call writes the whole cache: no state to keep
        Mirror& m = bd.scratch;
        if (m.floats < floats) {
            cudaStreamSynchronize(st);
            if (m.k) cudaFree(m.k);
            if (m.v) cudaFree(m.v);
            m.k = m.v = nullptr;
            m.floats = 0;
            VOXQ_CUDA_TRY(cudaMalloc(&m.k, floats * sizeof(float)));
            VOXQ_CUDA_TRY(cudaMalloc(&m.v, floats * sizeof(float)));
            m.floats = floats;
        }
        m.BK = BK;
        m.max_seq = max_seq;
        m.hd = hd;
        m.valid = 0;
        *out = &m;
        return VOXCPM_SUCCESS;
    }
    auto it = bd.mirrors.find(ck->data);
    if (it != bd.mirrors.end() && (it->second.floats != floats || it->second.hd != hd || it->second.BK != BK)) {
        spare_put(bd, it->second.floats, it->second.k);
        spare_put(bd, it->second.floats, it->second.v);
        bd.mirrors.erase(it);
        it = bd.mirrors.end();
    }
    if (it == bd.mirrors.end()) {
        if (bd.mirrors.size() >= (size_t)kMaxMirrors) {  // evict the least recently used
            auto lru = bd.mirrors.begin();
            for (auto m = bd.mirrors.begin(); m != bd.mirrors.end(); ++m)
                if (m->second.used < lru->second.used) lru = m;
            spare_put(bd, lru->second.floats, lru->second.k);
            spare_put(bd, lru->second.floats, lru->second.v);
            bd.mirrors.erase(lru);
        }
        Mirror m;
        m.k = dev_alloc(bd, floats);
        m.v = dev_alloc(bd, floats);
        if (!m.k || !m.v) return VOXCPM_ERR_OOM;
        m.floats = floats;
        m.BK = BK;
        m.max_seq = max_seq;
        m.hd = hd;
        it = bd.mirrors.emplace(ck->data, std::move(m)).first;
    }
    Mirror& m = it->second;
    m.used = ++bd.clock;
    if (pos == 0) m.valid = 0;
    if (m.valid > pos) m.valid = pos;
    // the host row the mirror last wrote must still be there
    if (m.valid > 0) {
        const float* hrow = ck->data + (size_t)(m.valid - 1) * hd;
        if ((int)m.last_row.size() != hd || memcmp(hrow, m.last_row.data(), (size_t)hd * sizeof(float)) != 0)
            m.valid = 0;
    }
    if (m.valid < pos) {  // rows [valid, pos) from the host cache
        const int r0 = m.valid, rows = pos - r0;
        const size_t n = (size_t)BK * rows * hd;
        if (!grow(&bd.h_stage, &bd.h_stage_floats, 2 * n, true, st)) return VOXCPM_ERR_OOM;
        for (int kv = 0; kv < 2; kv++) {
            const float* src = kv ? cv->data : ck->data;
            float* stage = bd.h_stage + kv * n;
            for (int bk = 0; bk < BK; bk++)
                memcpy(stage + (size_t)bk * rows * hd, src + ((size_t)bk * max_seq + r0) * hd,
                       (size_t)rows * hd * sizeof(float));
        }
        float* tmp = dev_alloc(bd, 2 * n);
        if (!tmp) return VOXCPM_ERR_OOM;
        VOXQ_CUDA_TRY(cudaMemcpyAsync(tmp, bd.h_stage, 2 * n * sizeof(float), cudaMemcpyHostToDevice, st));
        const int grid = (int)((n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024);
        cache_fill_kernel<<<grid, 256, 0, st>>>(tmp, m.k, BK, rows, hd, max_seq, r0);
        cache_fill_kernel<<<grid, 256, 0, st>>>(tmp + n, m.v, BK, rows, hd, max_seq, r0);
        VOXQ_CUDA_TRY(cudaGetLastError());
        VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
        cudaFree(tmp);  // rare: a cache the mirror cannot vouch for
        m.valid = pos;
        m.last_row.assign(ck->data + (size_t)(pos - 1) * hd, ck->data + (size_t)pos * hd);
    }
    *out = &m;
    return VOXCPM_SUCCESS;
}

bool is_host_f32(const Tensor* t) { return t && t->data && !t->is_cuda && !t->is_fp16; }

// Tensor-core attention for many query rows (attn_mma_kernel) unless
// VOXQ_ATTN_MMA=0 selects the CUDA-core kernel (attn_tiled_kernel).
bool attn_mma_enabled() {
    static const bool v = [] {
        const char* e = getenv("VOXQ_ATTN_MMA");
        return !(e && e[0] == '0');
    }();
    return v;
}

// attn_mma_kernel needs more than the default 48 KB of dynamic shared memory
// (68 KB at head_dim 128); the opt-in is a per-device function attribute.
cudaError_t attn_mma_prepare() {
    static std::mutex mu;
    static bool done[16] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(mu);
    if (dev >= 0 && dev < 16 && done[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(attn_mma_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             attn_mma_smem_bytes<128>());
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attn_mma_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 attn_mma_smem_bytes<64>());
    if (e == cudaSuccess && dev >= 0 && dev < 16) done[dev] = true;
    return e;
}

VoxCPMError project(const float* a, int M, int K, const voxq_qweight& w, float* out, const float* residual,
                    const voxq_qweight* up, cudaStream_t st) {
    voxq_epilogue epi = {nullptr, residual, w.N, up};
    return voxq_matmul_nt_q(a, M, K, &w, out, w.N, (residual || up) ? &epi : nullptr, st);
}

// A block's resolved weights: the seven projections (quantized device
// weights) and the two norm weights (device copies).
struct BlockW {
    voxq_qweight wq, wk, wv, wo, w1, w2, w3;
    const float* wn1 = nullptr;
    const float* wn2 = nullptr;
    float eps1 = 0.f, eps2 = 0.f;
    int D = 0, H = 0, KVH = 0, hd = 0, F = 0;
};

// false: not a block the device path takes (the caller runs the host code).
bool block_weights(const voxq_block_desc* blk, BlockW* w) {
    if (!blk || !blk->rms_attn || !blk->attn || !blk->rms_ffn || !blk->ffn) return false;
    const voxq_attention_desc& at = *blk->attn;
    const voxq_swiglu_desc& ff = *blk->ffn;
    w->D = at.d_model;
    w->H = at.n_heads;
    w->KVH = at.n_kv_heads;
    w->hd = at.head_dim;
    w->F = ff.d_ff;
    if (w->D != ff.d_model || w->H < 1 || w->KVH < 1 || w->H % w->KVH || w->hd < 4 || w->hd % 4 ||
        w->hd > kMaxHeadDim)
        return false;
    if (!device_qweight(at.wq, &w->wq) || !device_qweight(at.wk, &w->wk) || !device_qweight(at.wv, &w->wv) ||
        !device_qweight(at.wo, &w->wo) || !device_qweight(ff.w1, &w->w1) || !device_qweight(ff.w2, &w->w2) ||
        !device_qweight(ff.w3, &w->w3))
        return false;
    const int D = w->D, qk = w->H * w->hd, kv = w->KVH * w->hd, F = w->F;
    if (w->wq.N != qk || w->wq.K != D || w->wk.N != kv || w->wk.K != D || w->wv.N != kv || w->wv.K != D ||
        w->wo.N != D || w->wo.K != qk || w->w1.N != F || w->w1.K != D || w->w3.N != F || w->w3.K != D ||
        w->w2.N != D || w->w2.K != F || w->w1.qtype != w->w3.qtype || w->w1.q8_signed != w->w3.q8_signed)
        return false;
    w->eps1 = blk->rms_attn->eps;
    w->eps2 = blk->rms_ffn->eps;
    return true;
}

VoxCPMError block_norms(BlockDev& bd, const voxq_block_desc* blk, BlockW* w, cudaStream_t st) {
    VoxCPMError e = norm_weight(bd, blk->rms_attn->weight, st, &w->wn1);
    if (!e) e = norm_weight(bd, blk->rms_ffn->weight, st, &w->wn2);
    return e;
}

uint64_t block_weight_bytes(const BlockW& w) {
    uint64_t wb = 0;
    for (const voxq_qweight* q : {&w.wq, &w.wk, &w.wv, &w.wo, &w.w1, &w.w2, &w.w3})
        wb += voxq_codes_bytes(q->N, q->K, q->qtype) + voxq_scales_bytes(q->N, q->K, q->qtype);
    return wb;
}

inline size_t al64(size_t n) { return (n + 63) & ~(size_t)63; }  // 256-byte aligned parts

// The block's intermediate activations for M rows.
struct Scratch {
    float *n, *q, *k, *v, *qr, *ao, *h, *n2, *g;
};
size_t scratch_floats(int M, const BlockW& w) {
    const size_t nx = (size_t)M * w.D, nq = (size_t)M * w.H * w.hd, nk = (size_t)M * w.KVH * w.hd;
    return 3 * al64(nx) + 3 * al64(nq) + 2 * al64(nk) + al64((size_t)M * w.F);
}
Scratch scratch_at(float* p, int M, const BlockW& w) {
    const size_t nx = (size_t)M * w.D, nq = (size_t)M * w.H * w.hd, nk = (size_t)M * w.KVH * w.hd;
    Scratch s;
    s.n = p;
    s.q = s.n + al64(nx);
    s.k = s.q + al64(nq);
    s.v = s.k + al64(nk);
    s.qr = s.v + al64(nk);
    s.ao = s.qr + al64(nq);
    s.h = s.ao + al64(nq);
    s.n2 = s.h + al64(nx);
    s.g = s.n2 + al64(nx);
    return s;
}

// Enqueues the block on device rows: x [B*seq][D] -> out [B*seq][D] (out may
// be x).  K/V rows go into the mirror at [pos, pos + seq) and, when kn / vn
// are given, into them ([B][KVH][seq][hd], for the host write-back).
VoxCPMError block_core(const BlockW& w, const Scratch& sc, const float* d_x, float* d_o, int B, int seq,
                       const Mirror* mr, int max_seq, int pos, const float* d_mask, int mrows, int mcols,
                       const float* d_freqs, float* d_kn, float* d_vn, cudaStream_t st, float* part_buf = nullptr,
                       size_t part_floats = 0) {
    const int M = B * seq, D = w.D, H = w.H, KVH = w.KVH, hd = w.hd, F = w.F, qk = H * hd, L = pos + seq;
    VoxCPMError e = VOXCPM_SUCCESS;
    // n = RMSNorm(x)
    rmsnorm_kernel<<<M, kBlockThreads, 0, st>>>(d_x, w.wn1, w.eps1, sc.n, D);
    VOXQ_CUDA_TRY(cudaGetLastError());
    // q, k, v
    if (M <= 8) {
        voxq_gemv_item it[3] = {};
        const voxq_qweight* ws[3] = {&w.wq, &w.wk, &w.wv};
        float* outs[3] = {sc.q, sc.k, sc.v};
        for (int i = 0; i < 3; i++) {
            it[i].w = *ws[i];
            it[i].a = sc.n;
            it[i].out = outs[i];
            it[i].M = M;
            it[i].lda = D;
            it[i].ldo = ws[i]->N;
        }
        e = voxq_gemv_batch(it, 3, st);
    } else {
        e = project(sc.n, M, D, w.wq, sc.q, nullptr, nullptr, st);
        if (!e) e = project(sc.n, M, D, w.wk, sc.k, nullptr, nullptr, st);
        if (!e) e = project(sc.n, M, D, w.wv, sc.v, nullptr, nullptr, st);
    }
    if (e) return e;
    // RoPE, cache rows [pos, pos + seq)
    rope_cache_kernel<<<dim3(M, H + 2 * KVH), 64, 0, st>>>(sc.q, sc.k, sc.v, d_freqs, sc.qr, mr->k, mr->v, d_kn, d_vn,
                                                          seq, H, KVH, hd, max_seq, pos);
    VOXQ_CUDA_TRY(cudaGetLastError());
    // attention over [0, L)
    const int smem = (kMaxHeadDim + L) * (int)sizeof(float);
    static std::once_flag once;
    std::call_once(once, [] {
        cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (kMaxHeadDim + kMaxCacheLen) * (int)sizeof(float));
    });
    const int G = H / KVH;
    const float inv_scale = 1.0f / sqrtf((float)hd);
    if (seq * G >= 64 && 64 % G == 0 && (hd == 64 || hd == 128)) {
        // many query rows: tiled, key / value tiles shared by 64 query vectors; a call that
        // continues a long cache (pos > 0) with too few query tiles to fill the GPU also splits
        // the keys (at least 8 tiles each) and combines the splits in a second kernel
        const int nqt = (seq + 64 / G - 1) / (64 / G), ctas = nqt * KVH * B;
        int nsplit = 1;
        if (pos > 0 && part_buf) {
            const int want = (2 * device_sm_count() + ctas - 1) / ctas, most = (L + 8 * kFK - 1) / (8 * kFK);
            nsplit = std::max(1, std::min(std::min(want, most), 64));
            if ((size_t)ctas * nsplit * 64 * (hd + 2) > part_floats) nsplit = 1;
        }
        const dim3 grid((unsigned)(nqt * nsplit), (unsigned)KVH, (unsigned)B);
        if (attn_mma_enabled()) {
            // both products on the tensor cores (split TF32), same grid and partial records
            VOXQ_CUDA_TRY(attn_mma_prepare());
            if (hd == 128)
                attn_mma_kernel<128><<<grid, kMThreads, attn_mma_smem_bytes<128>(), st>>>(
                    sc.qr, mr->k, mr->v, d_mask, mrows, mcols, sc.ao, seq, H, KVH, max_seq, L, inv_scale, nsplit,
                    part_buf);
            else
                attn_mma_kernel<64><<<grid, kMThreads, attn_mma_smem_bytes<64>(), st>>>(
                    sc.qr, mr->k, mr->v, d_mask, mrows, mcols, sc.ao, seq, H, KVH, max_seq, L, inv_scale, nsplit,
                    part_buf);
        } else if (hd == 128) {
            attn_tiled_kernel<128><<<grid, kFThreads, 0, st>>>(sc.qr, mr->k, mr->v, d_mask, mrows, mcols, sc.ao, seq,
                                                                H, KVH, max_seq, L, inv_scale, nsplit, part_buf);
        } else {
            attn_tiled_kernel<64><<<grid, kFThreads, 0, st>>>(sc.qr, mr->k, mr->v, d_mask, mrows, mcols, sc.ao, seq, H,
                                                               KVH, max_seq, L, inv_scale, nsplit, part_buf);
        }
        if (nsplit > 1) {
            VOXQ_CUDA_TRY(cudaGetLastError());
            const int64_t threads = (int64_t)ctas * 64 * 32;
            const int blocks = (int)((threads + 255) / 256);
            if (hd == 128)
                attn_combine_kernel<128><<<blocks, 256, 0, st>>>(part_buf, sc.ao, seq, H, KVH, B, nqt, nsplit);
            else
                attn_combine_kernel<64><<<blocks, 256, 0, st>>>(part_buf, sc.ao, seq, H, KVH, B, nqt, nsplit);
        }
    } else {
        attn_kernel<<<dim3(seq, H, B), kAttnThreads, smem, st>>>(sc.qr, mr->k, mr->v, d_mask, mrows, mcols, sc.ao, seq,
                                                                H, KVH, hd, max_seq, L, inv_scale);
    }
    VOXQ_CUDA_TRY(cudaGetLastError());
    // h = x + a Wo^T ; n2 = RMSNorm(h) ; g = silu(n2 W1^T) * (n2 W3^T) ; o = h + g W2^T
    e = project(sc.ao, M, qk, w.wo, sc.h, d_x, nullptr, st);
    if (e) return e;
    rmsnorm_kernel<<<M, kBlockThreads, 0, st>>>(sc.h, w.wn2, w.eps2, sc.n2, D);
    VOXQ_CUDA_TRY(cudaGetLastError());
    e = project(sc.n2, M, D, w.w1, sc.g, nullptr, &w.w3, st);
    if (!e) e = project(sc.g, M, F, w.w2, d_o, sc.h, nullptr, st);
    return e;
}

}  // namespace

void block_cache_clear() {
    std::lock_guard<std::mutex> lk(g_blk_mu);
    for (BlockDev& bd : g_blk) {
        for (auto& m : bd.mirrors) {
            cudaFree(m.second.k);
            cudaFree(m.second.v);
        }
        for (auto& s : bd.spare) cudaFree(s.second);
        for (auto& n : bd.norms) cudaFree(n.second.p);
        for (auto& g : bd.graphs) cudaGraphExecDestroy(g.second);
        if (bd.scratch.k) cudaFree(bd.scratch.k);
        if (bd.scratch.v) cudaFree(bd.scratch.v);
        if (bd.arena) cudaFree(bd.arena);
        if (bd.dit_arena) cudaFree(bd.dit_arena);
        if (bd.h_stage) cudaFreeHost(bd.h_stage);
        if (bd.attn_part) cudaFree(bd.attn_part);
        if (bd.mask_dev) cudaFree(bd.mask_dev);
        bd = BlockDev();
    }
}

}  // namespace voxq

using namespace voxq;

extern "C" VoxCPMError voxq_transformer_block_forward(const voxq_block_desc* blk, const Tensor* x, Tensor* cache_k,
                                                      Tensor* cache_v, const Tensor* mask, const Tensor* freqs_cis,
                                                      int pos, Tensor* out) {
    constexpr VoxCPMError kHost = VOXCPM_ERR_CUDA_NOT_FOUND;  // "run the host code instead"
    if (!x || !out || !cache_k || !cache_v) return kHost;
    cudaStream_t st = (cudaStream_t)library_stream();
    if (!st) return kHost;
    BlockW w;
    if (!block_weights(blk, &w)) return kHost;
    // shapes the kernels take; anything else (including the reference's own
    // shape errors) goes to the host code
    if (!is_host_f32(x) || !is_host_f32(out) || x->ndim != 3 || out->ndim != 3) return kHost;
    const int B = x->shape[0], seq = x->shape[1], D = x->shape[2];
    if (out->shape[0] != B || out->shape[1] != seq || out->shape[2] != D || B < 1 || seq < 1 || D != w.D)
        return kHost;
    const int KVH = w.KVH, hd = w.hd;
    if (!is_host_f32(cache_k) || !is_host_f32(cache_v) || cache_k->ndim != 4 || cache_v->ndim != 4) return kHost;
    const int max_seq = cache_k->shape[2];
    for (int i = 0; i < 4; i++)
        if (cache_v->shape[i] != cache_k->shape[i]) return kHost;
    if (cache_k->shape[0] != B || cache_k->shape[1] != KVH || cache_k->shape[3] != hd) return kHost;
    const int L = pos + seq;  // cache length after this call
    if (pos < 0 || L > max_seq || L > kMaxCacheLen) return kHost;
    if (mask && (!is_host_f32(mask) || mask->ndim != 2)) return kHost;
    const int half = hd / 2;
    if (freqs_cis && (!is_host_f32(freqs_cis) || freqs_cis->size < (size_t)L * half * 2)) return kHost;
    const int kv = KVH * hd, M = B * seq;
    const int dev = current_device();
    if (dev < 0 || dev >= 16) return kHost;

    std::lock_guard<std::mutex> lk(g_blk_mu);
    BlockDev& bd = g_blk[dev];
    VoxCPMError e = block_norms(bd, blk, &w, st);
    if (e) return e;

    // device arena: x | block scratch | out | new K rows | new V rows | freqs rows | mask rows
    const int mcols = mask ? (mask->shape[1] < L ? mask->shape[1] : L) : 0;
    const int mrows = mask ? (mask->shape[0] < seq ? mask->shape[0] : seq) : 0;
    const size_t nx = (size_t)M * D, nk = (size_t)M * kv;
    const size_t nf = freqs_cis ? (size_t)seq * half * 2 : 0, nm = (size_t)mrows * mcols;
    const size_t off_s = al64(nx), off_o = off_s + scratch_floats(M, w), off_kn = off_o + al64(nx),
                 off_vn = off_kn + al64(nk), off_f = off_vn + al64(nk), off_m = off_f + al64(nf),
                 total = off_m + al64(nm);
    if (!grow(&bd.arena, &bd.arena_floats, total, false, st)) return VOXCPM_ERR_OOM;
    // pinned staging: uploads x | freqs rows | mask rows, downloads out | knew | vnew
    const size_t up_n = al64(nx) + al64(nf) + al64(nm), down_n = al64(nx) + 2 * al64(nk);
    if (!grow(&bd.h_stage, &bd.h_stage_floats, up_n + down_n, true, st)) return VOXCPM_ERR_OOM;

    Mirror* mr = nullptr;
    e = mirror_for(bd, cache_k, cache_v, B * KVH, max_seq, hd, pos, seq == max_seq, st, &mr);
    if (e) return e;
    // key-split partials for a continuation of a long cache through the tiled attention
    const bool graph_call = pos == 0 && seq == max_seq;
    if (pos > 0) {
        const int G = w.H / KVH;
        if (seq * G >= 64 && 64 % G == 0 && (hd == 64 || hd == 128)) {
            const size_t ctas = (size_t)((seq + 64 / G - 1) / (64 / G)) * KVH * B;
            if (!grow(&bd.attn_part, &bd.attn_part_floats, (ctas + 2 * (size_t)device_sm_count()) * 64 * (hd + 2),
                      false, st))
                return VOXCPM_ERR_OOM;
        }
    }
    // mask rows: outside graph calls, re-uploaded only when they differ from the last upload
    const bool mask_cached = nm && !graph_call;
    bool mask_upload = false;
    if (mask_cached) {
        bool same = bd.mask_dev && bd.mask_rows == mrows && bd.mask_cols == mcols;
        for (int r = 0; same && r < mrows; r++)
            same = memcmp(bd.mask_host.data() + (size_t)r * mcols, mask->data + (size_t)r * mask->shape[1],
                          (size_t)mcols * sizeof(float)) == 0;
        if (!same) {
            if (!grow(&bd.mask_dev, &bd.mask_dev_floats, nm, false, st)) return VOXCPM_ERR_OOM;
            bd.mask_host.resize(nm);
            for (int r = 0; r < mrows; r++)
                memcpy(bd.mask_host.data() + (size_t)r * mcols, mask->data + (size_t)r * mask->shape[1],
                       (size_t)mcols * sizeof(float));
            bd.mask_rows = mrows;
            bd.mask_cols = mcols;
            mask_upload = true;
        }
    }

    float* A = bd.arena;
    float *d_x = A, *d_o = A + off_o, *d_kn = A + off_kn, *d_vn = A + off_vn, *d_f = A + off_f, *d_m = A + off_m;
    const float* d_mask = nm ? (mask_cached ? bd.mask_dev : d_m) : nullptr;
    const Scratch sc = scratch_at(A + off_s, M, w);
    float* hs = bd.h_stage;
    memcpy(hs, x->data, nx * sizeof(float));
    if (nf) memcpy(hs + al64(nx), freqs_cis->data + (size_t)pos * half * 2, nf * sizeof(float));
    if (mask_upload)
        memcpy(hs + al64(nx) + al64(nf), bd.mask_host.data(), nm * sizeof(float));
    else if (nm && !mask_cached)
        for (int r = 0; r < mrows; r++)
            memcpy(hs + al64(nx) + al64(nf) + (size_t)r * mcols, mask->data + (size_t)r * mask->shape[1],
                   (size_t)mcols * sizeof(float));
    float* hd_out = hs + up_n;
    // everything from the upload to the downloads, on `st`
    auto enqueue = [&]() -> VoxCPMError {
        VOXQ_CUDA_TRY(cudaMemcpyAsync(d_x, hs, nx * sizeof(float), cudaMemcpyHostToDevice, st));
        if (nf) VOXQ_CUDA_TRY(cudaMemcpyAsync(d_f, hs + al64(nx), nf * sizeof(float), cudaMemcpyHostToDevice, st));
        if (nm && (!mask_cached || mask_upload))
            VOXQ_CUDA_TRY(cudaMemcpyAsync(mask_cached ? bd.mask_dev : d_m, hs + al64(nx) + al64(nf),
                                          nm * sizeof(float), cudaMemcpyHostToDevice, st));
        const VoxCPMError ce = block_core(w, sc, d_x, d_o, B, seq, mr, max_seq, pos, d_mask, mrows, mcols,
                                          nf ? d_f : nullptr, d_kn, d_vn, st, bd.attn_part, bd.attn_part_floats);
        if (ce) return ce;
        // downloads: out, new cache rows (the caller waits once)
        VOXQ_CUDA_TRY(cudaMemcpyAsync(hd_out, d_o, nx * sizeof(float), cudaMemcpyDeviceToHost, st));
        VOXQ_CUDA_TRY(cudaMemcpyAsync(hd_out + al64(nx), d_kn, nk * sizeof(float), cudaMemcpyDeviceToHost, st));
        VOXQ_CUDA_TRY(cudaMemcpyAsync(hd_out + al64(nx) + al64(nk), d_vn, nk * sizeof(float), cudaMemcpyDeviceToHost,
                                      st));
        return VOXCPM_SUCCESS;
    };
    // A fill call (the whole cache written at pos 0) repeats with identical
    // pointers and sizes (the LocDiT runs 12 blocks x 20 forwards per patch):
    // its launches are captured once into a CUDA graph and replayed.
    if (pos == 0 && seq == max_seq) {
        std::vector<uint64_t> key = {(uint64_t)(uintptr_t)blk, (uint64_t)B, (uint64_t)seq, (uint64_t)D,
                                     (uint64_t)(uintptr_t)mr->k, (uint64_t)(uintptr_t)mr->v,
                                     (uint64_t)(uintptr_t)bd.arena, (uint64_t)(uintptr_t)bd.h_stage,
                                     (uint64_t)(uintptr_t)w.wn1, (uint64_t)(uintptr_t)w.wn2,
                                     (uint64_t)mrows, (uint64_t)mcols, (uint64_t)nf};
        uint32_t eb[2];
        memcpy(&eb[0], &w.eps1, 4);
        memcpy(&eb[1], &w.eps2, 4);
        key.push_back(((uint64_t)eb[0] << 32) | eb[1]);
        for (const voxq_qweight* q : {&w.wq, &w.wk, &w.wv, &w.wo, &w.w1, &w.w2, &w.w3}) {
            key.push_back((uint64_t)(uintptr_t)q->codes);
            key.push_back((uint64_t)(uintptr_t)q->scales);
        }
        auto g = bd.graphs.find(key);
        if (g != bd.graphs.end()) {
            VOXQ_CUDA_TRY(cudaGraphLaunch(g->second, st));
        } else if (bd.seen[key]++ >= 1 && bd.graphs.size() < kMaxGraphs) {
            cudaGraph_t graph = nullptr;
            cudaGraphExec_t exec = nullptr;
            bool ok = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
            const VoxCPMError ce = ok ? enqueue() : VOXCPM_ERR_INTERNAL;
            if (ok) ok = cudaStreamEndCapture(st, &graph) == cudaSuccess && ce == VOXCPM_SUCCESS;
            if (ok) ok = cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
            if (graph) cudaGraphDestroy(graph);
            cudaGetLastError();
            if (ok) {
                bd.graphs[key] = exec;
                VOXQ_CUDA_TRY(cudaGraphLaunch(exec, st));
            } else {  // not capturable here: plain launches
                if (exec) cudaGraphExecDestroy(exec);
                e = enqueue();
                if (e) return e;
            }
        } else {
            e = enqueue();
            if (e) return e;
        }
    } else {
        e = enqueue();
        if (e) return e;
    }
    VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
    memcpy(out->data, hd_out, nx * sizeof(float));
    for (int kvs = 0; kvs < 2; kvs++) {
        const float* src = hd_out + al64(nx) + kvs * al64(nk);
        float* dst = kvs ? cache_v->data : cache_k->data;
        for (int bk = 0; bk < B * KVH; bk++)
            memcpy(dst + ((size_t)bk * max_seq + pos) * hd, src + (size_t)bk * seq * hd, (size_t)seq * hd * sizeof(float));
    }
    count_matmul_traffic(7, block_weight_bytes(w));
    mr->valid = L;
    mr->last_row.assign(cache_k->data + (size_t)(L - 1) * hd, cache_k->data + (size_t)L * hd);
    return VOXCPM_SUCCESS;
}

namespace voxq {
namespace {

// Sinusoidal embedding of the reference (src/loc_dit.c:35-50): row[2i] =
// sin(t f_i), row[2i + 1] = cos(t f_i), f_i = 1 / 10000^(2i / D), on the host
// with the same libm calls.
void sinusoidal(float t, int D, float* row) {
    const int half = D / 2;
    for (int i = 0; i < half; i++) {
        const float inv_freq = 1.0f / powf(10000.0f, 2.0f * (float)i / (float)D);
        const float val = t * inv_freq;
        row[2 * i] = sinf(val);
        row[2 * i + 1] = cosf(val);
    }
}

int ew(int n) { return (n + 255) / 256 > 0 ? (n + 255) / 256 : 1; }

}  // namespace
}  // namespace voxq

extern "C" VoxCPMError voxq_locdit_sample(const voxq_locdit_desc* dit, const Tensor* mu, const Tensor* cond,
                                          int n_timesteps, float cfg_value, const Tensor* x_init, Tensor* out) {
    constexpr VoxCPMError kHost = VOXCPM_ERR_CUDA_NOT_FOUND;
    if (!dit || !mu || !cond || !x_init || !out || n_timesteps < 1 || !dit->layers || dit->n_layers < 1 ||
        !dit->output_norm)
        return kHost;
    cudaStream_t st = (cudaStream_t)library_stream();
    if (!st) return kHost;
    const int D = dit->d_model, F = dit->feat_dim;
    if (!is_host_f32(mu) || mu->ndim != 2 || mu->shape[0] != 1 || mu->shape[1] != D) return kHost;
    if (!is_host_f32(out) || out->ndim != 3 || out->shape[0] != 1 || out->shape[1] != F) return kHost;
    const int P = out->shape[2];
    if (!is_host_f32(x_init) || x_init->ndim != 3 || x_init->shape[0] != 1 || x_init->shape[1] != F ||
        x_init->shape[2] != P || P < 1)
        return kHost;
    if (cond->ndim != 3 || cond->shape[0] != 1 || cond->shape[1] != F || cond->is_cuda || cond->is_fp16) return kHost;
    const int Tc = cond->shape[2];
    if (Tc > 0 && !cond->data) return kHost;
    if (cfg_value < 0.0f) cfg_value = 0.0f;
    const int nb = (cfg_value > 1.0f && Tc > 0) ? 2 : 1;
    const int S = 1 + P + Tc, M = nb * S;
    // weights
    voxq_qweight win, wc, wout, wt1, wt2, wd1, wd2;
    if (!device_qweight(dit->in_proj_weight, &win) || !device_qweight(dit->out_proj_weight, &wout) ||
        !device_qweight(dit->time_mlp_1_weight, &wt1) || !device_qweight(dit->time_mlp_2_weight, &wt2) ||
        !device_qweight(dit->delta_mlp_1_weight, &wd1) || !device_qweight(dit->delta_mlp_2_weight, &wd2))
        return kHost;
    if (Tc > 0 && !device_qweight(dit->cond_proj_weight, &wc)) return kHost;
    if (win.N != D || win.K != F || wout.N != F || wout.K != D || wt1.N != D || wt1.K != D || wt2.N != D ||
        wt2.K != D || wd1.N != D || wd1.K != D || wd2.N != D || wd2.K != D || (Tc > 0 && (wc.N != D || wc.K != F)))
        return kHost;
    std::vector<BlockW> bw(dit->n_layers);
    for (int l = 0; l < dit->n_layers; l++) {
        if (!block_weights(&dit->layers[l], &bw[l]) || bw[l].D != D) return kHost;
        if (S > kMaxCacheLen) return kHost;
    }
    const int dev = current_device();
    if (dev < 0 || dev >= 16) return kHost;

    std::lock_guard<std::mutex> lk(g_blk_mu);
    BlockDev& bd = g_blk[dev];
    VoxCPMError e = VOXCPM_SUCCESS;
    for (int l = 0; l < dit->n_layers; l++) {
        e = block_norms(bd, &dit->layers[l], &bw[l], st);
        if (e) return e;
    }
    // biases and the output norm weight: cached device copies of host tensors
    const float *b_in = nullptr, *b_c = nullptr, *b_out = nullptr, *b_t1 = nullptr, *b_t2 = nullptr,
                *b_d1 = nullptr, *b_d2 = nullptr, *w_on = nullptr;
    const Tensor* bt[8] = {dit->in_proj_bias,  dit->cond_proj_bias,  dit->out_proj_bias,  dit->time_mlp_1_bias,
                           dit->time_mlp_2_bias, dit->delta_mlp_1_bias, dit->delta_mlp_2_bias, dit->output_norm->weight};
    const float** bp[8] = {&b_in, &b_c, &b_out, &b_t1, &b_t2, &b_d1, &b_d2, &w_on};
    for (int i = 0; i < 8; i++) {
        e = norm_weight(bd, bt[i], st, bp[i]);
        if (e) return e;
    }
    // arena: seq | block scratch | K | V | small buffers
    int maxKVH = 0, maxhd = 0;
    size_t scr = 0;
    for (auto& w : bw) {
        maxKVH = std::max(maxKVH, w.KVH);
        maxhd = std::max(maxhd, w.hd);
        scr = std::max(scr, scratch_floats(M, w));
    }
    const size_t nseq = (size_t)M * D, nkv = (size_t)nb * maxKVH * S * maxhd;
    const size_t o_scr = al64(nseq), o_k = o_scr + scr, o_v = o_k + al64(nkv), o_x = o_v + al64(nkv),
                 o_xp = o_x + al64((size_t)F * P), o_xpr = o_xp + al64((size_t)P * F),
                 o_cp = o_xpr + al64((size_t)P * D), o_ct = o_cp + al64((size_t)Tc * F),
                 o_cr = o_ct + al64((size_t)Tc * D), o_mu = o_cr + al64((size_t)Tc * D), o_emb = o_mu + al64((size_t)D),
                 o_hid = o_emb + al64((size_t)D), o_tf = o_hid + al64((size_t)D), o_df = o_tf + al64((size_t)D),
                 o_gc = o_df + al64((size_t)D), o_xs = o_gc + al64((size_t)D), o_vr = o_xs + al64((size_t)nb * P * D),
                 total = o_vr + al64((size_t)nb * P * F);
    if (!grow(&bd.dit_arena, &bd.dit_arena_floats, total, false, st)) return VOXCPM_ERR_OOM;
    const size_t hs_n = (size_t)n_timesteps * 2 * D + (size_t)F * P + (size_t)F * Tc + (size_t)F * P + (size_t)D;
    if (!grow(&bd.h_stage, &bd.h_stage_floats, hs_n, true, st)) return VOXCPM_ERR_OOM;
    float* A = bd.dit_arena;
    float *d_seq = A, *d_k = A + o_k, *d_v = A + o_v, *d_x = A + o_x, *d_xperm = A + o_xp, *d_xproj = A + o_xpr,
          *d_cperm = A + o_cp, *d_cond = A + o_ct, *d_crows = A + o_cr, *d_emb = A + o_emb, *d_hid = A + o_hid,
          *d_tf = A + o_tf, *d_df = A + o_df, *d_gc = A + o_gc, *d_xs = A + o_xs, *d_vr = A + o_vr,
          *d_mu = A + o_mu;
    // host side: every step's two embeddings, x_init, cond
    float* hs = bd.h_stage;
    const float sigma_min = 1e-6f;
    const float dt = (1.0f - sigma_min) / (float)n_timesteps;
    for (int i = 0; i < n_timesteps; i++) {
        const float t_cur = 1.0f - (float)i * dt;
        sinusoidal(t_cur, D, hs + (size_t)i * 2 * D);
        sinusoidal(dt, D, hs + (size_t)i * 2 * D + D);
    }
    float* h_x = hs + (size_t)n_timesteps * 2 * D;
    memcpy(h_x, x_init->data, (size_t)F * P * sizeof(float));
    float* h_c = h_x + (size_t)F * P;
    if (Tc > 0) memcpy(h_c, cond->data, (size_t)F * Tc * sizeof(float));
    float* h_out = h_c + (size_t)F * Tc;
    float* h_mu = h_out + (size_t)F * P;
    memcpy(h_mu, mu->data, (size_t)D * sizeof(float));
    // upload: x_init -> d_x, mu -> d_mu, cond -> d_cond (as [F][Tc] then transposed to [Tc][F])
    VOXQ_CUDA_TRY(cudaMemcpyAsync(d_x, h_x, (size_t)F * P * sizeof(float), cudaMemcpyHostToDevice, st));
    VOXQ_CUDA_TRY(cudaMemcpyAsync(d_mu, h_mu, (size_t)D * sizeof(float), cudaMemcpyHostToDevice, st));
    if (Tc > 0) {
        VOXQ_CUDA_TRY(cudaMemcpyAsync(d_cperm, h_c, (size_t)F * Tc * sizeof(float), cudaMemcpyHostToDevice, st));
        transpose_kernel<<<ew(F * Tc), 256, 0, st>>>(d_cperm, d_cond, F, Tc);
        // condition rows [Tc][D] = cond^T Wc^T + bc (constant over the steps)
        voxq_epilogue epi = {b_c, nullptr, 0, nullptr};
        e = voxq_matmul_nt_q(d_cond, Tc, F, &wc, d_crows, D, &epi, st);
        if (e) return e;
    }
    // the scratch K/V of every block: a fresh cache filled whole (pos 0, length S)
    Mirror kvm;
    kvm.k = d_k;
    kvm.v = d_v;
    uint64_t traffic = 0;
    for (int i = 0; i < n_timesteps; i++) {
        // time / delta features: Linear-SiLU-Linear of the step's embeddings
        VOXQ_CUDA_TRY(cudaMemcpyAsync(d_emb, hs + (size_t)i * 2 * D, (size_t)D * sizeof(float),
                                      cudaMemcpyHostToDevice, st));
        voxq_epilogue e1 = {b_t1, nullptr, 0, nullptr}, e2 = {b_t2, nullptr, 0, nullptr};
        e = voxq_matmul_nt_q(d_emb, 1, D, &wt1, d_hid, D, &e1, st);
        if (e) return e;
        silu_inplace_kernel<<<ew(D), 256, 0, st>>>(d_hid, D);
        e = voxq_matmul_nt_q(d_hid, 1, D, &wt2, d_tf, D, &e2, st);
        if (e) return e;
        VOXQ_CUDA_TRY(cudaMemcpyAsync(d_emb, hs + (size_t)i * 2 * D + D, (size_t)D * sizeof(float),
                                      cudaMemcpyHostToDevice, st));
        voxq_epilogue e3 = {b_d1, nullptr, 0, nullptr}, e4 = {b_d2, nullptr, 0, nullptr};
        e = voxq_matmul_nt_q(d_emb, 1, D, &wd1, d_hid, D, &e3, st);
        if (e) return e;
        silu_inplace_kernel<<<ew(D), 256, 0, st>>>(d_hid, D);
        e = voxq_matmul_nt_q(d_hid, 1, D, &wd2, d_df, D, &e4, st);
        if (e) return e;
        add_vec_kernel<<<ew(D), 256, 0, st>>>(d_tf, d_df, d_gc, D);
        // input projection of x_t: [F][P] -> [P][F] -> [P][D] + b_in
        transpose_kernel<<<ew(F * P), 256, 0, st>>>(d_x, d_xperm, F, P);
        voxq_epilogue ei = {b_in, nullptr, 0, nullptr};
        e = voxq_matmul_nt_q(d_xperm, P, F, &win, d_xproj, D, &ei, st);
        if (e) return e;
        // the branches' sequences, the blocks, the x rows, the output norm and projection
        dit_seq_kernel<<<ew((int)std::min<size_t>(nseq, 1 << 20)), 256, 0, st>>>(d_seq, d_mu, d_xproj, d_crows,
                                                                                   b_c, d_gc, nb, P, Tc, D);
        VOXQ_CUDA_TRY(cudaGetLastError());
        for (int l = 0; l < dit->n_layers; l++) {
            const Scratch sc = scratch_at(A + o_scr, M, bw[l]);
            e = block_core(bw[l], sc, d_seq, d_seq, nb, S, &kvm, S, 0, nullptr, 0, 0, nullptr, nullptr, nullptr, st);
            if (e) return e;
            traffic += block_weight_bytes(bw[l]);
        }
        dit_slice_kernel<<<ew(nb * P * D), 256, 0, st>>>(d_seq, d_xs, nb, P, S, D);
        rmsnorm_kernel<<<nb * P, kBlockThreads, 0, st>>>(d_xs, w_on, dit->output_norm->eps, d_xs, D);
        voxq_epilogue eo = {b_out, nullptr, 0, nullptr};
        e = voxq_matmul_nt_q(d_xs, nb * P, D, &wout, d_vr, F, &eo, st);
        if (e) return e;
        dit_step_kernel<<<ew(F * P), 256, 0, st>>>(d_x, d_vr, nb, P, F, cfg_value, dt);
        VOXQ_CUDA_TRY(cudaGetLastError());
    }
    VOXQ_CUDA_TRY(cudaMemcpyAsync(h_out, d_x, (size_t)F * P * sizeof(float), cudaMemcpyDeviceToHost, st));
    VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
    memcpy(out->data, h_out, (size_t)F * P * sizeof(float));
    count_matmul_traffic((uint64_t)n_timesteps * (7 * dit->n_layers + 6) + (Tc > 0 ? 1 : 0), traffic);
    return VOXCPM_SUCCESS;
}

extern "C" VoxCPMError voxq_locenc_forward(const voxq_locenc_desc* enc, const Tensor* audio_feats, Tensor* out) {
    constexpr VoxCPMError kHost = VOXCPM_ERR_CUDA_NOT_FOUND;
    if (!enc || !audio_feats || !out || !enc->layers || enc->n_layers < 1 || !enc->output_norm ||
        !enc->special_token)
        return kHost;
    cudaStream_t st = (cudaStream_t)library_stream();
    if (!st) return kHost;
    const int D = enc->d_model;
    if (!is_host_f32(audio_feats) || audio_feats->ndim != 4 || !is_host_f32(out) || out->ndim != 3) return kHost;
    const int B = audio_feats->shape[0], T = audio_feats->shape[1], P = audio_feats->shape[2],
              F = audio_feats->shape[3];
    if (B < 1 || T < 1 || P < 1 || F < 1 || out->shape[0] != B || out->shape[1] != T || out->shape[2] != D)
        return kHost;
    if (!is_host_f32(enc->special_token) || enc->special_token->size < (size_t)D) return kHost;
    voxq_qweight win;
    if (!device_qweight(enc->in_proj_weight, &win) || win.N != D || win.K != F) return kHost;
    const int S = T * (P + 1), M = B * S;
    if (S > kMaxCacheLen) return kHost;
    std::vector<BlockW> bw(enc->n_layers);
    for (int l = 0; l < enc->n_layers; l++)
        if (!block_weights(&enc->layers[l], &bw[l]) || bw[l].D != D) return kHost;
    const int dev = current_device();
    if (dev < 0 || dev >= 16) return kHost;

    std::lock_guard<std::mutex> lk(g_blk_mu);
    BlockDev& bd = g_blk[dev];
    VoxCPMError e = VOXCPM_SUCCESS;
    for (int l = 0; l < enc->n_layers; l++) {
        e = block_norms(bd, &enc->layers[l], &bw[l], st);
        if (e) return e;
    }
    const float *b_in = nullptr, *d_special = nullptr, *w_on = nullptr;
    e = norm_weight(bd, enc->in_proj_bias, st, &b_in);
    if (!e) e = norm_weight(bd, enc->special_token, st, &d_special);
    if (!e) e = norm_weight(bd, enc->output_norm->weight, st, &w_on);
    if (e) return e;
    // arena: sequence | block scratch | K | V | features | projections | cls rows
    int maxKVH = 0, maxhd = 0;
    size_t scr = 0;
    for (auto& w : bw) {
        maxKVH = std::max(maxKVH, w.KVH);
        maxhd = std::max(maxhd, w.hd);
        scr = std::max(scr, scratch_floats(M, w));
    }
    const size_t nx = (size_t)M * D, nkv = (size_t)B * maxKVH * S * maxhd, nf = (size_t)B * T * P * F,
                 np = (size_t)B * T * P * D, nc = (size_t)B * T * D;
    const size_t o_scr = al64(nx), o_k = o_scr + scr, o_v = o_k + al64(nkv), o_f = o_v + al64(nkv),
                 o_p = o_f + al64(nf), o_c = o_p + al64(np), total = o_c + al64(nc);
    if (!grow(&bd.dit_arena, &bd.dit_arena_floats, total, false, st)) return VOXCPM_ERR_OOM;
    if (!grow(&bd.h_stage, &bd.h_stage_floats, al64(nf) + nc, true, st)) return VOXCPM_ERR_OOM;
    float* A = bd.dit_arena;
    float *d_x = A, *d_feats = A + o_f, *d_proj = A + o_p, *d_cls = A + o_c;
    float* h_f = bd.h_stage;
    float* h_out = bd.h_stage + al64(nf);
    memcpy(h_f, audio_feats->data, nf * sizeof(float));
    VOXQ_CUDA_TRY(cudaMemcpyAsync(d_feats, h_f, nf * sizeof(float), cudaMemcpyHostToDevice, st));
    // input projection + bias (src/loc_enc.c:76-101)
    voxq_epilogue ei = {b_in, nullptr, 0, nullptr};
    e = voxq_matmul_nt_q(d_feats, B * T * P, F, &win, d_proj, D, &ei, st);
    if (e) return e;
    enc_seq_kernel<<<ew((int)std::min<size_t>(nx, 1 << 20)), 256, 0, st>>>(d_x, d_proj, d_special, B, T, P, D);
    VOXQ_CUDA_TRY(cudaGetLastError());
    // the layers, in place, each over a fresh scratch cache (pos 0, length S)
    Mirror kvm;
    kvm.k = A + o_k;
    kvm.v = A + o_v;
    uint64_t traffic = (uint64_t)voxq_codes_bytes(win.N, win.K, win.qtype) + voxq_scales_bytes(win.N, win.K, win.qtype);
    for (int l = 0; l < enc->n_layers; l++) {
        const Scratch sc = scratch_at(A + o_scr, M, bw[l]);
        e = block_core(bw[l], sc, d_x, d_x, B, S, &kvm, S, 0, nullptr, 0, 0, nullptr, nullptr, nullptr, st);
        if (e) return e;
        traffic += block_weight_bytes(bw[l]);
    }
    // first token of each step, output norm (src/loc_enc.c:168-186)
    enc_cls_kernel<<<ew((int)nc), 256, 0, st>>>(d_x, d_cls, B * T, P, D);
    rmsnorm_kernel<<<B * T, kBlockThreads, 0, st>>>(d_cls, w_on, enc->output_norm->eps, d_cls, D);
    VOXQ_CUDA_TRY(cudaGetLastError());
    VOXQ_CUDA_TRY(cudaMemcpyAsync(h_out, d_cls, nc * sizeof(float), cudaMemcpyDeviceToHost, st));
    VOXQ_CUDA_TRY(cudaStreamSynchronize(st));
    memcpy(out->data, h_out, nc * sizeof(float));
    count_matmul_traffic(1 + 7 * (uint64_t)enc->n_layers, traffic);
    return VOXCPM_SUCCESS;
}

extern "C" void voxq_block_cache_clear(void) { block_cache_clear(); }
