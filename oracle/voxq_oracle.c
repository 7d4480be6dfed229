/*
 * voxq_oracle.c -- CPU restatement of the reference's quantized-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load it.  The product path (libvoxq.so) never links or calls it.
 *
 * What it restates (reference paths are relative to the voxcpm2-c project):
 *   - scripts/quantize.py:42-54   quantize_q4_block   (32 f32 -> 20 bytes)
 *   - scripts/quantize.py:56-67   dequantize_q4_block
 *   - scripts/quantize.py:69-75   quantize_q8_block   (32 f32 -> 40 bytes)
 *   - scripts/quantize.py:77-82   dequantize_q8_block (signed int8 read)
 *   - scripts/quantize.py:239-260 flattened-tensor blocking, zero-padded tail
 *   - scripts/quantize.py:88-104  compute_tensor_size (payload part)
 *   - src/tensor.c:617-678        tensor_matmul_nt, one sequential fp32
 *                                 accumulator over k per output
 *   - src/tensor.c:339-371        xorshift64 + Box-Muller normal generator
 *   - include/tensor.h:350-371    fp16 -> fp32 decode
 *
 * Parity is pinned by tests/golden (fixtures produced by running the
 * reference's quantize.py / gen_test_data.py and the reference tensor.c).
 *
 * numpy 2 (NEP 50) arithmetic that quantize.py performs, restated exactly:
 *   w_min, w_max   numpy reductions over the float32 block (NaN propagates)
 *   scale          (double(w_max) - double(w_min)) / 15.0 or / 255.0 in
 *                  double, or 1.0 when w_max == w_min
 *   t              float32(x - float32(w_min))                  (RN)
 *   r              float32(t / float32(scale))                  (RN, IEEE div)
 *   q              rint(r) (ties to even), clipped to [0,15] / [0,255];
 *                  NaN becomes code 0 (what the x86 cast gives)
 *   Q4 trailer     half(scale) rounded directly from the double, half(w_min)
 *   Q8 trailer     float(scale), float(w_min); codes stored as the low byte
 *                  (int8 wrap of codes 128..255)
 *
 * numpy's float32 min/max reduction on an AVX-512 host (the one the golden
 * fixtures were made on) visits a 32-element block as: seed r = x[0];
 * 16 vector lanes take v[i] = op(r, x[1+i]); the lanes are folded as
 * 8 <- (hi, lo), 4 <- (hi, lo), 4 <- (j, j^2), 1 <- (0, 1); the scalar tail
 * x[17..31] follows.  Every step keeps its SECOND operand on a tie, which only
 * matters for the sign of a zero min/max in blocks holding both +0 and -0.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#define QBLK 32

/* ------------------------------------------------------------------ */
/* numpy-order min/max over one 32-element block                       */
/* ------------------------------------------------------------------ */

/* op(a, x) for min: a if a < x else x (tie keeps x, the second operand). */
static inline float sel_min(float a, float x) { return (a < x) ? a : x; }
static inline float sel_max(float a, float x) { return (a > x) ? a : x; }

static float block_reduce(const float* b, int is_max) {
    for (int i = 0; i < QBLK; i++)
        if (isnan(b[i])) return b[i];
    float v[16];
    for (int i = 0; i < 16; i++)
        v[i] = is_max ? sel_max(b[0], b[1 + i]) : sel_min(b[0], b[1 + i]);
    float t3[8], t6[4], t8[4];
    for (int j = 0; j < 8; j++)
        t3[j] = is_max ? sel_max(v[8 + j], v[j]) : sel_min(v[8 + j], v[j]);
    for (int j = 0; j < 4; j++)
        t6[j] = is_max ? sel_max(t3[4 + j], t3[j]) : sel_min(t3[4 + j], t3[j]);
    for (int j = 0; j < 4; j++)
        t8[j] = is_max ? sel_max(t6[j], t6[j ^ 2]) : sel_min(t6[j], t6[j ^ 2]);
    float r = is_max ? sel_max(t8[0], t8[1]) : sel_min(t8[0], t8[1]);
    for (int i = 17; i < QBLK; i++)
        r = is_max ? sel_max(r, b[i]) : sel_min(r, b[i]);
    return r;
}

/* ------------------------------------------------------------------ */
/* IEEE binary64 -> binary16, round to nearest even, computed directly  */
/* from the double (no intermediate float rounding).                    */
/* ------------------------------------------------------------------ */
uint16_t oracle_double_to_half(double d) {
    uint64_t bits;
    memcpy(&bits, &d, 8);
    uint16_t sign = (uint16_t)((bits >> 48) & 0x8000u);
    int exp = (int)((bits >> 52) & 0x7ff);
    uint64_t mant = bits & ((1ull << 52) - 1);
    if (exp == 0x7ff) {
        if (mant == 0) return sign | 0x7c00u;
        uint16_t m = (uint16_t)(mant >> 42);
        if (m == 0) m = 0x200;
        return sign | 0x7c00u | m;
    }
    if (exp == 0) return sign; /* double zero / subnormal: far below 2^-25 */
    int e = exp - 1023;
    if (e > 15) return sign | 0x7c00u;
    if (e >= -14) {
        uint64_t hm = mant >> 42;
        uint64_t rem = mant & ((1ull << 42) - 1);
        uint64_t half = 1ull << 41;
        uint32_t h = ((uint32_t)(e + 15) << 10) + (uint32_t)hm;
        if (rem > half || (rem == half && (hm & 1))) h += 1;
        if (h >= 0x7c00u) h = 0x7c00u;
        return sign | (uint16_t)h;
    }
    /* binary16 subnormal: value / 2^-24, rounded to an integer 0..1024 */
    int s = 28 - e; /* >= 43 */
    if (s > 53) return sign;
    uint64_t sig = mant | (1ull << 52);
    uint64_t hm = sig >> s;
    uint64_t rem = sig & ((1ull << s) - 1);
    uint64_t half = 1ull << (s - 1);
    if (rem > half || (rem == half && (hm & 1))) hm += 1;
    return sign | (uint16_t)hm;
}

/* include/tensor.h:350-371 */
float oracle_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t mant = h & 0x3ff;
    uint32_t u;
    if (exp == 0) {
        if (mant == 0) {
            u = sign;
        } else {
            int e = 1;
            while (!(mant & 0x400)) { mant <<= 1; e--; }
            mant &= 0x3ff;
            u = sign | ((uint32_t)(e + 112) << 23) | (mant << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7f800000u | (mant << 13);
    } else {
        u = sign | ((exp + 112) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* ------------------------------------------------------------------ */
/* Block quantizers                                                     */
/* ------------------------------------------------------------------ */

/* Codes for one block; levels = 15 or 255.  Returns the double scale. */
static double block_codes(const float* b, double levels, uint8_t* q, float* wmin_out) {
    float mn = block_reduce(b, 0);
    float mx = block_reduce(b, 1);
    double dmin = (double)mn, dmax = (double)mx;
    double scale = (dmax != dmin) ? (dmax - dmin) / levels : 1.0;
    volatile float fscale = (float)scale;
    for (int i = 0; i < QBLK; i++) {
        volatile float t = b[i] - mn;
        volatile float r = t / fscale;
        float rr = rintf(r);
        if (isnan(rr)) {
            q[i] = 0;
            continue;
        }
        if (rr < 0.0f) rr = 0.0f;
        if (rr > (float)levels) rr = (float)levels;
        q[i] = (uint8_t)(int)rr;
    }
    *wmin_out = mn;
    return scale;
}

void oracle_quantize_q4_block(const float* b, uint8_t* out20) {
    uint8_t q[QBLK];
    float mn;
    double scale = block_codes(b, 15.0, q, &mn);
    for (int i = 0; i < 16; i++) out20[i] = (uint8_t)((q[2 * i] << 4) | q[2 * i + 1]);
    uint16_t hs = oracle_double_to_half(scale);
    uint16_t hm = oracle_double_to_half((double)mn);
    out20[16] = (uint8_t)(hs & 0xff);
    out20[17] = (uint8_t)(hs >> 8);
    out20[18] = (uint8_t)(hm & 0xff);
    out20[19] = (uint8_t)(hm >> 8);
}

void oracle_quantize_q8_block(const float* b, uint8_t* out40) {
    uint8_t q[QBLK];
    float mn;
    double scale = block_codes(b, 255.0, q, &mn);
    memcpy(out40, q, QBLK);
    float fs = (float)scale;
    memcpy(out40 + 32, &fs, 4);
    memcpy(out40 + 36, &mn, 4);
}

/* Quantize a flattened tensor of n elements (scripts/quantize.py:239-260):
 * ceil(n/32) blocks, the last one zero-padded.  Returns bytes written. */
size_t oracle_quantize(const float* src, size_t n, int qtype, uint8_t* dst) {
    size_t nb = (n + QBLK - 1) / QBLK;
    size_t bb = (qtype == 2) ? 20 : 40;
    float pad[QBLK];
    for (size_t b = 0; b < nb; b++) {
        const float* blk = src + b * QBLK;
        if ((b + 1) * QBLK > n) {
            size_t have = n - b * QBLK;
            memset(pad, 0, sizeof(pad));
            memcpy(pad, blk, have * sizeof(float));
            blk = pad;
        }
        if (qtype == 2)
            oracle_quantize_q4_block(blk, dst + b * bb);
        else
            oracle_quantize_q8_block(blk, dst + b * bb);
    }
    return nb * bb;
}

/* Dequantize n elements.  Q4: f32(q) * f32(half scale) + f32(half min), two
 * roundings (scripts/quantize.py:56-67).  Q8: code read as int8 when
 * q8_signed (scripts/quantize.py:79 literally) or as uint8 otherwise. */
void oracle_dequantize(const uint8_t* src, size_t n, int qtype, int q8_signed, float* dst) {
    size_t nb = (n + QBLK - 1) / QBLK;
    for (size_t b = 0; b < nb; b++) {
        float w[QBLK];
        if (qtype == 2) {
            const uint8_t* p = src + b * 20;
            float s = oracle_half_to_float((uint16_t)(p[16] | (p[17] << 8)));
            float m = oracle_half_to_float((uint16_t)(p[18] | (p[19] << 8)));
            for (int i = 0; i < 16; i++) {
                volatile float a0 = (float)((p[i] >> 4) & 0xf) * s;
                volatile float a1 = (float)(p[i] & 0xf) * s;
                w[2 * i] = a0 + m;
                w[2 * i + 1] = a1 + m;
            }
        } else {
            const uint8_t* p = src + b * 40;
            float s, m;
            memcpy(&s, p + 32, 4);
            memcpy(&m, p + 36, 4);
            for (int i = 0; i < QBLK; i++) {
                float qf = q8_signed ? (float)(int8_t)p[i] : (float)p[i];
                volatile float a = qf * s;
                w[i] = a + m;
            }
        }
        size_t have = (b + 1) * QBLK <= n ? QBLK : n - b * QBLK;
        memcpy(dst + b * QBLK, w, have * sizeof(float));
    }
}

/* ------------------------------------------------------------------ */
/* Matmul: out[M,N] = A[M,K] . W[N,K]^T (src/tensor.c:666-675)           */
/* ------------------------------------------------------------------ */

/* One sequential fp32 accumulator per output, as the reference loop. */
void oracle_matmul_nt(const float* a, const float* w, float* out, int M, int N, int K) {
    for (int i = 0; i < M; i++)
        for (int j = 0; j < N; j++) {
            float sum = 0.0f;
            const float* ar = a + (size_t)i * K;
            const float* wr = w + (size_t)j * K;
            for (int k = 0; k < K; k++) sum += ar[k] * wr[k];
            out[(size_t)i * N + j] = sum;
        }
}

/* fp64 reference and the tolerance scale sum_k |a_ik w_jk| / sqrt(K). */
void oracle_matmul_nt_f64(const float* a, const float* w, double* out, double* absscale,
                          int M, int N, int K) {
    double rk = 1.0 / sqrt((double)K);
    for (int i = 0; i < M; i++)
        for (int j = 0; j < N; j++) {
            double s = 0.0, sa = 0.0;
            const float* ar = a + (size_t)i * K;
            const float* wr = w + (size_t)j * K;
            for (int k = 0; k < K; k++) {
                double p = (double)ar[k] * (double)wr[k];
                s += p;
                sa += fabs(p);
            }
            out[(size_t)i * N + j] = s;
            absscale[(size_t)i * N + j] = sa * rk;
        }
}

/* ------------------------------------------------------------------ */
/* Synthetic inputs: xorshift64 + Box-Muller (src/tensor.c:339-371)     */
/* ------------------------------------------------------------------ */

static inline uint64_t xorshift64(uint64_t* s) {
    uint64_t x = *s;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *s = x;
    return x;
}

/* Fills out[0..n) with N(0,1) * mult; the seed must be non-zero.  As in the
 * reference, an odd n leaves the last element untouched (set here to 0). */
void oracle_rand_normal(uint64_t* seed, float* out, size_t n, float mult) {
    size_t i = 0;
    for (; i + 1 < n; i += 2) {
        double u1 = (double)xorshift64(seed) / (double)UINT64_MAX;
        double u2 = (double)xorshift64(seed) / (double)UINT64_MAX;
        if (u1 < 1e-15) u1 = 1e-15;
        double r = sqrt(-2.0 * log(u1));
        double th = 2.0 * 3.14159265358979323846 * u2;
        out[i] = (float)(r * cos(th)) * mult;
        out[i + 1] = (float)(r * sin(th)) * mult;
    }
    if (i < n) out[i] = 0.0f;
}

/* ------------------------------------------------------------------ */
/* AudioVAE convolutions (src/nn.c:765-834 conv1d_forward,             */
/* src/nn.c:864-931 conv1d_transpose_forward): same loop order, fp32    */
/* accumulation.  `absout` (may be NULL) receives the same sums of      */
/* |w x| -- the scale the parity tests measure errors against.          */
/* ------------------------------------------------------------------ */

void oracle_conv1d(const float* x, const float* w, const float* b, float* out, float* absout, int B, int Cin,
                   int Tin, int Cout, int Kw, int stride, int pad, int groups) {
    const int Tout = (Tin + 2 * pad - Kw) / stride + 1;
    const int ipg = groups > 0 ? Cin / groups : Cin, opg = groups > 0 ? Cout / groups : Cout;
    for (int n = 0; n < B; n++)
        for (int o = 0; o < Cout; o++) {
            const int c0 = (opg > 0 ? o / opg : 0) * ipg;
            for (int t = 0; t < Tout; t++) {
                float sum = b ? b[o] : 0.0f, asum = b ? fabsf(b[o]) : 0.0f;
                for (int c = c0; c < c0 + ipg; c++)
                    for (int k = 0; k < Kw; k++) {
                        const int ti = t * stride + k - pad;
                        if (ti < 0 || ti >= Tin) continue;
                        const float p = w[((size_t)o * ipg + (size_t)(c - c0)) * Kw + k] *
                                        x[((size_t)n * Cin + c) * Tin + ti];
                        sum += p;
                        asum += fabsf(p);
                    }
                out[((size_t)n * Cout + o) * Tout + t] = sum;
                if (absout) absout[((size_t)n * Cout + o) * Tout + t] = asum;
            }
        }
}

void oracle_conv1d_transpose(const float* x, const float* w, const float* b, float* out, float* absout, int B,
                             int Cin, int Tin, int Cout, int Kw, int stride, int pad) {
    const int Tout = (Tin - 1) * stride - 2 * pad + Kw;
    memset(out, 0, (size_t)B * Cout * Tout * sizeof(float));
    if (absout) memset(absout, 0, (size_t)B * Cout * Tout * sizeof(float));
    for (int n = 0; n < B; n++) {
        for (int c = 0; c < Cin; c++)
            for (int ti = 0; ti < Tin; ti++) {
                const float xv = x[((size_t)n * Cin + c) * Tin + ti];
                for (int k = 0; k < Kw; k++) {
                    const int to = ti * stride + k - pad;
                    if (to < 0 || to >= Tout) continue;
                    for (int o = 0; o < Cout; o++) {
                        const float p = w[((size_t)c * Cout + o) * Kw + k] * xv;
                        out[((size_t)n * Cout + o) * Tout + to] += p;
                        if (absout) absout[((size_t)n * Cout + o) * Tout + to] += fabsf(p);
                    }
                }
            }
        if (b)
            for (int o = 0; o < Cout; o++)
                for (int t = 0; t < Tout; t++) {
                    out[((size_t)n * Cout + o) * Tout + t] += b[o];
                    if (absout) absout[((size_t)n * Cout + o) * Tout + t] += fabsf(b[o]);
                }
    }
}
