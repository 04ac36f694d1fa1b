/*
 * CPU ORACLE -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of NanoCamelid's x86 portable (scalar) decode path.  It is
 * the checker the GPU product is compared against and the timed CPU baseline; it
 * is never linked into, called by, or shipped with the product library.  Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU arms load it.
 *
 * The reference is Rust and cannot be built here (no cargo/rustc, no network), so
 * this file restates the algorithm function by function.  Every function names
 * the reference file:line it follows.  Numerics mirrored exactly:
 *   - f32 arithmetic in the reference's operation order, no FMA contraction
 *     (built with -ffp-contract=off), sequential left-to-right sums;
 *   - Rust f32::round == C roundf (half away from zero); `as i8`/`as i32`
 *     saturate and map NaN to 0 (sat_i32 below);
 *   - transcendentals (powf, sinf, cosf, expf, sqrtf) from the same glibc libm
 *     that Rust's std calls on Linux.
 * Parity pins: tests/test_oracle_kat.py checks this file against every known-answer
 * test the reference's q8.rs / inference.rs hold for the path.
 */
#define _GNU_SOURCE
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#define QK 32
#define QKK 256
enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

/* ------------------------------------------------------------------ f16 */
/* q8.rs:3599-3622 f16_bits_to_f32 (exact, subnormals normalised). */
static float bits_f32(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t f32_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

float orc_f16_to_f32(uint16_t bits) {
    uint32_t sign = (uint32_t)(bits & 0x8000) << 16;
    uint32_t exponent = (bits >> 10) & 0x1f;
    uint32_t fraction = bits & 0x03ff;
    if (exponent == 0) {
        if (fraction == 0) return bits_f32(sign);
        int32_t e = -14;
        uint32_t m = fraction;
        while ((m & 0x0400) == 0) { m <<= 1; e -= 1; }
        m &= 0x03ff;
        return bits_f32(sign | ((uint32_t)(e + 127) << 23) | (m << 13));
    }
    if (exponent == 0x1f) return bits_f32(sign | 0x7f800000u | (fraction << 13));
    return bits_f32(sign | ((exponent + 112) << 23) | (fraction << 13));
}

/* q8.rs:3644-3673 fast_f32_to_f16: TRUNCATES the mantissa, flushes f32 denormals. */
uint16_t orc_f32_to_f16(float value) {
    uint32_t bits = f32_bits(value);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
    int32_t exponent = (int32_t)((bits >> 23) & 0xff);
    uint32_t fraction = bits & 0x007fffff;
    if (exponent == 0) return sign;
    if (exponent == 0xff) {
        if (fraction == 0) return sign | 0x7c00;
        return (uint16_t)(sign | 0x7c00 | (fraction >> 13) | 1);
    }
    int32_t he = exponent - 127 + 15;
    if (he >= 0x1f) return sign | 0x7c00;
    if (he <= 0) {
        if (he < -10) return sign;
        uint32_t mant = (fraction | 0x00800000u) >> (14 - he);
        return (uint16_t)(sign | mant);
    }
    return (uint16_t)(sign | ((uint16_t)he << 10) | (fraction >> 13));
}

/* Rust `f as i32`: saturating, NaN -> 0. */
static int32_t sat_i32(float f) {
    if (f != f) return 0;
    if (f >= 2147483647.0f) return 2147483647;
    if (f <= -2147483648.0f) return (-2147483647 - 1);
    return (int32_t)f;
}
static float rd16(const uint8_t* p) { return orc_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* ------------------------------------------------------------------ block formats */
size_t orc_block_bytes(int t) {
    return t == T_Q4_0 ? 18 : t == T_Q8_0 ? 34 : t == T_Q4_K ? 144 : t == T_Q6_K ? 210 : t == T_F32 ? 4 : t == T_F16 ? 2 : 0;
}
size_t orc_block_elems(int t) { return (t == T_Q4_K || t == T_Q6_K) ? QKK : (t == T_Q4_0 || t == T_Q8_0) ? QK : 1; }

/* q8.rs:539-546 Q4_0Block::unpack_values: low nibble -> j, high nibble -> j+16, minus 8. */
void orc_q4_0_unpack(const uint8_t* blk, int8_t out[32]) {
    for (int j = 0; j < 16; ++j) {
        out[j] = (int8_t)((blk[2 + j] & 0x0f) - 8);
        out[j + 16] = (int8_t)((blk[2 + j] >> 4) - 8);
    }
}

/* q8.rs:3376-3382 dot_i8_scalar. */
int32_t orc_dot_i8(const int8_t* a, const int8_t* b, int n) {
    int32_t s = 0;
    for (int i = 0; i < n; ++i) s += (int32_t)a[i] * (int32_t)b[i];
    return s;
}

/* q8.rs:2699-2702 dot_q4_0_q8_0_scalar / Q8_0Block::dot_i32 (q8.rs:505).  The sums are
 * exact in int32, so the loops are written to vectorise. */
static inline int32_t q4_0_dot(const uint8_t* blk, const int8_t* x) {
    int32_t s = 0;
    for (int j = 0; j < 16; ++j) {
        s += ((int32_t)(blk[2 + j] & 0x0f) - 8) * (int32_t)x[j];
        s += ((int32_t)(blk[2 + j] >> 4) - 8) * (int32_t)x[j + 16];
    }
    return s;
}
static inline int32_t q8_0_dot(const uint8_t* blk, const int8_t* x) {
    int32_t s = 0;
    for (int j = 0; j < 32; ++j) s += (int32_t)(int8_t)blk[2 + j] * (int32_t)x[j];
    return s;
}
int32_t orc_block_dot(int t, const uint8_t* blk, const int8_t* x) {
    return t == T_Q4_0 ? q4_0_dot(blk, x) : q8_0_dot(blk, x);
}

/* q8.rs:2009-2018 q4_k_scale_min. */
void orc_q4_k_scale_min(int idx, const uint8_t* sc, uint8_t* s, uint8_t* m) {
    if (idx < 4) { *s = sc[idx] & 63; *m = sc[idx + 4] & 63; }
    else {
        *s = (uint8_t)((sc[idx + 4] & 0x0f) | ((sc[idx - 4] >> 6) << 4));
        *m = (uint8_t)((sc[idx + 4] >> 4) | ((sc[idx] >> 6) << 4));
    }
}

/* Integer half of q8.rs:1338-1376 dot_q8_scaled_preloaded: per 32-sub-block
 * weighted sum Σ q·x (q in 0..15) and activation sum Σ x, sub-block order 0..7. */
void orc_q4_k_int_sums(const uint8_t* blk, const int8_t* x, int32_t wsum[8], int32_t asum[8]) {
    const uint8_t* v = blk + 16;
    for (int p = 0; p < 4; ++p) {
        int32_t lw = 0, la = 0, hw = 0, ha = 0;
        for (int l = 0; l < 32; ++l) {
            uint8_t byte = v[p * 32 + l];
            int32_t lx = x[p * 64 + l], hx = x[p * 64 + 32 + l];
            lw += (int32_t)(byte & 0x0f) * lx; la += lx;
            hw += (int32_t)(byte >> 4) * hx; ha += hx;
        }
        wsum[2 * p] = lw; asum[2 * p] = la; wsum[2 * p + 1] = hw; asum[2 * p + 1] = ha;
    }
}

/* q8.rs:1249-1269 unpack + q8.rs:1338-1376 dot_q8_scaled_preloaded (f32 combine). */
float orc_q4_k_dot(const uint8_t* blk, const int8_t* x, const float* xs) {
    float d = rd16(blk), dmin = rd16(blk + 2);
    float scales[8], mins[8];
    for (int p = 0; p < 4; ++p) {
        uint8_t ls, lm, hs, hm;
        orc_q4_k_scale_min(2 * p, blk + 4, &ls, &lm);
        orc_q4_k_scale_min(2 * p + 1, blk + 4, &hs, &hm);
        scales[2 * p] = d * (float)ls; scales[2 * p + 1] = d * (float)hs;
        mins[2 * p] = dmin * (float)lm; mins[2 * p + 1] = dmin * (float)hm;
    }
    int32_t ws[8], as[8];
    orc_q4_k_int_sums(blk, x, ws, as);
    float sum = 0.0f;
    for (int j = 0; j < 8; ++j) sum += xs[j] * (scales[j] * (float)ws[j] - mins[j] * (float)as[j]);
    return sum;
}

/* q8.rs:1240-1269 Q4KBlock::dequantize. */
void orc_q4_k_dequant(const uint8_t* blk, float out[256]) {
    float d = rd16(blk), dmin = rd16(blk + 2);
    for (int p = 0; p < 4; ++p) {
        uint8_t ls, lm, hs, hm;
        orc_q4_k_scale_min(2 * p, blk + 4, &ls, &lm);
        orc_q4_k_scale_min(2 * p + 1, blk + 4, &hs, &hm);
        float lsc = d * (float)ls, hsc = d * (float)hs, lmn = dmin * (float)lm, hmn = dmin * (float)hm;
        for (int l = 0; l < 32; ++l) {
            uint8_t byte = blk[16 + p * 32 + l];
            out[p * 64 + l] = lsc * (float)(byte & 0x0f) - lmn;
            out[p * 64 + 32 + l] = hsc * (float)(byte >> 4) - hmn;
        }
    }
}

/* q8.rs:2026-2090 Q6KBlock: ql[128] | qh[64] | scales i8[16] | d f16.  Each 128-value
 * half n holds four 32-lanes: q1 (ql low nibble, qh bits 0-1), q2 (ql+32 low, bits 2-3),
 * q3 (ql high, bits 4-5), q4 (ql+32 high, bits 6-7), each minus 32; lane l of quarter
 * j uses scale (n/128)*8 + j*2 + l/16. */
static inline void q6k_quad(const uint8_t* blk, int half, int l, int q[4]) {
    const uint8_t* ql = blk + half * 64;
    const uint8_t qh = blk[128 + half * 32 + l];
    q[0] = (int)(int8_t)((ql[l] & 0x0f) | ((qh & 0x03) << 4)) - 32;
    q[1] = (int)(int8_t)((ql[l + 32] & 0x0f) | (((qh >> 2) & 0x03) << 4)) - 32;
    q[2] = (int)(int8_t)((ql[l] >> 4) | (((qh >> 4) & 0x03) << 4)) - 32;
    q[3] = (int)(int8_t)((ql[l + 32] >> 4) | (((qh >> 6) & 0x03) << 4)) - 32;
}

/* q8.rs:2056-2090 dequantize: out = d * scale * q (left to right). */
void orc_q6_k_dequant(const uint8_t* blk, float out[256]) {
    const float d = rd16(blk + 208);
    const int8_t* sc = (const int8_t*)(blk + 192);
    for (int half = 0; half < 2; ++half)
        for (int l = 0; l < 32; ++l) {
            int q[4]; q6k_quad(blk, half, l, q);
            for (int j = 0; j < 4; ++j)
                out[half * 128 + j * 32 + l] = d * (float)sc[half * 8 + l / 16 + 2 * j] * (float)q[j];
        }
}

/* q8.rs:2092-2150 dot_q8_scaled (the x86 path of inference.rs:3074-3086): per
 * 128-half, c[j][h] = (d * scale) * x_scale; then one f32 sum over the 256 products
 * (c * q) * x in the order l = 0..15 (low scales) then 16..31 (high scales), and
 * within each l the quarters q1..q4. */
float orc_q6_k_dot(const uint8_t* blk, const int8_t* x, const float* xs) {
    const float d = rd16(blk + 208);
    const int8_t* sc = (const int8_t*)(blk + 192);
    float ws[16];
    for (int i = 0; i < 16; ++i) ws[i] = d * (float)sc[i];
    float sum = 0.0f;
    for (int half = 0; half < 2; ++half) {
        const int n = half * 128, so = half * 8, xo = n / 32;
        float c[4][2];
        for (int j = 0; j < 4; ++j) {
            c[j][0] = ws[so + 2 * j] * xs[xo + j];
            c[j][1] = ws[so + 2 * j + 1] * xs[xo + j];
        }
        for (int l = 0; l < 32; ++l) {
            int q[4]; q6k_quad(blk, half, l, q);
            const int hi = l >= 16;
            for (int j = 0; j < 4; ++j) sum += c[j][hi] * (float)q[j] * (float)x[n + j * 32 + l];
        }
    }
    return sum;
}

/* model.rs:1109-1132 load_f32_or_f16 for Q8_0 / Q4_0 / Q4_K / Q6_K / F32 / F16 rows. */
void orc_dequant_row(int t, const uint8_t* row, int cols, float* out) {
    if (t == T_F32) { memcpy(out, row, (size_t)cols * 4); return; }
    if (t == T_F16) { for (int i = 0; i < cols; ++i) out[i] = rd16(row + 2 * i); return; }
    if (t == T_Q4_K) { for (int b = 0; b < cols / QKK; ++b) orc_q4_k_dequant(row + (size_t)b * 144, out + b * QKK); return; }
    if (t == T_Q6_K) { for (int b = 0; b < cols / QKK; ++b) orc_q6_k_dequant(row + (size_t)b * 210, out + b * QKK); return; }
    int nb = cols / QK;
    for (int b = 0; b < nb; ++b) {
        const uint8_t* blk = row + (size_t)b * orc_block_bytes(t);
        float scale = rd16(blk);
        if (t == T_Q4_0) {
            int8_t v[32]; orc_q4_0_unpack(blk, v);
            for (int i = 0; i < 32; ++i) out[b * 32 + i] = (float)v[i] * scale;
        } else {
            const int8_t* v = (const int8_t*)(blk + 2);
            for (int i = 0; i < 32; ++i) out[b * 32 + i] = (float)v[i] * scale;
        }
    }
}

/* ------------------------------------------------------------------ quantizers */
/* inference.rs:991-1029 quantize_f32_to_q8_0_scalar (x86 path). Scale stored as f32. */
void orc_quantize_q8_0(const float* x, int n, int8_t* xq, float* xs) {
    for (int b = 0; b < n / 32; ++b) {
        const float* c = x + b * 32;
        float max_abs = 0.0f;
        for (int i = 0; i < 32; ++i) { float a = fabsf(c[i]); if (a > max_abs) max_abs = a; }
        float scale = max_abs / 127.0f;
        xs[b] = scale;
        if (scale > 0.0f) {
            float inv = 1.0f / scale;
            for (int i = 0; i < 32; ++i) {
                float q = roundf(c[i] * inv);
                if (q < -127.0f) q = -127.0f;
                if (q > 127.0f) q = 127.0f;
                xq[b * 32 + i] = (int8_t)q;
            }
        } else {
            memset(xq + b * 32, 0, 32);
        }
    }
}

/* q8.rs:2389-2440 quantize_f32_matrix_to_q8_0_blocks (f16-truncated scale), one block. */
void orc_quantize_block_q8_0(const float* c, uint8_t* o) {
    float max_abs = 0.0f;
    for (int i = 0; i < 32; ++i) { float a = fabsf(c[i]); if (a > max_abs) max_abs = a; }
    float scale = max_abs / 127.0f;
    int8_t q[32]; memset(q, 0, 32);
    if (scale > 0.0f) {
        float inv = 1.0f / scale;
        for (int i = 0; i < 32; ++i) {
            float t = roundf(c[i] * inv);
            if (t < -127.0f) t = -127.0f;
            if (t > 127.0f) t = 127.0f;
            q[i] = (int8_t)t;
        }
    }
    uint16_t sb = orc_f32_to_f16(scale);
    o[0] = sb & 0xff; o[1] = sb >> 8; memcpy(o + 2, q, 32);
}
void orc_quantize_matrix_q8_0(const float* v, long rows, int cols, uint8_t* out) {
    int nb = cols / 32;
    #pragma omp parallel for schedule(static) if (rows >= 128)
    for (long r = 0; r < rows; ++r)
        for (int b = 0; b < nb; ++b) orc_quantize_block_q8_0(v + r * cols + b * 32, out + ((size_t)r * nb + b) * 34);
}

/* q8.rs:2442-2488 quantize_f32_matrix_to_q4_0_blocks: d = signed-max/-8, q = trunc(x*id + 8.5). */
void orc_quantize_block_q4_0(const float* c, uint8_t* o) {
    float amax = 0.0f, mx = 0.0f;
    for (int i = 0; i < 32; ++i) { float a = fabsf(c[i]); if (a > amax) { amax = a; mx = c[i]; } }
    float d = mx / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    for (int j = 0; j < 16; ++j) {
        float x0 = c[j] * id + 8.5f;
        float x1 = c[j + 16] * id + 8.5f;
        int32_t q0 = sat_i32(x0), q1 = sat_i32(x1);
        q0 = q0 < 0 ? 0 : q0 > 15 ? 15 : q0;
        q1 = q1 < 0 ? 0 : q1 > 15 ? 15 : q1;
        o[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
    uint16_t sb = orc_f32_to_f16(d);
    o[0] = sb & 0xff; o[1] = sb >> 8;
}
void orc_quantize_matrix_q4_0(const float* v, long rows, int cols, uint8_t* out) {
    int nb = cols / 32;
    #pragma omp parallel for schedule(static) if (rows >= 128)
    for (long r = 0; r < rows; ++r)
        for (int b = 0; b < nb; ++b) orc_quantize_block_q4_0(v + r * cols + b * 32, out + ((size_t)r * nb + b) * 18);
}

/* ------------------------------------------------------------------ GEMV */
/* One output row, reference order.  Q4_0 / Q8_0: inference.rs:1146-1199 (matmul_q8_0),
 * 2641-2667 (matmul_q4_0), 2886-2935 (1x4 swizzled chunk; same per-row formula):
 *   sum += w_scale * x_scale * (float)dot   sequentially in block order.
 * Q4_K: inference.rs:3089-3135: sum += dot_q8_scaled_preloaded(block) per super-block. */
static float row_dot(int t, const uint8_t* row, int cols, const int8_t* xq, const float* xs) {
    float sum = 0.0f;
    if (t == T_Q4_K) {
        for (int b = 0; b < cols / QKK; ++b) sum += orc_q4_k_dot(row + (size_t)b * 144, xq + b * QKK, xs + b * 8);
        return sum;
    }
    if (t == T_Q6_K) {   /* inference.rs:3074-3086 */
        for (int b = 0; b < cols / QKK; ++b) sum += orc_q6_k_dot(row + (size_t)b * 210, xq + b * QKK, xs + b * 8);
        return sum;
    }
    size_t bb = orc_block_bytes(t);
    for (int b = 0; b < cols / QK; ++b) {
        const uint8_t* blk = row + b * bb;
        int32_t d = orc_block_dot(t, blk, xq + b * 32);
        sum += rd16(blk) * xs[b] * (float)d;
    }
    return sum;
}

size_t orc_row_bytes(int t, int cols) { return (size_t)cols / orc_block_elems(t) * orc_block_bytes(t); }

/* inference.rs:1201-1244 matmul_quantized: out fully overwritten; rows in parallel
 * (inference.rs:34-50: rayon only when rows >= 128; per-row order unchanged). */
void orc_matmul_quantized(int t, const uint8_t* w, long rows, int cols, const int8_t* xq, const float* xs, float* out) {
    size_t rb = orc_row_bytes(t, cols);
    #pragma omp parallel for schedule(static) if (rows >= 128)
    for (long r = 0; r < rows; ++r) out[r] = row_dot(t, w + r * rb, cols, xq, xs);
}

/* inference.rs:1246-1303,1343-1418,2006-2132 matmul_quantized_batch: out[token][row];
 * each token's row uses the single-token formula. */
void orc_matmul_quantized_batch(int t, const uint8_t* w, long rows, int cols, int ntok, const int8_t* xq, const float* xs, float* out) {
    size_t rb = orc_row_bytes(t, cols);
    int nbs = cols / 32;
    if (t != T_Q4_0 && t != T_Q8_0) {
        #pragma omp parallel for schedule(static) if (rows >= 128)
        for (long r = 0; r < rows; ++r)
            for (int k = 0; k < ntok; ++k) out[(size_t)k * rows + r] = row_dot(t, w + r * rb, cols, xq + (size_t)k * cols, xs + (size_t)k * nbs);
        return;
    }
    /* Q4_0 / Q8_0: the same per-token sums (block order, one f32 accumulator per token),
     * walking each weight block once for all tokens. */
    #pragma omp parallel
    {
        float* acc = (float*)malloc(sizeof(float) * (size_t)ntok);
        size_t bb = orc_block_bytes(t);
        #pragma omp for schedule(static)
        for (long r = 0; r < rows; ++r) {
            const uint8_t* row = w + r * rb;
            for (int k = 0; k < ntok; ++k) acc[k] = 0.0f;
            for (int b = 0; b < nbs; ++b) {
                const uint8_t* blk = row + b * bb;
                const float d = rd16(blk);
                int8_t wv[32];
                if (t == T_Q4_0) orc_q4_0_unpack(blk, wv);
                else memcpy(wv, blk + 2, 32);
                for (int k = 0; k < ntok; ++k) {
                    const int8_t* x = xq + (size_t)k * cols + b * 32;
                    int32_t dot = 0;
                    for (int j = 0; j < 32; ++j) dot += (int32_t)wv[j] * (int32_t)x[j];
                    acc[k] += d * xs[(size_t)k * nbs + b] * (float)dot;
                }
            }
            for (int k = 0; k < ntok; ++k) out[(size_t)k * rows + r] = acc[k];
        }
        free(acc);
    }
}

/* Per-block integer dot dump (the bit-exact gate): Q4_0/Q8_0 -> rows x (cols/32) i32;
 * Q4_K -> rows x (cols/32) x {wsum, asum}. */
void orc_block_dots(int t, const uint8_t* w, long rows, int cols, const int8_t* xq, int32_t* out) {
    size_t rb = orc_row_bytes(t, cols);
    int nb = cols / 32;
    for (long r = 0; r < rows; ++r) {
        const uint8_t* row = w + r * rb;
        if (t == T_Q4_K) {
            for (int s = 0; s < cols / QKK; ++s) {
                int32_t ws[8], as[8];
                orc_q4_k_int_sums(row + (size_t)s * 144, xq + s * QKK, ws, as);
                for (int j = 0; j < 8; ++j) {
                    out[((size_t)r * nb + s * 8 + j) * 2] = ws[j];
                    out[((size_t)r * nb + s * 8 + j) * 2 + 1] = as[j];
                }
            }
        } else {
            for (int b = 0; b < nb; ++b) out[(size_t)r * nb + b] = orc_block_dot(t, row + b * orc_block_bytes(t), xq + b * 32);
        }
    }
}

/* ------------------------------------------------------------------ elementwise */
/* inference.rs:697-706 rms_norm. */
void orc_rms_norm(float* out, const float* x, const float* w, int n, float eps) {
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) sum += x[i] * x[i];
    float scale = 1.0f / sqrtf(sum / (float)n + eps);
    for (int i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

/* inference.rs:860-900 cached_rope_angles (no rope-scaling keys): (sin, cos) per pair. */
void orc_rope_angles(int pos, int rope_dim, float base, float* sin_out, float* cos_out) {
    for (int i = 0; i < rope_dim / 2; ++i) {
        float theta = powf(base, -((float)(i * 2)) / (float)rope_dim);
        float angle = (float)pos * theta;
        sin_out[i] = sinf(angle);
        cos_out[i] = cosf(angle);
    }
}

/* inference.rs:904-933 apply_rope_cached, NORM style (interleaved pairs 2i, 2i+1). */
void orc_apply_rope(float* data, int pos, int heads, int hd, int rope_dim, float base) {
    float s[512], c[512];
    orc_rope_angles(pos, rope_dim, base, s, c);
    for (int h = 0; h < heads; ++h)
        for (int i = 0; i < rope_dim / 2; ++i) {
            float* d = data + h * hd + 2 * i;
            float x0 = d[0], x1 = d[1];
            d[0] = x0 * c[i] - x1 * s[i];
            d[1] = x0 * s[i] + x1 * c[i];
        }
}

/* inference.rs:3367-3390 fused_silu_mul: g * (1/(1+exp(-g))) * u. */
void orc_silu_mul(float* out, const float* g, const float* u, int n) {
    for (int i = 0; i < n; ++i) {
        float sig = 1.0f / (1.0f + expf(-g[i]));
        out[i] = g[i] * sig * u[i];
    }
}

/* inference.rs:3522-3540 softmax. */
static void softmax(float* x, int n) {
    float mx = -INFINITY;
    for (int i = 0; i < n; ++i) if (x[i] > mx) mx = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) { x[i] = expf(x[i] - mx); sum += x[i]; }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; ++i) x[i] *= inv;
}

/* inference.rs:4242-4292 apply_attention_head (f32 cache, x86 path): scores via
 * dot_f32_scalar (3570-3573), softmax, then out += score * v (add_weighted_f32_scalar
 * 3619-3623) over p = 0..pos.  `out` must be zeroed by the caller (4660). */
void orc_attention(float* out, const float* q, const float* kc, const float* vc, int pos,
                   int heads, int kv_heads, int hd, int kv_width) {
    int kv_mul = heads / kv_heads;
    float scale = 1.0f / sqrtf((float)hd);
    float* scores = (float*)malloc(sizeof(float) * (size_t)(pos + 1));
    for (int h = 0; h < heads; ++h) {
        int kvh = h / kv_mul;
        const float* qh = q + h * hd;
        for (int p = 0; p <= pos; ++p) {
            const float* k = kc + (size_t)p * kv_width + kvh * hd;
            float s = 0.0f;
            for (int d = 0; d < hd; ++d) s += qh[d] * k[d];
            scores[p] = s * scale;
        }
        softmax(scores, pos + 1);
        float* o = out + h * hd;
        for (int p = 0; p <= pos; ++p) {
            const float* v = vc + (size_t)p * kv_width + kvh * hd;
            for (int d = 0; d < hd; ++d) o[d] += scores[p] * v[d];
        }
    }
    free(scores);
}

/* inference.rs:4298-4317 quantize_row_to_q8_0_blocks (the Q8_0 KV-cache store): per 32
 * values scale = max|x|/127, inv = 1/scale (0 for a zero block), q = clamp(round(x*inv)),
 * the scale stored as f16 with the truncating encode (q8.rs fast_f32_to_f16). */
void orc_kv_quantize_row_q8_0(const float* x, int n, uint8_t* out) {
    for (int b = 0; b < n / 32; ++b) {
        const float* c = x + b * 32;
        uint8_t* o = out + (size_t)b * 34;
        float mx = 0.0f;
        for (int i = 0; i < 32; ++i) { float a = fabsf(c[i]); if (a > mx) mx = a; }
        float scale = mx / 127.0f, inv = scale > 0.0f ? 1.0f / scale : 0.0f;
        uint16_t sb = orc_f32_to_f16(scale);
        o[0] = sb & 0xff; o[1] = sb >> 8;
        for (int i = 0; i < 32; ++i) {
            float q = roundf(c[i] * inv);
            q = q < -127.0f ? -127.0f : q > 127.0f ? 127.0f : q;
            o[2 + i] = (uint8_t)(int8_t)q;
        }
    }
}

/* inference.rs:539-568 store_kv for the F16 cache: truncating f16 encode per value. */
void orc_kv_store_f16(const float* x, int n, uint16_t* out) {
    for (int i = 0; i < n; ++i) out[i] = orc_f32_to_f16(x[i]);
}

/* inference.rs:4242-4458 apply_attention_head over an F16 (kind 1) or Q8_0 (kind 2)
 * cache; kind 0 is the f32 cache of orc_attention.
 *   F16: each K / V head row is decoded to f32, then the f32 path (dot_f32, softmax,
 *        add_weighted).
 *   Q8_0: q_head is quantised like the store; score = (sum over blocks of
 *        (s_q * s_k) * dot_i32) * scale; V blocks decoded as q * s, then add_weighted.
 * `out` must be zeroed by the caller. */
void orc_attention_kv(int kind, float* out, const float* q, const void* kc, const void* vc, int pos, int heads,
                      int kv_heads, int hd, int kv_width) {
    if (kind == 0) { orc_attention(out, q, (const float*)kc, (const float*)vc, pos, heads, kv_heads, hd, kv_width); return; }
    int kv_mul = heads / kv_heads;
    float scale = 1.0f / sqrtf((float)hd);
    float* scores = malloc(sizeof(float) * (size_t)(pos + 1));
    float* row = malloc(sizeof(float) * (size_t)hd);
    uint8_t* qb = malloc((size_t)(hd / 32) * 34);
    const int bph = hd / 32, bpw = kv_width / 32;
    for (int h = 0; h < heads; ++h) {
        int kvh = h / kv_mul;
        const float* qh = q + h * hd;
        if (kind == 2) orc_kv_quantize_row_q8_0(qh, hd, qb);
        for (int p = 0; p <= pos; ++p) {
            float sc;
            if (kind == 1) {
                const uint16_t* k = (const uint16_t*)kc + (size_t)p * kv_width + kvh * hd;
                for (int d = 0; d < hd; ++d) row[d] = orc_f16_to_f32(k[d]);
                float s = 0.0f;
                for (int d = 0; d < hd; ++d) s += qh[d] * row[d];
                sc = s;
            } else {
                const uint8_t* k = (const uint8_t*)kc + ((size_t)p * bpw + (size_t)kvh * bph) * 34;
                float acc = 0.0f;
                for (int b = 0; b < bph; ++b) {
                    const uint8_t* kb = k + (size_t)b * 34;
                    const uint8_t* qq = qb + (size_t)b * 34;
                    int32_t dot = 0;
                    for (int i = 0; i < 32; ++i) dot += (int32_t)(int8_t)qq[2 + i] * (int32_t)(int8_t)kb[2 + i];
                    acc += rd16(qq) * rd16(kb) * (float)dot;   /* q8.rs:509-511 scaled_dot_f32 */
                }
                sc = acc;
            }
            scores[p] = sc * scale;
        }
        softmax(scores, pos + 1);
        float* o = out + h * hd;
        for (int p = 0; p <= pos; ++p) {
            if (kind == 1) {
                const uint16_t* v = (const uint16_t*)vc + (size_t)p * kv_width + kvh * hd;
                for (int d = 0; d < hd; ++d) row[d] = orc_f16_to_f32(v[d]);
            } else {
                const uint8_t* v = (const uint8_t*)vc + ((size_t)p * bpw + (size_t)kvh * bph) * 34;
                for (int b = 0; b < bph; ++b) {
                    float sb = rd16(v + (size_t)b * 34);
                    for (int i = 0; i < 32; ++i) row[b * 32 + i] = (float)(int8_t)v[(size_t)b * 34 + 2 + i] * sb;
                }
            }
            for (int d = 0; d < hd; ++d) o[d] += scores[p] * row[d];
        }
    }
    free(scores); free(row); free(qb);
}

/* inference.rs:4834-4845 sample_logits(temperature 0): first max, strict >. */
int orc_argmax(const float* x, long n) {
    float mv = x[0]; long mi = 0;
    for (long i = 0; i < n; ++i) if (x[i] > mv) { mv = x[i]; mi = i; }
    return (int)mi;
}

/* ------------------------------------------------------------------ GGUF reader */
/* gguf.rs:454-551 read_file: v2/v3 header, metadata, tensor table, aligned data. */
typedef struct { char name[96]; int type; int ndim; uint64_t dims[4]; uint64_t off; } orc_tensor;
typedef struct {
    const uint8_t* map; size_t size; int fd;
    orc_tensor* tensors; int ntensors;
    uint64_t data_start, alignment;
    /* llama hparams (model.rs:48-185) */
    uint32_t ctx, emb, layers, ffn, heads, kv_heads, vocab, head_dim, rope_dim;
    float rope_base, eps;
    char arch[32];
} orc_gguf;

typedef struct { const uint8_t* p; const uint8_t* end; int err; } rd_t;
static uint64_t rd_u(rd_t* r, int n) {
    if (r->p + n > r->end) { r->err = 1; return 0; }
    uint64_t v = 0; for (int i = 0; i < n; ++i) v |= (uint64_t)r->p[i] << (8 * i);
    r->p += n; return v;
}
static int value_size(int t) { switch (t) { case 0: case 1: case 7: return 1; case 2: case 3: return 2; case 4: case 5: case 6: return 4; case 10: case 11: case 12: return 8; default: return -1; } }
static void skip_value(rd_t* r, int t) {
    if (t == 8) { uint64_t n = rd_u(r, 8); r->p += n; return; }
    if (t == 9) { int et = (int)rd_u(r, 4); uint64_t n = rd_u(r, 8); for (uint64_t i = 0; i < n && !r->err; ++i) skip_value(r, et); return; }
    int s = value_size(t); if (s < 0) { r->err = 1; return; } r->p += s;
}

static orc_tensor* find_tensor(orc_gguf* g, const char* name) {
    for (int i = 0; i < g->ntensors; ++i) if (!strcmp(g->tensors[i].name, name)) return &g->tensors[i];
    return NULL;
}

orc_gguf* orc_gguf_open(const char* path) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return NULL;
    struct stat st; fstat(fd, &st);
    const uint8_t* map = (const uint8_t*)mmap(NULL, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (map == MAP_FAILED) { close(fd); return NULL; }
    orc_gguf* g = (orc_gguf*)calloc(1, sizeof(orc_gguf));
    g->map = map; g->size = (size_t)st.st_size; g->fd = fd; g->alignment = 32;
    g->rope_base = 10000.0f; g->eps = 1e-5f;
    rd_t r = { map, map + st.st_size, 0 };
    if (memcmp(map, "GGUF", 4)) goto fail;
    r.p += 4;
    uint32_t ver = (uint32_t)rd_u(&r, 4);
    if (ver < 2 || ver > 3) goto fail;
    uint64_t nt = rd_u(&r, 8), nkv = rd_u(&r, 8);
    for (uint64_t i = 0; i < nkv && !r.err; ++i) {
        uint64_t kl = rd_u(&r, 8);
        char key[128] = {0}; memcpy(key, r.p, kl < 127 ? kl : 127); r.p += kl;
        int t = (int)rd_u(&r, 4);
        const uint8_t* vp = r.p;
        if (!strcmp(key, "general.architecture") && t == 8) {
            uint64_t n = rd_u(&r, 8); memcpy(g->arch, r.p, n < 31 ? n : 31); r.p += n; continue;
        }
        skip_value(&r, t);
        uint64_t u = 0; float f = 0;
        if (t == 4 || t == 5) u = vp[0] | (vp[1] << 8) | (vp[2] << 16) | ((uint32_t)vp[3] << 24);
        if (t == 10) memcpy(&u, vp, 8);
        if (t == 6) memcpy(&f, vp, 4);
        const char* k = strchr(key, '.'); k = k ? k + 1 : key;
        if (!strcmp(key, "general.alignment")) g->alignment = u;
        else if (!strncmp(key, "llama.", 6)) {
            if (!strcmp(k, "context_length")) g->ctx = (uint32_t)u;
            else if (!strcmp(k, "embedding_length")) g->emb = (uint32_t)u;
            else if (!strcmp(k, "block_count")) g->layers = (uint32_t)u;
            else if (!strcmp(k, "feed_forward_length")) g->ffn = (uint32_t)u;
            else if (!strcmp(k, "attention.head_count")) g->heads = (uint32_t)u;
            else if (!strcmp(k, "attention.head_count_kv")) g->kv_heads = (uint32_t)u;
            else if (!strcmp(k, "vocab_size")) g->vocab = (uint32_t)u;
            else if (!strcmp(k, "attention.key_length")) g->head_dim = (uint32_t)u;
            else if (!strcmp(k, "rope.dimension_count")) g->rope_dim = (uint32_t)u;
            else if (!strcmp(k, "rope.freq_base")) g->rope_base = f;
            else if (!strcmp(k, "attention.layer_norm_rms_epsilon")) g->eps = f;
        }
    }
    g->tensors = (orc_tensor*)calloc(nt ? nt : 1, sizeof(orc_tensor));
    g->ntensors = (int)nt;
    for (uint64_t i = 0; i < nt && !r.err; ++i) {
        uint64_t nl = rd_u(&r, 8);
        memcpy(g->tensors[i].name, r.p, nl < 95 ? nl : 95); r.p += nl;
        g->tensors[i].ndim = (int)rd_u(&r, 4);
        for (int d = 0; d < g->tensors[i].ndim && d < 4; ++d) g->tensors[i].dims[d] = rd_u(&r, 8);
        g->tensors[i].type = (int)rd_u(&r, 4);
        g->tensors[i].off = rd_u(&r, 8);
    }
    if (r.err) goto fail;
    uint64_t pos = (uint64_t)(r.p - map);
    g->data_start = (pos + g->alignment - 1) / g->alignment * g->alignment;
    if (g->kv_heads == 0) g->kv_heads = g->heads;
    if (g->heads == 0 || g->emb % g->heads) goto fail;
    if (g->head_dim == 0) g->head_dim = g->emb / g->heads;
    if (g->rope_dim == 0) g->rope_dim = g->head_dim;
    if (g->vocab == 0) {
        orc_tensor* te = find_tensor(g, "token_embd.weight");
        if (!te) goto fail;
        g->vocab = (uint32_t)(te->dims[0] == g->emb ? te->dims[1] : te->dims[0]);
    }
    return g;
fail:
    munmap((void*)map, (size_t)st.st_size); close(fd); free(g->tensors); free(g);
    return NULL;
}

static const uint8_t* tensor_data(orc_gguf* g, orc_tensor* t) { return g->map + g->data_start + t->off; }

/* ------------------------------------------------------------------ model */
typedef struct { int type; long rows; int cols; const uint8_t* data; uint8_t* owned; } qmat;
typedef struct {
    float* attn_norm; float* ffn_norm;
    qmat wq, wk, wv, wo, w1, w2, w3;
} orc_layer;

typedef struct {
    orc_gguf* g;
    int emb, layers, ffn, heads, kv_heads, hd, vocab, rope_dim, ctx, qw, kvw;
    float eps, base;
    int embd_type; const uint8_t* embd;      /* token_embd raw rows, dequantised on demand */
    float* out_norm;
    qmat head;                                 /* untied output.weight or tied Q4_0 requant */
    orc_layer* L;
    float *kc, *vc;                            /* [layer][ctx][kv_width] f32, inference.rs:505-547 */
    int kv_kind;                               /* 0 f32, 1 F16, 2 Q8_0 storage (inference.rs:505-599) */
    uint8_t *kq, *vq;                          /* the F16 / Q8_0 caches when kv_kind != 0 */
    /* workspace (inference.rs:601-695) */
    float *hidden, *residual, *norm_x, *q, *k, *v, *att, *gate, *up, *gu, *logits;
    int8_t* xq; float* xs;
} orc_model;

static float* load_f32(orc_gguf* g, const char* name, long n) {
    orc_tensor* t = find_tensor(g, name);
    if (!t) return NULL;
    float* out = (float*)malloc(sizeof(float) * (size_t)n);
    orc_dequant_row(t->type, tensor_data(g, t), (int)n, out);
    return out;
}
static int load_q(orc_gguf* g, const char* name, qmat* m) {
    orc_tensor* t = find_tensor(g, name);
    if (!t || t->ndim != 2) return -1;
    m->type = t->type; m->cols = (int)t->dims[0]; m->rows = (long)t->dims[1];
    m->data = tensor_data(g, t); m->owned = NULL;
    return 0;
}

void orc_embed_row(const orc_model* m, int token, float* out) {
    orc_dequant_row(m->embd_type, m->embd + (size_t)token * orc_row_bytes(m->embd_type, m->emb), m->emb, out);
}

/* model.rs:471-508: the tied head is the Q4_0 re-quantisation of the dequantised f32
 * token_embd table, block by block (q8.rs:2442-2488). */
static void tied_head(orc_model* m) {
    long V = m->vocab; int H = m->emb, nb = H / 32;
    m->head.type = T_Q4_0; m->head.rows = V; m->head.cols = H;
    m->head.owned = (uint8_t*)malloc((size_t)V * nb * 18);
    m->head.data = m->head.owned;
    #pragma omp parallel
    {
        float* row = (float*)malloc(sizeof(float) * H);
        #pragma omp for schedule(static)
        for (long r = 0; r < V; ++r) {
            orc_embed_row(m, (int)r, row);
            for (int b = 0; b < nb; ++b) orc_quantize_block_q4_0(row + b * 32, m->head.owned + ((size_t)r * nb + b) * 18);
        }
        free(row);
    }
}

/* KV cache [layer][ctx][kv_width] f32 (inference.rs:505-547) and the per-token workspace
 * (inference.rs:601-695). */
static void alloc_workspace(orc_model* m) {
    size_t kvn = (size_t)m->layers * m->ctx * m->kvw;
    m->kc = (float*)calloc(kvn, 4); m->vc = (float*)calloc(kvn, 4);
    int mx = m->emb > m->qw ? m->emb : m->qw; if (m->ffn > mx) mx = m->ffn;
    m->hidden = calloc(m->emb, 4); m->residual = calloc(m->emb, 4); m->norm_x = calloc(m->emb, 4);
    m->q = calloc(m->qw, 4); m->k = calloc(m->kvw, 4); m->v = calloc(m->kvw, 4); m->att = calloc(m->qw, 4);
    m->gate = calloc(m->ffn, 4); m->up = calloc(m->ffn, 4); m->gu = calloc(m->ffn, 4);
    m->logits = calloc(m->vocab, 4); m->xq = calloc(mx, 1); m->xs = calloc(mx / 32 + 1, 4);
}

/* model.rs:461-545 LlamaWeights::load.  Tied head (model.rs:471-532, default
 * NANOCAMELID_Q4_HEAD=on via model.rs:1429-1442): Q4_0 re-quantisation of the
 * dequantised f32 token_embd table, block by block. */
orc_model* orc_model_load(const char* path, int ctx_limit) {
    orc_gguf* g = orc_gguf_open(path);
    if (!g) return NULL;
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->g = g; m->emb = g->emb; m->layers = g->layers; m->ffn = g->ffn; m->heads = g->heads;
    m->kv_heads = g->kv_heads; m->hd = g->head_dim; m->vocab = g->vocab; m->rope_dim = g->rope_dim;
    m->eps = g->eps; m->base = g->rope_base;
    m->ctx = (ctx_limit > 0 && ctx_limit < (int)g->ctx) ? ctx_limit : (int)g->ctx;
    m->qw = m->heads * m->hd; m->kvw = m->kv_heads * m->hd;
    orc_tensor* te = find_tensor(g, "token_embd.weight");
    if (!te) return NULL;
    m->embd_type = te->type; m->embd = tensor_data(g, te);
    m->out_norm = load_f32(g, "output_norm.weight", m->emb);
    if (load_q(g, "output.weight", &m->head) != 0) tied_head(m);
    m->L = (orc_layer*)calloc(m->layers, sizeof(orc_layer));
    char nm[128];
    for (int i = 0; i < m->layers; ++i) {
        orc_layer* l = &m->L[i];
#define LQ(field, s) snprintf(nm, sizeof nm, "blk.%d." s ".weight", i); if (load_q(g, nm, &l->field)) return NULL;
        snprintf(nm, sizeof nm, "blk.%d.attn_norm.weight", i); l->attn_norm = load_f32(g, nm, m->emb);
        snprintf(nm, sizeof nm, "blk.%d.ffn_norm.weight", i); l->ffn_norm = load_f32(g, nm, m->emb);
        LQ(wq, "attn_q") LQ(wk, "attn_k") LQ(wv, "attn_v") LQ(wo, "attn_output")
        LQ(w1, "ffn_gate") LQ(w3, "ffn_up") LQ(w2, "ffn_down")
#undef LQ
    }
    alloc_workspace(m);
    return m;
}

/* ------------------------------------------------------------------ synthetic models
 * The BASELINE configs are random-init models (weights ~ N(0, 0.02), quantised; norms
 * all ones; no checkpoint exists).  The generator that defines those weights is restated
 * here independently of the product library, so that the CPU baseline builds its model in
 * host memory without loading the product or writing a multi-GB GGUF file:
 *   key(tensor)   = splitmix64(FNV-1a64(name) ^ splitmix64(seed))
 *   value(key, i) = (sum of the four 16-bit lanes of splitmix64(key + i) - 131070) * C,
 *                   C = 0.02 sqrt(3) / 65536 rounded to f32 (Irwin-Hall(4), integer only),
 *   element i = row * cols + col of the full tensor;
 * then each block goes through the reference's matrix quantisers (Q4_0 q8.rs:2442-2488,
 * Q8_0 q8.rs:2389-2440).  The reference has no Q4_K encoder (it only decodes Q4_K,
 * q8.rs:1193-1376); the Q4_K blocks are a min/max encoder with 6-bit scales packed the way
 * q8.rs:2009-2018 reads them.  tests/test_cpu_host.py checks every block type against the
 * product's host generator byte for byte. */
typedef struct {
    int32_t emb, layers, heads, kv_heads, head_dim, ffn, vocab, ctx;
    float rope_base, eps;
    int32_t tied, t_embd, t_attn, t_ffn, t_out;
    uint64_t seed;
    int32_t t_down;   /* ffn_down type (0: t_ffn) */
} orc_synth_spec;

static uint64_t syn_mix(uint64_t x) {   /* splitmix64 */
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static float syn_value(uint64_t key, uint64_t idx) {
    uint64_t h = syn_mix(key + idx);
    int s = (int)(h & 0xffff) + (int)((h >> 16) & 0xffff) + (int)((h >> 32) & 0xffff) + (int)(h >> 48);
    return (float)(s - 131070) * 0x1.1bc77ap-21f;
}
uint64_t orc_synth_key(uint64_t seed, const char* name) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (const char* p = name; *p; ++p) { h ^= (uint8_t)*p; h *= 0x100000001b3ull; }
    return syn_mix(h ^ syn_mix(seed));
}

/* Q4_K: per 32-value sub-block j the range [min(0, lo), hi] on a 15-step grid; scales and
 * mins as 6-bit multiples of d = max(scale)/63 and dmin = max(min)/63 (f16, truncated). */
static void syn_encode_q4_k(const float* v, uint8_t* o) {
    float scf[8], mnf[8], maxsc = 0.0f, maxmn = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float lo = v[32 * j], hi = v[32 * j];
        for (int l = 1; l < 32; ++l) { float x = v[32 * j + l]; if (x < lo) lo = x; if (x > hi) hi = x; }
        if (lo > 0.0f) lo = 0.0f;
        scf[j] = (hi - lo) / 15.0f;
        mnf[j] = -lo;
        if (scf[j] > maxsc) maxsc = scf[j];
        if (mnf[j] > maxmn) maxmn = mnf[j];
    }
    uint16_t db = orc_f32_to_f16(maxsc / 63.0f), mb = orc_f32_to_f16(maxmn / 63.0f);
    float dd = orc_f16_to_f32(db), dm = orc_f16_to_f32(mb);
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        float a = dd > 0.0f ? roundf(scf[j] / dd) : 0.0f;
        float b = dm > 0.0f ? roundf(mnf[j] / dm) : 0.0f;
        sc[j] = a < 0.0f ? 0 : (a > 63.0f ? 63 : (int)a);
        mn[j] = b < 0.0f ? 0 : (b > 63.0f ? 63 : (int)b);
    }
    o[0] = db & 0xff; o[1] = db >> 8; o[2] = mb & 0xff; o[3] = mb >> 8;
    uint8_t* s = o + 4;
    for (int j = 0; j < 4; ++j) {   /* the inverse of q8.rs:2009-2018 */
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    for (int p = 0; p < 4; ++p)
        for (int l = 0; l < 32; ++l) {
            int q[2];
            for (int h = 0; h < 2; ++h) {
                int j = 2 * p + h;
                float ds = dd * (float)sc[j], dmv = dm * (float)mn[j];
                float t = ds > 0.0f ? roundf((v[32 * j + l] + dmv) / ds) : 0.0f;
                q[h] = t < 0.0f ? 0 : (t > 15.0f ? 15 : (int)t);
            }
            o[16 + 32 * p + l] = (uint8_t)(q[0] | (q[1] << 4));
        }
}

/* Q6_K (the reference has no encoder, q8.rs:2026-2090 only decodes): per 16-value group
 * an i8 scale round(group_max|x|/31 / d), d = max(group_max|x|/31) / 127 (f16, truncated),
 * 6-bit q = round(x / (d scale)) + 32 clamped to 0..63, its low nibble in ql and its top two
 * bits in qh where q8.rs:2069-2077 reads them. */
static void syn_encode_q6_k(const float* v, uint8_t* o) {
    float gs[16], maxgs = 0.0f;
    for (int g = 0; g < 16; ++g) {
        float amax = 0.0f;
        for (int i = 0; i < 16; ++i) { float a = fabsf(v[16 * g + i]); if (a > amax) amax = a; }
        gs[g] = amax / 31.0f;
        if (gs[g] > maxgs) maxgs = gs[g];
    }
    uint16_t db = orc_f32_to_f16(maxgs / 127.0f);
    float d = orc_f16_to_f32(db);
    int sc[16];
    for (int g = 0; g < 16; ++g) {
        float a = d > 0.0f ? roundf(gs[g] / d) : 0.0f;
        sc[g] = a < 0.0f ? 0 : (a > 127.0f ? 127 : (int)a);
        o[192 + g] = (uint8_t)(int8_t)sc[g];
    }
    memset(o, 0, 192);
    for (int e = 0; e < 256; ++e) {
        float step = d * (float)sc[e / 16];
        float t = step > 0.0f ? roundf(v[e] / step) : 0.0f;
        int q = (t < -32.0f ? -32 : (t > 31.0f ? 31 : (int)t)) + 32;
        int half = e / 128, j = (e % 128) / 32, l = e % 32;
        o[64 * half + l + 32 * (j & 1)] |= (uint8_t)((q & 15) << (j >= 2 ? 4 : 0));
        o[128 + 32 * half + l] |= (uint8_t)((q >> 4) << (2 * j));
    }
    o[208] = db & 0xff; o[209] = db >> 8;
}

/* Rows [r0, r0 + nrows) x columns [c0, c0 + ncols) of a synthetic tensor `cols` wide,
 * raw blocks, row-major, no padding. */
void orc_synth_tensor(int type, uint64_t key, long r0, long nrows, long c0, long ncols, long cols, uint8_t* out) {
    int be = (int)orc_block_elems(type), bb = (int)orc_block_bytes(type);
    long bpr = ncols / be;
    size_t rb = (size_t)bpr * bb;
    #pragma omp parallel for schedule(static)
    for (long r = 0; r < nrows; ++r) {
        float v[256];
        for (long b = 0; b < bpr; ++b) {
            uint64_t base = (uint64_t)(r0 + r) * (uint64_t)cols + (uint64_t)(c0 + b * be);
            uint8_t* o = out + (size_t)r * rb + (size_t)b * bb;
            for (int i = 0; i < be; ++i) v[i] = syn_value(key, base + i);
            if (type == T_Q4_0) orc_quantize_block_q4_0(v, o);
            else if (type == T_Q8_0) orc_quantize_block_q8_0(v, o);
            else if (type == T_Q4_K) syn_encode_q4_k(v, o);
            else if (type == T_Q6_K) syn_encode_q6_k(v, o);
            else if (type == T_F32) memcpy(o, &v[0], 4);
            else { uint16_t h = orc_f32_to_f16(v[0]); o[0] = h & 0xff; o[1] = h >> 8; }
        }
    }
}

static uint8_t* syn_alloc_tensor(const orc_synth_spec* sp, const char* name, int type, long rows, long cols) {
    uint8_t* d = (uint8_t*)malloc(orc_row_bytes(type, (int)cols) * (size_t)rows);
    if (d) orc_synth_tensor(type, orc_synth_key(sp->seed, name), 0, rows, 0, cols, cols, d);
    return d;
}
static int syn_mat(const orc_synth_spec* sp, const char* name, int type, long rows, int cols, qmat* m) {
    m->type = type; m->rows = rows; m->cols = cols;
    m->owned = syn_alloc_tensor(sp, name, type, rows, cols);
    m->data = m->owned;
    return m->owned ? 0 : -1;
}
static float* syn_ones(int n) {
    float* v = (float*)malloc(4 * (size_t)n);
    for (int i = 0; i < n; ++i) v[i] = 1.0f;
    return v;
}

/* The synthetic model in host memory, exactly as orc_model_load would read it from the
 * synthetic GGUF file of the same spec (rope_dim = head_dim; context = spec ctx). */
orc_model* orc_model_create_synthetic(const orc_synth_spec* sp, int ctx_limit) {
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->emb = sp->emb; m->layers = sp->layers; m->ffn = sp->ffn; m->heads = sp->heads; m->kv_heads = sp->kv_heads;
    m->hd = sp->head_dim; m->vocab = sp->vocab; m->rope_dim = sp->head_dim; m->eps = sp->eps; m->base = sp->rope_base;
    m->ctx = (ctx_limit > 0 && ctx_limit < sp->ctx) ? ctx_limit : sp->ctx;
    m->qw = m->heads * m->hd; m->kvw = m->kv_heads * m->hd;
    const int H = m->emb, F = m->ffn, QW = m->qw, KW = m->kvw;
    m->embd_type = sp->t_embd;
    m->embd = syn_alloc_tensor(sp, "token_embd.weight", sp->t_embd, m->vocab, H);
    if (!m->embd) return NULL;
    m->out_norm = syn_ones(H);
    if (sp->tied) tied_head(m);
    else if (syn_mat(sp, "output.weight", sp->t_out, m->vocab, H, &m->head)) return NULL;
    m->L = (orc_layer*)calloc(m->layers, sizeof(orc_layer));
    char nm[128];
    for (int i = 0; i < m->layers; ++i) {
        orc_layer* l = &m->L[i];
        l->attn_norm = syn_ones(H);
        l->ffn_norm = syn_ones(H);
#define SQ(field, s, t, r, c) snprintf(nm, sizeof nm, "blk.%d." s ".weight", i); if (syn_mat(sp, nm, t, r, c, &l->field)) return NULL;
        SQ(wq, "attn_q", sp->t_attn, QW, H) SQ(wk, "attn_k", sp->t_attn, KW, H) SQ(wv, "attn_v", sp->t_attn, KW, H)
        SQ(wo, "attn_output", sp->t_attn, H, QW) SQ(w1, "ffn_gate", sp->t_ffn, F, H) SQ(w3, "ffn_up", sp->t_ffn, F, H)
        SQ(w2, "ffn_down", sp->t_down ? sp->t_down : sp->t_ffn, H, F)
#undef SQ
    }
    alloc_workspace(m);
    return m;
}

/* Fills K/V of positions [0, npos) of every layer with seeded values of the size the
 * projections produce (|x| < 0.5), so that a decode step at position npos does the same
 * attention work as after an npos-token prompt (the timed CPU sample of long contexts). */
void orc_model_fill_kv(orc_model* m, int npos, uint64_t seed) {
    if (npos > m->ctx) npos = m->ctx;
    size_t per = (size_t)npos * m->kvw;
    #pragma omp parallel for schedule(static)
    for (int li = 0; li < m->layers; ++li) {
        size_t lo = (size_t)li * m->ctx * m->kvw;
        uint64_t kk = orc_synth_key(seed, "kv.k") + (uint64_t)li * per, kv = orc_synth_key(seed, "kv.v") + (uint64_t)li * per;
        for (size_t i = 0; i < per; ++i) {
            m->kc[lo + i] = syn_value(kk, i) * 16.0f;
            m->vc[lo + i] = syn_value(kv, i) * 16.0f;
        }
    }
}

/* Bytes of one cached K (or V) row of kv_width values in the cache's storage type. */
static size_t kv_row_bytes(const orc_model* m) {
    return m->kv_kind == 1 ? 2 * (size_t)m->kvw : m->kv_kind == 2 ? (size_t)m->kvw / 32 * 34 : 4 * (size_t)m->kvw;
}

/* inference.rs:512-531: the cache storage the reference picks (NANOCAMELID_KV_CACHE_Q8 when
 * kv_width is a multiple of 32, else NANOCAMELID_KV_CACHE_F16, else f32); kind 1 F16,
 * kind 2 Q8_0.  Clears the cache. */
int orc_model_set_kv_kind(orc_model* m, int kind) {
    if (kind == 2 && m->kvw % 32) kind = 0;
    m->kv_kind = kind;
    free(m->kq); free(m->vq); m->kq = m->vq = NULL;
    if (kind) {
        size_t n = kv_row_bytes(m) * (size_t)m->layers * m->ctx;
        m->kq = calloc(n, 1); m->vq = calloc(n, 1);
    }
    return kind;
}

int orc_model_info(const orc_model* m, int* out) {
    out[0] = m->emb; out[1] = m->layers; out[2] = m->ffn; out[3] = m->heads; out[4] = m->kv_heads;
    out[5] = m->hd; out[6] = m->vocab; out[7] = m->rope_dim; out[8] = m->ctx; out[9] = m->head.type;
    return 10;
}
void orc_model_reset(orc_model* m) {
    size_t kvn = (size_t)m->layers * m->ctx * m->kvw;
    memset(m->kc, 0, kvn * 4); memset(m->vc, 0, kvn * 4);
    if (m->kv_kind) {
        size_t n = kv_row_bytes(m) * (size_t)m->layers * m->ctx;
        memset(m->kq, 0, n); memset(m->vq, 0, n);
    }
}
const uint8_t* orc_model_head_blocks(const orc_model* m) { return m->head.data; }
float* orc_model_hidden(orc_model* m) { return m->hidden; }

static void mm(const qmat* w, const int8_t* xq, const float* xs, float* out) {
    orc_matmul_quantized(w->type, w->data, w->rows, w->cols, xq, xs, out);
}

/* inference.rs:539-568 store_kv at (layer, pos). */
static void kv_store(orc_model* m, int li, int pos, const float* k, const float* v) {
    size_t lo = (size_t)li * m->ctx * m->kvw;
    if (m->kv_kind == 0) {
        memcpy(m->kc + lo + (size_t)pos * m->kvw, k, 4 * (size_t)m->kvw);
        memcpy(m->vc + lo + (size_t)pos * m->kvw, v, 4 * (size_t)m->kvw);
        return;
    }
    size_t off = ((size_t)li * m->ctx + pos) * kv_row_bytes(m);
    if (m->kv_kind == 1) {
        orc_kv_store_f16(k, m->kvw, (uint16_t*)(m->kq + off));
        orc_kv_store_f16(v, m->kvw, (uint16_t*)(m->vq + off));
    } else {
        orc_kv_quantize_row_q8_0(k, m->kvw, m->kq + off);
        orc_kv_quantize_row_q8_0(v, m->kvw, m->vq + off);
    }
}

/* inference.rs:4142-4292 (+ 4319-4458 for the F16 / Q8_0 caches) over layer li. */
static void kv_attend(orc_model* m, int li, float* out, const float* q, int pos) {
    if (m->kv_kind == 0) {
        size_t lo = (size_t)li * m->ctx * m->kvw;
        orc_attention(out, q, m->kc + lo, m->vc + lo, pos, m->heads, m->kv_heads, m->hd, m->kvw);
        return;
    }
    size_t off = (size_t)li * m->ctx * kv_row_bytes(m);
    orc_attention_kv(m->kv_kind, out, q, m->kq + off, m->vq + off, pos, m->heads, m->kv_heads, m->hd, m->kvw);
}

/* inference.rs:4505-4781 run_layer_range (dense FFN) for one token at `pos`. */
static void run_layers(orc_model* m, int pos) {
    for (int li = 0; li < m->layers; ++li) {
        orc_layer* l = &m->L[li];
        memcpy(m->residual, m->hidden, 4 * (size_t)m->emb);
        orc_rms_norm(m->norm_x, m->hidden, l->attn_norm, m->emb, m->eps);
        orc_quantize_q8_0(m->norm_x, m->emb, m->xq, m->xs);
        mm(&l->wq, m->xq, m->xs, m->q);
        mm(&l->wk, m->xq, m->xs, m->k);
        mm(&l->wv, m->xq, m->xs, m->v);
        orc_apply_rope(m->q, pos, m->heads, m->hd, m->rope_dim, m->base);
        orc_apply_rope(m->k, pos, m->kv_heads, m->hd, m->rope_dim, m->base);
        kv_store(m, li, pos, m->k, m->v);
        memset(m->att, 0, 4 * (size_t)m->qw);
        kv_attend(m, li, m->att, m->q, pos);
        orc_quantize_q8_0(m->att, m->qw, m->xq, m->xs);
        mm(&l->wo, m->xq, m->xs, m->hidden);
        for (int i = 0; i < m->emb; ++i) m->hidden[i] += m->residual[i];
        memcpy(m->residual, m->hidden, 4 * (size_t)m->emb);
        orc_rms_norm(m->norm_x, m->hidden, l->ffn_norm, m->emb, m->eps);
        orc_quantize_q8_0(m->norm_x, m->emb, m->xq, m->xs);
        mm(&l->w1, m->xq, m->xs, m->gate);
        mm(&l->w3, m->xq, m->xs, m->up);
        orc_silu_mul(m->gu, m->gate, m->up, m->ffn);
        orc_quantize_q8_0(m->gu, m->ffn, m->xq, m->xs);
        mm(&l->w2, m->xq, m->xs, m->hidden);
        for (int i = 0; i < m->emb; ++i) m->hidden[i] += m->residual[i];
    }
}

/* inference.rs:4783-4832 compute_logits_from_hidden (quantised head). */
void orc_compute_logits(orc_model* m, const float* hidden, float* logits) {
    float* nx = (float*)malloc(4 * (size_t)m->emb);
    int8_t* xq = (int8_t*)malloc(m->emb); float* xs = (float*)malloc(4 * (size_t)(m->emb / 32));
    orc_rms_norm(nx, hidden, m->out_norm, m->emb, m->eps);
    orc_quantize_q8_0(nx, m->emb, xq, xs);
    mm(&m->head, xq, xs, logits);
    free(nx); free(xq); free(xs);
}

/* inference.rs:3649-3670 forward_pass -> 4460-4492 forward_pass_inner.  Returns the
 * greedy token (sample_logits temperature 0); logits copied out when non-NULL. */
int orc_forward_pass(orc_model* m, int token, int pos, float* logits_out) {
    orc_embed_row(m, token, m->hidden);
    run_layers(m, pos);
    orc_compute_logits(m, m->hidden, m->logits);
    if (logits_out) memcpy(logits_out, m->logits, 4 * (size_t)m->vocab);
    return orc_argmax(m->logits, m->vocab);
}

/* bin/cluster_tp_node.rs:808-875 run_reference: prompt token by token, then greedy
 * decode of n_gen tokens (each generated token is fed back). */
int orc_generate(orc_model* m, const int* prompt, int n_prompt, int n_gen, int* out, float* last_logits) {
    int pos = 0, next = 0;
    for (int i = 0; i < n_prompt; ++i) next = orc_forward_pass(m, prompt[i], pos++, NULL);
    for (int g = 0; g < n_gen && pos < m->ctx; ++g) {
        out[g] = next;
        next = orc_forward_pass(m, next, pos++, (g + 1 == n_gen) ? last_logits : NULL);
    }
    return next;
}

/* inference.rs:3695-3744 prefill_pass_batch + 3747-4111 run_layer_range_batch: per
 * token the single-token formulas, KV stored for the whole batch before attention.
 * Writes the final hidden of each token into hidden_out[n][emb]. */
void orc_prefill_batch(orc_model* m, const int* tokens, int n, int start_pos, float* hidden_out) {
    int H = m->emb, F = m->ffn, QW = m->qw, KW = m->kvw;
    float* hid = malloc(4 * (size_t)n * H); float* res = malloc(4 * (size_t)n * H);
    float* nx = malloc(4 * (size_t)n * H); float* q = malloc(4 * (size_t)n * QW);
    float* k = malloc(4 * (size_t)n * KW); float* v = malloc(4 * (size_t)n * KW);
    float* att = malloc(4 * (size_t)n * QW); float* g = malloc(4 * (size_t)n * F);
    float* u = malloc(4 * (size_t)n * F); float* gu = malloc(4 * (size_t)n * F);
    int mx = F > QW ? F : QW; if (H > mx) mx = H;
    int8_t* xq = malloc((size_t)n * mx); float* xs = malloc(4 * (size_t)n * (mx / 32));
    for (int t = 0; t < n; ++t) orc_embed_row(m, tokens[t], hid + (size_t)t * H);
    for (int li = 0; li < m->layers; ++li) {
        orc_layer* l = &m->L[li];
        memcpy(res, hid, 4 * (size_t)n * H);
        for (int t = 0; t < n; ++t) {
            orc_rms_norm(nx + (size_t)t * H, hid + (size_t)t * H, l->attn_norm, H, m->eps);
            orc_quantize_q8_0(nx + (size_t)t * H, H, xq + (size_t)t * H, xs + (size_t)t * (H / 32));
        }
        orc_matmul_quantized_batch(l->wq.type, l->wq.data, l->wq.rows, H, n, xq, xs, q);
        orc_matmul_quantized_batch(l->wk.type, l->wk.data, l->wk.rows, H, n, xq, xs, k);
        orc_matmul_quantized_batch(l->wv.type, l->wv.data, l->wv.rows, H, n, xq, xs, v);
        for (int t = 0; t < n; ++t) {
            int pos = start_pos + t;
            orc_apply_rope(q + (size_t)t * QW, pos, m->heads, m->hd, m->rope_dim, m->base);
            orc_apply_rope(k + (size_t)t * KW, pos, m->kv_heads, m->hd, m->rope_dim, m->base);
            kv_store(m, li, pos, k + (size_t)t * KW, v + (size_t)t * KW);
        }
        memset(att, 0, 4 * (size_t)n * QW);
        for (int t = 0; t < n; ++t) kv_attend(m, li, att + (size_t)t * QW, q + (size_t)t * QW, start_pos + t);
        for (int t = 0; t < n; ++t) orc_quantize_q8_0(att + (size_t)t * QW, QW, xq + (size_t)t * QW, xs + (size_t)t * (QW / 32));
        orc_matmul_quantized_batch(l->wo.type, l->wo.data, H, QW, n, xq, xs, hid);
        for (size_t i = 0; i < (size_t)n * H; ++i) hid[i] += res[i];
        memcpy(res, hid, 4 * (size_t)n * H);
        for (int t = 0; t < n; ++t) {
            orc_rms_norm(nx + (size_t)t * H, hid + (size_t)t * H, l->ffn_norm, H, m->eps);
            orc_quantize_q8_0(nx + (size_t)t * H, H, xq + (size_t)t * H, xs + (size_t)t * (H / 32));
        }
        orc_matmul_quantized_batch(l->w1.type, l->w1.data, F, H, n, xq, xs, g);
        orc_matmul_quantized_batch(l->w3.type, l->w3.data, F, H, n, xq, xs, u);
        orc_silu_mul(gu, g, u, n * F);
        for (int t = 0; t < n; ++t) orc_quantize_q8_0(gu + (size_t)t * F, F, xq + (size_t)t * F, xs + (size_t)t * (F / 32));
        orc_matmul_quantized_batch(l->w2.type, l->w2.data, H, F, n, xq, xs, hid);
        for (size_t i = 0; i < (size_t)n * H; ++i) hid[i] += res[i];
    }
    memcpy(hidden_out, hid, 4 * (size_t)n * H);
    free(hid); free(res); free(nx); free(q); free(k); free(v); free(att); free(g); free(u); free(gu); free(xq); free(xs);
}

/* orc_generate with the prompt ingested `chunk` rows per orc_prefill_batch pass (the
 * reference's batched prefill; every row equals the one-token step, inference.rs:6866-6913),
 * then the greedy loop of bin/cluster_tp_node.rs:808-875. */
int orc_generate_batched(orc_model* m, const int* prompt, int n_prompt, int n_gen, int chunk, int* out, float* last_logits) {
    if (chunk < 1) chunk = 1;
    float* hid = (float*)malloc(4 * (size_t)chunk * m->emb);
    int next = 0, pos = 0;
    for (int c0 = 0; c0 < n_prompt; c0 += chunk) {
        int n = n_prompt - c0 < chunk ? n_prompt - c0 : chunk;
        orc_prefill_batch(m, prompt + c0, n, c0, hid);
        if (c0 + n == n_prompt) {
            orc_compute_logits(m, hid + (size_t)(n - 1) * m->emb, m->logits);
            next = orc_argmax(m->logits, m->vocab);
        }
    }
    free(hid);
    pos = n_prompt;
    for (int g = 0; g < n_gen && pos < m->ctx; ++g) {
        out[g] = next;
        next = orc_forward_pass(m, next, pos++, (g + 1 == n_gen) ? last_logits : NULL);
    }
    return next;
}

/* speculative.rs:299-494 speculative_decoding_step (greedy, no stop tokens).
 * `tlogit_tok` / `dlogit_tok` carry the argmax of the target/draft logits left by
 * the previous pass.  Appends accepted tokens to out; returns the count and
 * updates *pos, the argmaxes and stats[0..1] (drafted, accepted). */
static int spec_step(orc_model* tgt, orc_model* dr, int* pos, int* tlogit_tok, int* dlogit_tok, int k, int* out, int* stats) {
    int start = *pos;
    int maxd = k;
    if (tgt->ctx - (start + 1) < maxd) maxd = tgt->ctx - (start + 1);
    if (dr->ctx - (start + 1) < maxd) maxd = dr->ctx - (start + 1);
    if (maxd <= 0) return 0;
    int drafted[64]; int nd = 0, cur = start;
    while (nd < maxd) {
        int t = *dlogit_tok;
        drafted[nd++] = t;
        *dlogit_tok = orc_forward_pass(dr, t, cur, NULL);
        cur++;
    }
    float* hb = malloc(4 * (size_t)nd * tgt->emb);
    orc_prefill_batch(tgt, drafted, nd, start, hb);
    float* lg = malloc(4 * (size_t)tgt->vocab);
    int nacc = 0, rejected = 0;
    stats[0] += nd;
    for (int i = 0; i < nd; ++i) {
        int tt;
        if (i == 0) tt = *tlogit_tok;
        else { orc_compute_logits(tgt, hb + (size_t)(i - 1) * tgt->emb, lg); tt = orc_argmax(lg, tgt->vocab); }
        if (drafted[i] == tt) { out[nacc++] = tt; stats[1]++; }
        else {
            rejected = 1; out[nacc++] = tt;
            *tlogit_tok = orc_forward_pass(tgt, tt, start + i, NULL);
            *dlogit_tok = orc_forward_pass(dr, tt, start + i, NULL);
            *pos = start + i + 1;
            break;
        }
    }
    if (!rejected) {
        orc_compute_logits(tgt, hb + (size_t)(nd - 1) * tgt->emb, lg);
        int tr = orc_argmax(lg, tgt->vocab);
        out[nacc++] = tr;
        *tlogit_tok = orc_forward_pass(tgt, tr, start + nd, NULL);
        *dlogit_tok = orc_forward_pass(dr, tr, start + nd, NULL);
        *pos = start + nd + 1;
    }
    free(hb); free(lg);
    return nacc;
}

/* main.rs:9604-9830 speculative chat loop shape: prompt through both models token by
 * token, then speculative steps until n_gen tokens.  Returns tokens produced. */
int orc_spec_generate(orc_model* tgt, orc_model* dr, const int* prompt, int n_prompt, int n_gen, int k, int* out, int* stats) {
    int pos = 0, tt = 0, dt = 0, n = 0;
    stats[0] = stats[1] = 0;
    for (int i = 0; i < n_prompt; ++i) { tt = orc_forward_pass(tgt, prompt[i], pos, NULL); dt = orc_forward_pass(dr, prompt[i], pos, NULL); pos++; }
    int buf[80];
    while (n < n_gen) {
        int c = spec_step(tgt, dr, &pos, &tt, &dt, k, buf, stats);
        if (c == 0) break;
        for (int i = 0; i < c && n < n_gen; ++i) out[n++] = buf[i];
    }
    return n;
}

/* speculative.rs:80-105 NGramDrafter::draft: the longest suffix n-gram of history
 * (max_ngram down to min_ngram) with an earlier occurrence, the most recent one; its
 * continuation (up to max_tokens, inside history) is the draft. */
int orc_ngram_draft(const int* h, int len, int max_tokens, int max_ngram, int min_ngram, int* out) {
    if (max_tokens <= 0 || min_ngram <= 0 || len <= min_ngram) return 0;
    int max_n = max_ngram < len - 1 ? max_ngram : len - 1;
    for (int n = max_n; n >= min_ngram; --n) {
        const int* pat = h + len - n;
        for (int start = len - n - 1; start >= 0; --start) {
            if (memcmp(h + start, pat, sizeof(int) * (size_t)n) == 0) {
                int cs = start + n, ce = cs + max_tokens < len ? cs + max_tokens : len;
                if (cs < ce) {
                    memcpy(out, h + cs, sizeof(int) * (size_t)(ce - cs));
                    return ce - cs;
                }
                break;
            }
        }
    }
    return 0;
}

/* speculative.rs:122-297 ngram_speculative_step at temperature 0 (no stop tokens),
 * driven as main.rs:9720-9760: k per step = min(k, remaining - 1); drafts bounded by
 * max_batch - 1 and the context; t0 and the drafts verified as batch rows (each row =
 * a one-token forward pass at its position), a corrective pass on the first mismatch. */
int orc_ngram_generate(orc_model* m, const int* prompt, int n_prompt, int n_gen, int k, int max_ngram, int min_ngram,
                       int max_batch, int* out, int* stats) {
    stats[0] = stats[1] = 0;
    int* hist = malloc(sizeof(int) * (size_t)(n_prompt + n_gen + 2));
    int* drafts = malloc(sizeof(int) * (size_t)(k + 1));
    int len = 0, pos = 0, pred = 0, n = 0;
    for (int i = 0; i < n_prompt; ++i) { pred = orc_forward_pass(m, prompt[i], pos++, NULL); hist[len++] = prompt[i]; }
    while (n < n_gen && pos < m->ctx) {
        int cur_k = k < n_gen - n - 1 ? k : n_gen - n - 1;
        int t0 = pred;
        hist[len] = t0;
        int nd = cur_k > 0 ? orc_ngram_draft(hist, len + 1, cur_k, max_ngram, min_ngram, drafts) : 0;
        if (nd > max_batch - 1) nd = max_batch - 1;
        if (nd > m->ctx - (pos + 1)) nd = m->ctx - (pos + 1);
        if (nd <= 0) {
            out[n++] = t0; hist[len++] = t0;
            pred = orc_forward_pass(m, t0, pos, NULL);
            pos += 1;
            continue;
        }
        stats[0] += nd;
        int g[65];
        g[0] = orc_forward_pass(m, t0, pos, NULL);
        for (int i = 0; i < nd; ++i) g[i + 1] = orc_forward_pass(m, drafts[i], pos + 1 + i, NULL);
        out[n++] = t0; hist[len++] = t0;
        int all = 1;
        for (int i = 0; i < nd; ++i) {
            int tt = g[i];
            if (drafts[i] == tt) {
                stats[1]++;
                out[n++] = tt; hist[len++] = tt;
            } else {
                out[n++] = tt; hist[len++] = tt;
                pred = orc_forward_pass(m, tt, pos + i + 1, NULL);
                pos = pos + i + 2;
                all = 0;
                break;
            }
        }
        if (all) { pred = g[nd]; pos = pos + nd + 1; }
    }
    free(hist); free(drafts);
    return n;
}

/* ------------------------------------------------------------------ tensor parallel */
/* tp.rs:641-660 validate_shares + tp.rs:662-701 shard_geometry.
 * out: q_start q_heads kv_start kv_heads ffn_start ffn_len head_row_start head_rows. */
int orc_shard_geometry(int heads, int kv_total, int ffn, int vocab, const int* shares, int n, int idx, int* out) {
    int sum = 0;
    for (int i = 0; i < n; ++i) { sum += shares[i]; if (shares[i] == 0) return -2; }
    if (sum != kv_total) return -1;
    for (int i = 0; i < n; ++i) if (((long)ffn * shares[i]) % ((long)kv_total * 32)) return -3;
    if (idx < 0 || idx >= n) return -4;
    int qpk = heads / kv_total, kv_start = 0;
    for (int i = 0; i < idx; ++i) kv_start += shares[i];
    int unit = ffn / kv_total;
    long acc = 0, hs = 0, he = 0;
    for (int i = 0; i < n; ++i) {
        if (i == idx) hs = acc;
        acc += ((long)vocab * shares[i] / kv_total) & ~3L;
        if (i == idx) he = acc;
    }
    out[0] = kv_start * qpk; out[1] = shares[idx] * qpk; out[2] = kv_start; out[3] = shares[idx];
    out[4] = kv_start * unit; out[5] = shares[idx] * unit;
    out[6] = (int)hs; out[7] = (idx + 1 == n) ? (int)(vocab - hs) : (int)(he - hs);
    return 0;
}

typedef struct {
    int q0, qh, k0, kh, f0, fl, h0, hr;
    qmat *wq, *wk, *wv, *wo, *w1, *w3, *w2;   /* per layer */
    float *kc, *vc;
    qmat head;
} orc_shard;
typedef struct { orc_model* m; int n; orc_shard* s; } orc_tp;

/* tp.rs:41-49 slice_rows / row_run. */
static qmat slice_rows(const qmat* w, long r0, long r1) {
    qmat o = *w; size_t rb = orc_row_bytes(w->type, w->cols);
    o.rows = r1 - r0; o.owned = malloc(rb * (size_t)o.rows);
    memcpy(o.owned, w->data + rb * r0, rb * (size_t)o.rows); o.data = o.owned; return o;
}
/* tp.rs:61-118 slice_cols / col_gather (block-aligned column slices). */
static qmat slice_cols(const qmat* w, int c0, int c1) {
    qmat o = *w; int be = (int)orc_block_elems(w->type); size_t bb = orc_block_bytes(w->type);
    size_t rb = orc_row_bytes(w->type, w->cols), nrb = (size_t)(c1 - c0) / be * bb;
    o.cols = c1 - c0; o.owned = malloc(nrb * (size_t)w->rows);
    for (long r = 0; r < w->rows; ++r) memcpy(o.owned + nrb * r, w->data + rb * r + (size_t)c0 / be * bb, nrb);
    o.data = o.owned; return o;
}

/* tp.rs:125-199 build_tp_shards + tp.rs:541-570 build_tp_head_shards (tied and untied
 * heads both become row slices of the same head blocks; per-block requantisation makes
 * the tied slices identical to slicing the full requantised head). */
orc_tp* orc_tp_build(orc_model* m, const int* shares, int n) {
    orc_tp* tp = calloc(1, sizeof(orc_tp)); tp->m = m; tp->n = n; tp->s = calloc(n, sizeof(orc_shard));
    for (int i = 0; i < n; ++i) {
        int geo[8];
        if (orc_shard_geometry(m->heads, m->kv_heads, m->ffn, m->vocab, shares, n, i, geo)) return NULL;
        orc_shard* s = &tp->s[i];
        s->q0 = geo[0]; s->qh = geo[1]; s->k0 = geo[2]; s->kh = geo[3]; s->f0 = geo[4]; s->fl = geo[5];
        s->h0 = geo[6]; s->hr = geo[7];
        s->wq = calloc(m->layers, sizeof(qmat)); s->wk = calloc(m->layers, sizeof(qmat)); s->wv = calloc(m->layers, sizeof(qmat));
        s->wo = calloc(m->layers, sizeof(qmat)); s->w1 = calloc(m->layers, sizeof(qmat)); s->w3 = calloc(m->layers, sizeof(qmat));
        s->w2 = calloc(m->layers, sizeof(qmat));
        int hd = m->hd;
        for (int l = 0; l < m->layers; ++l) {
            orc_layer* L = &m->L[l];
            s->wq[l] = slice_rows(&L->wq, (long)s->q0 * hd, (long)(s->q0 + s->qh) * hd);
            s->wk[l] = slice_rows(&L->wk, (long)s->k0 * hd, (long)(s->k0 + s->kh) * hd);
            s->wv[l] = slice_rows(&L->wv, (long)s->k0 * hd, (long)(s->k0 + s->kh) * hd);
            s->wo[l] = slice_cols(&L->wo, s->q0 * hd, (s->q0 + s->qh) * hd);
            s->w1[l] = slice_rows(&L->w1, s->f0, s->f0 + s->fl);
            s->w3[l] = slice_rows(&L->w3, s->f0, s->f0 + s->fl);
            s->w2[l] = slice_cols(&L->w2, s->f0, s->f0 + s->fl);
        }
        size_t kvn = (size_t)m->layers * m->ctx * s->kh * hd;
        s->kc = calloc(kvn, 4); s->vc = calloc(kvn, 4);
        s->head = slice_rows(&m->head, s->h0, s->h0 + s->hr);
    }
    return tp;
}
void orc_tp_reset(orc_tp* tp) {
    for (int i = 0; i < tp->n; ++i) {
        size_t kvn = (size_t)tp->m->layers * tp->m->ctx * tp->s[i].kh * tp->m->hd;
        memset(tp->s[i].kc, 0, kvn * 4); memset(tp->s[i].vc, 0, kvn * 4);
    }
}

/* tp.rs:226-428 tp_forward_token_reduced with the fixed-order reducer of
 * cluster_tp_node.rs:1154-1180: hidden = ((0 + p0) + p1) + ... then + residual.
 * Then head_shard_argmax (tp.rs:576-611) on every shard and the strict->, lowest
 * row_start merge (cluster_tp_node.rs:1185-1204).  Returns the greedy token. */
int orc_tp_forward(orc_tp* tp, int token, int pos, float* logits_out) {
    orc_model* m = tp->m; int H = m->emb, hd = m->hd;
    float* part = malloc(4 * (size_t)H);
    orc_embed_row(m, token, m->hidden);
    for (int li = 0; li < m->layers; ++li) {
        orc_layer* L = &m->L[li];
        memcpy(m->residual, m->hidden, 4 * (size_t)H);
        orc_rms_norm(m->norm_x, m->hidden, L->attn_norm, H, m->eps);
        for (int i = 0; i < H; ++i) m->hidden[i] = 0.0f;
        for (int si = 0; si < tp->n; ++si) {
            orc_shard* s = &tp->s[si];
            int qw = s->qh * hd, kw = s->kh * hd;
            orc_quantize_q8_0(m->norm_x, H, m->xq, m->xs);
            mm(&s->wq[li], m->xq, m->xs, m->q);
            mm(&s->wk[li], m->xq, m->xs, m->k);
            mm(&s->wv[li], m->xq, m->xs, m->v);
            orc_apply_rope(m->q, pos, s->qh, hd, m->rope_dim, m->base);
            orc_apply_rope(m->k, pos, s->kh, hd, m->rope_dim, m->base);
            size_t lo = (size_t)li * m->ctx * kw;
            memcpy(s->kc + lo + (size_t)pos * kw, m->k, 4 * (size_t)kw);
            memcpy(s->vc + lo + (size_t)pos * kw, m->v, 4 * (size_t)kw);
            memset(m->att, 0, 4 * (size_t)qw);
            orc_attention(m->att, m->q, s->kc + lo, s->vc + lo, pos, s->qh, s->kh, hd, kw);
            orc_quantize_q8_0(m->att, qw, m->xq, m->xs);
            mm(&s->wo[li], m->xq, m->xs, part);
            for (int i = 0; i < H; ++i) m->hidden[i] += part[i];
        }
        for (int i = 0; i < H; ++i) m->hidden[i] += m->residual[i];
        memcpy(m->residual, m->hidden, 4 * (size_t)H);
        orc_rms_norm(m->norm_x, m->hidden, L->ffn_norm, H, m->eps);
        for (int i = 0; i < H; ++i) m->hidden[i] = 0.0f;
        for (int si = 0; si < tp->n; ++si) {
            orc_shard* s = &tp->s[si];
            orc_quantize_q8_0(m->norm_x, H, m->xq, m->xs);
            mm(&s->w1[li], m->xq, m->xs, m->gate);
            mm(&s->w3[li], m->xq, m->xs, m->up);
            orc_silu_mul(m->gu, m->gate, m->up, s->fl);
            orc_quantize_q8_0(m->gu, s->fl, m->xq, m->xs);
            mm(&s->w2[li], m->xq, m->xs, part);
            for (int i = 0; i < H; ++i) m->hidden[i] += part[i];
        }
        for (int i = 0; i < H; ++i) m->hidden[i] += m->residual[i];
    }
    float* nx = malloc(4 * (size_t)H); int8_t* xq = malloc(H); float* xs = malloc(4 * (size_t)(H / 32));
    orc_rms_norm(nx, m->hidden, m->out_norm, H, m->eps);
    orc_quantize_q8_0(nx, H, xq, xs);
    int best = 0; float bv = 0.0f;
    for (int si = 0; si < tp->n; ++si) {
        orc_shard* s = &tp->s[si];
        float* lg = logits_out ? logits_out + s->h0 : malloc(4 * (size_t)s->hr);
        mm(&s->head, xq, xs, lg);
        int loc = orc_argmax(lg, s->hr);
        if (si == 0 || lg[loc] > bv) { bv = lg[loc]; best = s->h0 + loc; }
        if (!logits_out) free(lg);
    }
    free(nx); free(xq); free(xs); free(part);
    return best;
}

int orc_tp_generate(orc_tp* tp, const int* prompt, int n_prompt, int n_gen, int* out) {
    int pos = 0, next = 0;
    for (int i = 0; i < n_prompt; ++i) next = orc_tp_forward(tp, prompt[i], pos++, NULL);
    for (int g = 0; g < n_gen && pos < tp->m->ctx; ++g) { out[g] = next; next = orc_tp_forward(tp, next, pos++, NULL); }
    return next;
}

/* Debug view of the workspace (same `which` codes as the product's ncm_debug_read). */
float* orc_model_buf(orc_model* m, int which, int layer) {
    size_t lo = (size_t)layer * m->ctx * m->kvw;
    switch (which) {
        case 0: return m->hidden;
        case 1: return m->q;
        case 2: return m->att;
        case 3: return m->gu;
        case 4: return m->kc + lo;
        case 5: return m->vc + lo;
        case 6: return m->logits;
        default: return NULL;
    }
}
