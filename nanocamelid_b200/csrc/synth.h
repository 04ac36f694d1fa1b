// Synthetic random-init weights, shared by the host GGUF writer (gguf.cpp) and the
// on-device initialiser (kernels.cu) so that both produce the same bytes.
//
// BASELINE.json's configs are random-init models: weights ~ N(0, 0.02), quantised
// with the reference's own quantisers.  There is no checkpoint to download, so this
// generator defines the weights:
//   value(tensor, i) = (sum of four 16-bit lanes of splitmix64(key + i) - 131070) * C
// an Irwin-Hall(4) approximation of N(0, 0.02) that needs only integer arithmetic and
// one f32 multiply, so host and device agree bit for bit (no libm involved).
//
// Quantisers:
//   Q4_0 : q8.rs:2442-2488 quantize_f32_matrix_to_q4_0_blocks (d = signed-max/-8,
//          q = trunc(x*id + 8.5) clamped to 0..15, f16 scale truncated).
//   Q8_0 : q8.rs:2389-2440 quantize_f32_matrix_to_q8_0_blocks.
//   Q6_K : the reference only decodes Q6_K (q8.rs:2026-2090); this encoder is our own
//          (per 16-value group an i8 scale, d = max group scale / 127, 6-bit values
//          q + 32 split into ql nibbles and qh bit pairs as q8.rs:2069-2077 reads them).
//   Q4_K : the reference only decodes Q4_K (q8.rs:1193-1376); this encoder is our own
//          (per 32-sub-block min/max, 6-bit scales/mins packed as q8.rs:2009-2018 reads
//          them).  Any valid encoder serves: the oracle and the GPU read the same bytes.
// All f32 operations are single IEEE operations (no FMA: host built with
// -ffp-contract=off, device with -fmad=false) and f16 encoding truncates as
// q8.rs:3644-3673 fast_f32_to_f16 does.
#pragma once
#include <stdint.h>
#include <string.h>
#include <math.h>

#if defined(__CUDACC__)
#define NCM_HD __host__ __device__ __forceinline__
#else
#define NCM_HD static inline
#endif

enum { NCM_T_F32 = 0, NCM_T_F16 = 1, NCM_T_Q4_0 = 2, NCM_T_Q8_0 = 8, NCM_T_Q4_K = 12, NCM_T_Q6_K = 14 };

// 0.02 * sqrt(3) / 65536 rounded to f32 (written in hex so every compiler agrees).
#define NCM_SYNTH_SCALE 0x1.1bc77ap-21f

NCM_HD uint64_t ncm_splitmix64(uint64_t x) {
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

NCM_HD float ncm_synth_value(uint64_t key, uint64_t idx) {
    uint64_t h = ncm_splitmix64(key + idx);
    int s = (int)(h & 0xffff) + (int)((h >> 16) & 0xffff) + (int)((h >> 32) & 0xffff) + (int)(h >> 48);
    return (float)(s - 131070) * NCM_SYNTH_SCALE;
}

NCM_HD float ncm_bits_f32(uint32_t b) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(b);
#else
    float f; memcpy(&f, &b, 4); return f;
#endif
}
NCM_HD uint32_t ncm_f32_bits(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t b; memcpy(&b, &f, 4); return b;
#endif
}

// q8.rs:3626-3642 fast_f16_to_f32 (exact).
NCM_HD float ncm_f16_to_f32(uint16_t bits) {
    uint32_t sign = (uint32_t)(bits & 0x8000) << 16;
    uint32_t e = (bits >> 10) & 0x1f, f = bits & 0x3ff;
    if (e == 0) {
        if (f == 0) return ncm_bits_f32(sign);
        int32_t ex = -14;
        while ((f & 0x400) == 0) { f <<= 1; ex -= 1; }
        f &= 0x3ff;
        return ncm_bits_f32(sign | ((uint32_t)(ex + 127) << 23) | (f << 13));
    }
    if (e == 0x1f) return ncm_bits_f32(sign | 0x7f800000u | (f << 13));
    return ncm_bits_f32(sign | ((e + 112) << 23) | (f << 13));
}

// q8.rs:3644-3673 fast_f32_to_f16: mantissa truncation, f32 denormals flush to +-0.
NCM_HD uint16_t ncm_f32_to_f16_trunc(float v) {
    uint32_t bits = ncm_f32_bits(v);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
    int32_t ex = (int32_t)((bits >> 23) & 0xff);
    uint32_t fr = bits & 0x7fffff;
    if (ex == 0) return sign;
    if (ex == 0xff) return fr == 0 ? (uint16_t)(sign | 0x7c00) : (uint16_t)(sign | 0x7c00 | (fr >> 13) | 1);
    int32_t he = ex - 127 + 15;
    if (he >= 0x1f) return (uint16_t)(sign | 0x7c00);
    if (he <= 0) {
        if (he < -10) return sign;
        return (uint16_t)(sign | ((fr | 0x800000u) >> (14 - he)));
    }
    return (uint16_t)(sign | ((uint16_t)he << 10) | (fr >> 13));
}

// Rust `f as i32`: saturating, NaN -> 0.
NCM_HD int32_t ncm_sat_i32(float f) {
    if (f != f) return 0;
    if (f >= 2147483647.0f) return 2147483647;
    if (f <= -2147483648.0f) return -2147483647 - 1;
    return (int32_t)f;
}

NCM_HD void ncm_put16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)(v & 0xff); p[1] = (uint8_t)(v >> 8); }

NCM_HD void ncm_encode_q4_0(const float* c, uint8_t* o) {
    float amax = 0.0f, mx = 0.0f;
    for (int i = 0; i < 32; ++i) { float a = fabsf(c[i]); if (a > amax) { amax = a; mx = c[i]; } }
    float d = mx / -8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    for (int j = 0; j < 16; ++j) {
        float x0 = c[j] * id + 8.5f;
        float x1 = c[j + 16] * id + 8.5f;
        int32_t q0 = ncm_sat_i32(x0), q1 = ncm_sat_i32(x1);
        q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
        q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
        o[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
    ncm_put16(o, ncm_f32_to_f16_trunc(d));
}

NCM_HD void ncm_encode_q8_0(const float* c, uint8_t* o) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) { float a = fabsf(c[i]); if (a > amax) amax = a; }
    float scale = amax / 127.0f;
    for (int i = 0; i < 32; ++i) o[2 + i] = 0;
    if (scale > 0.0f) {
        float inv = 1.0f / scale;
        for (int i = 0; i < 32; ++i) {
            float t = roundf(c[i] * inv);
            t = t < -127.0f ? -127.0f : (t > 127.0f ? 127.0f : t);
            o[2 + i] = (uint8_t)(int8_t)t;
        }
    }
    ncm_put16(o, ncm_f32_to_f16_trunc(scale));
}

NCM_HD void ncm_encode_q4_k(const float* v, uint8_t* o) {
    float scf[8], mnf[8], maxsc = 0.0f, maxmn = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float mn = v[32 * j], mx = v[32 * j];
        for (int l = 1; l < 32; ++l) { float x = v[32 * j + l]; if (x < mn) mn = x; if (x > mx) mx = x; }
        if (mn > 0.0f) mn = 0.0f;
        scf[j] = (mx - mn) / 15.0f;
        mnf[j] = -mn;
        if (scf[j] > maxsc) maxsc = scf[j];
        if (mnf[j] > maxmn) maxmn = mnf[j];
    }
    uint16_t db = ncm_f32_to_f16_trunc(maxsc / 63.0f), mb = ncm_f32_to_f16_trunc(maxmn / 63.0f);
    float dd = ncm_f16_to_f32(db), dm = ncm_f16_to_f32(mb);
    int sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
        float a = dd > 0.0f ? roundf(scf[j] / dd) : 0.0f;
        float b = dm > 0.0f ? roundf(mnf[j] / dm) : 0.0f;
        sc[j] = a < 0.0f ? 0 : (a > 63.0f ? 63 : (int)a);
        m[j] = b < 0.0f ? 0 : (b > 63.0f ? 63 : (int)b);
    }
    ncm_put16(o, db);
    ncm_put16(o + 2, mb);
    uint8_t* s = o + 4;
    for (int j = 0; j < 4; ++j) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
    }
    for (int p = 0; p < 4; ++p)
        for (int l = 0; l < 32; ++l) {
            int q[2];
            for (int h = 0; h < 2; ++h) {
                int j = 2 * p + h;
                float ds = dd * (float)sc[j], dmv = dm * (float)m[j];
                float t = ds > 0.0f ? roundf((v[32 * j + l] + dmv) / ds) : 0.0f;
                q[h] = t < 0.0f ? 0 : (t > 15.0f ? 15 : (int)t);
            }
            o[16 + 32 * p + l] = (uint8_t)(q[0] | (q[1] << 4));
        }
}

// Q6_K block (210 bytes): ql[128] | qh[64] | scales i8[16] | d f16.  Element e of the
// block: half = e / 128, quarter j = (e % 128) / 32, l = e % 32; its low 4 bits are the
// low (j = 0, 1) or high (j = 2, 3) nibble of ql[64 half + l + 32 (j & 1)], its high 2
// bits are bits 2j, 2j+1 of qh[32 half + l]; value = d * scales[e / 16] * (q - 32).
NCM_HD void ncm_encode_q6_k(const float* v, uint8_t* o) {
    float gs[16], maxgs = 0.0f;
    for (int g = 0; g < 16; ++g) {
        float amax = 0.0f;
        for (int i = 0; i < 16; ++i) { float a = fabsf(v[16 * g + i]); if (a > amax) amax = a; }
        gs[g] = amax / 31.0f;
        if (gs[g] > maxgs) maxgs = gs[g];
    }
    uint16_t db = ncm_f32_to_f16_trunc(maxgs / 127.0f);
    float d = ncm_f16_to_f32(db);
    int sc[16];
    for (int g = 0; g < 16; ++g) {
        float a = d > 0.0f ? roundf(gs[g] / d) : 0.0f;
        sc[g] = a < 0.0f ? 0 : (a > 127.0f ? 127 : (int)a);
        o[192 + g] = (uint8_t)(int8_t)sc[g];
    }
    for (int i = 0; i < 192; ++i) o[i] = 0;
    for (int e = 0; e < 256; ++e) {
        float step = d * (float)sc[e / 16];
        float t = step > 0.0f ? roundf(v[e] / step) : 0.0f;
        int q = (t < -32.0f ? -32 : (t > 31.0f ? 31 : (int)t)) + 32;
        int half = e / 128, j = (e % 128) / 32, l = e % 32;
        int qi = 64 * half + l + 32 * (j & 1);
        o[qi] |= (uint8_t)((q & 15) << (j >= 2 ? 4 : 0));
        o[128 + 32 * half + l] |= (uint8_t)((q >> 4) << (2 * j));
    }
    ncm_put16(o + 208, db);
}

NCM_HD int ncm_type_block_elems(int t) {
    return (t == NCM_T_Q4_K || t == NCM_T_Q6_K) ? 256 : (t == NCM_T_Q4_0 || t == NCM_T_Q8_0) ? 32 : 1;
}
NCM_HD int ncm_type_block_bytes(int t) {
    return t == NCM_T_Q4_0 ? 18 : t == NCM_T_Q8_0 ? 34 : t == NCM_T_Q4_K ? 144 : t == NCM_T_Q6_K ? 210
         : t == NCM_T_F32 ? 4 : t == NCM_T_F16 ? 2 : 0;
}

// Encode one block (or one element for F32/F16) of global tensor row `r` starting at
// column `c` (cols = full tensor width) into `o`.
NCM_HD void ncm_synth_block(int type, uint64_t key, uint64_t r, uint64_t c, uint64_t cols, uint8_t* o) {
    uint64_t base = r * cols + c;
    if (type == NCM_T_F32 || type == NCM_T_F16) {
        float v = ncm_synth_value(key, base);
        if (type == NCM_T_F32) { uint32_t b = ncm_f32_bits(v); o[0] = b & 0xff; o[1] = (b >> 8) & 0xff; o[2] = (b >> 16) & 0xff; o[3] = b >> 24; }
        else ncm_put16(o, ncm_f32_to_f16_trunc(v));
        return;
    }
    if (type == NCM_T_Q4_K || type == NCM_T_Q6_K) {
        float v[256];
        for (int i = 0; i < 256; ++i) v[i] = ncm_synth_value(key, base + i);
        if (type == NCM_T_Q4_K) ncm_encode_q4_k(v, o);
        else ncm_encode_q6_k(v, o);
        return;
    }
    float v[32];
    for (int i = 0; i < 32; ++i) v[i] = ncm_synth_value(key, base + i);
    if (type == NCM_T_Q4_0) ncm_encode_q4_0(v, o); else ncm_encode_q8_0(v, o);
}

// Per-tensor stream key: FNV-1a of the GGUF tensor name mixed with the model seed.
static inline uint64_t ncm_synth_key(uint64_t seed, const char* name) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (const char* p = name; *p; ++p) { h ^= (uint8_t)*p; h *= 0x100000001b3ull; }
    return ncm_splitmix64(h ^ ncm_splitmix64(seed));
}
