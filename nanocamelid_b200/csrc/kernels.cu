// sm_100a kernels of the decode hot path.
//
// The GEMV (the whole decode cost: every weight byte is read once per token) streams
// raw GGUF quant blocks from HBM into shared memory with the bulk-copy (TMA) engine,
// `nstages` row tiles in flight per CTA, completion tracked by mbarriers.  The
// activation vector is quantised to Q8_0 once per CTA, straight into registers, in the
// kernel prologue (optionally after the RMSNorm), while the first weight tiles are
// already in flight; programmatic dependent launch lets the next kernel's weight
// prefetch start before this kernel finishes.  Each thread owns fixed 64-column
// "units" (two Q8 activation blocks) of every row, so its activation registers are
// reused across all rows the CTA streams; the per-block integer dots are dp4a sums,
// exact in int32 and bit-identical to the reference's scalar dot.  Epilogues fuse what
// follows each projection in the reference layer loop (inference.rs:4505-4781).
#include <cuda_runtime.h>
#include <stdint.h>
#include <math.h>
#include "ncm_internal.h"
#include "common.cuh"
#include "synth.h"

namespace ncm {

static int g_num_sms = 0;
int num_sms() {
    if (!g_num_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

// ------------------------------------------------------------------ activation (Q8_0)
// Activation registers of one 64-column unit: two Q8_0 blocks.
struct XUnit {
    uint32_t w[16];   // 64 int8 values, 4 per word, element order
    float s[2];       // per-block f32 scale (inference.rs:1008 stores the f32 scale)
    int sum[2];       // per-block sum of the int8 values (for the Q4_0 -8 offset and Q4_K mins)
};

// inference.rs:991-1029 quantize_f32_to_q8_0_scalar for one 32-value block:
// scale = max|x|/127, q = round_half_away(x * (1/scale)) clamped to +-127; zero block -> 0.
__device__ __forceinline__ void quant_block32(const float* v, uint32_t* w, float& s, int& sum) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) { float a = fabsf(v[i]); if (a > amax) amax = a; }
    float scale = amax / 127.0f;
    s = scale;
    int acc = 0;
    if (scale > 0.0f) {
        float inv = 1.0f / scale;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            uint32_t word = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float q = roundf(v[4 * k + j] * inv);
                q = fminf(fmaxf(q, -127.0f), 127.0f);
                int qi = (int)q;
                acc += qi;
                word |= ((uint32_t)(qi & 0xff)) << (8 * j);
            }
            w[k] = word;
        }
    } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = 0;
    }
    sum = acc;
}

// ------------------------------------------------------------------ unit dots
// Q4_0 unit = blocks 2u, 2u+1 = 36 bytes (nine 32-bit words, 4-byte aligned): nine
// LDS.32 per lane with a 9-word stride, conflict-free across the warp.
// q8.rs:2699-2702 dot = sum((nib-8)*x) = sum(nib*x) - 8*sum(x), exact in int32; the
// block term is w_scale * x_scale * (float)dot as in inference.rs:2663.
__device__ __forceinline__ void dots_q4_0(const uint8_t* row, int u, const XUnit& x, int& dA, int& dB, float& sA,
                                          float& sB) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(row + 36 * u);
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = p[i];
    sA = f16_bits_to_f32(w[0] & 0xffff);
    sB = f16_bits_to_f32(w[4] >> 16);
    int a = 0, b = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t q = __funnelshift_r(w[i], w[i + 1], 16);
        a = __dp4a((int)(q & 0x0f0f0f0fu), (int)x.w[i], a);
        a = __dp4a((int)((q >> 4) & 0x0f0f0f0fu), (int)x.w[4 + i], a);
        uint32_t r = w[5 + i];
        b = __dp4a((int)(r & 0x0f0f0f0fu), (int)x.w[8 + i], b);
        b = __dp4a((int)((r >> 4) & 0x0f0f0f0fu), (int)x.w[12 + i], b);
    }
    dA = a - 8 * x.sum[0];
    dB = b - 8 * x.sum[1];
}

// Q8_0 unit = 68 bytes (17 words, conflict-free stride): q8.rs:505 dot_i32.
__device__ __forceinline__ void dots_q8_0(const uint8_t* row, int u, const XUnit& x, int& dA, int& dB, float& sA,
                                          float& sB) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(row + 68 * u);
    uint32_t w[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) w[i] = p[i];
    sA = f16_bits_to_f32(w[0] & 0xffff);
    sB = f16_bits_to_f32(w[8] >> 16);
    int a = 0, b = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        a = __dp4a((int)__funnelshift_r(w[i], w[i + 1], 16), (int)x.w[i], a);
        b = __dp4a((int)w[9 + i], (int)x.w[8 + i], b);
    }
    dA = a;
    dB = b;
}

// q8.rs:2009-2018 q4_k_scale_min over the 12 packed scale bytes held in 3 words.
__device__ __forceinline__ uint32_t sbyte(uint32_t s0, uint32_t s1, uint32_t s2, int i) {
    uint32_t w = i < 4 ? s0 : (i < 8 ? s1 : s2);
    return (w >> (8 * (i & 3))) & 0xff;
}
__device__ __forceinline__ void q4k_scale_min(int idx, uint32_t s0, uint32_t s1, uint32_t s2, int& sc, int& m) {
    if (idx < 4) {
        sc = sbyte(s0, s1, s2, idx) & 63;
        m = sbyte(s0, s1, s2, idx + 4) & 63;
    } else {
        sc = (sbyte(s0, s1, s2, idx + 4) & 0x0f) | ((sbyte(s0, s1, s2, idx - 4) >> 6) << 4);
        m = (sbyte(s0, s1, s2, idx + 4) >> 4) | ((sbyte(s0, s1, s2, idx) >> 6) << 4);
    }
}

// Q4_K unit u = sub-block pair (u & 3) of super-block (u >> 2): 16-byte header shared by
// four lanes (broadcast) + 32 bytes of nibbles (two LDS.128, conflict-free).
// Integer sums of q8.rs:1350-1368; f32 combine of q8.rs:1370-1373.
__device__ __forceinline__ float unit_q4_k(const uint8_t* row, int u, const XUnit& x, int* ints) {
    const uint8_t* sb = row + 144 * (u >> 2);
    const int pr = u & 3;
    uint4 h = *reinterpret_cast<const uint4*>(sb);
    uint4 q0 = *reinterpret_cast<const uint4*>(sb + 16 + 32 * pr);
    uint4 q1 = *reinterpret_cast<const uint4*>(sb + 32 + 32 * pr);
    uint32_t q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    int wl = 0, wh = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        wl = __dp4a((int)(q[i] & 0x0f0f0f0fu), (int)x.w[i], wl);
        wh = __dp4a((int)((q[i] >> 4) & 0x0f0f0f0fu), (int)x.w[8 + i], wh);
    }
    float d = f16_bits_to_f32(h.x & 0xffff), dmin = f16_bits_to_f32(h.x >> 16);
    int sl, ml, sh, mh;
    q4k_scale_min(2 * pr, h.y, h.z, h.w, sl, ml);
    q4k_scale_min(2 * pr + 1, h.y, h.z, h.w, sh, mh);
    if (ints) { ints[0] = wl; ints[1] = x.sum[0]; ints[2] = wh; ints[3] = x.sum[1]; }
    float scl = d * (float)sl, mnl = dmin * (float)ml;
    float sch = d * (float)sh, mnh = dmin * (float)mh;
    float lo = x.s[0] * (scl * (float)wl - mnl * (float)x.sum[0]);
    float hi = x.s[1] * (sch * (float)wh - mnh * (float)x.sum[1]);
    return lo + hi;
}

template <int QT>
__device__ __forceinline__ float unit_dot(const uint8_t* row, int u, const XUnit& x) {
    if constexpr (QT == NCM_T_Q4_K) {
        return unit_q4_k(row, u, x, nullptr);
    } else {
        int dA, dB;
        float sA, sB;
        if constexpr (QT == NCM_T_Q4_0) dots_q4_0(row, u, x, dA, dB, sA, sB);
        else dots_q8_0(row, u, x, dA, dB, sA, sB);
        return sA * x.s[0] * (float)dA + sB * x.s[1] * (float)dB;
    }
}

// ------------------------------------------------------------------ prologue
template <int NPT, int IN>
__device__ __forceinline__ void load_activation(const GemvParams& p, XUnit (&xr)[NPT], int li, float* red) {
    const int tid = threadIdx.x;
    if constexpr (IN == IN_Q8) {
#pragma unroll
        for (int k = 0; k < NPT; ++k) {
            int u = li + 256 * k;
            if (u < p.units) {
                const uint4* src = reinterpret_cast<const uint4*>(p.xq + 64 * u);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    uint4 v = src[i];
                    xr[k].w[4 * i] = v.x; xr[k].w[4 * i + 1] = v.y; xr[k].w[4 * i + 2] = v.z; xr[k].w[4 * i + 3] = v.w;
                }
                xr[k].s[0] = p.xs[2 * u];
                xr[k].s[1] = p.xs[2 * u + 1];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    int s = 0;
#pragma unroll
                    for (int i = 0; i < 8; ++i) s = __dp4a((int)xr[k].w[8 * h + i], 0x01010101, s);
                    xr[k].sum[h] = s;
                }
            }
        }
    } else {
        float scale = 1.0f;
        if constexpr (IN == IN_F32_RMS) {
            // inference.rs:697-706: scale = 1/sqrt(sum(x^2)/n + eps).
            float tot;
            if (p.ssq_tok) {
                // Layer 0: the input is a dequantised embedding row whose normalised values
                // sit exactly on Q8 rounding ties, so the sum must round exactly as the
                // reference's sequential loop does: precomputed per vocab row at load.
                tot = p.ssq_tok[p.tokens[p.state[ST_POS]]];
            } else {
                // Tree sum (sequential in the reference; within f32 rounding).
                float ss = 0.0f;
                for (int i = tid * 4; i < p.cols; i += 4 * kThreads) {
                    float4 v = *reinterpret_cast<const float4*>(p.x + i);
                    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(NCM_FULL, ss, o);
                if ((tid & 31) == 0) red[tid >> 5] = ss;
                __syncthreads();
                tot = 0.0f;
#pragma unroll
                for (int w = 0; w < kThreads / 32; ++w) tot += red[w];
            }
            scale = 1.0f / sqrtf(tot / (float)p.cols + p.eps);
        }
#pragma unroll
        for (int k = 0; k < NPT; ++k) {
            int u = li + 256 * k;
            if (u < p.units) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float v[32];
                    const float4* src = reinterpret_cast<const float4*>(p.x + 64 * u + 32 * h);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        float4 t = src[i];
                        v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
                    }
                    if constexpr (IN == IN_F32_RMS) {
                        const float4* nw = reinterpret_cast<const float4*>(p.norm_w + 64 * u + 32 * h);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            float4 t = nw[i];
                            // inference.rs:704 out = x * scale * weight
                            v[4 * i] = v[4 * i] * scale * t.x;
                            v[4 * i + 1] = v[4 * i + 1] * scale * t.y;
                            v[4 * i + 2] = v[4 * i + 2] * scale * t.z;
                            v[4 * i + 3] = v[4 * i + 3] * scale * t.w;
                        }
                    }
                    quant_block32(v, &xr[k].w[8 * h], xr[k].s[h], xr[k].sum[h]);
                }
            }
        }
    }
}

// ------------------------------------------------------------------ GEMV
struct TileCursor {
    int seg, n;
};
__device__ __forceinline__ TileCursor tile_at(const GemvParams& p, int cur, int r_end) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSeg; ++i)
        if (i < p.nseg && cur >= p.seg[i].row_begin) s = i;
    int seg_end = p.seg[s].row_begin + p.seg[s].rows;
    int n = min(p.tile_rows, min(r_end, seg_end) - cur);
    return {s, n};
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

template <int QT, int NPT, int IN, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr bool DUAL = (EPI == EPI_SILU);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    float* part = reinterpret_cast<float*>(smem + p.part_off);
    uint8_t* stages = smem + p.stage_off;
    __shared__ float red[32];
    __shared__ int s_abort;
    __shared__ float s_bv;
    __shared__ int s_bi;
    __shared__ int s_last;

    const int tid = threadIdx.x;
    const int R = p.total_rows;
    const int nb = gridDim.x;
    const int r_begin = (int)(((long long)blockIdx.x * R / nb)) & ~1;
    const int r_end = (blockIdx.x + 1 == nb) ? R : ((int)(((long long)(blockIdx.x + 1) * R / nb)) & ~1);
    const int half_off = p.tile_rows * p.pitch;   // DUAL: second matrix inside a stage
    const uint64_t limit_ns = 4000000000ull;

    // (1) barriers, then weight prefetch (weights never change: legal before the
    // dependency wait of programmatic dependent launch).
    int icur = r_begin;
    uint64_t pol = 0;
    if (tid == 0) {
        for (int s = 0; s < p.nstages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
        s_abort = 0;
        s_bv = -INFINITY;
        s_bi = 0x7fffffff;
        pol = l2_evict_first_policy();
        for (int s = 0; s < p.nstages && icur < r_end; ++s) {
            TileCursor tc = tile_at(p, icur, r_end);
            uint32_t bytes = (uint32_t)(tc.n * p.pitch);
            const Seg& sg = p.seg[tc.seg];
            size_t off = (size_t)(icur - sg.row_begin) * p.pitch;
            mbar_arrive_expect_tx(&full[s], DUAL ? 2 * bytes : bytes);
            bulk_g2s(stages + (size_t)s * p.stage_bytes, sg.w + off, bytes, &full[s], pol);
            if (DUAL) bulk_g2s(stages + (size_t)s * p.stage_bytes + half_off, sg.w2 + off, bytes, &full[s], pol);
            icur += tc.n;
        }
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();

    // (2) activation -> registers.
    const int pp = p.pp, G = p.groups, np = p.nparts;
    const int g = tid / pp, li = tid % pp;
    XUnit xr[NPT];
    load_activation<NPT, IN>(p, xr, li, red);

    int pos = 0;
    if (EPI == EPI_QKV || EPI == EPI_ARGMAX) pos = p.state[ST_POS];

    float best_v = -INFINITY;
    int best_i = 0x7fffffff;

    // (3) stream the CTA's rows.
    int cur = r_begin, t = 0;
    while (cur < r_end) {
        TileCursor tc = tile_at(p, cur, r_end);
        const int s = t % p.nstages;
        const uint32_t par = (uint32_t)((t / p.nstages) & 1);
        if (!mbar_wait(&full[s], par, limit_ns)) {
            s_abort = 1;
            set_dev_error(p.err, NCM_DEVERR_MBAR_TIMEOUT);
        }
        const uint8_t* sb = stages + (size_t)s * p.stage_bytes;
        float* pb = part + (t & 1) * (p.tile_rows * np * (DUAL ? 2 : 1));
        const int iters = (tc.n + G - 1) / G;
        for (int j = 0; j < iters; ++j) {
            const int rho = g + j * G;
            const bool valid = rho < tc.n;
            const uint8_t* rowp = sb + (size_t)(valid ? rho : 0) * p.pitch;
            float acc = 0.0f, acc2 = 0.0f;
            if (valid) {
#pragma unroll
                for (int k = 0; k < NPT; ++k) {
                    int u = li + 256 * k;
                    if (u < p.units) {
                        acc += unit_dot<QT>(rowp, u, xr[k]);
                        if constexpr (DUAL) acc2 += unit_dot<QT>(rowp + half_off, u, xr[k]);
                    }
                }
            }
            if (pp <= 32) {
                for (int o = pp >> 1; o > 0; o >>= 1) {
                    acc += __shfl_xor_sync(NCM_FULL, acc, o);
                    if constexpr (DUAL) acc2 += __shfl_xor_sync(NCM_FULL, acc2, o);
                }
                if (li == 0 && valid) {
                    pb[rho * np] = acc;
                    if constexpr (DUAL) pb[(p.tile_rows + rho) * np] = acc2;
                }
            } else {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    acc += __shfl_xor_sync(NCM_FULL, acc, o);
                    if constexpr (DUAL) acc2 += __shfl_xor_sync(NCM_FULL, acc2, o);
                }
                if ((tid & 31) == 0 && valid) {
                    pb[rho * np + (li >> 5)] = acc;
                    if constexpr (DUAL) pb[(p.tile_rows + rho) * np + (li >> 5)] = acc2;
                }
            }
        }
        __syncthreads();
        if (s_abort) break;
        // stage s is free: refill it with the next pending tile.
        if (tid == 0 && icur < r_end) {
            TileCursor nc = tile_at(p, icur, r_end);
            uint32_t bytes = (uint32_t)(nc.n * p.pitch);
            const Seg& sg = p.seg[nc.seg];
            size_t off = (size_t)(icur - sg.row_begin) * p.pitch;
            mbar_arrive_expect_tx(&full[s], DUAL ? 2 * bytes : bytes);
            bulk_g2s(stages + (size_t)s * p.stage_bytes, sg.w + off, bytes, &full[s], pol);
            if (DUAL) bulk_g2s(stages + (size_t)s * p.stage_bytes + half_off, sg.w2 + off, bytes, &full[s], pol);
            icur += nc.n;
        }

        // (4) epilogue for this tile.
        const Seg& sg = p.seg[tc.seg];
        const int lrow0 = cur - sg.row_begin;   // segment-local first row
        if constexpr (EPI == EPI_QKV) {
            const int npairs = tc.n >> 1;
            for (int pr = tid; pr < npairs; pr += kThreads) {
                const int rho = 2 * pr;
                float v0 = 0.0f, v1 = 0.0f;
                for (int k = 0; k < np; ++k) { v0 += pb[rho * np + k]; v1 += pb[(rho + 1) * np + k]; }
                const int lr = lrow0 + rho;
                if (sg.kind != SEG_V) {
                    // inference.rs:904-933 apply_rope_cached, NORM pairs (2i, 2i+1).
                    const int i = (lr % p.head_dim) >> 1;
                    if (i < p.rope_half) {
                        float2 sc = p.rope[(size_t)pos * p.rope_half + i];
                        float x0 = v0, x1 = v1;
                        v0 = x0 * sc.y - x1 * sc.x;
                        v1 = x0 * sc.x + x1 * sc.y;
                    }
                }
                if (sg.kind == SEG_Q) {
                    sg.out[lr] = v0; sg.out[lr + 1] = v1;
                } else {
                    float* c = (sg.kind == SEG_K ? p.kcache : p.vcache) + (size_t)pos * p.kv_width;
                    c[lr] = v0; c[lr + 1] = v1;
                }
            }
        } else {
            for (int rho = tid; rho < tc.n; rho += kThreads) {
                float v = 0.0f;
                for (int k = 0; k < np; ++k) v += pb[rho * np + k];
                const int lr = lrow0 + rho;
                if constexpr (EPI == EPI_PLAIN) {
                    sg.out[lr] = v;
                } else if constexpr (EPI == EPI_RESID) {
                    sg.out[lr] += v;   // inference.rs:4670-4672 hidden[i] += residual[i]
                } else if constexpr (EPI == EPI_SILU) {
                    float u = 0.0f;
                    for (int k = 0; k < np; ++k) u += pb[(p.tile_rows + rho) * np + k];
                    // inference.rs:3385-3388 g * (1/(1+exp(-g))) * u
                    float sig = 1.0f / (1.0f + expf(-v));
                    sg.out[lr] = v * sig * u;
                } else if constexpr (EPI == EPI_ARGMAX) {
                    if (sg.out) sg.out[lr] = v;
                    if (better(v, lr, best_v, best_i)) { best_v = v; best_i = lr; }
                } else if constexpr (EPI == EPI_TP_RESID) {
                    // Partial row into slot [rank] of every GPU's receive area (NVLink
                    // stores for peers), tp.rs:357-359 "all-reduce #1/#2" summand.
                    const size_t idx = ((size_t)p.tp_slot * p.tp.world + p.tp.rank) * p.tp.H + lr;
                    for (int d = 0; d < p.tp.world; ++d) p.tp.recv[d][idx] = v;
                }
            }
        }
        cur += tc.n;
        ++t;
    }

    if constexpr (EPI == EPI_ARGMAX) {
        // CTA-local first-max, then the last CTA merges all CTAs (rows ascend with the
        // CTA index, so "larger value, ties to the lower row" == inference.rs:4838-4843).
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(NCM_FULL, best_v, o);
            int oi = __shfl_xor_sync(NCM_FULL, best_i, o);
            if (better(ov, oi, best_v, best_i)) { best_v = ov; best_i = oi; }
        }
        __shared__ float wv[kThreads / 32];
        __shared__ int wi[kThreads / 32];
        if ((tid & 31) == 0) { wv[tid >> 5] = best_v; wi[tid >> 5] = best_i; }
        __syncthreads();
        if (tid == 0) {
            float bv = wv[0];
            int bi = wi[0];
            for (int w = 1; w < kThreads / 32; ++w)
                if (better(wv[w], wi[w], bv, bi)) { bv = wv[w]; bi = wi[w]; }
            p.amax_part[blockIdx.x] = make_float2(bv, __int_as_float(bi));
            __threadfence();
            unsigned prev = atomicAdd(p.counter, 1u);
            s_last = (prev == (unsigned)nb - 1);
        }
        __syncthreads();
        if (s_last && tid == 0) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int c = 0; c < nb; ++c) {
                float2 e = __ldcg(&p.amax_part[c]);
                int ei = __float_as_int(e.y);
                if (better(e.x, ei, bv, bi)) { bv = e.x; bi = ei; }
            }
            int tok = p.head_row0 + bi;
            const unsigned epoch = (unsigned)p.state[ST_STEP] + 1u;
            if (p.head_out) {
                *p.head_out = make_float2(bv, __int_as_float(tok));
                *p.counter = 0u;
                return;
            }
            if (p.tp.world > 1) {
                // Argmax merge across shards (cluster_tp_node.rs:1185-1204): every rank
                // publishes (logit, token) to all ranks, then merges in rank order with
                // strict '>' so the lowest row range wins ties.
                const int W = p.tp.world, me = p.tp.rank;
                for (int d = 0; d < W; ++d) p.tp.hx[d][me] = make_float2(bv, __int_as_float(tok));
                __threadfence_system();
                for (int d = 0; d < W; ++d) st_release_sys(&p.tp.hflags[d][me], epoch);
                uint64_t t0 = global_timer_ns();
                bool ok = true;
                for (int src = 0; src < W; ++src) {
                    while (ld_acquire_sys(&p.tp.hflags[me][src]) < epoch) {
                        if (global_timer_ns() - t0 > p.tp.timeout_ns) { ok = false; break; }
                        __nanosleep(64);
                    }
                    if (!ok) break;
                }
                if (!ok) set_dev_error(p.err, NCM_DEVERR_PEER_TIMEOUT);
                float mv = 0.0f;
                int mt = 0;
                for (int src = 0; src < W; ++src) {
                    float2 e = __ldcg(&p.tp.hx[me][src]);
                    if (src == 0 || e.x > mv) { mv = e.x; mt = __float_as_int(e.y); }
                }
                tok = mt;
            }
            const int ps = p.state[ST_POS];
            if (ps + 1 < p.ctx && ps + 1 >= p.state[ST_NPROMPT]) p.tokens[ps + 1] = tok;
            p.state[ST_LAST_TOKEN] = tok;
            p.state[ST_POS] = ps + 1;
            p.state[ST_STEP] = (int)epoch;
            *p.counter = 0u;
        }
    }

    if constexpr (EPI == EPI_TP_RESID) {
        // Fused row-parallel reduction over NVLink (replaces the TCP star reducer,
        // cluster_tp_node.rs:1154-1180): publish, wait for every rank's slice of the
        // same rows, then sum in rank order on every GPU so all ranks hold identical
        // bits: hidden = ((0 + p0) + p1) + ... then += residual (tp.rs:349-363).
        __syncthreads();
        const int W = p.tp.world, me = p.tp.rank;
        const unsigned epoch = (unsigned)p.state[ST_STEP] + 1u;
        const size_t fslot = ((size_t)p.tp_slot * p.tp.grid_max + blockIdx.x) * W;
        if (tid == 0) {
            __threadfence_system();
            for (int d = 0; d < W; ++d) st_release_sys(&p.tp.flags[d][fslot + me], epoch);
        }
        if (tid < W) {
            uint64_t t0 = global_timer_ns();
            while (ld_acquire_sys(&p.tp.flags[me][fslot + tid]) < epoch) {
                if (global_timer_ns() - t0 > p.tp.timeout_ns) {
                    set_dev_error(p.err, NCM_DEVERR_PEER_TIMEOUT);
                    break;
                }
                __nanosleep(32);
            }
        }
        __syncthreads();
        const float* base = p.tp.recv[me] + (size_t)p.tp_slot * W * p.tp.H;
        for (int r = r_begin + tid; r < r_end; r += kThreads) {
            float s = 0.0f;
            for (int src = 0; src < W; ++src) s += __ldcg(base + (size_t)src * p.tp.H + r);
            p.hidden[r] += s;
        }
    }
}

// ------------------------------------------------------------------ GEMV planning / launch
void gemv_plan(int qtype, int cols, int rows_hint, bool dual, bool need_even, int world_grid, GemvParams& p, int& grid,
               size_t& smem) {
    const int units = cols / 64;
    p.units = units;
    p.cols = cols;
    if (units <= 256) {
        int pp = 1;
        while (pp < units) pp <<= 1;
        p.pp = pp;
        p.groups = kThreads / pp;
    } else {
        p.pp = kThreads;
        p.groups = 1;
    }
    p.nparts = p.pp > 32 ? p.pp / 32 : 1;
    const int row_bytes = p.pitch * (dual ? 2 : 1);
    const int target = 24 * 1024;
    int tr = target / row_bytes;
    if (tr < p.groups) tr = p.groups;          // groups is a power of two (may be 1)
    else tr = tr / p.groups * p.groups;
    if (tr > 256) tr = 256;
    if (need_even && (tr & 1)) tr += 1;        // RoPE pairs must share a tile
    p.tile_rows = tr;
    p.stage_bytes = (tr * row_bytes + 127) / 128 * 128;
    // 4 stages (~96 KB) keeps two CTAs per SM; very wide rows drop to 2-3 stages.
    int ns = (112 * 1024) / p.stage_bytes;
    p.nstages = ns > 4 ? 4 : (ns < 2 ? 2 : ns);
    p.part_off = 128;
    const int part_bytes = 2 * tr * p.nparts * (dual ? 2 : 1) * 4;
    p.stage_off = (p.part_off + part_bytes + 127) / 128 * 128;
    smem = (size_t)p.stage_off + (size_t)p.nstages * p.stage_bytes;
    int g = world_grid > 0 ? world_grid : num_sms();
    int maxg = (rows_hint + 1) / 2;
    if (maxg < 1) maxg = 1;
    grid = g < maxg ? g : maxg;
    (void)qtype;
}

template <int QT, int NPT, int IN, int EPI>
static int launch_t(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    static bool configured = false;
    const size_t smem = (size_t)p.stage_off + (size_t)p.nstages * p.stage_bytes;
    auto kern = gemv_kernel<QT, NPT, IN, EPI>;
    if (!configured) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, kern, p);
}

template <int QT, int NPT>
static int launch_mode(int in_mode, int epi, const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    if (in_mode == IN_F32_RMS && epi == EPI_QKV) return launch_t<QT, NPT, IN_F32_RMS, EPI_QKV>(p, grid, s, pdl);
    if (in_mode == IN_F32_RMS && epi == EPI_SILU) return launch_t<QT, NPT, IN_F32_RMS, EPI_SILU>(p, grid, s, pdl);
    if (in_mode == IN_F32_RMS && epi == EPI_ARGMAX) return launch_t<QT, NPT, IN_F32_RMS, EPI_ARGMAX>(p, grid, s, pdl);
    if (in_mode == IN_F32 && epi == EPI_RESID) return launch_t<QT, NPT, IN_F32, EPI_RESID>(p, grid, s, pdl);
    if (in_mode == IN_F32 && epi == EPI_TP_RESID) return launch_t<QT, NPT, IN_F32, EPI_TP_RESID>(p, grid, s, pdl);
    if (in_mode == IN_F32 && epi == EPI_PLAIN) return launch_t<QT, NPT, IN_F32, EPI_PLAIN>(p, grid, s, pdl);
    if (in_mode == IN_Q8 && epi == EPI_PLAIN) return launch_t<QT, NPT, IN_Q8, EPI_PLAIN>(p, grid, s, pdl);
    return (int)cudaErrorInvalidValue;
}

int gemv_launch(int qtype, int in_mode, int epi, GemvParams p, int grid, cudaStream_t s, bool pdl) {
    const int npt = p.units <= 256 ? 1 : (p.units + 255) / 256;
    if (npt > 2) return (int)cudaErrorInvalidValue;
    if (qtype == NCM_T_Q4_0) return npt == 1 ? launch_mode<NCM_T_Q4_0, 1>(in_mode, epi, p, grid, s, pdl)
                                             : launch_mode<NCM_T_Q4_0, 2>(in_mode, epi, p, grid, s, pdl);
    if (qtype == NCM_T_Q8_0) return npt == 1 ? launch_mode<NCM_T_Q8_0, 1>(in_mode, epi, p, grid, s, pdl)
                                             : launch_mode<NCM_T_Q8_0, 2>(in_mode, epi, p, grid, s, pdl);
    if (qtype == NCM_T_Q4_K) return npt == 1 ? launch_mode<NCM_T_Q4_K, 1>(in_mode, epi, p, grid, s, pdl)
                                             : launch_mode<NCM_T_Q4_K, 2>(in_mode, epi, p, grid, s, pdl);
    return (int)cudaErrorInvalidValue;
}

// ------------------------------------------------------------------ attention
// Decode attention over the f32 KV cache (inference.rs:4242-4292), split over
// positions: CTA (kv head, split) scores its positions for the head group, keeps
// softmax stats, accumulates V; the last CTA of a kv head merges the splits.
__global__ void __launch_bounds__(256) attn_kernel(const __grid_constant__ AttnParams a) {
    extern __shared__ __align__(16) float sh[];
    __shared__ float m_s[8], l_s[8];
    __shared__ int s_last;
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int kvh = blockIdx.x, split = blockIdx.y;
    const int pos = a.state[ST_POS];
    const int n = pos + 1;
    const int per = (n + a.nsplit - 1) / a.nsplit;
    const int p0 = split * per;
    const int p1 = min(n, p0 + per);
    const int np = max(0, p1 - p0);
    const int g = a.heads / a.kv_heads, hd = a.hd;
    float* qs = sh;                       // [g][hd]
    float* sc = sh + g * hd;              // [g][max_per]
    float* rd = sc + g * a.max_per;       // [256 / hd][g][hd]
    for (int i = tid; i < g * hd; i += 256) qs[i] = a.q[(size_t)kvh * g * hd + i];
    __syncthreads();
    const int dpl = hd / 32;
    for (int pi = warp; pi < np; pi += 8) {
        const float* kr = a.kc + (size_t)(p0 + pi) * a.kvw + (size_t)kvh * hd + lane * dpl;
        float kv[8];
        for (int j = 0; j < dpl; ++j) kv[j] = kr[j];
        for (int h = 0; h < g; ++h) {
            float d = 0.0f;
            for (int j = 0; j < dpl; ++j) d += qs[h * hd + lane * dpl + j] * kv[j];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(NCM_FULL, d, o);
            if (lane == 0) sc[h * a.max_per + pi] = d * a.scale;   // inference.rs:4256
        }
    }
    __syncthreads();
    if (warp < g) {
        float m = -INFINITY;
        for (int pi = lane; pi < np; pi += 32) m = fmaxf(m, sc[warp * a.max_per + pi]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(NCM_FULL, m, o));
        float l = 0.0f;
        for (int pi = lane; pi < np; pi += 32) {
            float e = expf(sc[warp * a.max_per + pi] - m);
            sc[warp * a.max_per + pi] = e;
            l += e;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(NCM_FULL, l, o);
        if (lane == 0) { m_s[warp] = m; l_s[warp] = l; }
    }
    __syncthreads();
    const int nsub = 256 / hd, d = tid % hd, sub = tid / hd;
    float acc[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) acc[h] = 0.0f;
    for (int pi = sub; pi < np; pi += nsub) {
        float v = a.vc[(size_t)(p0 + pi) * a.kvw + (size_t)kvh * hd + d];
#pragma unroll
        for (int h = 0; h < 8; ++h)
            if (h < g) acc[h] += sc[h * a.max_per + pi] * v;
    }
#pragma unroll
    for (int h = 0; h < 8; ++h)
        if (h < g) rd[(sub * g + h) * hd + d] = acc[h];
    __syncthreads();
    const int stride = hd + 2;
    for (int i = tid; i < g * hd; i += 256) {
        int h = i / hd, dd = i % hd;
        float s = 0.0f;
        for (int k = 0; k < nsub; ++k) s += rd[(k * g + h) * hd + dd];
        a.part[((size_t)(kvh * g + h) * a.nsplit + split) * stride + 2 + dd] = s;
    }
    if (tid < g) {
        float* pr = a.part + ((size_t)(kvh * g + tid) * a.nsplit + split) * stride;
        pr[0] = np > 0 ? m_s[tid] : -INFINITY;
        pr[1] = np > 0 ? l_s[tid] : 0.0f;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&a.counter[kvh], 1u) == (unsigned)a.nsplit - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = tid; i < g * hd; i += 256) {
        int h = i / hd, dd = i % hd;
        const float* base = a.part + (size_t)(kvh * g + h) * a.nsplit * stride;
        float M = -INFINITY;
        for (int c = 0; c < a.nsplit; ++c) M = fmaxf(M, __ldcg(base + (size_t)c * stride));
        float L = 0.0f, o = 0.0f;
        for (int c = 0; c < a.nsplit; ++c) {
            float mc = __ldcg(base + (size_t)c * stride);
            float f = expf(mc - M);
            L += __ldcg(base + (size_t)c * stride + 1) * f;
            o += __ldcg(base + (size_t)c * stride + 2 + dd) * f;
        }
        a.out[(size_t)(kvh * g + h) * hd + dd] = o / L;
    }
    if (tid == 0) a.counter[kvh] = 0u;
}

int attention_launch(const AttnParams& a, cudaStream_t s, bool pdl) {
    const int g = a.heads / a.kv_heads;
    const size_t smem = (size_t)(g * a.hd + g * a.max_per + 256 * g) * sizeof(float);
    static bool configured = false;
    if (!configured) {
        cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.kv_heads, a.nsplit);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, attn_kernel, a);
}

// ------------------------------------------------------------------ small kernels
// inference.rs:4494-4503 embed_token: one row of the dequantised token_embd table
// (model.rs:1109-1132 dequantisation, done on demand for the current token).
// One element of a dequantised row (model.rs:1109-1132 load_f32_or_f16 semantics).
__device__ __forceinline__ float dequant_elem(int type, const uint8_t* row, int i) {
    if (type == NCM_T_F32) return reinterpret_cast<const float*>(row)[i];
    if (type == NCM_T_F16) return f16_bits_to_f32(row[2 * i] | (row[2 * i + 1] << 8));
    if (type == NCM_T_Q4_K) {
        const uint8_t* b = row + (size_t)(i / 256) * 144;
        int e = i % 256, pr = e / 64, hi = (e % 64) / 32, l = e % 32;
        uint32_t s0 = *reinterpret_cast<const uint32_t*>(b + 4), s1 = *reinterpret_cast<const uint32_t*>(b + 8),
                 s2 = *reinterpret_cast<const uint32_t*>(b + 12);
        int sc, m;
        q4k_scale_min(2 * pr + hi, s0, s1, s2, sc, m);
        float d = f16_bits_to_f32(b[0] | (b[1] << 8)), dmin = f16_bits_to_f32(b[2] | (b[3] << 8));
        uint8_t byte = b[16 + pr * 32 + l];
        int q = hi ? (byte >> 4) : (byte & 0x0f);
        return (d * (float)sc) * (float)q - dmin * (float)m;   // q8.rs:1271-1292 dequantize
    }
    const int bb = ncm_type_block_bytes(type);
    const uint8_t* b = row + (size_t)(i / 32) * bb;
    float d = f16_bits_to_f32(b[0] | (b[1] << 8));
    int e = i % 32, q;
    if (type == NCM_T_Q4_0) q = (e < 16 ? (b[2 + e] & 0x0f) : (b[2 + e - 16] >> 4)) - 8;
    else q = (int)(int8_t)b[2 + e];
    return (float)q * d;
}

__global__ void embed_kernel(int type, const uint8_t* table, int64_t pitch, int emb, const int* tokens,
                             const int* state, float* hidden) {
    pdl_launch_dependents();
    pdl_wait();
    const int tok = tokens[state[ST_POS]];
    const uint8_t* row = table + (size_t)tok * pitch;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < emb; i += gridDim.x * blockDim.x)
        hidden[i] = dequant_elem(type, row, i);
}

// Sequential f32 sum of squares of every dequantised vocab row, in the reference's
// rms_norm loop order (inference.rs:698-701): one thread per row.
__global__ void embed_ssq_kernel(int type, const uint8_t* table, int64_t pitch, int emb, int vocab, float* out) {
    int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= vocab) return;
    const uint8_t* row = table + (size_t)r * pitch;
    float sum = 0.0f;
    for (int i = 0; i < emb; ++i) {
        float v = dequant_elem(type, row, i);
        sum += v * v;
    }
    out[r] = sum;
}
int embed_ssq_launch(int type, const uint8_t* table, int64_t pitch, int emb, int vocab, float* out, cudaStream_t s) {
    embed_ssq_kernel<<<(vocab + 127) / 128, 128, 0, s>>>(type, table, pitch, emb, vocab, out);
    return (int)cudaGetLastError();
}

static cudaLaunchConfig_t small_cfg(dim3 g, dim3 b, cudaStream_t s, bool pdl, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = g;
    cfg.blockDim = b;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

int embed_launch(int type, const uint8_t* table, int64_t pitch, int emb, const int* tokens, const int* state,
                 float* hidden, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = small_cfg(dim3((emb + 255) / 256), dim3(256), s, pdl, attr);
    return (int)cudaLaunchKernelEx(&cfg, embed_kernel, type, table, pitch, emb, tokens, state, hidden);
}

__global__ void resid_add_kernel(float* hidden, const float* part, int n) {
    pdl_launch_dependents();
    pdl_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) hidden[i] += part[i];
}
int resid_add_launch(float* hidden, const float* part, int n, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = small_cfg(dim3((n + 255) / 256), dim3(256), s, pdl, attr);
    return (int)cudaLaunchKernelEx(&cfg, resid_add_kernel, hidden, part, n);
}

// NCCL-baseline argmax merge over all-gathered (logit, token) pairs.
__global__ void argmax_merge_kernel(const float2* gathered, int world, int* tokens, int* state, int ctx) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x != 0) return;
    float mv = 0.0f;
    int mt = 0;
    for (int r = 0; r < world; ++r) {
        float2 e = gathered[r];
        if (r == 0 || e.x > mv) { mv = e.x; mt = __float_as_int(e.y); }
    }
    const int ps = state[ST_POS];
    if (ps + 1 < ctx && ps + 1 >= state[ST_NPROMPT]) tokens[ps + 1] = mt;
    state[ST_LAST_TOKEN] = mt;
    state[ST_POS] = ps + 1;
    state[ST_STEP] += 1;
}
int argmax_merge_launch(const float2* gathered, int world, int* tokens, int* state, int ctx, cudaStream_t s,
                        bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = small_cfg(dim3(1), dim3(32), s, pdl, attr);
    return (int)cudaLaunchKernelEx(&cfg, argmax_merge_kernel, gathered, world, tokens, state, ctx);
}

__global__ void advance_kernel(int* state) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) { state[ST_POS] += 1; state[ST_STEP] += 1; }
}
int advance_launch(int* state, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = small_cfg(dim3(1), dim3(32), s, pdl, attr);
    return (int)cudaLaunchKernelEx(&cfg, advance_kernel, state);
}

// Standalone activation quantiser (quantize_f32_to_q8_0 seam): one thread per block.
__global__ void quantize_kernel(const float* x, int nblocks, int8_t* xq, float* xs) {
    int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    float v[32];
    for (int i = 0; i < 32; ++i) v[i] = x[32 * b + i];
    uint32_t w[8];
    float s;
    int sum;
    quant_block32(v, w, s, sum);
    for (int k = 0; k < 8; ++k) reinterpret_cast<uint32_t*>(xq + 32 * b)[k] = w[k];
    xs[b] = s;
}
int quantize_launch(const float* x, int n, int8_t* xq, float* xs, cudaStream_t s) {
    int nb = n / 32;
    if (nb == 0) return 0;
    quantize_kernel<<<(nb + 127) / 128, 128, 0, s>>>(x, nb, xq, xs);
    return (int)cudaGetLastError();
}

// Per-block integer dots (debug seam of the bit-exact gate), computed with the same
// unit code as the GEMV.
__global__ void block_dots_kernel(int qtype, const uint8_t* w, int64_t rows, int cols, int64_t pitch,
                                  const int8_t* xq, int32_t* out) {
    const int units = cols / 64;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * units) return;
    int64_t r = idx / units;
    int u = (int)(idx % units);
    XUnit x;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(xq + 64 * u);
    for (int i = 0; i < 16; ++i) x.w[i] = src[i];
    x.s[0] = x.s[1] = 1.0f;
    for (int h = 0; h < 2; ++h) {
        int s = 0;
        for (int i = 0; i < 8; ++i) s = __dp4a((int)x.w[8 * h + i], 0x01010101, s);
        x.sum[h] = s;
    }
    const uint8_t* row = w + r * pitch;
    const int nb = cols / 32;
    if (qtype == NCM_T_Q4_K) {
        int ints[4];
        unit_q4_k(row, u, x, ints);
        int32_t* o = out + (r * nb + 2 * u) * 2;
        o[0] = ints[0]; o[1] = ints[1]; o[2] = ints[2]; o[3] = ints[3];
    } else {
        int dA, dB;
        float sA, sB;
        if (qtype == NCM_T_Q4_0) dots_q4_0(row, u, x, dA, dB, sA, sB);
        else dots_q8_0(row, u, x, dA, dB, sA, sB);
        out[r * nb + 2 * u] = dA;
        out[r * nb + 2 * u + 1] = dB;
    }
}
int block_dots_launch(int qtype, const uint8_t* w, int64_t rows, int cols, const int8_t* xq, int32_t* out,
                      cudaStream_t s) {
    int64_t pitch = (int64_t)cols / ncm_type_block_elems(qtype) * ncm_type_block_bytes(qtype);
    int64_t n = rows * (cols / 64);
    if (n == 0) return 0;
    block_dots_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(qtype, w, rows, cols, pitch, xq, out);
    return (int)cudaGetLastError();
}

// Multi-token GEMV (matmul_quantized_batch seam, speculative verify): one warp per row,
// each lane a set of units, every token's activation read from global (L1/L2 resident).
template <int QT>
__global__ void __launch_bounds__(256) gemv_batch_kernel(const uint8_t* w, int64_t rows, int cols, int64_t pitch,
                                                         int ntok, const int8_t* xq, const float* xs, float* out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = cols / 64;
    for (int64_t r = (int64_t)blockIdx.x * 8 + warp; r < rows; r += (int64_t)gridDim.x * 8) {
        const uint8_t* row = w + r * pitch;
        float acc[8];
        for (int t = 0; t < 8; ++t) acc[t] = 0.0f;
        for (int u = lane; u < units; u += 32) {
            for (int t = 0; t < ntok; ++t) {
                XUnit x;
                const uint32_t* src = reinterpret_cast<const uint32_t*>(xq + (size_t)t * cols + 64 * u);
                for (int i = 0; i < 16; ++i) x.w[i] = src[i];
                x.s[0] = xs[(size_t)t * (cols / 32) + 2 * u];
                x.s[1] = xs[(size_t)t * (cols / 32) + 2 * u + 1];
                for (int h = 0; h < 2; ++h) {
                    int s = 0;
                    for (int i = 0; i < 8; ++i) s = __dp4a((int)x.w[8 * h + i], 0x01010101, s);
                    x.sum[h] = s;
                }
                acc[t] += unit_dot<QT>(row, u, x);
            }
        }
        for (int t = 0; t < ntok; ++t) {
            float v = acc[t];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(NCM_FULL, v, o);
            if (lane == 0) out[(size_t)t * rows + r] = v;
        }
    }
}
int gemv_batch_launch(int qtype, const uint8_t* w, int64_t rows, int cols, int pitch, int ntok, const int8_t* xq,
                      const float* xs, float* out, cudaStream_t s) {
    if (rows == 0) return 0;
    int grid = (int)((rows + 7) / 8);
    int cap = num_sms() * 8;
    if (grid > cap) grid = cap;
    if (qtype == NCM_T_Q4_0) gemv_batch_kernel<NCM_T_Q4_0><<<grid, 256, 0, s>>>(w, rows, cols, pitch, ntok, xq, xs, out);
    else if (qtype == NCM_T_Q8_0) gemv_batch_kernel<NCM_T_Q8_0><<<grid, 256, 0, s>>>(w, rows, cols, pitch, ntok, xq, xs, out);
    else if (qtype == NCM_T_Q4_K) gemv_batch_kernel<NCM_T_Q4_K><<<grid, 256, 0, s>>>(w, rows, cols, pitch, ntok, xq, xs, out);
    else return (int)cudaErrorInvalidValue;
    return (int)cudaGetLastError();
}

// inference.rs:697-706 rms_norm (one CTA; tree sum of squares).
__global__ void rms_norm_kernel(float* out, const float* x, const float* w, int n, float eps) {
    __shared__ float red[32];
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(NCM_FULL, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int k = 0; k < (int)(blockDim.x / 32); ++k) tot += red[k];
    float scale = 1.0f / sqrtf(tot / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = x[i] * scale * w[i];
}
int rms_norm_launch(float* out, const float* x, const float* w, int n, float eps, cudaStream_t s) {
    rms_norm_kernel<<<1, 1024, 0, s>>>(out, x, w, n, eps);
    return (int)cudaGetLastError();
}

__global__ void silu_mul_kernel(float* out, const float* g, const float* u, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        float sig = 1.0f / (1.0f + expf(-g[i]));
        out[i] = g[i] * sig * u[i];
    }
}
int silu_mul_launch(float* out, const float* g, const float* u, int n, cudaStream_t s) {
    if (n == 0) return 0;
    silu_mul_kernel<<<(n + 255) / 256, 256, 0, s>>>(out, g, u, n);
    return (int)cudaGetLastError();
}

// On-device synthetic weights (synth.h): rows [r0, r0+nrows) x columns [c0, c0+ncols)
// of a tensor `full_cols` wide, one thread per block, row pitch `pitch`.
__global__ void synth_kernel(int type, uint64_t key, int64_t r0, int64_t nrows, int64_t c0, int64_t ncols,
                             int64_t full_cols, uint8_t* out, int64_t pitch) {
    const int be = ncm_type_block_elems(type), bb = ncm_type_block_bytes(type);
    const int64_t bpr = ncols / be;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= nrows * bpr) return;
    int64_t r = idx / bpr, b = idx % bpr;
    ncm_synth_block(type, key, (uint64_t)(r0 + r), (uint64_t)(c0 + b * be), (uint64_t)full_cols,
                    out + r * pitch + b * bb);
}
int synth_launch(int type, uint64_t key, int64_t r0, int64_t nrows, int64_t c0, int64_t ncols, int64_t full_cols,
                 uint8_t* out, int64_t pitch, cudaStream_t s) {
    int64_t n = nrows * (ncols / ncm_type_block_elems(type));
    if (n == 0) return 0;
    synth_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(type, key, r0, nrows, c0, ncols, full_cols, out, pitch);
    return (int)cudaGetLastError();
}

// Tied LM head (model.rs:471-508 with q4_head_enabled, model.rs:1429-1442): the
// dequantised token_embd rows re-quantised with quantize_f32_matrix_to_q4_0_blocks.
__global__ void requant_q4_0_kernel(int src_type, const uint8_t* src, int64_t rows, int cols, int64_t src_pitch,
                                    uint8_t* dst, int64_t dst_pitch) {
    const int nb = cols / 32;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * nb) return;
    int64_t r = idx / nb;
    int b = (int)(idx % nb);
    float v[32];
    const uint8_t* row = src + r * src_pitch;
    if (src_type == NCM_T_Q4_K) {
        const uint8_t* sb = row + (size_t)(b / 8) * 144;
        int j = b % 8, pr = j / 2, hi = j % 2;
        uint32_t s0 = *reinterpret_cast<const uint32_t*>(sb + 4), s1 = *reinterpret_cast<const uint32_t*>(sb + 8),
                 s2 = *reinterpret_cast<const uint32_t*>(sb + 12);
        int sc, m;
        q4k_scale_min(j, s0, s1, s2, sc, m);
        float d = f16_bits_to_f32(sb[0] | (sb[1] << 8)), dmin = f16_bits_to_f32(sb[2] | (sb[3] << 8));
        float scl = d * (float)sc, mn = dmin * (float)m;
        for (int l = 0; l < 32; ++l) {
            uint8_t byte = sb[16 + pr * 32 + l];
            v[l] = scl * (float)(hi ? (byte >> 4) : (byte & 0x0f)) - mn;
        }
    } else if (src_type == NCM_T_F32) {
        for (int l = 0; l < 32; ++l) v[l] = reinterpret_cast<const float*>(row)[32 * b + l];
    } else if (src_type == NCM_T_F16) {
        for (int l = 0; l < 32; ++l) v[l] = f16_bits_to_f32(row[2 * (32 * b + l)] | (row[2 * (32 * b + l) + 1] << 8));
    } else {
        const int bb = ncm_type_block_bytes(src_type);
        const uint8_t* blk = row + (size_t)b * bb;
        float d = f16_bits_to_f32(blk[0] | (blk[1] << 8));
        for (int l = 0; l < 32; ++l) {
            int q = src_type == NCM_T_Q4_0 ? (l < 16 ? (blk[2 + l] & 0x0f) : (blk[2 + l - 16] >> 4)) - 8
                                           : (int)(int8_t)blk[2 + l];
            v[l] = (float)q * d;
        }
    }
    ncm_encode_q4_0(v, dst + r * dst_pitch + (size_t)b * 18);
}
int requant_q4_0_launch(int src_type, const uint8_t* src, int64_t rows, int cols, int64_t src_pitch, uint8_t* dst,
                        int64_t dst_pitch, cudaStream_t s) {
    int64_t n = rows * (cols / 32);
    if (n == 0) return 0;
    requant_q4_0_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(src_type, src, rows, cols, src_pitch, dst,
                                                                   dst_pitch);
    return (int)cudaGetLastError();
}

// Bounded-wait test: the same flag wait as EPI_TP_RESID on flags nobody sets.
__global__ void peer_timeout_kernel(TpComm c, int* err) {
    if (threadIdx.x >= c.world) return;
    uint64_t t0 = global_timer_ns();
    while (ld_acquire_sys(&c.flags[c.rank][threadIdx.x]) < 1u) {
        if (global_timer_ns() - t0 > c.timeout_ns) {
            set_dev_error(err, NCM_DEVERR_PEER_TIMEOUT);
            return;
        }
        __nanosleep(1000);
    }
}
int peer_timeout_test_launch(TpComm c, int* err, cudaStream_t s) {
    peer_timeout_kernel<<<1, 32, 0, s>>>(c, err);
    return (int)cudaGetLastError();
}

}  // namespace ncm
