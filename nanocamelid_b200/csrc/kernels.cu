// sm_100a kernels of the decode hot path.
//
// Parity contract: every f32 value is produced by the same operations in the same
// order as the reference's x86 scalar path (inference.rs / q8.rs), so GPU activations
// are bit-identical to the reference's wherever the reference itself is deterministic
// (the one exception is expf, see expf_cr).  This matters more than it looks: the
// activations are re-quantised to int8 before every projection, and with random-init
// weights a single last-bit difference that moves one value across a rounding tie
// changes an int8 and cascades into ~1e-2 logit differences.  So:
//   * GEMV row sums fold the per-block terms sequentially in block order, one lane per
//     row (inference.rs:1150-1160, 2659-2664, 3129-3133); the per-block integer dots,
//     which are exact, are spread over all threads;
//   * RMSNorm's sum of squares and the softmax denominator reproduce the reference's
//     sequential f32 fold exactly with a parallel algorithm (seq_sum_nonneg);
//   * attention scores, softmax weights and the V accumulation follow
//     inference.rs:4242-4292 term by term.
//
// GEMV data path: raw GGUF blocks are streamed by the TMA engine as 2-D tiles
// (box_rows rows x 512 columns) into a multi-stage shared-memory ring tracked by
// mbarriers; the activation vector is quantised to Q8_0 once per CTA into shared
// memory in the prologue, while the first tiles are in flight.  Programmatic dependent
// launch lets the next kernel's weight prefetch start before this kernel drains.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <math.h>
#include <algorithm>
#include <mutex>
#include <set>
#include <utility>
#include <type_traits>
#include "ncm_internal.h"
#include "common.cuh"
#include "synth.h"

namespace ncm {

int num_sms() {
    // every device of a B200 box has the same count; first call wins (thread-safe init)
    static const int n = [] {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    return n;
}

// Raises a kernel's dynamic shared-memory limit once per (kernel, device): the attribute
// is per device, and several host threads (one per shard) may launch at once.
static int set_smem_limit(const void* fn, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<const void*, int>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (done.count({fn, dev})) return 0;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done.insert({fn, dev});
    return (int)e;
}

EncodeTiledFn encode_tiled_fn() {
    static const EncodeTiledFn fn = [] {   // thread-safe one-time lookup
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return (EncodeTiledFn)p;
        return (EncodeTiledFn) nullptr;
    }();
    return fn;
}

// ------------------------------------------------------------------ exp
// The reference's exp is the host glibc expf (Rust f32::exp).  glibc's expf is not
// correctly rounded, so a device exp must reproduce its exceptions: exp() in double
// rounded to float is the correctly rounded value (up to CUDA's double exp landing
// within one double ulp of a float midpoint), and the inputs where glibc differs from
// it -- all of them lie within 2^-7 ulp of a float rounding midpoint -- are patched from
// an exception hash built on the host from this process's glibc (libm_table.cpp).
// Only values that close to a midpoint (~0.4% of inputs) probe the table, unless the
// host found an exception outside that window (another glibc): then every value probes.
// The table lives in a fixed in-library array (no device allocation), filled once per
// device; g_expf_tab stays null until then (correctly rounded exp without patches).
__device__ uint2 g_expf_store[kExpfTabEntries];
__device__ const uint32_t* g_expf_tab = nullptr;
__device__ uint32_t g_expf_mask = 0;
__device__ int g_expf_gate = 1;

__device__ __forceinline__ float expf_cr(float x) {
    const double yd = exp((double)x);
    const float y = (float)yd;
    const uint32_t* tab = g_expf_tab;
    if (tab != nullptr && y != 0.0f && !isinf(y)) {
        const double yy = (double)y;
        const double half = (yd >= yy ? ((double)nextafterf(y, INFINITY) - yy) : (yy - (double)nextafterf(y, 0.0f))) * 0.5;
        const double dist = fabs(yd - yy);
        if (!g_expf_gate || half - dist <= half * 0x1p-6) {
            const uint32_t key = __float_as_uint(x), mask = g_expf_mask;
            uint32_t h = (key * 2654435761u) & mask;
            for (int probe = 0; probe < 64; ++probe) {
                const uint2 e = reinterpret_cast<const uint2*>(tab)[h];
                if (e.x == key) return __uint_as_float(e.y);
                if (e.x == 0xffffffffu) break;
                h = (h + 1) & mask;
            }
        }
    }
    return y;
}

// Copies the host-built table (pairs {key, value}, power-of-two capacity <=
// kExpfTabEntries) into the in-library array of the current device and publishes it.
int expf_table_install(const uint32_t* host_tab, size_t entries, uint32_t mask, int gate) {
    if (entries > kExpfTabEntries || entries != (size_t)mask + 1) return (int)cudaErrorInvalidValue;
    cudaError_t e = cudaMemcpyToSymbol(g_expf_store, host_tab, entries * sizeof(uint2));
    void* dev = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&dev, g_expf_store);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_expf_mask, &mask, sizeof(mask));
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_expf_gate, &gate, sizeof(gate));
    const uint32_t* p = (const uint32_t*)dev;
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_expf_tab, &p, sizeof(p));
    return (int)e;
}

// ------------------------------------------------------------------ exact sequential sums
// Reproduces   s = 0.0f; for i in [0, n): s = RN(s + t(i))   for t(i) >= 0 exactly.
//
// Within one binade [2^e, 2^(e+1)) floats are a grid of spacing u, and for s = k*u,
// RN(s + t) = u * (k + rint(t/u)) unless t/u is an exact half-integer (a tie, whose
// result depends on the parity of k) or the sum leaves the binade.  So a run of terms
// that keeps the running value inside one binade adds a fixed integer number of ulps
// -- to the bit pattern of s -- independent of where in the binade it starts.
//
// Which binade the running value S(i) is in is certified from an approximate prefix
// A(i) computed in parallel: for nonnegative terms the sequential fold satisfies
// |S(i) - R(i)| <= gamma_i R(i), and any summation tree in which every term goes
// through at most d additions satisfies |A(i) - R(i)| <= gamma_d R(i), where R is the
// exact sum and gamma_k = k u / (1 - k u), u = 2^-24 (Higham, "Accuracy and Stability
// of Numerical Algorithms", 2nd ed., section 4.2).  A term is "certain" when
// A(i-1)(1 - mg) and A(i)(1 + mg) lie in the same binade, mg = 4 u (i + 128) covering
// both bounds (here d < 90) and the rounding of the two products; S(i-1) and S(i) are
// then provably in that binade and, barring a tie, the term adds rint(t/u) ulps.  The
// other terms ("uncertain": binade crossings, ties, the first terms) are listed in
// order; one thread walks the list, adding the ulp count of the certain run before
// each listed term to the bit pattern and the listed term itself with a real FADD --
// about one integer add and one FADD per binade crossing.
//
// Each thread owns a chunk of KM consecutive terms (KM odd, so a warp's reads hit
// distinct banks) held in registers; every per-term step is unrolled so that the
// terms' latencies overlap.  A list that would overflow falls back to a plain
// sequential fold.  Counts are kept modulo 2^32: only differences between consecutive
// list entries are used, each below 2^24.
constexpr int kSeqSerial = 256;   // one-warp sums of at most this many terms: plain fold

template <int NT>
struct SeqSumScratchT {
    static constexpr int kList = NT > 32 ? 512 : 128;   // uncertain terms per segment
    float lt[kList];                    // the uncertain terms, in order
    uint32_t lc[kList];                 // certain-term ulp count before each (mod 2^32)
    float wsum[NT / 32];                // per-warp totals for the block scans
    uint32_t wcnt[NT / 32], wunc[NT / 32];
    uint32_t tail;                      // certain-term ulp count of the whole segment
    int nlist;
    float result;
};
typedef SeqSumScratchT<kThreads> SeqSumScratch;
typedef SeqSumScratchT<32> SeqSumScratchW;

// 1/u for the binade with biased exponent e (24 <= e <= 253): 2^(150 - e), exact.
__device__ __forceinline__ float seq_inv_ulp(int e) { return __uint_as_float((uint32_t)(277 - e) << 23); }

// a = t / u (exact scaling) rounded to the nearest integer, with FADDs only: below 2^23,
// a + 2^23 lands in [2^23, 2^24) where the float grid is the integers, so the add rounds
// a half-even and the bit pattern holds the integer; from 2^23 on, a is an integer.
// False for a tie (|rint(a) - a| = 1/2, the subtraction is exact), for a >= 2^24 and NaN.
__device__ __forceinline__ bool seq_units(float a, uint32_t& c) {
    const float y = a + 8388608.0f;
    const bool lo = a < 8388608.0f;
    const float r = y - 8388608.0f;
    c = lo ? __float_as_uint(y) - 0x4b000000u : __float_as_uint(a) - 0x4a800000u;
    const bool ok = (a < 16777216.0f) & (!lo | (fabsf(r - a) != 0.5f));
    c = ok ? c : 0u;
    return ok;
}

// Term t at global index i, added to a running value whose approximate prefix is ae
// before and ai after the add: true when the running value provably stays in one
// binade and t is no tie there; c = t in ulps of that binade (0 otherwise).  With
// mg = (i + 128) 2^-22, "ae (1 - mg) and ai (1 + mg) in the binade of ae" is checked
// on the significand bits: frac(ae) >= mg and frac(ai) <= 1 - 2 mg with frac the
// fraction field in units of 2^-23, mg 2^23 = 2 (i + 128), plus one unit for the
// roundings of the comparison itself.
__device__ __forceinline__ bool seq_certain(float t, float ae, float ai, int i, uint32_t& c) {
    const uint32_t be = __float_as_uint(ae), bi = __float_as_uint(ai);
    const int e = (int)(be >> 23);
    const uint32_t m = 2u * (uint32_t)(i + 128) + 1u;
    const bool in = (e >= 24) & (e <= 253) & ((int)(bi >> 23) == e) & ((be & 0x7fffffu) >= m) &
                    ((bi & 0x7fffffu) + 2u * m <= 0x7fffffu);
    const bool ok = seq_units(t * seq_inv_ulp(in ? e : 150), c) & in;
    c = ok ? c : 0u;
    return ok;
}

// Adds the terms a0 .. a0+m-1 (m <= GS) to x in order with real FADDs.  All loads are
// issued before the first add.
template <int GS, class Term>
__device__ __forceinline__ float seq_fold(const Term& term, int a0, int m, float x) {
    float tv[GS];
#pragma unroll
    for (int q = 0; q < GS; ++q) tv[q] = q < m ? term(a0 + q) : 0.0f;
    asm volatile("" ::: "memory");
#pragma unroll
    for (int q = 0; q < GS; ++q) x = x + tv[q];   // + 0.0f is exact
    return x;
}

template <class T>
__device__ __forceinline__ T warp_incl_scan(T v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T t = __shfl_up_sync(NCM_FULL, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

// Barrier among the NT threads that take part: the whole CTA (BAR == 0) or named
// barrier BAR with NT threads (a CTA whose other warps run on).
template <int NT, int BAR>
__device__ __forceinline__ void group_sync() {
    if constexpr (BAR == 0) __syncthreads();
    else asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
}
template <int NT, int BAR>
__device__ __forceinline__ int group_sync_or(int pred) {
    if constexpr (BAR == 0) {
        return __syncthreads_or(pred);
    } else {
        int r;
        asm volatile("{ .reg .pred p, q; setp.ne.s32 p, %1, 0; bar.red.or.pred q, %2, %3, p; selp.s32 %0, 1, 0, q; }"
                     : "=r"(r) : "r"(pred), "n"(BAR), "n"(NT) : "memory");
        return r;
    }
}

// One segment (at most KM * NT terms) continuing from the exact value carry.
template <int NT, int KM, int BAR = 0, class Term>
__device__ float seq_sum_segment(const Term& term, int seg0, int segn, float carry, SeqSumScratchT<NT>& sc,
                                 int rank) {
    constexpr int kList = SeqSumScratchT<NT>::kList;
    const int lane = rank & 31, warp = rank >> 5;
    const bool member = rank < NT;
    const int i0 = member ? rank * KM : segn;
    // (1) the chunk into registers; approximate exclusive prefix of the chunk
    float v[KM];
#pragma unroll
    for (int q = 0; q < KM; ++q) v[q] = i0 + q < segn ? term(seg0 + i0 + q) : 0.0f;
    float loc[KM];
    float tot = 0.0f;
#pragma unroll
    for (int q = 0; q < KM; ++q) { tot = tot + v[q]; loc[q] = tot; }
    const float incl = warp_incl_scan(tot, lane);
    float excl = __shfl_up_sync(NCM_FULL, incl, 1);
    if (lane == 0) excl = 0.0f;
    float base = 0.0f;
    if (NT > 32) {
        if (member && lane == 31) sc.wsum[warp] = incl;
        group_sync<NT, BAR>();
        if (member)
            for (int w = 0; w < warp; ++w) base += sc.wsum[w];
    }
    const float off = base + excl;
    // (2) certify each term, four at a time: when the approximate prefix at both ends of
    // a run of four (widened by the error margin of its last index) lies in one binade,
    // S does too over the whole run (S is monotone), and a term of the run is uncertain
    // only if it is a tie; a run that straddles a binade edge is certified term by term.
    // A lane's runs take the same branch as its neighbours' except near the few binade
    // crossings, so the warp rarely executes both.  The first chunk of a sum (running
    // value near zero, crossing binades every few terms) is listed whole.
    uint32_t c[KM];
    uint64_t umask = 0;   // KM may exceed 32
    uint32_t cnt = 0;
    const int nq = min(KM, max(0, segn - i0));
    const bool first = seg0 + i0 == 0 && carry == 0.0f;
    constexpr int kRun = 4;
#pragma unroll
    for (int q0 = 0; q0 < KM; q0 += kRun) {
        const int q1 = q0 + kRun - 1 < KM - 1 ? q0 + kRun - 1 : KM - 1;
        const float alo = carry + (q0 ? off + loc[q0 - 1] : off);
        const float ahi = carry + (off + loc[q1]);
        const float mg = (float)(seg0 + i0 + q1 + 1 + 128) * 0x1p-22f;
        const int er = (int)(__float_as_uint(alo) >> 23);
        const bool run_ok = !first & (er >= 24) & (er <= 253) &
                            ((int)(__float_as_uint(alo * (1.0f - mg)) >> 23) == er) &
                            ((int)(__float_as_uint(ahi * (1.0f + mg)) >> 23) == er);
        if (run_ok) {
            const float inv = seq_inv_ulp(er);
#pragma unroll
            for (int q = q0; q <= q1; ++q) {
                uint32_t cq;
                const bool ok = seq_units(v[q] * inv, cq);   // padding terms are 0: ok, count 0
                c[q] = cq;
                umask |= ok ? 0ull : (1ull << q);
                cnt += cq;
            }
        } else if (first) {
#pragma unroll
            for (int q = q0; q <= q1; ++q) {
                c[q] = 0u;
                umask |= q < nq ? (1ull << q) : 0ull;
            }
        } else {
#pragma unroll
            for (int q = q0; q <= q1; ++q) {
                const float ae = carry + (q ? off + loc[q - 1] : off);
                const float ai = carry + (off + loc[q]);
                const bool valid = q < nq;
                uint32_t cq;
                const bool cert = seq_certain(v[q], ae, ai, seg0 + i0 + q, cq);
                c[q] = valid ? cq : 0u;
                umask |= (valid & !cert) ? (1ull << q) : 0ull;
                cnt += c[q];
            }
        }
    }
    const uint32_t nunc = __popcll(umask);
    // (3) list positions and count offsets (block scans of integers: exact)
    const uint32_t ci = warp_incl_scan(cnt, lane), ui = warp_incl_scan(nunc, lane);
    uint32_t cb = 0, ub = 0;
    if (NT > 32) {
        if (member && lane == 31) { sc.wcnt[warp] = ci; sc.wunc[warp] = ui; }
        group_sync<NT, BAR>();
        if (member)
            for (int w = 0; w < warp; ++w) { cb += sc.wcnt[w]; ub += sc.wunc[w]; }
    }
    if (rank == NT - 1) { sc.tail = cb + ci; sc.nlist = (int)(ub + ui); }
    uint32_t k = ub + ui - nunc, cr = cb + ci - cnt;
    int ovf = member && k + nunc > (uint32_t)kList;
    if (member && !ovf && umask) {
#pragma unroll
        for (int q = 0; q < KM; ++q) {
            if (umask & (1ull << q)) { sc.lt[k] = v[q]; sc.lc[k] = cr; ++k; }
            cr += c[q];
        }
    }
    if (NT > 32) ovf = group_sync_or<NT, BAR>(ovf); else ovf = __any_sync(NCM_FULL, ovf);
    // (4) the walk, by warp 0 in lockstep
    if (rank < 32) {
        float x = carry;
        if (ovf) {
            for (int i = 0; i < segn; i += 32) x = seq_fold<32>(term, seg0 + i, min(32, segn - i), x);
        } else {
            const int nlist = sc.nlist;
            uint32_t bits = __float_as_uint(x), prev = 0;
            int j = 0;
            for (; j + 8 <= nlist; j += 8) {
                float tk[8];
                uint32_t ck[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) { tk[q] = sc.lt[j + q]; ck[q] = sc.lc[j + q]; }
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    bits += ck[q] - prev;
                    prev = ck[q];
                    bits = __float_as_uint(__uint_as_float(bits) + tk[q]);
                }
            }
            for (; j < nlist; ++j) {
                const uint32_t cj = sc.lc[j];
                bits += cj - prev;
                prev = cj;
                bits = __float_as_uint(__uint_as_float(bits) + sc.lt[j]);
            }
            bits += sc.tail - prev;
            x = __uint_as_float(bits);
        }
        if (rank == 0) sc.result = x;
    }
    if (NT == 32) __syncwarp(); else group_sync<NT, BAR>();
    return sc.result;
}

// NT threads (one warp, or the whole 256-thread CTA) cooperate; `rank` is the thread's
// index among them; the terms are read through term(i).  All NT threads get the result;
// with NT > 32 every thread of the CTA must call (threads beyond NT only take part in
// the barriers).
template <int NT, int BAR = 0, class Term>
__device__ float seq_sum_nonneg(const Term& term, int n, SeqSumScratchT<NT>& sc, int rank) {
    if (n <= 0) return 0.0f;
    if (NT == 32 && n <= kSeqSerial) {
        float x = 0.0f;
        for (int i = 0; i < n; i += 32) x = seq_fold<32>(term, i, min(32, n - i), x);
        return x;
    }
    if (n <= 9 * NT) return seq_sum_segment<NT, 9, BAR>(term, 0, n, 0.0f, sc, rank);
    if (n <= 13 * NT) return seq_sum_segment<NT, 13, BAR>(term, 0, n, 0.0f, sc, rank);
    if (n <= 17 * NT) return seq_sum_segment<NT, 17, BAR>(term, 0, n, 0.0f, sc, rank);
    if (n <= 25 * NT) return seq_sum_segment<NT, 25, BAR>(term, 0, n, 0.0f, sc, rank);
    float x = 0.0f;
    for (int seg0 = 0; seg0 < n; seg0 += 33 * NT)
        x = seq_sum_segment<NT, 33, BAR>(term, seg0, min(n - seg0, 33 * NT), x, sc, rank);
    return x;
}

// ------------------------------------------------------------------ activation (Q8_0)
// inference.rs:991-1029 quantize_f32_to_q8_0_scalar for one 32-value block:
// scale = max|x|/127 (kept as f32), q = round_half_away(x * (1/scale)) clamped to
// +-127; zero block -> scale 0, values 0.
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

// Activation of one 64-column unit (two Q8_0 blocks).
struct XUnit {
    uint32_t w[16];
    float s[2];
    int sum[2];
};

// Shared-memory layout of the quantised activation: unit g at xq + 80 g (64 bytes +
// 16 padding so that eight consecutive units hit distinct 16-byte bank groups).
__device__ __forceinline__ void load_xunit(const uint8_t* smem, const GemvParams& p, int g, XUnit& x) {
    const uint4* src = reinterpret_cast<const uint4*>(smem + p.xq_off + 80 * g);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint4 v = src[i];
        x.w[4 * i] = v.x; x.w[4 * i + 1] = v.y; x.w[4 * i + 2] = v.z; x.w[4 * i + 3] = v.w;
    }
    float2 s = reinterpret_cast<const float2*>(smem + p.xs_off)[g];
    int2 c = reinterpret_cast<const int2*>(smem + p.xsum_off)[g];
    x.s[0] = s.x; x.s[1] = s.y;
    x.sum[0] = c.x; x.sum[1] = c.y;
}

// ------------------------------------------------------------------ per-unit block terms
// Q4_0 unit = blocks 2u, 2u+1 (36 bytes, nine words): q8.rs:2699-2702 dot =
// sum((nib-8)*x) = sum(nib*x) - 8*sum(x) exact in int32; term = d_w * x_scale *
// (float)dot as inference.rs:2663 (left to right).
__device__ __forceinline__ void terms_q4_0(const uint8_t* row, int u, const XUnit& x, float& t0, float& t1, int* dots) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(row + 36 * u);
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = p[i];
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
    a -= 8 * x.sum[0];
    b -= 8 * x.sum[1];
    if (dots) { dots[0] = a; dots[1] = b; }
    t0 = f16_bits_to_f32(w[0] & 0xffff) * x.s[0] * (float)a;
    t1 = f16_bits_to_f32(w[4] >> 16) * x.s[1] * (float)b;
}

// Q8_0 unit = 68 bytes (17 words): q8.rs:505 dot_i32; inference.rs:1157.
__device__ __forceinline__ void terms_q8_0(const uint8_t* row, int u, const XUnit& x, float& t0, float& t1, int* dots) {
    const uint32_t* p = reinterpret_cast<const uint32_t*>(row + 68 * u);
    uint32_t w[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) w[i] = p[i];
    int a = 0, b = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        a = __dp4a((int)__funnelshift_r(w[i], w[i + 1], 16), (int)x.w[i], a);
        b = __dp4a((int)w[9 + i], (int)x.w[8 + i], b);
    }
    if (dots) { dots[0] = a; dots[1] = b; }
    t0 = f16_bits_to_f32(w[0] & 0xffff) * x.s[0] * (float)a;
    t1 = f16_bits_to_f32(w[8] >> 16) * x.s[1] * (float)b;
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

// Q4_K unit u = sub-block pair (u & 3) of super-block (u >> 2) counted from `row`:
// terms of sub-blocks 2p and 2p+1 exactly as q8.rs:1370-1373 (x_scale * (d*sc *
// sum(q*x) - dmin*m * sum(x))), with d*sc and dmin*m formed as in q8.rs:1260-1263.
__device__ __forceinline__ void terms_q4_k(const uint8_t* row, int u, const XUnit& x, float& t0, float& t1, int* ints) {
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
    if (ints) { ints[0] = wl; ints[1] = x.sum[0]; ints[2] = wh; ints[3] = x.sum[1]; }
    float d = f16_bits_to_f32(h.x & 0xffff), dmin = f16_bits_to_f32(h.x >> 16);
    int sl, ml, sh, mh;
    q4k_scale_min(2 * pr, h.y, h.z, h.w, sl, ml);
    q4k_scale_min(2 * pr + 1, h.y, h.z, h.w, sh, mh);
    const float scl = d * (float)sl, mnl = dmin * (float)ml;
    const float sch = d * (float)sh, mnh = dmin * (float)mh;
    t0 = x.s[0] * (scl * (float)wl - mnl * (float)x.sum[0]);
    t1 = x.s[1] * (sch * (float)wh - mnh * (float)x.sum[1]);
}

// Four rows' terms of unit u, every shared-memory load issued before the first dot so
// that the rows' latency chains overlap (same arithmetic per row as the one-row forms).
template <int QT, int N>
__device__ __forceinline__ void unit_terms_n(const uint8_t* const (&rows)[N], int u, const XUnit& x, float (&t0)[N],
                                             float (&t1)[N]) {
    if constexpr (QT == NCM_T_Q4_0) {
        uint32_t w[N][9];
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const uint32_t* p = reinterpret_cast<const uint32_t*>(rows[i] + 36 * u);
#pragma unroll
            for (int j = 0; j < 9; ++j) w[i][j] = p[j];
        }
#pragma unroll
        for (int i = 0; i < N; ++i) {
            int a = 0, b = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t q = __funnelshift_r(w[i][k], w[i][k + 1], 16);
                a = __dp4a((int)(q & 0x0f0f0f0fu), (int)x.w[k], a);
                a = __dp4a((int)((q >> 4) & 0x0f0f0f0fu), (int)x.w[4 + k], a);
                const uint32_t r = w[i][5 + k];
                b = __dp4a((int)(r & 0x0f0f0f0fu), (int)x.w[8 + k], b);
                b = __dp4a((int)((r >> 4) & 0x0f0f0f0fu), (int)x.w[12 + k], b);
            }
            a -= 8 * x.sum[0];
            b -= 8 * x.sum[1];
            t0[i] = f16_bits_to_f32(w[i][0] & 0xffff) * x.s[0] * (float)a;
            t1[i] = f16_bits_to_f32(w[i][4] >> 16) * x.s[1] * (float)b;
        }
    } else if constexpr (QT == NCM_T_Q8_0) {
        uint32_t w[N][17];
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const uint32_t* p = reinterpret_cast<const uint32_t*>(rows[i] + 68 * u);
#pragma unroll
            for (int j = 0; j < 17; ++j) w[i][j] = p[j];
        }
#pragma unroll
        for (int i = 0; i < N; ++i) {
            int a = 0, b = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                a = __dp4a((int)__funnelshift_r(w[i][k], w[i][k + 1], 16), (int)x.w[k], a);
                b = __dp4a((int)w[i][9 + k], (int)x.w[8 + k], b);
            }
            t0[i] = f16_bits_to_f32(w[i][0] & 0xffff) * x.s[0] * (float)a;
            t1[i] = f16_bits_to_f32(w[i][8] >> 16) * x.s[1] * (float)b;
        }
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i) terms_q4_k(rows[i], u, x, t0[i], t1[i], nullptr);
    }
}

template <int QT>
__device__ __forceinline__ void unit_terms(const uint8_t* row, int u, const XUnit& x, float& t0, float& t1) {
    if constexpr (QT == NCM_T_Q4_0) terms_q4_0(row, u, x, t0, t1, nullptr);
    else if constexpr (QT == NCM_T_Q8_0) terms_q8_0(row, u, x, t0, t1, nullptr);
    else terms_q4_k(row, u, x, t0, t1, nullptr);
}

// ------------------------------------------------------------------ TMA
// 2-D tiled load (plain, no cluster multicast); x = word column (a multiple of 4 words,
// i.e. 16 bytes), y = row.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// Copies n floats (n a multiple of 4, both pointers 16-byte aligned) from global to
// shared memory with up to eight float4 loads per thread in flight.
__device__ __forceinline__ void stage_f32(float* dst, const float* src, int n, int tid, int nthreads) {
    const int n4 = n >> 2;
    for (int base = 0; base < n4; base += 8 * nthreads) {
        float4 r[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = base + k * nthreads + tid;
            if (i < n4) r[k] = reinterpret_cast<const float4*>(src)[i];
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = base + k * nthreads + tid;
            if (i < n4) reinterpret_cast<float4*>(dst)[i] = r[k];
        }
    }
}

// GEMV block: warps 0-7 compute, 8-9 fold, 10 produces (see ncm_qgemv_kernel).
constexpr int kComputeThreads = 256;
constexpr int kFoldBase = 256;      // first fold thread
constexpr int kProducer = 320;      // producer thread
constexpr int kGemvThreads = 352;
typedef SeqSumScratchT<kGemvThreads> GemvSeqScratch;

// ------------------------------------------------------------------ prologue
// Quantises the activation (optionally RMS-normalised) into shared memory.
template <int IN>
__device__ void gemv_prologue(uint8_t* smem, const GemvParams& p, GemvSeqScratch& sc) {
    const int tid = threadIdx.x;
    const int nblk = p.nchunk * 16;     // padded block count (tail blocks zero)
    float2* xs = reinterpret_cast<float2*>(smem + p.xs_off);
    int2* xsum = reinterpret_cast<int2*>(smem + p.xsum_off);
    if constexpr (IN == IN_Q8) {
        for (int g = tid; g < nblk / 2; g += blockDim.x) {
            uint4* dst = reinterpret_cast<uint4*>(smem + p.xq_off + 80 * g);
            if (2 * g < p.nb) {
                // an odd block count leaves the second block of the last unit empty
                const bool two = 2 * g + 1 < p.nb;
                const uint4* src = reinterpret_cast<const uint4*>(p.xq + 64 * g);
                int s0 = 0, s1 = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    uint4 v = (i < 2 || two) ? src[i] : make_uint4(0, 0, 0, 0);
                    dst[i] = v;
                    int a = i < 2 ? s0 : s1;
                    a = __dp4a((int)v.x, 0x01010101, a);
                    a = __dp4a((int)v.y, 0x01010101, a);
                    a = __dp4a((int)v.z, 0x01010101, a);
                    a = __dp4a((int)v.w, 0x01010101, a);
                    if (i < 2) s0 = a; else s1 = a;
                }
                xs[g] = make_float2(p.xs[2 * g], two ? p.xs[2 * g + 1] : 0.0f);
                xsum[g] = make_int2(s0, s1);
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) dst[i] = make_uint4(0, 0, 0, 0);
                xs[g] = make_float2(0.0f, 0.0f);
                xsum[g] = make_int2(0, 0);
            }
        }
    } else {
        float scale = 1.0f;
        // the input vector, staged with coalesced loads
        float* xf = reinterpret_cast<float*>(smem + p.xf_off);
        stage_f32(xf, p.x, p.cols, tid, blockDim.x);
        __syncthreads();
        if (tid == 0 && p.dbg_ts) p.dbg_ts[(size_t)blockIdx.x * 16 + 12] = global_timer_ns();
        if constexpr (IN == IN_F32_RMS) {
            float tot;
            if (p.ssq_tok) {
                // Layer 0: sum of squares of the embedding row, folded sequentially at load.
                tot = p.ssq_tok[p.tokens[p.state[ST_POS]]];
            } else {
                // inference.rs:698-701: sum += val * val, sequential.
                if (p.tune & 1) {
                    // measurement knob: an unordered tree sum (wrong last bits) to time the exact sum
                    float part = 0.0f;
                    for (int i = tid; i < p.cols; i += blockDim.x) part += xf[i] * xf[i];
                    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(NCM_FULL, part, o);
                    if ((tid & 31) == 0) sc.wsum[tid >> 5] = part;
                    __syncthreads();
                    tot = 0.0f;
                    for (int w = 0; w < kGemvThreads / 32; ++w) tot += sc.wsum[w];
                    __syncthreads();
                } else {
                    tot = seq_sum_nonneg<kGemvThreads>([&](int i) { float v = xf[i]; return v * v; }, p.cols, sc, tid);
                }
            }
            scale = 1.0f / sqrtf(tot / (float)p.cols + p.eps);
            if (tid == 0 && p.dbg_ts) p.dbg_ts[(size_t)blockIdx.x * 16 + 13] = global_timer_ns();
        }
        // Four lanes per 32-value block (quantize_f32_to_q8_0, inference.rs:991-1029):
        // lane li takes elements 8c .. 8c+7 with c = (li + b) & 3 (bank rotation); the
        // block max and the value sum are reduced inside the quad (both order free),
        // every element is rounded exactly as in the one-thread quantiser.
        const int li = tid & 3;
        const unsigned qmask = 0xFu << (tid & 28);
        for (int b = tid >> 2; b < ((p.tune & 2) ? 0 : nblk); b += blockDim.x >> 2) {
            uint32_t* dst = reinterpret_cast<uint32_t*>(smem + p.xq_off + 80 * (b >> 1) + 32 * (b & 1));
            const int c = (li + b) & 3;
            if (b < p.nb) {
                float v[8];
                const float4* xb = reinterpret_cast<const float4*>(xf) + 8 * b + 2 * c;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float4 x4 = xb[h];
                    if constexpr (IN == IN_F32_RMS) {
                        const float4 w4 = reinterpret_cast<const float4*>(smem + p.nw_off)[8 * b + 2 * c + h];
                        // inference.rs:704 out = x * scale * weight
                        v[4 * h] = x4.x * scale * w4.x;
                        v[4 * h + 1] = x4.y * scale * w4.y;
                        v[4 * h + 2] = x4.z * scale * w4.z;
                        v[4 * h + 3] = x4.w * scale * w4.w;
                    } else {
                        v[4 * h] = x4.x; v[4 * h + 1] = x4.y; v[4 * h + 2] = x4.z; v[4 * h + 3] = x4.w;
                    }
                }
                float amax = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
                amax = fmaxf(amax, __shfl_xor_sync(qmask, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(qmask, amax, 2));
                const float scale_b = amax / 127.0f;
                uint32_t w0 = 0, w1 = 0;
                int sum = 0;
                if (scale_b > 0.0f) {
                    const float inv = 1.0f / scale_b;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        float q = roundf(v[i] * inv);
                        q = fminf(fmaxf(q, -127.0f), 127.0f);
                        const int qi = (int)q;
                        sum += qi;
                        const uint32_t byte = (uint32_t)(qi & 0xff) << (8 * (i & 3));
                        if (i < 4) w0 |= byte; else w1 |= byte;
                    }
                }
                sum += __shfl_xor_sync(qmask, sum, 1);
                sum += __shfl_xor_sync(qmask, sum, 2);
                dst[2 * c] = w0;
                dst[2 * c + 1] = w1;
                if (li == 0) {
                    reinterpret_cast<float*>(xs)[b] = scale_b;
                    reinterpret_cast<int*>(xsum)[b] = sum;
                }
            } else {
                dst[2 * c] = 0;
                dst[2 * c + 1] = 0;
                if (li == 0) {
                    reinterpret_cast<float*>(xs)[b] = 0.0f;
                    reinterpret_cast<int*>(xsum)[b] = 0;
                }
            }
        }
    }
}

// ------------------------------------------------------------------ GEMV
struct TileCursor {
    int seg, n;
};
// With p.fused the segments' matrices lie back to back in one buffer under one tensor
// map (tm[0]): tiles run across segment boundaries and each row finds its segment in the
// epilogue.  Otherwise a tile stays inside one segment (its own tensor map).
__device__ __forceinline__ int seg_of(const GemvParams& p, int row) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSeg; ++i)
        if (i < p.nseg && row >= p.seg[i].row_begin) s = i;
    return s;
}
__device__ __forceinline__ TileCursor tile_at(const GemvParams& p, int cur, int r_end) {
    if (p.fused) return {0, min(p.box_rows, r_end - cur)};
    const int s = seg_of(p, cur);
    const int seg_end = p.seg[s].row_begin + p.seg[s].rows;
    const int n = min(p.box_rows, min(r_end, seg_end) - cur);
    return {s, n};
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
    return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// L2 prefetch (cp.async.bulk.prefetch.L2) of up to pf_bytes of this CTA's share of the
// next kernel's weight rows: the rows [b R / grid, (b+1) R / grid) of the next launch's
// fused row space (both matrices of a dual pair).  Row pitches are multiples of 16 bytes.
__device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__device__ __forceinline__ void prefetch_l2(const uint8_t* a, int64_t bytes) {
    for (int64_t o = 0; o < bytes; o += 32768) {
        const uint32_t n = (uint32_t)min64(32768, bytes - o);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a + o), "r"(n) : "memory");
    }
}
__device__ void prefetch_next_weights(const GemvParams& p) {
    if (p.pf_nmat == 0 || (int)blockIdx.x >= p.pf_grid) return;
    const int b = blockIdx.x;
    int64_t budget = p.pf_bytes;
    if (p.pf_dual) {
        const int R = p.pf_rows[0];
        const int r0 = (int)((long long)b * R / p.pf_grid), r1 = (int)((long long)(b + 1) * R / p.pf_grid);
        for (int m = 0; m < p.pf_nmat; ++m)
            prefetch_l2(p.pf_base[m] + (int64_t)r0 * p.pf_pitch[m],
                        min64((int64_t)(r1 - r0) * p.pf_pitch[m], budget / p.pf_nmat));
        return;
    }
    int R = 0;
    for (int m = 0; m < p.pf_nmat; ++m) R += p.pf_rows[m];
    const int r0 = (int)((long long)b * R / p.pf_grid), r1 = (int)((long long)(b + 1) * R / p.pf_grid);
    int seg0 = 0;
    for (int m = 0; m < p.pf_nmat && budget > 0; ++m) {
        const int lo = max(r0, seg0), hi = min(r1, seg0 + p.pf_rows[m]);
        if (lo < hi) {
            const int64_t n = min64((int64_t)(hi - lo) * p.pf_pitch[m], budget);
            prefetch_l2(p.pf_base[m] + (int64_t)(lo - seg0) * p.pf_pitch[m], n);
            budget -= n;
        }
        seg0 += p.pf_rows[m];
    }
}

// Warp roles: warps 0-7 compute per-block terms, warps 8-9 fold them row by row (and run
// the epilogue), warp 10 issues the TMA loads.  Hand-offs use mbarriers only:
//   full[s]   (TMA -> compute)            empty[s]  (compute -> producer: stage s reusable)
//   tfull[s]  (compute -> fold: terms of stage s written)
//   tempty[s] (fold -> compute: term slot s folded)
// The eight compute warps form p.cgroups groups (4 by default: two warps each); group g
// works on the stages t with t % cgroups == g, so four stages' dot products are in
// progress at once and the latency of one stage's shared-memory loads, dp4a chains and
// term stores overlaps the others' (one group per stage left the SM mostly waiting).

// quantize_f32_to_q8_0 (inference.rs:991-1029) of one 32-value block held one value per
// lane: scale = max|x| / 127, q = round(x * (1 / scale)) clamped to +-127 (zero block:
// scale 0, values 0).  Writes this lane's int8, returns the block scale.
__device__ __forceinline__ float q8_block_quantise(float v, int8_t* q_out) {
    float amax = fabsf(v);
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) amax = fmaxf(amax, __shfl_xor_sync(NCM_FULL, amax, k));
    const float scale = amax / 127.0f;
    int q = 0;
    if (scale > 0.0f) {
        const float inv = 1.0f / scale;
        q = (int)fminf(fmaxf(roundf(v * inv), -127.0f), 127.0f);
    }
    *q_out = (int8_t)q;
    return scale;
}

// Measurement probe: when p.dbg_ts is set, per-CTA global-timer stamps (ns) of the
// pipeline's phases: [0] entry, [1] after the PDL wait, [2] prologue done, [3] last TMA
// issued, [4] last fold done, [5] fold-thread time in tile epilogues, [6] exit,
// [7] compute warp 0: waiting for stage data, [8] waiting for a free term slot,
// [9] fold warp 0: waiting for terms, [10] producer: waiting for a free stage,
// [11] compute warp 0: end of its loop.
#define NCM_TS(i, v) do { if (p.dbg_ts) p.dbg_ts[(size_t)blockIdx.x * 16 + (i)] = (v); } while (0)

template <int QT, int IN, int EPI>
__global__ void __launch_bounds__(kGemvThreads, 1) ncm_qgemv_kernel(const __grid_constant__ GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr bool DUAL = (EPI == EPI_SILU);
    __shared__ GemvSeqScratch sc;
    __shared__ int s_last;
    __shared__ float xchg[kMaxFold];
    __shared__ float wv[2];
    __shared__ int wi[2];

    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + 8;
    uint64_t* tfull = full + 16;
    uint64_t* tempty = full + 24;
    float* tbuf = reinterpret_cast<float*>(smem + p.t_off);
    uint8_t* stages = smem + p.stage_off;
    const int tid = threadIdx.x, lane = tid & 31;
    const int R = p.total_rows;
    const int nbk = gridDim.x;
    const int ralign = p.row_align;
    const int r_begin = (int)(((long long)blockIdx.x * R / nbk)) & ~(ralign - 1);
    const int r_end = (blockIdx.x + 1 == nbk) ? R : ((int)(((long long)(blockIdx.x + 1) * R / nbk)) & ~(ralign - 1));
    const int box_bytes = p.box_rows * p.chunk_bytes;
    const int box2_off = (box_bytes + 127) & ~127;   // tensor-TMA destinations are 128-byte aligned
    const int ns = p.nstages;
    const uint64_t limit_ns = 4000000000ull;

    if (tid == 0) {
        for (int s = 0; s < ns; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kComputeThreads / 32 / p.cgroups);
            mbar_init(&tfull[s], kComputeThreads / 32 / p.cgroups);
            mbar_init(&tempty[s], 2);
        }
        fence_mbar_init();
    }
    __syncthreads();

    // (1) producer: first stages before the PDL wait (weights are constant).
    int icur = r_begin, ichunk = 0, tprod = 0;
    uint64_t pol = 0;
    uint64_t tpw = 0;
    auto issue = [&]() {
        const int s = tprod % ns;
        const uint64_t tp0 = p.dbg_ts ? global_timer_ns() : 0;
        if (tprod >= ns && !mbar_wait(&empty[s], (uint32_t)(((tprod / ns) & 1) ^ 1), limit_ns))
            set_dev_error(p.err, NCM_DEVERR_MBAR_TIMEOUT);
        if (p.dbg_ts) tpw += global_timer_ns() - tp0;
        TileCursor tc = tile_at(p, icur, r_end);
        const int y = icur - p.seg[tc.seg].row_begin;
        const int x = ichunk * p.chunk_words;
        mbar_arrive_expect_tx(&full[s], DUAL ? 2 * box_bytes : box_bytes);
        tma_load_2d(stages + (size_t)s * p.stage_bytes, &p.tm[tc.seg], x, y, &full[s], pol);
        if (DUAL) tma_load_2d(stages + (size_t)s * p.stage_bytes + box2_off, &p.tm2, x, y, &full[s], pol);
        if (++ichunk == p.nchunk) { ichunk = 0; icur += tc.n; }
        ++tprod;
    };
    if (tid == kProducer) {
        pol = l2_evict_first_policy();
        while (tprod < ns && icur < r_end) issue();
    }
    if constexpr (IN == IN_F32_RMS) {
        // norm weights are constant: stage them before waiting for the previous kernel
        stage_f32(reinterpret_cast<float*>(smem + p.nw_off), p.norm_w, p.cols, tid, blockDim.x);
    }
    if (tid == 0 && p.dbg_ts) NCM_TS(0, global_timer_ns());
    pdl_launch_dependents();
    pdl_wait();
    if (tid == 0 && p.dbg_ts) NCM_TS(1, global_timer_ns());

    // (2) activation -> shared memory (all threads).
    gemv_prologue<IN>(smem, p, sc);
    __syncthreads();
    if (tid == 0 && p.dbg_ts) NCM_TS(2, global_timer_ns());

    if (tid == kProducer) {
        while (icur < r_end) issue();
        if (p.dbg_ts) { NCM_TS(3, global_timer_ns()); NCM_TS(10, tpw); }
        // Every load of this CTA is issued: HBM would idle through this kernel's tail, the
        // kernel boundary and the next kernel's prologue, so stream the start of the next
        // kernel's weights into L2 now (its first tiles then come from L2).
        prefetch_next_weights(p);
    } else if (tid < kComputeThreads) {
        // (3a) compute warps in G groups of 8/G warps: group gi takes the stages t with
        // t % G == gi, so G stages are worked on at once.  Lane = (unit u = lane & 7, row
        // group v0 = lane >> 3); warp wi of the group takes the virtual rows
        // v0 + 4 wi + (32 / G) j, j < 2 G.
        uint64_t twait = 0, tslot = 0;
        auto compute = [&](auto gc) {
            constexpr int G = decltype(gc)::value;
            constexpr int WPG = kComputeThreads / 32 / G;   // warps per group
            const int w = tid >> 5, gi = w / WPG, wi = w % WPG, u = lane & 7, v0 = lane >> 3;
            int t = 0;
            for (int cur = r_begin; cur < r_end;) {
                const int n = tile_at(p, cur, r_end).n;
                const int vrows = DUAL ? 2 * p.box_rows : n;
                for (int c = 0; c < p.nchunk; ++c, ++t) {
                    if (t % G != gi) continue;
                    const int s = t % ns;
                    const uint32_t use = (uint32_t)(t / ns);
                    const uint64_t tw0 = (p.dbg_ts && tid == 0) ? global_timer_ns() : 0;
                    if (!mbar_wait(&full[s], use & 1, limit_ns)) set_dev_error(p.err, NCM_DEVERR_MBAR_TIMEOUT);
                    if (p.dbg_ts && tid == 0) twait += global_timer_ns() - tw0;
                    const uint64_t tw1 = (p.dbg_ts && tid == 0) ? global_timer_ns() : 0;
                    if (use > 0 && !mbar_wait(&tempty[s], (use - 1) & 1, limit_ns))
                        set_dev_error(p.err, NCM_DEVERR_MBAR_TIMEOUT);
                    if (p.dbg_ts && tid == 0) tslot += global_timer_ns() - tw1;
                    const uint8_t* sb = stages + (size_t)s * p.stage_bytes;
                    float* T = tbuf + s * (kMaxFold * kTStride);
                    XUnit x;
                    load_xunit(smem, p, c * kUnits + u, x);
                    constexpr int NJ = 2 * G;
                    const uint8_t* rp[NJ];
                    bool ok[NJ];
                    int vr[NJ];
#pragma unroll
                    for (int j = 0; j < NJ; ++j) {
                        vr[j] = v0 + 4 * wi + (32 / G) * j;
                        const int mat = DUAL ? (vr[j] >= p.box_rows) : 0;
                        const int r = vr[j] - mat * p.box_rows;
                        ok[j] = vr[j] < vrows && r < n;
                        rp[j] = sb + mat * box2_off + (ok[j] ? r : 0) * p.chunk_bytes;
                    }
                    float t0[NJ], t1[NJ];
                    // Rows grow with j, so the j that reach a row of a short tile are a
                    // prefix, and its length is the same for the whole warp (v0 = 0 is the
                    // warp's lowest row).  A tile with fewer rows than the 64 lanes (the
                    // fused q/k/v tiles, 36 rows on the 70B shape; wo / w2 at 55-56) then
                    // computes only the rows it holds, one row at a time; the terms and
                    // their fold are unchanged.  Measured on the 70B decode step: +1.8 %
                    // tokens/s over the full-width form; two-row pieces gave +0.1 %.
                    const int nact = DUAL ? NJ : min(NJ, max(0, (n - 4 * wi + (32 / G) - 1) / (32 / G)));
                    if (DUAL || nact == NJ || (p.tune & 16)) {
                        unit_terms_n<QT, NJ>(rp, u, x, t0, t1);
                    } else {
#pragma unroll
                        for (int j = 0; j < NJ; ++j) {
                            if (j < nact) {
                                const uint8_t* rq[1] = {rp[j]};
                                float q0[1], q1[1];
                                unit_terms_n<QT, 1>(rq, u, x, q0, q1);
                                t0[j] = q0[0];
                                t1[j] = q1[0];
                            }
                        }
                    }
#pragma unroll
                    for (int j = 0; j < NJ; ++j) {
                        if (ok[j]) {
                            float* trow = T + vr[j] * kTStride;
                            trow[2 * u] = t0[j];
                            trow[2 * u + 1] = t1[j];
                        }
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&empty[s]);
                        mbar_arrive(&tfull[s]);
                    }
                }
                cur += n;
            }
        };
        if (p.cgroups == 4) compute(std::integral_constant<int, 4>{});
        else if (p.cgroups == 2) compute(std::integral_constant<int, 2>{});
        else compute(std::integral_constant<int, 1>{});
        if (tid == 0 && p.dbg_ts) { NCM_TS(7, twait); NCM_TS(8, tslot); NCM_TS(11, global_timer_ns()); }
    } else if (tid < kProducer) {
        // (3b) fold warps: sequential per-row sums in block order, then the epilogue.
        const int f = tid - kFoldBase;
        int pos = 0;
        if (EPI == EPI_QKV || EPI == EPI_ARGMAX) pos = p.state[ST_POS];
        float best_v = -INFINITY;
        int best_i = 0x7fffffff;
        const int nsb = p.nb / 8;
        int t = 0;
        uint64_t tepi = 0, tfw = 0;
        for (int cur = r_begin; cur < r_end;) {
            const TileCursor tc = tile_at(p, cur, r_end);
            const int n = tc.n;
            const bool live = DUAL ? (f < 2 * p.box_rows && (f % p.box_rows) < n) : (f < n);
            float acc = 0.0f;
            const float* trow0 = tbuf + f * kTStride;
            for (int c = 0; c < p.nchunk; ++c, ++t) {
                const int s = t % ns;
                const uint32_t use = (uint32_t)(t / ns);
                const uint64_t tf0 = (p.dbg_ts && f == 0) ? global_timer_ns() : 0;
                if (!mbar_wait(&tfull[s], use & 1, limit_ns)) set_dev_error(p.err, NCM_DEVERR_MBAR_TIMEOUT);
                if (p.dbg_ts && f == 0) tfw += global_timer_ns() - tf0;
                if (live) {
                    // all 16 terms into registers first, then the in-order adds
                    const float* trow = trow0 + s * (kMaxFold * kTStride);
                    float tv[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) tv[j] = trow[j];
                    asm volatile("" ::: "memory");
                    if constexpr (QT == NCM_T_Q4_K) {
                        const int nsbc = min(2, nsb - 2 * c);
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            if (q < nsbc) {
                                float ssum = 0.0f;   // q8.rs:1342 sum starts at 0 per super-block
#pragma unroll
                                for (int j = 0; j < 8; ++j) ssum += tv[8 * q + j];
                                acc += ssum;         // inference.rs:3129 row sum += block result
                            }
                        }
                    } else {
                        const int nbc = min(16, p.nb - 16 * c);
                        if (nbc == 16) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) acc += tv[j];
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                if (j < nbc) acc += tv[j];
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[s]);
            }

            const uint64_t te0 = (p.dbg_ts && f == 0) ? global_timer_ns() : 0;
            // tile epilogue (rows cur .. cur+n-1 of segment tc.seg)
            const Seg& sg = p.seg[tc.seg];
            const int lrow0 = cur - sg.row_begin;
            if constexpr (EPI == EPI_QKV) {
                const float other = __shfl_xor_sync(NCM_FULL, acc, 1);
                if (f < n) {
                    // the row's own segment (tiles of a fused q/k/v buffer span segments)
                    const Seg& sg = p.seg[p.fused ? seg_of(p, cur + f) : tc.seg];
                    const int lr = cur + f - sg.row_begin;
                    float v = acc;
                    if (sg.kind != SEG_V) {
                        // inference.rs:904-933 apply_rope_cached, NORM pairs (2i, 2i+1).
                        const int i = (lr % p.head_dim) >> 1;
                        if (i < p.rope_half) {
                            const float2 scs = p.rope[(size_t)pos * p.rope_half + i];
                            const float x0 = (f & 1) ? other : acc;
                            const float x1 = (f & 1) ? acc : other;
                            v = (f & 1) ? (x0 * scs.x + x1 * scs.y) : (x0 * scs.y - x1 * scs.x);
                        }
                    }
                    if (sg.kind == SEG_Q) sg.out[lr] = v;
                    else ((sg.kind == SEG_K ? p.kcache : p.vcache) + (p.kv_stage ? (size_t)0 : (size_t)pos * p.kv_width))[lr] = v;
                }
            } else if constexpr (EPI == EPI_SILU) {
                if (f >= p.box_rows && f < p.box_rows + n) xchg[f - p.box_rows] = acc;
                asm volatile("bar.sync 1, 64;" ::: "memory");
                float o = 0.0f;
                if (f < n) {
                    const float g = acc, uu = xchg[f];
                    // inference.rs:3385-3388: sigmoid = 1/(1+exp(-g)); g * sigmoid * u
                    const float sig = 1.0f / (1.0f + expf_cr(-g));
                    o = g * sig * uu;
                    sg.out[lrow0 + f] = o;
                }
                if (p.qout && f < 32) {
                    // The tile is one 32-row block (box_rows == 32, 32-aligned row ranges):
                    // fold warp 8 holds it and quantises it for the down projection.
                    const float scale = q8_block_quantise(o, p.qout + lrow0 + f);
                    if (f == 0) p.qout_s[lrow0 >> 5] = scale;
                }
                asm volatile("bar.sync 1, 64;" ::: "memory");
            } else {
                if (f < n) {
                    const int lr = lrow0 + f;
                    if constexpr (EPI == EPI_PLAIN) {
                        sg.out[lr] = acc;
                    } else if constexpr (EPI == EPI_RESID) {
                        sg.out[lr] += acc;   // inference.rs:4670-4672 / 4744-4746
                    } else if constexpr (EPI == EPI_ARGMAX) {
                        if (sg.out) sg.out[lr] = acc;
                        if (better(acc, lr, best_v, best_i)) { best_v = acc; best_i = lr; }
                    } else if constexpr (EPI == EPI_TP_RESID) {
                        // Partial row into slot [rank] of every GPU's receive area (NVLink
                        // stores for peers): the summands of tp.rs:357-359 / 418-420.
                        const size_t idx = ((size_t)p.tp_slot * p.tp.world + p.tp.rank) * p.tp.H + lr;
                        for (int d = 0; d < p.tp.world; ++d) p.tp.recv[d][idx] = acc;
                    }
                }
            }
            if (p.dbg_ts && f == 0) tepi += global_timer_ns() - te0;
            cur += n;
        }
        if (p.dbg_ts && f == 0) { NCM_TS(4, global_timer_ns()); NCM_TS(5, tepi); NCM_TS(9, tfw); }
        if constexpr (EPI == EPI_ARGMAX) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                float ov = __shfl_xor_sync(NCM_FULL, best_v, o);
                int oi = __shfl_xor_sync(NCM_FULL, best_i, o);
                if (better(ov, oi, best_v, best_i)) { best_v = ov; best_i = oi; }
            }
            if (lane == 0) { wv[f >> 5] = best_v; wi[f >> 5] = best_i; }
        }
    }
    __syncthreads();

    if constexpr (EPI == EPI_ARGMAX) {
        // CTA first-max over its rows, then the last CTA merges every CTA (rows ascend
        // with the CTA index, so "larger value, ties to the lower row" reproduces the
        // strict '>' scan of inference.rs:4838-4843).
        if (tid == 0) {
            float bv = wv[0];
            int bi = wi[0];
            if (better(wv[1], wi[1], bv, bi)) { bv = wv[1]; bi = wi[1]; }
            p.amax_part[blockIdx.x] = make_float2(bv, __int_as_float(bi));
            __threadfence();
            unsigned prev = atomicAdd(p.counter, 1u);
            s_last = (prev == (unsigned)nbk - 1);
        }
        __syncthreads();
        if (s_last && tid == 0) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int c = 0; c < nbk; ++c) {
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
                fence_acq_rel_sys();
                for (int d = 0; d < W; ++d) st_relaxed_sys(&p.tp.hflags[d][me], epoch);
                bool ok = true;
                for (int src = 0; src < W && ok; ++src) ok = wait_flag_sys(&p.tp.hflags[me][src], epoch, p.tp.timeout_ns);
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
        // cluster_tp_node.rs:1154-1180): publish, wait for every rank's slice of the same
        // rows, then sum in rank order on every GPU so all ranks hold identical bits:
        // hidden = ((0 + p0) + p1) + ... then += residual (tp.rs:349-363).
        const int W = p.tp.world, me = p.tp.rank;
        const unsigned epoch = (unsigned)p.state[ST_STEP] + 1u;
        const size_t fslot = ((size_t)p.tp_slot * p.tp.grid_max + blockIdx.x) * W;
        if (tid == 0) {
            // the CTA's peer stores are ordered before this fence by the barrier above
            fence_acq_rel_sys();
            for (int d = 0; d < W; ++d) st_relaxed_sys(&p.tp.flags[d][fslot + me], epoch);
        }
        if (tid < W && !wait_flag_sys(&p.tp.flags[me][fslot + tid], epoch, p.tp.timeout_ns))
            set_dev_error(p.err, NCM_DEVERR_PEER_TIMEOUT);
        __syncthreads();
        const float* base = p.tp.recv[me] + (size_t)p.tp_slot * W * p.tp.H;
        for (int r = r_begin + tid; r < r_end; r += blockDim.x) {
            float s = 0.0f;
            for (int src = 0; src < W; ++src) s += __ldcg(base + (size_t)src * p.tp.H + r);
            p.hidden[r] += s;
        }
    }
    if (tid == 0 && p.dbg_ts) NCM_TS(6, global_timer_ns());
}

// ------------------------------------------------------------------ GEMV planning / launch
int gemv_tensor_map(CUtensorMap* tm, const void* base, int64_t rows, int pitch, int chunk_words, int box_rows) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return (int)cudaErrorNotSupported;
    cuuint64_t gdim[2] = {(cuuint64_t)(pitch / 4), (cuuint64_t)rows};
    cuuint64_t gstride[1] = {(cuuint64_t)pitch};
    cuuint32_t box[2] = {(cuuint32_t)chunk_words, (cuuint32_t)box_rows};
    cuuint32_t estride[2] = {1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), gdim, gstride, box, estride,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

constexpr int kGemvSmemLimit = 220 * 1024;

int gemv_plan(int qtype, int cols, int rows, bool dual, int in_mode, GemvParams& p) {
    p.cols = cols;
    p.nb = cols / 32;
    p.nchunk = (cols + kChunkCols - 1) / kChunkCols;
    p.chunk_bytes = qtype == NCM_T_Q8_0 ? 16 * 34 : 288;
    p.chunk_words = p.chunk_bytes / 4;
    p.total_rows = rows;
    int grid = num_sms();
    if (p.cgroups != 1 && p.cgroups != 2 && p.cgroups != 4) p.cgroups = 4;
    if (p.row_align < 2) p.row_align = 2;
    const int ra = p.row_align;
    int maxg = (rows + ra - 1) / ra;
    if (maxg < 1) maxg = 1;
    if (grid > maxg) grid = maxg;
    const int per_cta = (rows + grid - 1) / grid;
    // rows per tile: a stage (one tile x 512 columns) stays near 18 KB so that eight
    // stages fit beside the activation.  The CTA's rows are split into equal tiles (a
    // TMA box always brings box_rows rows, so a short last tile would fetch rows that
    // are not used).
    int maxr = qtype == NCM_T_Q8_0 ? 32 : 64;
    if (dual) maxr /= 2;
    const int span = per_cta + ra;   // the most rows a CTA's aligned range can hold
    const int ntiles = (span + maxr - 1) / maxr;
    int br = (span + ntiles - 1) / ntiles;
    br = (br + ra - 1) / ra * ra;
    if (br > maxr) br = maxr;
    if (br < 2) br = 2;
    p.box_rows = br;
    p.stage_bytes = (br * p.chunk_bytes + 127) / 128 * 128 * (dual ? 2 : 1);
    const int units = p.nchunk * kUnits;
    int off = 256;   // full / empty / tfull / tempty mbarriers
    p.xq_off = off;
    off += units * 80;
    p.xs_off = off;
    off += units * 8;
    p.xsum_off = off;
    off += units * 8;
    off = (off + 127) / 128 * 128;
    // The f32 staging of the input and the term buffers (one slot per stage) are live
    // at different times.  The stage count is the largest that fits the budget.
    p.xf_off = off;
    p.t_off = off;
    const int base = off;
    int ns = kMaxStages;
    for (; ns >= 2; --ns) {
        int o = base;
        int shared_region = ns * kMaxFold * kTStride * 4;
        if (in_mode != IN_Q8 && cols * 4 > shared_region) shared_region = cols * 4;
        o += (shared_region + 127) / 128 * 128;
        p.nw_off = o;
        if (in_mode == IN_F32_RMS) o += (cols * 4 + 127) / 128 * 128;
        p.stage_off = o;
        if (o + ns * p.stage_bytes <= kGemvSmemLimit) break;
    }
    if (ns < 2) return -1;
    p.nstages = ns;
    p.smem_bytes = p.stage_off + ns * p.stage_bytes;
    return grid;
}

template <int QT, int IN, int EPI>
static int launch_t(const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    auto kern = ncm_qgemv_kernel<QT, IN, EPI>;
    if (int r = set_smem_limit((const void*)kern, kGemvSmemLimit)) return r;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = p.smem_bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, kern, p);
}

template <int QT>
static int launch_mode(int in_mode, int epi, const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    if (in_mode == IN_F32_RMS && epi == EPI_QKV) return launch_t<QT, IN_F32_RMS, EPI_QKV>(p, grid, s, pdl);
    if (in_mode == IN_F32_RMS && epi == EPI_SILU) return launch_t<QT, IN_F32_RMS, EPI_SILU>(p, grid, s, pdl);
    if (in_mode == IN_F32_RMS && epi == EPI_ARGMAX) return launch_t<QT, IN_F32_RMS, EPI_ARGMAX>(p, grid, s, pdl);
    if (in_mode == IN_F32 && epi == EPI_RESID) return launch_t<QT, IN_F32, EPI_RESID>(p, grid, s, pdl);
    if (in_mode == IN_F32 && epi == EPI_TP_RESID) return launch_t<QT, IN_F32, EPI_TP_RESID>(p, grid, s, pdl);
    if (in_mode == IN_F32 && epi == EPI_PLAIN) return launch_t<QT, IN_F32, EPI_PLAIN>(p, grid, s, pdl);
    if (in_mode == IN_Q8 && epi == EPI_PLAIN) return launch_t<QT, IN_Q8, EPI_PLAIN>(p, grid, s, pdl);
    if (in_mode == IN_Q8 && epi == EPI_RESID) return launch_t<QT, IN_Q8, EPI_RESID>(p, grid, s, pdl);
    if (in_mode == IN_Q8 && epi == EPI_TP_RESID) return launch_t<QT, IN_Q8, EPI_TP_RESID>(p, grid, s, pdl);
    return (int)cudaErrorInvalidValue;
}

int gemv_launch(int qtype, int in_mode, int epi, const GemvParams& p, int grid, cudaStream_t s, bool pdl) {
    if (qtype == NCM_T_Q4_0) return launch_mode<NCM_T_Q4_0>(in_mode, epi, p, grid, s, pdl);
    if (qtype == NCM_T_Q8_0) return launch_mode<NCM_T_Q8_0>(in_mode, epi, p, grid, s, pdl);
    if (qtype == NCM_T_Q4_K) return launch_mode<NCM_T_Q4_K>(in_mode, epi, p, grid, s, pdl);
    return (int)cudaErrorInvalidValue;
}

// ------------------------------------------------------------------ attention
// inference.rs:4242-4292 apply_attention_head, f32 cache, term by term.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// 16-byte vector access is used when every base pointer is 16-byte aligned (rows of
// q / K / V start at multiples of head_dim, a multiple of 32 floats).
__device__ __forceinline__ bool attn_vec_ok(const AttnParams& a) {
    return (((uintptr_t)a.q | (uintptr_t)a.kc | (uintptr_t)a.vc) & 15) == 0 && (a.kvw & 3) == 0;
}

// Scores over a Q8_0 cache (inference.rs:4319-4357 apply_attention_head_q8_0): q_head is
// quantised like the store (per 32 values, f16-truncated scale), then per position
// score = (sum over blocks, in order, of (s_q * s_k) * dot_i32) * scale (q8.rs:509-511).
// The CTA's 32 positions x hd/32 blocks of K are copied into shared memory as words
// (the 34-byte blocks are only 2-byte aligned) with their scales decoded.
__device__ void attn_scores_q8(const AttnParams& a, const float* qsrc, float* scores, int kvh, int g, int p0, int np,
                               float* qbuf, float* kbuf) {
    // in the kernel's K tile buffer: [pos][block][8 words] (hd <= 256, padded) + scales;
    // in its q buffer: [head][block][8 words] + scales
    uint32_t* kw_s = reinterpret_cast<uint32_t*>(kbuf);
    float* ksc = kbuf + 32 * 8 * 8 + 32;
    uint32_t (*qw_s)[64] = reinterpret_cast<uint32_t (*)[64]>(qbuf);
    float (*qsc)[8] = reinterpret_cast<float (*)[8]>(qbuf + 8 * 64);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, hd = a.hd, bph = hd / 32, bpw = a.kvw / 32;
    const uint8_t* kb = reinterpret_cast<const uint8_t*>(a.kc_raw);
    for (int i = tid; i < np * bph; i += 256) {
        const int pp = i / bph, b = i % bph;
        const uint16_t* src = reinterpret_cast<const uint16_t*>(kb + ((size_t)(p0 + pp) * bpw + (size_t)kvh * bph + b) * 34);
        ksc[pp * 8 + b] = f16_bits_to_f32(src[0]);
        uint32_t* dst = kw_s + (pp * 8 + b) * 8 + pp;   // + pp: rotate banks across positions
#pragma unroll
        for (int k = 0; k < 8; ++k) dst[k] = (uint32_t)src[1 + 2 * k] | ((uint32_t)src[2 + 2 * k] << 16);
    }
    // quantize_row_to_q8_0_blocks (inference.rs:4298-4317) of each query head of the group
    for (int i = warp; i < g * bph; i += 8) {
        const int h = i / bph, b = i % bph;
        const float x = qsrc[h * hd + 32 * b + lane];
        float mx = fabsf(x);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(NCM_FULL, mx, o));
        const float sc = mx / 127.0f, inv = sc > 0.0f ? 1.0f / sc : 0.0f;
        const int q = (int)fminf(fmaxf(roundf(x * inv), -127.0f), 127.0f);
        // pack four lanes' bytes into a word
        const uint32_t byte = (uint32_t)(q & 0xff) << (8 * (lane & 3));
        uint32_t w = byte;
        w |= __shfl_xor_sync(NCM_FULL, w, 1);
        w |= __shfl_xor_sync(NCM_FULL, w, 2);
        if ((lane & 3) == 0) qw_s[h][b * 8 + (lane >> 2)] = w;
        if (lane == 0) qsc[h][b] = f16_bits_to_f32(ncm_f32_to_f16_trunc(sc));
    }
    __syncthreads();
    for (int h = warp; h < g; h += 8) {
        if (lane < np) {
            float acc = 0.0f;
            for (int b = 0; b < bph; ++b) {
                const uint32_t* kr = kw_s + (lane * 8 + b) * 8 + lane;
                int dot = 0;
#pragma unroll
                for (int k = 0; k < 8; ++k) dot = __dp4a((int)qw_s[h][b * 8 + k], (int)kr[k], dot);
                acc += qsc[h][b] * ksc[lane * 8 + b] * (float)dot;
            }
            scores[(size_t)(kvh * g + h) * a.ctx + p0 + lane] = acc * a.scale;
        }
    }
}

// Stage 1 (attn_scores_kernel): scores[h][p] = dot_f32(q_h, k_p) * scale with the dot a
// sequential sum over head_dim (inference.rs:3570-3573, 4256); grid (kv head, 32
// positions), warp = query head of the group, lane = position.  The K tile is loaded
// with all its loads in flight at once, then transposed into a padded shared array.
// One (kv head, 32-position tile, row) item by 256 threads (BAR: 0 = the whole CTA, else
// the named barrier of the 256 threads); qs / ks are the shared tiles (8 x 256 and
// 32 x 257 floats).  Activations written by other CTAs of the same launch are read
// through L2 (ld.global.cg).
template <int BAR>
__device__ void attn_scores_body(const AttnParams& a, int kvh, int ty, int tz, float* qs, float* ks) {
    const int pos = (a.pos_override >= 0 ? a.pos_override : __ldcg(&a.state[ST_POS])) + tz;
    const int n = pos + 1;
    const int p0 = ty * 32;
    if (p0 >= n) return;
    const int g = a.heads / a.kv_heads, hd = a.hd;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int np = min(32, n - p0);
    const float* qsrc = a.q + (size_t)tz * a.tok_stride + (size_t)kvh * g * hd;
    float* scores = a.scores + (size_t)tz * a.heads * a.ctx;
    const float* ksrc = a.kc + (size_t)p0 * a.kvw + (size_t)kvh * hd;
    if constexpr (BAR == 0) {
        if (a.kv_kind == KV_Q8_0) {
            attn_scores_q8(a, qsrc, scores, kvh, g, p0, np, qs, ks);
            return;
        }
    }
    if (a.kv_kind == KV_F16) {
        // decode_f16_head (inference.rs:4453-4458): exact f16 -> f32, then the f32 path
        const uint16_t* k16 = reinterpret_cast<const uint16_t*>(a.kc_raw) + (size_t)p0 * a.kvw + (size_t)kvh * hd;
        for (int i = tid; i < g * hd; i += 256) qs[i] = __ldcg(&qsrc[i]);
        for (int i = tid; i < np * hd; i += 256)
            ks[(i / hd) * (hd + 1) + i % hd] = f16_bits_to_f32(__ldcg(&k16[(size_t)(i / hd) * a.kvw + i % hd]));
    } else if (attn_vec_ok(a)) {
        const int per = hd >> 2;                 // float4 per row
        float4 qv[2], kv[8];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = tid + 256 * k;
            if (i < g * per) qv[k] = __ldcg(reinterpret_cast<const float4*>(qsrc) + i);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = tid + 256 * k;
            if (i < np * per) kv[k] = __ldcg(reinterpret_cast<const float4*>(ksrc + (size_t)(i / per) * a.kvw + 4 * (i % per)));
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = tid + 256 * k;
            if (i < g * per) reinterpret_cast<float4*>(qs)[i] = qv[k];
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int i = tid + 256 * k;
            if (i < np * per) {
                float* d = ks + (i / per) * (hd + 1) + 4 * (i % per);
                d[0] = kv[k].x; d[1] = kv[k].y; d[2] = kv[k].z; d[3] = kv[k].w;
            }
        }
    } else {
        for (int i = tid; i < g * hd; i += 256) qs[i] = __ldcg(&qsrc[i]);
        for (int i = tid; i < np * hd; i += 256)
            ks[(i / hd) * (hd + 1) + i % hd] = __ldcg(&ksrc[(size_t)(i / hd) * a.kvw + i % hd]);
    }
    group_sync<256, BAR>();
    for (int h = warp; h < g; h += 8) {
        if (lane < np) {
            const float* q = qs + h * hd;
            const float* k = ks + lane * (hd + 1);
            float s = 0.0f;
#pragma unroll 8
            for (int d = 0; d < hd; ++d) s += q[d] * k[d];
            scores[(size_t)(kvh * g + h) * a.ctx + p0 + lane] = s * a.scale;
        }
    }
}

__global__ void __launch_bounds__(256) attn_scores_kernel(const __grid_constant__ AttnParams a) {
    __shared__ __align__(16) float qs[8 * 256];
    __shared__ float ks[32 * 257];
    pdl_launch_dependents();
    pdl_wait();
    attn_scores_body<0>(a, blockIdx.x, blockIdx.y, blockIdx.z, qs, ks);
}

// Stage 2 (attn_softmax_kernel): one CTA of 256 threads per (query head, row).  softmax
// (inference.rs:3522-3540): max (order free), e_p = exp(s_p - max), the sequential sum of
// the e_p (seq_sum_nonneg, exact), inv = 1 / sum, w_p = e_p * inv; the weights overwrite
// the scores in place.  e is a shared buffer of at least pos + 1 floats, red 8 floats.
template <int BAR>
__device__ void attn_softmax_body(const AttnParams& a, int h, int tz, float* e, SeqSumScratch& sc, float* red) {
    const int pos = (a.pos_override >= 0 ? a.pos_override : __ldcg(&a.state[ST_POS])) + tz;
    const int n = pos + 1;
    const int tid = threadIdx.x & 255, warp = tid >> 5, lane = tid & 31;
    float* srow = a.scores + ((size_t)tz * a.heads + h) * a.ctx;
    constexpr int kReg = 8;   // rows up to 2048 positions stay in registers
    float r[kReg];
    float mx = -INFINITY;
    if (n <= kReg * 256) {
#pragma unroll
        for (int k = 0; k < kReg; ++k) r[k] = tid + 256 * k < n ? __ldcg(&srow[tid + 256 * k]) : -INFINITY;
#pragma unroll
        for (int k = 0; k < kReg; ++k) mx = fmaxf(mx, r[k]);   // max is order independent (no NaNs)
    } else {
        for (int p = tid; p < n; p += 256) {
            const float v = __ldcg(&srow[p]);
            e[p] = v;
            mx = fmaxf(mx, v);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(NCM_FULL, mx, o));
    if (lane == 0) red[warp] = mx;
    group_sync<256, BAR>();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
    if (n <= kReg * 256) {
#pragma unroll
        for (int k = 0; k < kReg; ++k)
            if (tid + 256 * k < n) {
                r[k] = expf_cr(r[k] - mx);
                e[tid + 256 * k] = r[k];
            }
    } else {
        for (int p = tid; p < n; p += 256) e[p] = expf_cr(e[p] - mx);
    }
    group_sync<256, BAR>();
    const float sum = seq_sum_nonneg<256, BAR>([&](int i) { return e[i]; }, n, sc, tid);
    const float inv = 1.0f / sum;
    if (n <= kReg * 256) {
#pragma unroll
        for (int k = 0; k < kReg; ++k)
            if (tid + 256 * k < n) srow[tid + 256 * k] = r[k] * inv;
    } else {
        for (int p = tid; p < n; p += 256) srow[p] = e[p] * inv;
    }
}

__global__ void __launch_bounds__(256) attn_softmax_kernel(const __grid_constant__ AttnParams a) {
    extern __shared__ __align__(16) float e[];
    __shared__ SeqSumScratch sc;
    __shared__ float red[8];
    pdl_launch_dependents();
    pdl_wait();
    attn_softmax_body<0>(a, blockIdx.x, blockIdx.z, e, sc, red);
}

// Stage 3 (attn_av_kernel): out[d] = sum_p w_p * v_p[d], sequential over p per (head, dim)
// (attn_output zeroed, add_weighted_f32_scalar inference.rs:3619-3623).  One item = (kv
// head, 32-dimension block, group of W * HPW query heads of that kv head, row): lane =
// dimension, warp w carries the chains of HPW heads (independent adds that interleave:
// one chain alone stalls on each add's latency), and a warp's output per head is one
// Q8_0 block for the output projection.  The item's V columns (128 bytes a position,
// shared by all its heads) and weights stream through a ring of kAvStages chunks of
// kAvChunk positions by cp.async, so the loads of later chunks are in flight while a
// chunk's chains run.  buf holds kAvStages * av_stage_floats(W * HPW) floats.
constexpr int kAvChunk = 64;
constexpr int kAvStages = 4;
__host__ __device__ constexpr int av_stage_floats(int heads) { return kAvChunk * 32 + heads * kAvChunk; }

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int W, int HPW>
__device__ void attn_av_body(const AttnParams& a, int kvh, int db, int hgrp, int tz, float* buf, int rank) {
    constexpr int NT = W * 32, HC = W * HPW;   // threads, heads of the item
    const int pos = (a.pos_override >= 0 ? a.pos_override : __ldcg(&a.state[ST_POS])) + tz;
    const int n = pos + 1;
    const int g = a.heads / a.kv_heads;
    const int warp = rank >> 5, lane = rank & 31;
    const int h0 = kvh * g + hgrp * HC;
    const int d0 = db * 32;
    const float* wbase = a.scores + ((size_t)tz * a.heads + h0) * a.ctx;
    const bool vec = a.kv_kind == KV_F32 && attn_vec_ok(a);
    const float* vsrc = a.vc + (size_t)kvh * a.hd + d0;
    const int nchunk = (n + kAvChunk - 1) / kAvChunk;
    constexpr int SF = av_stage_floats(HC);
    auto stage = [&](int k) {
        float* vs = buf + (k % kAvStages) * SF;
        float* ws = vs + kAvChunk * 32;
        const int c0 = k * kAvChunk, np = min(kAvChunk, n - c0);
        if (vec) {
            for (int i = rank; i < np * 8; i += NT) cp_async16(vs + 4 * i, vsrc + (size_t)(c0 + (i >> 3)) * a.kvw + 4 * (i & 7));
        } else if (a.kv_kind == KV_F16) {
            // decode_f16_head (inference.rs:4453-4458)
            const uint16_t* v16 = reinterpret_cast<const uint16_t*>(a.vc_raw) + (size_t)kvh * a.hd + d0;
            for (int i = rank; i < np * 32; i += NT)
                vs[i] = f16_bits_to_f32(__ldcg(&v16[(size_t)(c0 + (i >> 5)) * a.kvw + (i & 31)]));
        } else if (a.kv_kind == KV_Q8_0) {
            // inference.rs:4369-4379: value = q as f32 * block scale (one 34-byte block)
            const uint8_t* vb = reinterpret_cast<const uint8_t*>(a.vc_raw);
            const int bpw = a.kvw / 32;
            for (int i = rank; i < np * 32; i += NT) {
                const uint8_t* blk = vb + ((size_t)(c0 + (i >> 5)) * bpw + (size_t)(kvh * a.hd + d0) / 32) * 34;
                vs[i] = (float)(int8_t)blk[2 + (i & 31)] * f16_bits_to_f32((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
            }
        } else {
            for (int i = rank; i < np * 32; i += NT) vs[i] = __ldcg(&vsrc[(size_t)(c0 + (i >> 5)) * a.kvw + (i & 31)]);
        }
        for (int p = rank; p < np; p += NT) {
#pragma unroll
            for (int hh = 0; hh < HC; ++hh) cp_async4(ws + hh * kAvChunk + p, wbase + (size_t)hh * a.ctx + c0 + p);
        }
    };
#pragma unroll
    for (int k = 0; k < kAvStages - 1; ++k) {
        if (k < nchunk) stage(k);
        cp_async_commit();
    }
    float acc[HPW];
#pragma unroll
    for (int j = 0; j < HPW; ++j) acc[j] = 0.0f;
    for (int k = 0; k < nchunk; ++k) {
        if (k + kAvStages - 1 < nchunk) stage(k + kAvStages - 1);
        cp_async_commit();
        cp_async_wait_group<kAvStages - 1>();   // chunk k has landed (this thread's copies)
        group_sync<NT, 0>();                     // ... and every thread's
        const float* vs = buf + (k % kAvStages) * SF;
        const float* ws = vs + kAvChunk * 32 + warp * HPW * kAvChunk;
        const int np = min(kAvChunk, n - k * kAvChunk);
        int p = 0;
        // 8 positions a step, every shared-memory load issued before the first add (each
        // chain's adds stay in position order)
        for (; p + 8 <= np; p += 8) {
            float vv[8], wv[HPW][8];
#pragma unroll
            for (int q = 0; q < 8; ++q) vv[q] = vs[(p + q) * 32 + lane];
#pragma unroll
            for (int j = 0; j < HPW; ++j) {
                const float4 x0 = *reinterpret_cast<const float4*>(ws + j * kAvChunk + p);
                const float4 x1 = *reinterpret_cast<const float4*>(ws + j * kAvChunk + p + 4);
                wv[j][0] = x0.x; wv[j][1] = x0.y; wv[j][2] = x0.z; wv[j][3] = x0.w;
                wv[j][4] = x1.x; wv[j][5] = x1.y; wv[j][6] = x1.z; wv[j][7] = x1.w;
            }
#pragma unroll
            for (int q = 0; q < 8; ++q)
#pragma unroll
                for (int j = 0; j < HPW; ++j) acc[j] += wv[j][q] * vv[q];
        }
        for (; p < np; ++p) {
            const float v = vs[p * 32 + lane];
#pragma unroll
            for (int j = 0; j < HPW; ++j) acc[j] += ws[j * kAvChunk + p] * v;
        }
        group_sync<NT, 0>();                     // the slot may be refilled
    }
#pragma unroll
    for (int j = 0; j < HPW; ++j) {
        const int h = h0 + warp * HPW + j;
        a.out[(size_t)tz * a.tok_stride + (size_t)h * a.hd + d0 + lane] = acc[j];
        if (a.out_q) {
            // quantize_f32_to_q8_0 of this 32-value block for the output projection
            // (inference.rs:991-1029)
            float amax = fabsf(acc[j]);
#pragma unroll
            for (int k = 16; k > 0; k >>= 1) amax = fmaxf(amax, __shfl_xor_sync(NCM_FULL, amax, k));
            const float scale = amax / 127.0f;
            int q = 0;
            if (scale > 0.0f) {
                const float inv = 1.0f / scale;
                q = (int)fminf(fmaxf(roundf(acc[j] * inv), -127.0f), 127.0f);
            }
            const size_t o = (size_t)h * a.hd + d0;
            a.out_q[o + lane] = (int8_t)q;
            if (lane == 0) a.out_s[o >> 5] = scale;
        }
    }
}

// The same V items with the f32 cache's chunks brought by the TMA engine: one 2-D tiled
// load (32 floats x kAvChunk positions of this kv head's dimension block) per chunk into
// a ring of kAvStages slots tracked by mbarriers, issued by thread 0; the weights still
// come by cp.async.  One chain per thread (W warps = W query heads).
// One chunk of a V chain: acc += w_p * v_p[lane] for p = 0 .. np-1 in order (ws: the
// chunk's weights, vs: its [position][32] values, both in shared memory, ws 16-byte
// aligned).  A full chunk runs as four groups of 16 positions with the next group's
// loads issued before the current group's adds, so only the adds' own latency is serial.
__device__ __forceinline__ float av_chunk_chain(const float* ws, const float* vs, int np, int lane, float acc) {
    if (np == kAvChunk) {
        float wv[2][16], vv[2][16];
        auto load = [&](int gq, int b) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 w4 = *reinterpret_cast<const float4*>(ws + 16 * gq + 4 * q);
                wv[b][4 * q] = w4.x; wv[b][4 * q + 1] = w4.y; wv[b][4 * q + 2] = w4.z; wv[b][4 * q + 3] = w4.w;
            }
#pragma unroll
            for (int q = 0; q < 16; ++q) vv[b][q] = vs[(16 * gq + q) * 32 + lane];
        };
        load(0, 0);
        asm volatile("" ::: "memory");
#pragma unroll
        for (int gq = 0; gq < kAvChunk / 16; ++gq) {
            if (gq + 1 < kAvChunk / 16) load(gq + 1, (gq + 1) & 1);
            asm volatile("" ::: "memory");   // the next group's loads stay ahead of these adds
#pragma unroll
            for (int q = 0; q < 16; ++q) acc += wv[gq & 1][q] * vv[gq & 1][q];
        }
        return acc;
    }
    int p = 0;
    for (; p + 16 <= np; p += 16) {
        float wv[16], vv[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 w4 = *reinterpret_cast<const float4*>(ws + p + 4 * q);
            wv[4 * q] = w4.x; wv[4 * q + 1] = w4.y; wv[4 * q + 2] = w4.z; wv[4 * q + 3] = w4.w;
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) vv[q] = vs[(p + q) * 32 + lane];
#pragma unroll
        for (int q = 0; q < 16; ++q) acc += wv[q] * vv[q];
    }
    for (; p < np; ++p) acc += ws[p] * vs[p * 32 + lane];
    return acc;
}

template <int W>
__global__ void __launch_bounds__(W * 32) attn_av_tma_kernel(const __grid_constant__ AttnParams a) {
    extern __shared__ __align__(128) float buf[];   // [slot][kAvChunk][32] V, then [slot][W][kAvChunk] w
    __shared__ __align__(8) uint64_t full[kAvStages];
    constexpr int NT = W * 32;
    const int rank = threadIdx.x, warp = rank >> 5, lane = rank & 31;
    if (rank == 0) {
        for (int k = 0; k < kAvStages; ++k) mbar_init(&full[k], 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();
    const int nd = a.hd / 32;
    const int kvh = blockIdx.x, db = blockIdx.y % nd, hgrp = blockIdx.y / nd, tz = blockIdx.z;
    const int pos = (a.pos_override >= 0 ? a.pos_override : __ldcg(&a.state[ST_POS])) + tz;
    const int n = pos + 1;
    const int g = a.heads / a.kv_heads;
    const int h0 = kvh * g + hgrp * W;
    const int d0 = db * 32;
    const float* wbase = a.scores + ((size_t)tz * a.heads + h0) * a.ctx;
    const int nchunk = (n + kAvChunk - 1) / kAvChunk;
    float* vbuf = buf;
    float* wbuf = buf + kAvStages * kAvChunk * 32;
    const uint64_t limit_ns = 1000000000ull;
    const uint64_t pol = l2_evict_first_policy();
    auto issue_v = [&](int k) {   // thread 0
        uint64_t* bar = &full[k % kAvStages];
        mbar_arrive_expect_tx(bar, kAvChunk * 32 * 4);
        tma_load_2d(vbuf + (k % kAvStages) * kAvChunk * 32, &a.vmap, kvh * a.hd + d0, k * kAvChunk, bar, pol);
    };
    auto stage_w = [&](int k) {
        float* ws = wbuf + (k % kAvStages) * W * kAvChunk;
        const int c0 = k * kAvChunk, np = min(kAvChunk, n - c0);
        for (int p = rank; p < np; p += NT) {
#pragma unroll
            for (int hh = 0; hh < W; ++hh) cp_async4(ws + hh * kAvChunk + p, wbase + (size_t)hh * a.ctx + c0 + p);
        }
    };
#pragma unroll
    for (int k = 0; k < kAvStages - 1; ++k) {
        if (k < nchunk) {
            if (rank == 0) issue_v(k);
            stage_w(k);
        }
        cp_async_commit();
    }
    float acc = 0.0f;
    bool ok = true;
    for (int k = 0; k < nchunk; ++k) {
        if (k + kAvStages - 1 < nchunk) {
            if (rank == 0) issue_v(k + kAvStages - 1);
            stage_w(k + kAvStages - 1);
        }
        cp_async_commit();
        cp_async_wait_group<kAvStages - 1>();
        if (!mbar_wait(&full[k % kAvStages], (uint32_t)((k / kAvStages) & 1), limit_ns)) {
            if (a.err) set_dev_error(a.err, NCM_DEVERR_MBAR_TIMEOUT);
            ok = false;
        }
        if (!__syncthreads_and(ok)) {
            // a load that never landed: wait (bounded) for the copies still in flight
            cp_async_wait_group<0>();
            if (rank == 0)
                for (int j = k; j < nchunk && j < k + kAvStages; ++j)
                    mbar_wait(&full[j % kAvStages], (uint32_t)((j / kAvStages) & 1), 100000000ull);
            return;
        }
        const float* vs = vbuf + (k % kAvStages) * kAvChunk * 32;
        const float* ws = wbuf + (k % kAvStages) * W * kAvChunk + warp * kAvChunk;
        const int np = min(kAvChunk, n - k * kAvChunk);
        acc = av_chunk_chain(ws, vs, np, lane, acc);
        __syncthreads();   // the slot may be refilled
    }
    const int h = h0 + warp;
    a.out[(size_t)tz * a.tok_stride + (size_t)h * a.hd + d0 + lane] = acc;
    if (a.out_q) {
        float amax = fabsf(acc);   // quantize_f32_to_q8_0 of this block (inference.rs:991-1029)
#pragma unroll
        for (int k = 16; k > 0; k >>= 1) amax = fmaxf(amax, __shfl_xor_sync(NCM_FULL, amax, k));
        const float scale = amax / 127.0f;
        int q = 0;
        if (scale > 0.0f) {
            const float inv = 1.0f / scale;
            q = (int)fminf(fmaxf(roundf(acc * inv), -127.0f), 127.0f);
        }
        const size_t o = (size_t)h * a.hd + d0;
        a.out_q[o + lane] = (int8_t)q;
        if (lane == 0) a.out_s[o >> 5] = scale;
    }
}

// Softmax and V accumulation in one launch (f32 cache through the TMA ring): one
// 256-thread CTA per (kv head, 32-dimension block, W query heads).  The first V chunks
// are requested before anything else, so they arrive while the softmax runs; then four
// warps per head compute that head's softmax (as attn_softmax_kernel: max, exp, the exact
// sequential sum, * 1/sum) into shared memory -- each of the head's hd/32 CTAs computes
// it, in parallel -- and warps 0 .. W-1 run the V chains as attn_av_tma_kernel does.  It
// saves the softmax launch and its round trip through global memory.
constexpr int kSvThreads = 256;
template <int W>
__global__ void __launch_bounds__(kSvThreads) attn_sv_kernel(const __grid_constant__ AttnParams a) {
    extern __shared__ __align__(128) float buf[];   // V ring [S][kAvChunk][32] | w [W][ctx4]
    __shared__ __align__(8) uint64_t full[kAvStages];
    __shared__ SeqSumScratchT<128> sc[W];
    __shared__ float red[8];
    constexpr int S = kAvStages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int k = 0; k < S; ++k) mbar_init(&full[k], 1);
        fence_mbar_init();
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();
    const int nd = a.hd / 32;
    const int kvh = blockIdx.x, db = blockIdx.y % nd, hgrp = blockIdx.y / nd, tz = blockIdx.z;
    const int pos = (a.pos_override >= 0 ? a.pos_override : __ldcg(&a.state[ST_POS])) + tz;
    const int n = pos + 1;
    const int g = a.heads / a.kv_heads;
    const int h0 = kvh * g + hgrp * W;
    const int d0 = db * 32;
    const int ctx4 = (a.ctx + 3) & ~3;
    float* vbuf = buf;
    float* wsm = buf + S * kAvChunk * 32;
    const int nchunk = (n + kAvChunk - 1) / kAvChunk;
    const uint64_t limit_ns = 1000000000ull;
    const uint64_t pol = l2_evict_first_policy();
    auto issue_v = [&](int k) {   // thread 0
        uint64_t* bar = &full[k % S];
        mbar_arrive_expect_tx(bar, kAvChunk * 32 * 4);
        tma_load_2d(vbuf + (k % S) * kAvChunk * 32, &a.vmap, kvh * a.hd + d0, k * kAvChunk, bar, pol);
    };
    if (tid == 0)
        for (int k = 0; k < S - 1 && k < nchunk; ++k) issue_v(k);
    // ---- softmax of head h0 + j by warps 4j .. 4j+3 (inference.rs:3522-3540)
    const int j = warp >> 2, t = tid & 127;
    if (j < W) {
        const float* srow = a.scores + ((size_t)tz * a.heads + h0 + j) * a.ctx;
        float* e = wsm + j * ctx4;
        float mx = -INFINITY;
        for (int p = t; p < n; p += 128) {
            const float v = __ldcg(&srow[p]);
            e[p] = v;
            mx = fmaxf(mx, v);   // max is order independent (no NaNs)
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(NCM_FULL, mx, o));
        if (lane == 0) red[warp] = mx;
        if (j == 0) group_sync<128, 1>(); else group_sync<128, 2>();
        mx = fmaxf(fmaxf(red[4 * j], red[4 * j + 1]), fmaxf(red[4 * j + 2], red[4 * j + 3]));
        for (int p = t; p < n; p += 128) e[p] = expf_cr(e[p] - mx);
        float sum;
        if (j == 0) {
            group_sync<128, 1>();
            sum = seq_sum_nonneg<128, 1>([&](int i) { return e[i]; }, n, sc[0], t);
        } else {
            group_sync<128, 2>();
            sum = seq_sum_nonneg<128, 2>([&](int i) { return e[i]; }, n, sc[W - 1], t);
        }
        const float inv = 1.0f / sum;
        for (int p = t; p < n; p += 128) e[p] = e[p] * inv;
    }
    __syncthreads();
    // ---- V chains: warp h < W, lane = dimension
    float acc = 0.0f;
    for (int k = 0; k < nchunk; ++k) {
        if (tid == 0 && k + S - 1 < nchunk) issue_v(k + S - 1);
        bool ok = mbar_wait(&full[k % S], (uint32_t)((k / S) & 1), limit_ns);
        if (!ok && a.err) set_dev_error(a.err, NCM_DEVERR_MBAR_TIMEOUT);
        if (!__syncthreads_and(ok)) {
            // a load that never landed: wait (bounded) for the copies still in flight
            if (tid == 0)
                for (int q = k; q < nchunk && q < k + S; ++q)
                    mbar_wait(&full[q % S], (uint32_t)((q / S) & 1), 100000000ull);
            return;
        }
        if (warp < W) {
            const float* vs = vbuf + (k % S) * kAvChunk * 32;
            const int c0 = k * kAvChunk;
            const float* ws = wsm + warp * ctx4 + c0;
            const int np = min(kAvChunk, n - c0);
            acc = av_chunk_chain(ws, vs, np, lane, acc);
        }
        __syncthreads();   // the slot may be refilled
    }
    if (warp < W) {
        const int h = h0 + warp;
        a.out[(size_t)tz * a.tok_stride + (size_t)h * a.hd + d0 + lane] = acc;
        if (a.out_q) {
            float amax = fabsf(acc);   // quantize_f32_to_q8_0 of this block (inference.rs:991-1029)
#pragma unroll
            for (int k = 16; k > 0; k >>= 1) amax = fmaxf(amax, __shfl_xor_sync(NCM_FULL, amax, k));
            const float scale = amax / 127.0f;
            int q = 0;
            if (scale > 0.0f) {
                const float inv = 1.0f / scale;
                q = (int)fminf(fmaxf(roundf(acc * inv), -127.0f), 127.0f);
            }
            const size_t o = (size_t)h * a.hd + d0;
            a.out_q[o + lane] = (int8_t)q;
            if (lane == 0) a.out_s[o >> 5] = scale;
        }
    }
}

template <int W, int HPW>
__global__ void __launch_bounds__(W * 32) attn_av_kernel(const __grid_constant__ AttnParams a) {
    extern __shared__ __align__(16) float buf[];
    pdl_launch_dependents();
    pdl_wait();
    const int nd = a.hd / 32;
    attn_av_body<W, HPW>(a, blockIdx.x, blockIdx.y % nd, blockIdx.y / nd, blockIdx.z, buf, threadIdx.x);
}

// The V cache of a layer as a 2-D tensor map: {kvw floats, ctx rows}, box 32 x kAvChunk.
static int encode_v_map(AttnParams& a) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (!enc) return (int)cudaErrorNotSupported;
    cuuint64_t gdim[2] = {(cuuint64_t)a.kvw, (cuuint64_t)a.ctx};
    cuuint64_t gstride[1] = {(cuuint64_t)a.kvw * 4};
    cuuint32_t box[2] = {32, (cuuint32_t)kAvChunk};
    cuuint32_t estride[2] = {1, 1};
    CUresult cr = enc(&a.vmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(a.vc), gdim, gstride, box, estride,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return cr == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

int attention_launch(const AttnParams& a0, cudaStream_t s, bool pdl) {
    constexpr int kMaxSmem = 200 * 1024;
    AttnParams a = a0;
    const int g = a.heads / a.kv_heads;
    if (a.hd % 32 || a.heads % a.kv_heads || (size_t)a.ctx * 4 > (size_t)kMaxSmem) return (int)cudaErrorInvalidValue;
    if (int r = set_smem_limit((const void*)attn_softmax_kernel, kMaxSmem)) return r;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const int nz = a.ntok > 1 ? a.ntok : 1;
    cfg.gridDim = dim3(a.kv_heads, (a.ctx + 31) / 32, nz);
    int r = (int)cudaLaunchKernelEx(&cfg, attn_scores_kernel, a);
    if (r) return r;
    const int w = g % 2 == 0 ? 2 : 1;
    const size_t sv_smem = (size_t)kAvStages * kAvChunk * 32 * 4 + (size_t)w * ((a.ctx + 3) & ~3) * 4;
    if (a.vmap_on && a.sv_on && a.kv_kind == KV_F32 && (((uintptr_t)a.vc) & 15) == 0 && (a.kvw & 3) == 0 &&
        sv_smem <= (size_t)kMaxSmem && encode_v_map(a) == 0) {
        // softmax and V accumulation in one launch
        if (int r2 = set_smem_limit((const void*)attn_sv_kernel<1>, kMaxSmem)) return r2;
        if (int r2 = set_smem_limit((const void*)attn_sv_kernel<2>, kMaxSmem)) return r2;
        cfg.gridDim = dim3(a.kv_heads, (a.hd / 32) * (g / w), nz);
        cfg.blockDim = dim3(kSvThreads);
        cfg.dynamicSmemBytes = sv_smem;
        if (w == 2) return (int)cudaLaunchKernelEx(&cfg, attn_sv_kernel<2>, a);
        return (int)cudaLaunchKernelEx(&cfg, attn_sv_kernel<1>, a);
    }
    // the softmax of the last row reaches position pos + ntok - 1 (at most ctx - 1)
    cfg.gridDim = dim3(a.heads, 1, nz);
    cfg.dynamicSmemBytes = (size_t)a.ctx * 4;
    r = (int)cudaLaunchKernelEx(&cfg, attn_softmax_kernel, a);
    if (r) return r;
    // heads per item: two warps of one chain each when the group allows (measured on the
    // 70B shape at 1k positions: more chains per warp, or more heads per item, are slower
    // -- the items then stream their V slices with fewer CTAs)
    if (a.vmap_on && a.kv_kind == KV_F32 && (((uintptr_t)a.vc) & 15) == 0 && (a.kvw & 3) == 0 &&
        encode_v_map(a) == 0) {
        cfg.gridDim = dim3(a.kv_heads, (a.hd / 32) * (g / w), nz);
        cfg.blockDim = dim3(w * 32);
        cfg.dynamicSmemBytes = (size_t)kAvStages * kAvChunk * (32 + w) * 4;
        if (w == 2) return (int)cudaLaunchKernelEx(&cfg, attn_av_tma_kernel<2>, a);
        return (int)cudaLaunchKernelEx(&cfg, attn_av_tma_kernel<1>, a);
    }
    cfg.gridDim = dim3(a.kv_heads, (a.hd / 32) * (g / w), nz);
    cfg.blockDim = dim3(w * 32);
    cfg.dynamicSmemBytes = (size_t)kAvStages * av_stage_floats(w) * 4;
    if (w == 2) return (int)cudaLaunchKernelEx(&cfg, attn_av_kernel<2, 1>, a);
    return (int)cudaLaunchKernelEx(&cfg, attn_av_kernel<1, 1>, a);
}

// store_kv (inference.rs:539-568) for the F16 cache (fast_f32_to_f16 per value) and the
// Q8_0 cache (quantize_row_to_q8_0_blocks, inference.rs:4298-4317: scale = max|x|/127,
// inv = 1/scale or 0, q = round(x * inv) clamped, scale stored as truncated f16): one warp
// per 32-value block, grid (blocks, token).
__global__ void kv_store_kernel(int kind, const float* sk, const float* sv, int kw, uint8_t* kc, uint8_t* vc,
                                const int* pos_dev) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.y, lane = threadIdx.x & 31;
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= kw / 32) return;
    const int pos = pos_dev[0] + t;
    for (int which = 0; which < 2; ++which) {
        const float x = (which ? sv : sk)[(size_t)t * kw + 32 * b + lane];
        uint8_t* cache = which ? vc : kc;
        if (kind == KV_F16) {
            reinterpret_cast<uint16_t*>(cache)[(size_t)pos * kw + 32 * b + lane] = ncm_f32_to_f16_trunc(x);
        } else {
            float mx = fabsf(x);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(NCM_FULL, mx, o));
            const float sc = mx / 127.0f, inv = sc > 0.0f ? 1.0f / sc : 0.0f;
            const int q = (int)fminf(fmaxf(roundf(x * inv), -127.0f), 127.0f);
            uint8_t* blk = cache + ((size_t)pos * (kw / 32) + b) * 34;
            blk[2 + lane] = (uint8_t)(int8_t)q;
            if (lane == 0) {
                const uint16_t h = ncm_f32_to_f16_trunc(sc);
                blk[0] = (uint8_t)(h & 0xff);
                blk[1] = (uint8_t)(h >> 8);
            }
        }
    }
}

// ------------------------------------------------------------------ small kernels
static cudaLaunchConfig_t small_cfg(dim3 g, dim3 b, cudaStream_t s, bool pdl, cudaLaunchAttribute* attr);
int kv_store_launch(int kind, const float* sk, const float* sv, int ntok, int kw, void* kc, void* vc,
                    const int* pos_dev, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    const int nb = kw / 32;
    cudaLaunchConfig_t cfg = small_cfg(dim3((nb + 7) / 8, ntok), dim3(256), s, pdl, attr);
    return (int)cudaLaunchKernelEx(&cfg, kv_store_kernel, kind, sk, sv, kw, (uint8_t*)kc, (uint8_t*)vc, pos_dev);
}

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

// inference.rs:4494-4503 embed_token: one row of the dequantised token_embd table,
// dequantised on demand for the current token.
// A step that starts at or past the context limit (the caller decoded more tokens than
// the context holds) would store K/V past the cache: the position is clamped to the last
// slot here, before any later kernel of the step reads it (they all read it after their
// dependent-launch wait), and the error word tells the host.
__global__ void embed_kernel(int type, const uint8_t* table, int64_t pitch, int emb, const int* tokens,
                             int* state, int ctx, int* err, float* hidden) {
    pdl_launch_dependents();
    pdl_wait();
    int ps = state[ST_POS];
    if (ps >= ctx || ps < 0) {
        ps = ps < 0 ? 0 : ctx - 1;
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            state[ST_POS] = ps;
            set_dev_error(err, NCM_DEVERR_CTX_FULL);
        }
    }
    const int tok = tokens[ps];
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

int embed_launch(int type, const uint8_t* table, int64_t pitch, int emb, const int* tokens, int* state, int ctx,
                 int* err, float* hidden, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = small_cfg(dim3((emb + 255) / 256), dim3(256), s, pdl, attr);
    return (int)cudaLaunchKernelEx(&cfg, embed_kernel, type, table, pitch, emb, tokens, state, ctx, err, hidden);
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

// ------------------------------------------------------------------ multi-row TP reductions
// The row-parallel sum of a multi-row pass (tp.rs:349-363, every row): each CTA takes a
// slice of the ntok x H partials, stores it into slot [me] of every rank's receive area
// (NVLink stores for peers), publishes one flag per rank after a system-scope fence, waits
// (bounded) for the same CTA of every rank, then sums the slice in rank order from 0.0f
// and adds it to the residual -- the same bits on every rank, and the same bits as the
// one-row fused reduction and the host reducer.
__global__ void tp_rows_reduce_kernel(const __grid_constant__ TpRows t, const float* part, float* hidden, int n) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ unsigned s_epoch;
    if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile unsigned*>(&t.ctr[0]) + 1u;
    __syncthreads();
    const unsigned epoch = s_epoch;
    const int W = t.world, me = t.rank;
    const size_t par = (size_t)(epoch & 1u) * W;
    const int slice = (n + gridDim.x - 1) / gridDim.x;
    const int lo = blockIdx.x * slice, hi = min(n, lo + slice);
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = part[i];
        for (int d = 0; d < W; ++d) t.rrecv[d][(par + me) * t.stride + i] = v;
    }
    __syncthreads();
    unsigned* fl = nullptr;
    if (threadIdx.x == 0) {
        fence_acq_rel_sys();
        for (int d = 0; d < W; ++d) st_relaxed_sys(&t.rflags[d][(size_t)blockIdx.x * W + me], epoch);
    }
    if ((int)threadIdx.x < W) {
        fl = &t.rflags[me][(size_t)blockIdx.x * W + threadIdx.x];
        if (!wait_flag_sys(fl, epoch, t.timeout_ns)) set_dev_error(t.err, NCM_DEVERR_PEER_TIMEOUT);
    }
    __syncthreads();
    const float* base = t.rrecv[me] + par * t.stride;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        float sum = 0.0f;
        for (int src = 0; src < W; ++src) sum += __ldcg(base + (size_t)src * t.stride + i);
        hidden[i] += sum;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // the last CTA of this rank to finish advances the epoch for the next use
        __threadfence();
        if (atomicAdd(&t.ctr[1], 1u) == gridDim.x - 1) {
            t.ctr[1] = 0u;
            t.ctr[0] = epoch;
            __threadfence();
        }
    }
}

int tp_rows_reduce_launch(const TpRows& t, const float* part, float* hidden, int n, cudaStream_t s) {
    const int grid = std::max(1, std::min(t.grid_max, (n + 1023) / 1024));
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = small_cfg(dim3(grid), dim3(256), s, true, attr);
    return (int)cudaLaunchKernelEx(&cfg, tp_rows_reduce_kernel, t, part, hidden, n);
}

// Each row's head pair (logit, global token) of this vocab shard to every rank, then the
// merge in rank order, the first strictly greater logit winning (cluster_tp_node.rs:
// 1185-1204, per row) -- one CTA, one thread per row.
__global__ void tp_rows_argmax_kernel(const __grid_constant__ TpRows t, const float2* pairs, int ntok,
                                      int* argmax_out) {
    pdl_launch_dependents();
    pdl_wait();
    const unsigned epoch = *reinterpret_cast<volatile unsigned*>(&t.ctr[2]) + 1u;
    const int W = t.world, me = t.rank;
    const size_t par = (size_t)(epoch & 1u) * W;
    const int r = threadIdx.x;
    if (r < ntok)
        for (int d = 0; d < W; ++d) t.hrecv[d][(par + me) * kMaxBatch + r] = pairs[r];
    __syncthreads();
    if (threadIdx.x == 0) {
        fence_acq_rel_sys();
        for (int d = 0; d < W; ++d) st_relaxed_sys(&t.hflags[d][me], epoch);
    }
    if ((int)threadIdx.x < W && !wait_flag_sys(&t.hflags[me][threadIdx.x], epoch, t.timeout_ns))
        set_dev_error(t.err, NCM_DEVERR_PEER_TIMEOUT);
    __syncthreads();
    if (r < ntok) {
        float mv = 0.0f;
        int mt = 0;
        for (int src = 0; src < W; ++src) {
            const float2 e = __ldcg(&t.hrecv[me][(par + src) * kMaxBatch + r]);
            if (src == 0 || e.x > mv) { mv = e.x; mt = __float_as_int(e.y); }
        }
        argmax_out[r] = mt;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        t.ctr[2] = epoch;
    }
}

int tp_rows_argmax_launch(const TpRows& t, const float2* pairs, int ntok, int* argmax_out, cudaStream_t s) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = small_cfg(dim3(1), dim3(32), s, true, attr);
    return (int)cudaLaunchKernelEx(&cfg, tp_rows_argmax_kernel, t, pairs, ntok, argmax_out);
}

// The NCCL variant's merge: gathered = [world][kMaxBatch] pairs after ncclAllGather.
__global__ void rows_argmax_merge_kernel(const float2* gathered, int world, int ntok, int* argmax_out) {
    pdl_launch_dependents();
    pdl_wait();
    const int r = threadIdx.x;
    if (r >= ntok) return;
    float mv = 0.0f;
    int mt = 0;
    for (int src = 0; src < world; ++src) {
        const float2 e = gathered[(size_t)src * kMaxBatch + r];
        if (src == 0 || e.x > mv) { mv = e.x; mt = __float_as_int(e.y); }
    }
    argmax_out[r] = mt;
}

int rows_argmax_merge_launch(const float2* gathered, int world, int ntok, int* argmax_out, cudaStream_t s) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = small_cfg(dim3(1), dim3(32), s, true, attr);
    return (int)cudaLaunchKernelEx(&cfg, rows_argmax_merge_kernel, gathered, world, ntok, argmax_out);
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
    const int nb = cols / 32, units = (nb + 1) / 2;
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * units) return;
    int64_t r = idx / units;
    int u = (int)(idx % units);
    const bool two = 2 * u + 1 < nb;   // the last unit of an odd block count holds one block
    XUnit x;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(xq + 64 * u);
    for (int i = 0; i < 16; ++i) x.w[i] = (i < 8 || two) ? src[i] : 0u;
    x.s[0] = x.s[1] = 1.0f;
    for (int h = 0; h < 2; ++h) {
        int s = 0;
        for (int i = 0; i < 8; ++i) s = __dp4a((int)x.w[8 * h + i], 0x01010101, s);
        x.sum[h] = s;
    }
    const uint8_t* row = w + r * pitch;
    float t0, t1;
    if (qtype == NCM_T_Q4_K) {
        int ints[4];
        terms_q4_k(row, u, x, t0, t1, ints);
        int32_t* o = out + (r * nb + 2 * u) * 2;
        o[0] = ints[0]; o[1] = ints[1]; o[2] = ints[2]; o[3] = ints[3];
    } else {
        int d[2];
        if (qtype == NCM_T_Q4_0) terms_q4_0(row, u, x, t0, t1, d);
        else terms_q8_0(row, u, x, t0, t1, d);
        out[r * nb + 2 * u] = d[0];
        if (two) out[r * nb + 2 * u + 1] = d[1];
    }
}
int block_dots_launch(int qtype, const uint8_t* w, int64_t rows, int cols, int64_t pitch, const int8_t* xq,
                      int32_t* out, cudaStream_t s) {
    int64_t n = rows * ((cols / 32 + 1) / 2);
    if (n == 0) return 0;
    block_dots_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(qtype, w, rows, cols, pitch, xq, out);
    return (int)cudaGetLastError();
}

// inference.rs:697-706 rms_norm (one CTA): sequential-order sum of squares.  x is staged
// in shared memory when it fits (the exact sum reads each term up to three times).
__global__ void rms_norm_kernel(float* out, const float* x, const float* w, int n, float eps, int staged) {
    extern __shared__ __align__(16) float xs[];
    __shared__ SeqSumScratch sc;
    float tot;
    if (staged) {
        for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = x[i];
        __syncthreads();
        tot = seq_sum_nonneg<kThreads>([&](int i) { float v = xs[i]; return v * v; }, n, sc, threadIdx.x);
    } else {
        tot = seq_sum_nonneg<kThreads>([&](int i) { float v = x[i]; return v * v; }, n, sc, threadIdx.x);
    }
    const float scale = 1.0f / sqrtf(tot / (float)n + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = x[i] * scale * w[i];
}
int rms_norm_launch(float* out, const float* x, const float* w, int n, float eps, cudaStream_t s) {
    constexpr int kMaxStaged = 48 * 1024;   // floats (192 KB)
    if (int r = set_smem_limit((const void*)rms_norm_kernel, kMaxStaged * 4)) return r;
    const int staged = n <= kMaxStaged;
    rms_norm_kernel<<<1, kThreads, staged ? (size_t)n * 4 : 0, s>>>(out, x, w, n, eps, staged);
    return (int)cudaGetLastError();
}

__global__ void silu_mul_kernel(float* out, const float* g, const float* u, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        float sig = 1.0f / (1.0f + expf_cr(-g[i]));
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
    for (int l = 0; l < 32; ++l) v[l] = dequant_elem(src_type, row, 32 * b + l);
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


// ================================================================== multi-row GEMV (verify)
// speculative.rs:381-389 prefill_pass_batch -> inference.rs:1246-1303
// matmul_quantized_batch: each of ntok <= 8 activation rows against the same weights,
// every row's result bit-identical to the one-row GEMV (inference.rs:6866-6913).
// The block dots come from int8 tensor-core MMA (mma.sync m16n8k32 s8): A = 16 weight
// rows (a slab) x one 32-column block straight from the raw GGUF bytes in shared memory
// (Q4_0 nibbles - 8, Q8_0 bytes, Q4_K unsigned nibbles), B = the block of 8 token rows.
// Lane (g, t) of an MMA holds the exact integer dots of slab rows g, g+8 and tokens 2t,
// 2t+1.  Warp roles per 512-column stage:
//   warps 0-7  split the stage's slabs x 16 blocks, turn each dot into its f32 term with
//              the one-row path's formula and store the lane's four terms (float4);
//   warps 8-9  fold warp f owns slab f: the terms in block order into the four row sums
//              (same lane layout), then the epilogue;
//   thread 320 issues the TMA loads.
// Hand-offs are mbarriers: full (TMA -> compute), empty (compute -> producer), tfull
// (compute -> fold), tempty (fold -> compute: term slot reusable).
constexpr int kBatchThreads = 352;
constexpr int kBatchFoldWarps = 2;
constexpr int kBatchProducer = 320;

__device__ __forceinline__ void mma_s8_16x8x32(int32_t c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 4 bytes at a 2-byte aligned shared-memory address.
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    if ((a & 3) == 0) return *reinterpret_cast<const uint32_t*>(p);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(p - 2);
    return __funnelshift_r(w[0], w[1], 16);
}

__device__ __forceinline__ TileCursor batch_tile_at(const BatchParams& p, int cur, int r_end) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSeg; ++i)
        if (i < p.nseg && cur >= p.seg[i].row_begin) s = i;
    const int seg_end = p.seg[s].row_begin + p.seg[s].rows;
    return {s, min(p.box_rows, min(r_end, seg_end) - cur)};
}

// Terms of blocks bl0 .. bl0+NB-1 of chunk c for slab rows ra, rb = ra + 8 of one
// matrix tile.  T points at this lane's float4 of block 0 (block bl at T[32 * bl]):
// {(ra, tok 2t), (ra, 2t+1), (rb, 2t), (rb, 2t+1)}.
template <int QT, int NB>
__device__ __forceinline__ void batch_terms(const uint8_t* tile, int cb, int ra, int g, int t, int c, int bl0,
                                            const uint8_t* xq, int xq_pitch, const float* xs, const int* xsum,
                                            int nb, int ntok, float4* T) {
    const uint8_t* rowa = tile + ra * cb;
    const uint8_t* rowb = rowa + 8 * cb;
    const bool tg = g < ntok;
    const uint8_t* xrow = xq + g * xq_pitch;
    const int ta = 2 * t, tb = 2 * t + 1;
    const bool va = ta < ntok, vb = tb < ntok;
    if constexpr (QT == NCM_T_Q4_0 || QT == NCM_T_Q8_0) {
        constexpr int BB = QT == NCM_T_Q4_0 ? 18 : 34;
        // every fragment load first, then the MMAs, so that loads of different blocks overlap
        uint32_t a[NB][4], bf[NB][2];
        float da[NB], db[NB], sa[NB], sb[NB];
#pragma unroll
        for (int q = 0; q < NB; ++q) {
            const int bl = bl0 + q, bg = min(16 * c + bl, nb - 1);   // blocks past nb: terms unused
            if constexpr (QT == NCM_T_Q4_0) {
                const uint32_t wa = ld_u32_a2(rowa + BB * bl + 2 + 4 * t), wb = ld_u32_a2(rowb + BB * bl + 2 + 4 * t);
                a[q][0] = __vsub4(wa & 0x0f0f0f0fu, 0x08080808u);
                a[q][2] = __vsub4((wa >> 4) & 0x0f0f0f0fu, 0x08080808u);
                a[q][1] = __vsub4(wb & 0x0f0f0f0fu, 0x08080808u);
                a[q][3] = __vsub4((wb >> 4) & 0x0f0f0f0fu, 0x08080808u);
            } else {
                a[q][0] = ld_u32_a2(rowa + BB * bl + 2 + 4 * t);
                a[q][2] = ld_u32_a2(rowa + BB * bl + 18 + 4 * t);
                a[q][1] = ld_u32_a2(rowb + BB * bl + 2 + 4 * t);
                a[q][3] = ld_u32_a2(rowb + BB * bl + 18 + 4 * t);
            }
            bf[q][0] = tg ? *reinterpret_cast<const uint32_t*>(xrow + 32 * bg + 4 * t) : 0u;
            bf[q][1] = tg ? *reinterpret_cast<const uint32_t*>(xrow + 32 * bg + 16 + 4 * t) : 0u;
            da[q] = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(rowa + BB * bl));
            db[q] = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(rowb + BB * bl));
            sa[q] = va ? xs[ta * nb + bg] : 0.0f;
            sb[q] = vb ? xs[tb * nb + bg] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < NB; ++q) {
            int32_t d[4] = {0, 0, 0, 0};
            mma_s8_16x8x32(d, a[q][0], a[q][1], a[q][2], a[q][3], bf[q][0], bf[q][1]);
            // inference.rs:2663 / 1157: d_w * x_scale * (dot as f32)
            T[32 * (bl0 + q)] = make_float4(da[q] * sa[q] * (float)d[0], da[q] * sb[q] * (float)d[1],
                                            db[q] * sa[q] * (float)d[2], db[q] * sb[q] * (float)d[3]);
        }
    } else {
        // Q4_K: block bl is sub-block j = bl % 8 of super-block bl / 8 (two per chunk)
#pragma unroll
        for (int q = 0; q < NB; ++q) {
            const int bl = bl0 + q, sbi = bl >> 3, j = bl & 7, pr = j >> 1, h = j & 1;
            if (2 * c + sbi >= nb / 8) continue;   // chunk tail: the fold skips these terms
            const int bg = 16 * c + bl;
            const uint8_t* sa_ = rowa + 144 * sbi;
            const uint8_t* sb_ = rowb + 144 * sbi;
            const uint4 ha = *reinterpret_cast<const uint4*>(sa_), hb = *reinterpret_cast<const uint4*>(sb_);
            const float dA = f16_bits_to_f32(ha.x & 0xffff), mA = f16_bits_to_f32(ha.x >> 16);
            const float dB = f16_bits_to_f32(hb.x & 0xffff), mB = f16_bits_to_f32(hb.x >> 16);
            const uint32_t wa0 = *reinterpret_cast<const uint32_t*>(sa_ + 16 + 32 * pr + 4 * t);
            const uint32_t wa1 = *reinterpret_cast<const uint32_t*>(sa_ + 32 + 32 * pr + 4 * t);
            const uint32_t wb0 = *reinterpret_cast<const uint32_t*>(sb_ + 16 + 32 * pr + 4 * t);
            const uint32_t wb1 = *reinterpret_cast<const uint32_t*>(sb_ + 32 + 32 * pr + 4 * t);
            const uint32_t a0 = (wa0 >> (4 * h)) & 0x0f0f0f0fu, a2 = (wa1 >> (4 * h)) & 0x0f0f0f0fu;
            const uint32_t a1 = (wb0 >> (4 * h)) & 0x0f0f0f0fu, a3 = (wb1 >> (4 * h)) & 0x0f0f0f0fu;
            uint32_t b0 = 0, b1 = 0;
            if (tg) {
                b0 = *reinterpret_cast<const uint32_t*>(xrow + 32 * bg + 4 * t);
                b1 = *reinterpret_cast<const uint32_t*>(xrow + 32 * bg + 16 + 4 * t);
            }
            int32_t d4[4] = {0, 0, 0, 0};
            mma_s8_16x8x32(d4, a0, a1, a2, a3, b0, b1);
            int scA, mnA, scB, mnB;
            q4k_scale_min(j, ha.y, ha.z, ha.w, scA, mnA);
            q4k_scale_min(j, hb.y, hb.z, hb.w, scB, mnB);
            const float sclA = dA * (float)scA, mnlA = mA * (float)mnA;
            const float sclB = dB * (float)scB, mnlB = mB * (float)mnB;
            const float sa = va ? xs[ta * nb + bg] : 0.0f, sb = vb ? xs[tb * nb + bg] : 0.0f;
            const float xa = va ? (float)xsum[ta * nb + bg] : 0.0f, xb = vb ? (float)xsum[tb * nb + bg] : 0.0f;
            // q8.rs:1370-1373: x_scale * (d*sc * sum(q*x) - dmin*m * sum(x))
            T[32 * bl] = make_float4(sa * (sclA * (float)d4[0] - mnlA * xa), sb * (sclA * (float)d4[1] - mnlA * xb),
                                     sa * (sclB * (float)d4[2] - mnlB * xa), sb * (sclB * (float)d4[3] - mnlB * xb));
        }
    }
}

// Folds one chunk's 16 terms (T as in batch_terms) into acc[4] in block order: Q4_0 /
// Q8_0 term by term (inference.rs row sum += block result); Q4_K per super-block from 0
// (q8.rs:1342) and then into the row sum (inference.rs:3129).
template <int QT>
__device__ __forceinline__ void batch_fold(const float4* T, int c, int nb, float acc[4]) {
    float4 tv[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) tv[j] = T[32 * j];
    asm volatile("" ::: "memory");
    if constexpr (QT == NCM_T_Q4_K) {
        const int nsbc = min(2, nb / 8 - 2 * c);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            if (q < nsbc) {
                float ss[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    ss[0] += tv[8 * q + j].x;
                    ss[1] += tv[8 * q + j].y;
                    ss[2] += tv[8 * q + j].z;
                    ss[3] += tv[8 * q + j].w;
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[i] += ss[i];
            }
        }
    } else {
        const int nbc = min(16, nb - 16 * c);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (j < nbc) {
                acc[0] += tv[j].x;
                acc[1] += tv[j].y;
                acc[2] += tv[j].z;
                acc[3] += tv[j].w;
            }
        }
    }
}

template <int QT, int EPI>
__global__ void __launch_bounds__(kBatchThreads, 1) ncm_qgemm_verify_kernel(const __grid_constant__ BatchParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr bool DUAL = (EPI == EPI_SILU);
    constexpr int NM = DUAL ? 2 : 1;
    __shared__ float wv[kBatchFoldWarps][kMaxBatch];
    __shared__ int wi[kBatchFoldWarps][kMaxBatch];
    __shared__ int s_last;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + 8;
    uint64_t* tfull = full + 16;
    uint64_t* tempty = full + 24;
    uint8_t* stages = smem + p.stage_off;
    float4* tbase = reinterpret_cast<float4*>(smem + p.t_off);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int R = p.total_rows, nbk = gridDim.x;
    const int r_begin = (int)(((long long)blockIdx.x * R / nbk)) & ~1;
    const int r_end = (blockIdx.x + 1 == nbk) ? R : ((int)(((long long)(blockIdx.x + 1) * R / nbk)) & ~1);
    const int box_bytes = p.box_rows * p.chunk_bytes;
    const int box2_off = (box_bytes + 127) & ~127;
    const int ns = p.nstages, S = p.nslab;
    const int tslot = NM * S * 16 * 32;   // float4 per term slot
    const uint64_t limit_ns = 4000000000ull;
    if (tid == 0) {
        for (int s = 0; s < ns; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 8 / p.cgroups);
            mbar_init(&tfull[s], 8 / p.cgroups);
            mbar_init(&tempty[s], kBatchFoldWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();
    int icur = r_begin, ichunk = 0, tprod = 0;
    uint64_t pol = 0;
    auto issue = [&]() {
        const int s = tprod % ns;
        if (tprod >= ns && !mbar_wait(&empty[s], (uint32_t)(((tprod / ns) & 1) ^ 1), limit_ns))
            set_dev_error(p.err, NCM_DEVERR_MBAR_TIMEOUT);
        const TileCursor tc = batch_tile_at(p, icur, r_end);
        const int y = icur - p.seg[tc.seg].row_begin;
        const int x = ichunk * p.chunk_words;
        mbar_arrive_expect_tx(&full[s], DUAL ? 2 * box_bytes : box_bytes);
        tma_load_2d(stages + (size_t)s * p.stage_bytes, &p.tm[tc.seg], x, y, &full[s], pol);
        if (DUAL) tma_load_2d(stages + (size_t)s * p.stage_bytes + box2_off, &p.tm2, x, y, &full[s], pol);
        if (++ichunk == p.nchunk) { ichunk = 0; icur += tc.n; }
        ++tprod;
    };
    if (tid == kBatchProducer) {
        pol = l2_evict_first_policy();
        while (tprod < ns && icur < r_end) issue();
    }
    pdl_launch_dependents();
    pdl_wait();
    // quantised rows, their scales and per-block sums into shared memory (or, for rows
    // too wide for it, read in place from global memory, where they stay L2-resident)
    const uint8_t* xq = p.x_global ? reinterpret_cast<const uint8_t*>(p.xq) : smem + p.xq_off;
    const float* xs = p.x_global ? p.xs : reinterpret_cast<const float*>(smem + p.xs_off);
    const int* xsum = p.x_global ? p.xsum : reinterpret_cast<const int*>(smem + p.xsum_off);
    const int xq_pitch = p.x_global ? p.cols : p.xq_pitch;
    if (p.x_global) {
        // nothing to stage
    } else if (p.xf) {
        uint8_t* xq_s = smem + p.xq_off;
        float* xs_s = reinterpret_cast<float*>(smem + p.xs_off);
        int* xsum_s = reinterpret_cast<int*>(smem + p.xsum_off);
        // f32 rows: quantize_f32_to_q8_0 (inference.rs:991-1029) here, four lanes per
        // 32-value block (quad max and sum reductions), every element rounded as in the
        // one-thread quantiser
        const int li = tid & 3;
        const unsigned qmask = 0xFu << (tid & 28);
        for (int i = tid >> 2; i < p.ntok * p.nb; i += blockDim.x >> 2) {
            const int tk = i / p.nb, b = i % p.nb;
            const float4* src = reinterpret_cast<const float4*>(p.xf + (size_t)tk * p.xf_stride) + 8 * b + 2 * li;
            const float4 x0 = src[0], x1 = src[1];
            const float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            float amax = 0.0f;
#pragma unroll
            for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
            amax = fmaxf(amax, __shfl_xor_sync(qmask, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(qmask, amax, 2));
            const float sb = amax / 127.0f;
            uint32_t w0 = 0, w1 = 0;
            int sum = 0;
            if (sb > 0.0f) {
                const float inv = 1.0f / sb;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    float q = roundf(v[k] * inv);
                    q = fminf(fmaxf(q, -127.0f), 127.0f);
                    const int qi = (int)q;
                    sum += qi;
                    const uint32_t byte = (uint32_t)(qi & 0xff) << (8 * (k & 3));
                    if (k < 4) w0 |= byte; else w1 |= byte;
                }
            }
            sum += __shfl_xor_sync(qmask, sum, 1);
            sum += __shfl_xor_sync(qmask, sum, 2);
            *reinterpret_cast<uint2*>(xq_s + tk * p.xq_pitch + 32 * b + 8 * li) = make_uint2(w0, w1);
            if (li == 0) {
                xs_s[i] = sb;
                xsum_s[i] = sum;
            }
        }
    } else {
        uint8_t* xq_s = smem + p.xq_off;
        float* xs_s = reinterpret_cast<float*>(smem + p.xs_off);
        int* xsum_s = reinterpret_cast<int*>(smem + p.xsum_off);
        const int n16 = p.cols / 16;
        for (int i = tid; i < p.ntok * n16; i += blockDim.x) {
            const int tk = i / n16, k = i % n16;
            *reinterpret_cast<uint4*>(xq_s + tk * p.xq_pitch + 16 * k) =
                *reinterpret_cast<const uint4*>(p.xq + (size_t)tk * p.cols + 16 * k);
        }
        for (int i = tid; i < p.ntok * p.nb; i += blockDim.x) {
            const int tk = i / p.nb, b = i % p.nb;
            xs_s[i] = p.xs[(size_t)tk * p.nb + b];
            const uint4* src = reinterpret_cast<const uint4*>(p.xq + (size_t)tk * p.cols + 32 * b);
            int sum = 0;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const uint4 v = src[k];
                sum = __dp4a((int)v.x, 0x01010101, sum);
                sum = __dp4a((int)v.y, 0x01010101, sum);
                sum = __dp4a((int)v.z, 0x01010101, sum);
                sum = __dp4a((int)v.w, 0x01010101, sum);
            }
            xsum_s[i] = sum;
        }
    }
    __syncthreads();
    const int pos0 = p.pos_dev ? *p.pos_dev : p.pos0;
    float best_v[2] = {-INFINITY, -INFINITY};
    int best_i[2] = {0x7fffffff, 0x7fffffff};
    if (tid == kBatchProducer) {
        while (icur < r_end) issue();
    } else if (warp < 8) {
        // compute: p.cgroups groups of 8 / cgroups warps, group gi on the stages t with
        // t % cgroups == gi (several stages in progress at once); warp wi of a group ->
        // slab wi % S, blocks bl0 .. bl0 + nbw - 1 of its stages, nbw = 16 S / (8 / cgroups)
        const int G = p.cgroups, WG = 8 / G, gi = warp / WG, wi = warp % WG;
        const int g = lane >> 2, t = lane & 3;
        const int sl = wi % S, nbw = 16 * S / WG, bl0 = (wi / S) * nbw;
        const int ra = 16 * sl + g;
        auto terms = [&](const uint8_t* tl, int c, float4* T) {
            if (nbw == 2) batch_terms<QT, 2>(tl, p.chunk_bytes, ra, g, t, c, bl0, xq, xq_pitch, xs, xsum, p.nb, p.ntok, T);
            else if (nbw == 4) batch_terms<QT, 4>(tl, p.chunk_bytes, ra, g, t, c, bl0, xq, xq_pitch, xs, xsum, p.nb, p.ntok, T);
            else batch_terms<QT, 8>(tl, p.chunk_bytes, ra, g, t, c, bl0, xq, xq_pitch, xs, xsum, p.nb, p.ntok, T);
        };
        int tc_ = 0;
        for (int cur = r_begin; cur < r_end;) {
            const int n = batch_tile_at(p, cur, r_end).n;
            const bool active = 16 * sl < n;
            for (int c = 0; c < p.nchunk; ++c, ++tc_) {
                if (tc_ % G != gi) continue;
                const int s = tc_ % ns;
                const uint32_t u = (uint32_t)(tc_ / ns);
                if (!mbar_wait(&full[s], u & 1, limit_ns)) set_dev_error(p.err, NCM_DEVERR_MBAR_TIMEOUT);
                if (u > 0 && !mbar_wait(&tempty[s], (u - 1) & 1, limit_ns)) set_dev_error(p.err, NCM_DEVERR_MBAR_TIMEOUT);
                if (active) {
                    const uint8_t* tile = stages + (size_t)s * p.stage_bytes;
                    float4* T = tbase + (size_t)s * tslot + sl * 16 * 32 + lane;
                    terms(tile, c, T);
                    if (DUAL) terms(tile + box2_off, c, T + S * 16 * 32);
                }
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&empty[s]);
                    mbar_arrive(&tfull[s]);
                }
            }
            cur += n;
        }
    } else if (warp < 8 + kBatchFoldWarps) {
        // fold warp f: slab f's rows ra / rb (tile-local) for tokens 2t / 2t+1
        const int f = warp - 8;
        const int g = lane >> 2, t = lane & 3;
        const int ra = 16 * f + g, rb = ra + 8;
        int tc_ = 0;
        for (int cur = r_begin; cur < r_end;) {
            const TileCursor tc = batch_tile_at(p, cur, r_end);
            const int n = tc.n;
            const bool active = f < S && 16 * f < n;
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, acc2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int c = 0; c < p.nchunk; ++c, ++tc_) {
                const int s = tc_ % ns;
                const uint32_t u = (uint32_t)(tc_ / ns);
                if (!mbar_wait(&tfull[s], u & 1, limit_ns)) set_dev_error(p.err, NCM_DEVERR_MBAR_TIMEOUT);
                if (active) {
                    const float4* T = tbase + (size_t)s * tslot + f * 16 * 32 + lane;
                    batch_fold<QT>(T, c, p.nb, acc);
                    if (DUAL) batch_fold<QT>(T + S * 16 * 32, c, p.nb, acc2);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[s]);
            }
            // tile epilogue
            const Seg& sg = p.seg[tc.seg];
            const int lrow0 = cur - sg.row_begin;
            float part[4];
            if (EPI == EPI_QKV) {
#pragma unroll
                for (int i = 0; i < 4; ++i) part[i] = __shfl_xor_sync(NCM_FULL, acc[i], 4);   // row ^ 1
            }
            if (active) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = (i < 2) ? ra : rb, tk = 2 * t + (i & 1);
                    if (r >= n || tk >= p.ntok) continue;
                    const int lr = lrow0 + r;
                    const float v = acc[i];
                    if constexpr (EPI == EPI_PLAIN) {
                        sg.out[(size_t)tk * p.out_stride + lr] = v;
                    } else if constexpr (EPI == EPI_RESID) {
                        p.hidden[(size_t)tk * p.hidden_stride + lr] += v;   // inference.rs:4670-4672
                    } else if constexpr (EPI == EPI_QKV) {
                        float o = v;
                        if (sg.kind != SEG_V) {
                            // inference.rs:904-933 apply_rope_cached at this token's position
                            const int ri = (lr % p.head_dim) >> 1;
                            if (ri < p.rope_half) {
                                const float2 scs = p.rope[(size_t)(pos0 + tk) * p.rope_half + ri];
                                const float x0 = (lr & 1) ? part[i] : v;
                                const float x1 = (lr & 1) ? v : part[i];
                                o = (lr & 1) ? (x0 * scs.x + x1 * scs.y) : (x0 * scs.y - x1 * scs.x);
                            }
                        }
                        if (sg.kind == SEG_Q) sg.out[(size_t)tk * p.out_stride + lr] = o;
                        else ((sg.kind == SEG_K ? p.kcache : p.vcache) +
                              (size_t)(p.kv_stage ? tk : pos0 + tk) * p.kv_width)[lr] = o;
                    } else if constexpr (EPI == EPI_SILU) {
                        const float gg = v, uu = acc2[i];
                        const float sig = 1.0f / (1.0f + expf_cr(-gg));   // inference.rs:3385-3388
                        sg.out[(size_t)tk * p.out_stride + lr] = gg * sig * uu;
                    } else if constexpr (EPI == EPI_ARGMAX) {
                        if (sg.out) sg.out[(size_t)tk * p.out_stride + lr] = v;
                        const int k = i & 1;
                        if (better(v, lr, best_v[k], best_i[k])) { best_v[k] = v; best_i[k] = lr; }
                    }
                }
            }
            cur += n;
        }
        if constexpr (EPI == EPI_ARGMAX) {
            // lanes with the same t hold the same two tokens: reduce over g (lane bits 2-4)
#pragma unroll
            for (int k = 0; k < 2; ++k) {
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    const float ov = __shfl_xor_sync(NCM_FULL, best_v[k], o);
                    const int oi = __shfl_xor_sync(NCM_FULL, best_i[k], o);
                    if (better(ov, oi, best_v[k], best_i[k])) { best_v[k] = ov; best_i[k] = oi; }
                }
            }
            if (lane < 4) {
                wv[f][2 * lane] = best_v[0]; wi[f][2 * lane] = best_i[0];
                wv[f][2 * lane + 1] = best_v[1]; wi[f][2 * lane + 1] = best_i[1];
            }
        }
    }
    __syncthreads();
    if constexpr (EPI == EPI_ARGMAX) {
        if (tid < p.ntok) {
            float bv = wv[0][tid];
            int bi = wi[0][tid];
            for (int w = 1; w < kBatchFoldWarps; ++w)
                if (better(wv[w][tid], wi[w][tid], bv, bi)) { bv = wv[w][tid]; bi = wi[w][tid]; }
            p.amax_part[(size_t)blockIdx.x * kMaxBatch + tid] = make_float2(bv, __int_as_float(bi));
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(p.counter, 1u) == (unsigned)nbk - 1;
        __syncthreads();
        if (s_last && tid < p.ntok) {
            __threadfence();
            float bv = -INFINITY;
            int bi = 0x7fffffff;
            for (int c = 0; c < nbk; ++c) {
                const float2 e = __ldcg(&p.amax_part[(size_t)c * kMaxBatch + tid]);
                const int ei = __float_as_int(e.y);
                if (better(e.x, ei, bv, bi)) { bv = e.x; bi = ei; }
            }
            if (p.pair_out) p.pair_out[tid] = make_float2(bv, __int_as_float(p.head_row0 + bi));   // shard's pair
            else p.argmax_out[tid] = p.head_row0 + bi;
        }
        __syncthreads();
        if (s_last && tid == 0) *p.counter = 0u;
    }
}

constexpr int kBatchSmemLimit = 220 * 1024;

int batch_plan(int qtype, int cols, int rows, bool dual, int ntok, BatchParams& p) {
    if (ntok < 1 || ntok > kMaxBatch || cols % 32) return -1;
    p.ntok = ntok;
    p.cols = cols;
    p.nb = cols / 32;
    p.nchunk = (cols + kChunkCols - 1) / kChunkCols;
    p.chunk_bytes = qtype == NCM_T_Q8_0 ? 16 * 34 : 288;
    p.chunk_words = p.chunk_bytes / 4;
    p.total_rows = rows;
    // one CTA per SM while every CTA keeps at least one 16-row slab
    int grid = num_sms();
    const int maxg = (rows + 15) / 16;
    if (grid > maxg) grid = maxg > 0 ? maxg : 1;
    const int per_cta = (rows + grid - 1) / grid;
    p.xq_pitch = cols + 16;   // distinct banks for the eight token rows of a fragment
    // Activation rows in shared memory when they fit beside a ring of at least four
    // stages; otherwise (wide inputs: the 70B down projection has 28672 columns) they are
    // read in place from global memory (x_global: xq / xs / xsum prepared by the caller).
    for (int xg = 0; xg < 2; ++xg) {
        int off = 256;            // full / empty / tfull / tempty mbarriers
        if (!xg) {
            p.xq_off = off;
            off += (ntok * p.xq_pitch + 127) / 128 * 128;
            p.xs_off = off;
            off += (ntok * p.nb * 4 + 127) / 128 * 128;
            p.xsum_off = off;
            off += (ntok * p.nb * 4 + 127) / 128 * 128;
        } else {
            if (p.xf) return -1;   // f32 rows are quantised into shared memory only
            p.xq_off = p.xs_off = p.xsum_off = off;
        }
        p.x_global = xg;
        p.stage_off = off;
        // slabs per tile: two (one per fold warp) unless the CTA's rows or the budget say one
        for (int S = std::min(2, (per_cta + 15) / 16); S >= 1; --S) {
            const int br = 16 * S;
            const int stage_bytes = (br * p.chunk_bytes + 127) / 128 * 128 * (dual ? 2 : 1);
            const int t_bytes = (dual ? 2 : 1) * S * 16 * 32 * 16;
            int ns = kMaxStages;
            while (ns > 2 && off + ns * (stage_bytes + t_bytes) > kBatchSmemLimit) --ns;
            if (off + ns * (stage_bytes + t_bytes) > kBatchSmemLimit || (!xg && ns < 4)) continue;
            p.nslab = S;
            if (p.cgroups != 1 && p.cgroups != 2 && p.cgroups != 4) p.cgroups = 2;
            if (S == 2 && p.cgroups == 4) p.cgroups = 2;
            p.box_rows = br;
            p.stage_bytes = stage_bytes;
            p.nstages = ns;
            p.t_off = off + ns * stage_bytes;
            p.smem_bytes = p.t_off + ns * t_bytes;
            return grid;
        }
    }
    return -1;
}

template <int QT, int EPI>
static int batch_launch_t(const BatchParams& p, int grid, cudaStream_t s, bool pdl) {
    auto kern = ncm_qgemm_verify_kernel<QT, EPI>;
    if (int r = set_smem_limit((const void*)kern, kBatchSmemLimit)) return r;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kBatchThreads);
    cfg.dynamicSmemBytes = p.smem_bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return (int)cudaLaunchKernelEx(&cfg, kern, p);
}

template <int QT>
static int batch_launch_q(int epi, const BatchParams& p, int grid, cudaStream_t s, bool pdl) {
    switch (epi) {
        case EPI_PLAIN: return batch_launch_t<QT, EPI_PLAIN>(p, grid, s, pdl);
        case EPI_RESID: return batch_launch_t<QT, EPI_RESID>(p, grid, s, pdl);
        case EPI_QKV: return batch_launch_t<QT, EPI_QKV>(p, grid, s, pdl);
        case EPI_SILU: return batch_launch_t<QT, EPI_SILU>(p, grid, s, pdl);
        case EPI_ARGMAX: return batch_launch_t<QT, EPI_ARGMAX>(p, grid, s, pdl);
        default: return (int)cudaErrorInvalidValue;
    }
}

int batch_gemv_launch(int qtype, int epi, const BatchParams& p, int grid, cudaStream_t s, bool pdl) {
    if (qtype == NCM_T_Q4_0) return batch_launch_q<NCM_T_Q4_0>(epi, p, grid, s, pdl);
    if (qtype == NCM_T_Q8_0) return batch_launch_q<NCM_T_Q8_0>(epi, p, grid, s, pdl);
    if (qtype == NCM_T_Q4_K) return batch_launch_q<NCM_T_Q4_K>(epi, p, grid, s, pdl);
    return (int)cudaErrorInvalidValue;
}

// Per token row: optional rms_norm (inference.rs:697-706; layer 0 reads the embedding
// row's sequential sum of squares) then quantize_f32_to_q8_0 (inference.rs:991-1029).
// Grid (token, split): every CTA of a token forms the same exact norm scale and
// quantises its share of the 32-value blocks, four lanes per block.
constexpr int kPrepSplit = 16;
// NT threads: 512 when the CTA folds an RMS sum (short per-thread chunks), else 256.
template <int NT>
__global__ void __launch_bounds__(NT) batch_prep_kernel(const float* x, int x_stride, int n, const float* norm_w,
                                                        float eps, const float* ssq_tab, const int* toks,
                                                        int8_t* xq, float* xs, int* xsum) {
    extern __shared__ __align__(16) float xr[];
    __shared__ SeqSumScratchT<NT> sc;
    pdl_launch_dependents();
    pdl_wait();
    const int tk = blockIdx.x, tid = threadIdx.x;
    const int nblk = n / 32;
    const int per = (nblk + gridDim.y - 1) / gridDim.y;
    const int b0 = blockIdx.y * per, b1 = min(nblk, b0 + per);
    const float* src = x + (size_t)tk * x_stride;
    float scale = 1.0f;
    if (norm_w) {
        if (ssq_tab) {
            scale = 1.0f / sqrtf(ssq_tab[toks[tk]] / (float)n + eps);
        } else {
            stage_f32(xr, src, n, tid, blockDim.x);
            __syncthreads();
            const float tot = seq_sum_nonneg<NT>([&](int i) { float v = xr[i]; return v * v; }, n, sc, tid);
            scale = 1.0f / sqrtf(tot / (float)n + eps);
        }
    }
    const int li = tid & 3;
    const unsigned qmask = 0xFu << (tid & 28);
    for (int b = b0 + (tid >> 2); b < b1; b += blockDim.x >> 2) {
        const int c = li;
        float v[8];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float4 x4 = reinterpret_cast<const float4*>(src)[8 * b + 2 * c + h];
            if (norm_w) {
                const float4 w4 = reinterpret_cast<const float4*>(norm_w)[8 * b + 2 * c + h];
                v[4 * h] = x4.x * scale * w4.x;
                v[4 * h + 1] = x4.y * scale * w4.y;
                v[4 * h + 2] = x4.z * scale * w4.z;
                v[4 * h + 3] = x4.w * scale * w4.w;
            } else {
                v[4 * h] = x4.x; v[4 * h + 1] = x4.y; v[4 * h + 2] = x4.z; v[4 * h + 3] = x4.w;
            }
        }
        float amax = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
        amax = fmaxf(amax, __shfl_xor_sync(qmask, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(qmask, amax, 2));
        const float sb = amax / 127.0f;
        uint32_t w0 = 0, w1 = 0;
        int sum = 0;
        if (sb > 0.0f) {
            const float inv = 1.0f / sb;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float q = roundf(v[i] * inv);
                q = fminf(fmaxf(q, -127.0f), 127.0f);
                sum += (int)q;
                const uint32_t byte = (uint32_t)((int)q & 0xff) << (8 * (i & 3));
                if (i < 4) w0 |= byte; else w1 |= byte;
            }
        }
        sum += __shfl_xor_sync(qmask, sum, 1);
        sum += __shfl_xor_sync(qmask, sum, 2);
        *reinterpret_cast<uint2*>(xq + (size_t)tk * n + 32 * b + 8 * c) = make_uint2(w0, w1);
        if (li == 0) {
            xs[(size_t)tk * nblk + b] = sb;
            if (xsum) xsum[(size_t)tk * nblk + b] = sum;
        }
    }
}

int batch_prep_launch(const float* x, int x_stride, int n, int ntok, const float* norm_w, float eps,
                      const float* ssq_tab, const int* toks, int8_t* xq, float* xs, int* xsum, cudaStream_t s,
                      bool pdl) {
    if (int r = set_smem_limit((const void*)batch_prep_kernel<256>, 128 * 1024)) return r;
    if (int r = set_smem_limit((const void*)batch_prep_kernel<512>, 128 * 1024)) return r;
    cudaLaunchAttribute attr[1];
    const int split = std::min(kPrepSplit, std::max(1, n / 32 / 64));
    const bool folds = norm_w && !ssq_tab;
    cudaLaunchConfig_t cfg = small_cfg(dim3(ntok, split), dim3(folds ? 512 : 256), s, pdl, attr);
    cfg.dynamicSmemBytes = folds ? (size_t)n * 4 : 0;
    if (folds)
        return (int)cudaLaunchKernelEx(&cfg, batch_prep_kernel<512>, x, x_stride, n, norm_w, eps, ssq_tab, toks, xq, xs,
                                       xsum);
    return (int)cudaLaunchKernelEx(&cfg, batch_prep_kernel<256>, x, x_stride, n, norm_w, eps, ssq_tab, toks, xq, xs,
                                   xsum);
}

// Per-block sums of quantised rows (the Q4_K min term needs sum(x) per 32-block).
__global__ void block_sums_kernel(const int8_t* xq, int64_t nblocks, int* xsum) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    const uint4* src = reinterpret_cast<const uint4*>(xq + 32 * b);
    int sum = 0;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint4 v = src[k];
        sum = __dp4a((int)v.x, 0x01010101, sum);
        sum = __dp4a((int)v.y, 0x01010101, sum);
        sum = __dp4a((int)v.z, 0x01010101, sum);
        sum = __dp4a((int)v.w, 0x01010101, sum);
    }
    xsum[b] = sum;
}
int block_sums_launch(const int8_t* xq, int64_t nblocks, int* xsum, cudaStream_t s) {
    if (nblocks <= 0) return 0;
    block_sums_kernel<<<(unsigned)((nblocks + 127) / 128), 128, 0, s>>>(xq, nblocks, xsum);
    return (int)cudaGetLastError();
}

__global__ void embed_rows_kernel(int type, const uint8_t* table, int64_t pitch, int emb, const int* toks,
                                  float* hidden) {
    pdl_launch_dependents();
    pdl_wait();
    const int tk = blockIdx.y;
    const uint8_t* row = table + (size_t)toks[tk] * pitch;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < emb; i += gridDim.x * blockDim.x)
        hidden[(size_t)tk * emb + i] = dequant_elem(type, row, i);
}

int embed_rows_launch(int type, const uint8_t* table, int64_t pitch, int emb, const int* toks, int ntok,
                      float* hidden, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = small_cfg(dim3((emb + 255) / 256, ntok), dim3(256), s, pdl, attr);
    return (int)cudaLaunchKernelEx(&cfg, embed_rows_kernel, type, table, pitch, emb, toks, hidden);
}


// ================================================================== Q6_K GEMV
// matmul_q6_k (inference.rs:3045-3087) over Q6KBlock::dot_q8_scaled (q8.rs:2092-2150),
// the x86 path: per super-block sum = 0, then for each 128-half the 256 products
// (c * q) * x, c = (d * scale) * x_scale, added one at a time in the order l = 0..15 then
// 16..31, quarters q1..q4 within each l; the row sum adds the super-block sums in order.
// That is one sequential f32 chain per row, so each thread owns one row.  The thread
// reads its row with 16-byte loads: a run of 8 super-blocks (1680 bytes) starts on a
// 16-byte boundary, so with the run unrolled every super-block's byte offset is a
// compile-time constant and its fields are assembled from the loaded words without
// dynamic register indexing.  The activation is staged once per CTA as f32 (exact).
template <int J>
__device__ __forceinline__ uint32_t q6_word(const uint4 (&u)[14], int i) {
    // 32-bit word i of super-block J of the run (its bytes 4i .. 4i+3)
    constexpr int off = (210 * J) & 15;
    const int b = off + 4 * i;                  // byte offset inside the 16-byte-aligned cover
    const int q = b >> 2, sh = (b & 3) * 8;
    auto w = [&](int k) -> uint32_t {
        if (k >= 56) return 0u;   // past the cover (only its unused high half is asked for)
        const uint4 v = u[k >> 2];
        return (k & 3) == 0 ? v.x : (k & 3) == 1 ? v.y : (k & 3) == 2 ? v.z : v.w;
    };
    return sh ? __funnelshift_r(w(q), w(q + 1), sh) : w(q);
}

template <int J>
__device__ __forceinline__ float q6k_block_sum(const uint4 (&u)[14], const float* x, const float* xs) {
    float ws[16];
    const uint32_t dw = q6_word<J>(u, 52);      // bytes 208..211: d at 208
    const float d = f16_bits_to_f32(dw & 0xffff);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t sw = q6_word<J>(u, 48 + i);   // scales 192 + 4i ..
#pragma unroll
        for (int b = 0; b < 4; ++b) ws[4 * i + b] = d * (float)(int)(int8_t)(sw >> (8 * b));
    }
    float sum = 0.0f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        float c[4][2];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            c[j][0] = ws[8 * half + 2 * j] * xs[4 * half + j];
            c[j][1] = ws[8 * half + 2 * j + 1] * xs[4 * half + j];
        }
        const float* xh = x + 128 * half;
#pragma unroll
        for (int l4 = 0; l4 < 8; ++l4) {
            const uint32_t a = q6_word<J>(u, 16 * half + l4);        // ql[64 half + 4 l4 ..]
            const uint32_t b = q6_word<J>(u, 16 * half + 8 + l4);    // ql[64 half + 32 + 4 l4 ..]
            const uint32_t h = q6_word<J>(u, 32 + 8 * half + l4);    // qh[32 half + 4 l4 ..]
            const uint32_t q1 = (a & 0x0f0f0f0fu) | ((h & 0x03030303u) << 4);
            const uint32_t q2 = (b & 0x0f0f0f0fu) | (((h >> 2) & 0x03030303u) << 4);
            const uint32_t q3 = ((a >> 4) & 0x0f0f0f0fu) | (((h >> 4) & 0x03030303u) << 4);
            const uint32_t q4 = ((b >> 4) & 0x0f0f0f0fu) | (((h >> 6) & 0x03030303u) << 4);
            const int hi = l4 >= 4;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int l = 4 * l4 + k;
                const float f1 = (float)((int)((q1 >> (8 * k)) & 0xff) - 32);
                const float f2 = (float)((int)((q2 >> (8 * k)) & 0xff) - 32);
                const float f3 = (float)((int)((q3 >> (8 * k)) & 0xff) - 32);
                const float f4 = (float)((int)((q4 >> (8 * k)) & 0xff) - 32);
                sum += c[0][hi] * f1 * xh[l];
                sum += c[1][hi] * f2 * xh[l + 32];
                sum += c[2][hi] * f3 * xh[l + 64];
                sum += c[3][hi] * f4 * xh[l + 96];
            }
        }
    }
    return sum;
}

template <int J>
__device__ __forceinline__ void q6k_run_step(const uint8_t* run, int nsb_left, const float* xr, const float* xsr,
                                             float& acc) {
    if (J >= nsb_left) return;
    uint4 u[14];
    const uint4* src = reinterpret_cast<const uint4*>(run + ((210 * J) & ~15));
    const int nu = ((((210 * J) & 15) + 210 + 15) >> 4);   // 16-byte words covering the block
#pragma unroll
    for (int i = 0; i < 14; ++i) u[i] = i < nu ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
    acc += q6k_block_sum<J>(u, xr + 256 * J, xsr + 8 * J);   // inference.rs:3082 sum += block dot
}

template <int EPI>
__global__ void __launch_bounds__(128) ncm_q6k_gemv_kernel(const __grid_constant__ Q6Params p) {
    extern __shared__ __align__(16) float q6x[];   // x as f32 [cols], then x scales [cols / 32]
    __shared__ float wv[4];
    __shared__ int wi[4];
    __shared__ int s_last;
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x, lane = tid & 31;
    float* xsf = q6x + p.cols;
    for (int i = tid; i < p.cols; i += blockDim.x) q6x[i] = (float)p.xq[i];
    for (int i = tid; i < p.cols / 32; i += blockDim.x) xsf[i] = p.xs[i];
    __syncthreads();
    const int r = blockIdx.x * blockDim.x + tid;
    const int nsb = p.cols / 256;
    float acc = 0.0f;
    if (r < p.rows) {
        const uint8_t* row = p.w + (size_t)r * p.pitch;
        for (int g = 0; g < nsb; g += 8) {
            const uint8_t* run = row + (size_t)g * 210;   // 1680 g / 8 bytes: 16-byte aligned
            const int left = nsb - g;
            const float* xr = q6x + 256 * g;
            const float* xsr = xsf + 8 * g;
            q6k_run_step<0>(run, left, xr, xsr, acc);
            q6k_run_step<1>(run, left, xr, xsr, acc);
            q6k_run_step<2>(run, left, xr, xsr, acc);
            q6k_run_step<3>(run, left, xr, xsr, acc);
            q6k_run_step<4>(run, left, xr, xsr, acc);
            q6k_run_step<5>(run, left, xr, xsr, acc);
            q6k_run_step<6>(run, left, xr, xsr, acc);
            q6k_run_step<7>(run, left, xr, xsr, acc);
        }
        if constexpr (EPI == EPI_PLAIN) p.out[r] = acc;
        else if constexpr (EPI == EPI_RESID) p.out[r] += acc;   // inference.rs:4744-4746
        else if (p.out) p.out[r] = acc;
    }
    if constexpr (EPI == EPI_ARGMAX) {
        // strict first-max (inference.rs:4838-4843): CTA, then the last CTA over all CTAs
        float bv = r < p.rows ? acc : -INFINITY;
        int bi = r < p.rows ? r : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(NCM_FULL, bv, o);
            const int oi = __shfl_xor_sync(NCM_FULL, bi, o);
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { wv[tid >> 5] = bv; wi[tid >> 5] = bi; }
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
                if (better(wv[w], wi[w], bv, bi)) { bv = wv[w]; bi = wi[w]; }
            p.amax_part[blockIdx.x] = make_float2(bv, __int_as_float(bi));
            __threadfence();
            s_last = atomicAdd(p.counter, 1u) == gridDim.x - 1;
        }
        __syncthreads();
        if (s_last && tid == 0) {
            __threadfence();
            bv = -INFINITY;
            bi = 0x7fffffff;
            for (int c = 0; c < (int)gridDim.x; ++c) {
                const float2 e = __ldcg(&p.amax_part[c]);
                const int ei = __float_as_int(e.y);
                if (better(e.x, ei, bv, bi)) { bv = e.x; bi = ei; }
            }
            const int tok = p.head_row0 + bi;
            if (p.head_out) {
                *p.head_out = make_float2(bv, __int_as_float(tok));
            } else {
                const int ps = p.state[ST_POS];
                if (ps + 1 < p.ctx && ps + 1 >= p.state[ST_NPROMPT]) p.tokens[ps + 1] = tok;
                p.state[ST_LAST_TOKEN] = tok;
                p.state[ST_POS] = ps + 1;
                p.state[ST_STEP] += 1;
            }
            *p.counter = 0u;
        }
    }
}

int q6k_gemv_launch(int epi, const Q6Params& p, cudaStream_t s, bool pdl) {
    if (p.cols % 256 || (p.pitch & 15) || ((uintptr_t)p.w & 15)) return (int)cudaErrorInvalidValue;
    const size_t smem = (size_t)p.cols * 4 + (size_t)(p.cols / 32) * 4;
    int threads = 128;
    while (threads > 32 && (int64_t)(p.rows + threads - 1) / threads < num_sms()) threads >>= 1;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = small_cfg(dim3((p.rows + threads - 1) / threads), dim3(threads), s, pdl, attr);
    cfg.dynamicSmemBytes = smem;
    const void* fn = epi == EPI_PLAIN ? (const void*)ncm_q6k_gemv_kernel<EPI_PLAIN>
                   : epi == EPI_RESID ? (const void*)ncm_q6k_gemv_kernel<EPI_RESID>
                                      : (const void*)ncm_q6k_gemv_kernel<EPI_ARGMAX>;
    if (int r = set_smem_limit(fn, 200 * 1024)) return r;
    if (smem > 200 * 1024) return (int)cudaErrorInvalidValue;
    if (epi == EPI_PLAIN) return (int)cudaLaunchKernelEx(&cfg, ncm_q6k_gemv_kernel<EPI_PLAIN>, p);
    if (epi == EPI_RESID) return (int)cudaLaunchKernelEx(&cfg, ncm_q6k_gemv_kernel<EPI_RESID>, p);
    if (epi == EPI_ARGMAX) return (int)cudaLaunchKernelEx(&cfg, ncm_q6k_gemv_kernel<EPI_ARGMAX>, p);
    return (int)cudaErrorInvalidValue;
}

}  // namespace ncm
