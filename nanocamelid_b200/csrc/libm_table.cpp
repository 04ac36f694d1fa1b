// Host side of the device expf that matches the reference's libm bit for bit.
//
// The reference computes exp with Rust's f32::exp, i.e. the host glibc expf
// (inference.rs:3385 silu, 3533 softmax).  glibc's expf is not correctly rounded: on
// this image (glibc 2.39) it differs from the correctly rounded result on roughly 1 in
// 5000 float inputs.  The device computes the correctly rounded value and patches those
// inputs from a table built here by asking this process's own glibc expf about every
// float whose exp neither underflows nor overflows (about 2.2e9 inputs, multithreaded,
// ~1-2 s).  The table is an open-addressing hash: key = input bits, value = glibc bits.
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <algorithm>
#include <cmath>
#include <thread>
#include <vector>

namespace ncm {

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

// Exceptions over [lo, hi) of float bit patterns (one sign).
static void scan_range(uint32_t lo, uint32_t hi, std::vector<uint64_t>* out) {
    for (uint64_t b = lo; b < hi; ++b) {
        const float x = u2f((uint32_t)b);
        const float g = expf(x);
        const float c = (float)exp((double)x);
        if (f2u(g) != f2u(c)) out->push_back((b << 32) | f2u(g));
    }
}

// True when the correctly rounded exp(x) is close enough to a float rounding midpoint
// for the device to consult the table: the same test as expf_cr, here with the host's
// double exp.
static bool near_midpoint(float x) {
    const double yd = exp((double)x);
    const float y = (float)yd;
    if (y == 0.0f || std::isinf(y)) return true;
    const double yy = (double)y;
    const double half = (yd >= yy ? ((double)nextafterf(y, INFINITY) - yy) : (yy - (double)nextafterf(y, 0.0f))) * 0.5;
    const double dist = fabs(yd - yy);
    // a margin of 2 over the device window covers the two libraries' double exp differing
    return half - dist <= half * 0x1p-7;
}

// Builds the exception hash.  Returns the table (pairs of uint32 {key, value}, EMPTY key
// 0xffffffff) with power-of-two capacity (at most max_entries); *mask = capacity - 1.
// Empty when even a half-full table of max_entries cannot hold them.
std::vector<uint32_t> build_expf_exceptions(int threads, uint32_t max_entries, uint32_t* mask, size_t* count,
                                            int* gate) {
    // x in (-104, 89): outside, expf is 0 / inf for both.
    const uint32_t pos_hi = f2u(89.0f);              // [+0, 89)
    const uint32_t neg_lo = 0x80000000u, neg_hi = f2u(-104.0f);   // [-0, -104)
    if (threads < 1) threads = 1;
    const int nt = threads * 2;
    std::vector<std::vector<uint64_t>> parts(nt);
    std::vector<std::thread> th;
    for (int k = 0; k < threads; ++k) {
        uint32_t a = (uint32_t)((uint64_t)pos_hi * k / threads), e = (uint32_t)((uint64_t)pos_hi * (k + 1) / threads);
        th.emplace_back(scan_range, a, e, &parts[k]);
        uint64_t span = (uint64_t)(neg_hi - neg_lo);
        uint32_t na = neg_lo + (uint32_t)(span * k / threads), ne = neg_lo + (uint32_t)(span * (k + 1) / threads);
        th.emplace_back(scan_range, na, ne, &parts[threads + k]);
    }
    for (auto& t : th) t.join();
    size_t n = 0;
    *gate = 1;
    for (auto& p : parts) {
        n += p.size();
        for (uint64_t e : p)
            if (!near_midpoint(u2f((uint32_t)(e >> 32)))) *gate = 0;
    }
    *count = n;
    size_t cap = 1;
    while (cap < 4 * n + 16) cap <<= 1;
    if (cap > max_entries) cap = max_entries;
    if (cap < 2 * n + 16) return {};
    std::vector<uint32_t> tab(2 * cap, 0xffffffffu);
    for (auto& p : parts)
        for (uint64_t e : p) {
            uint32_t key = (uint32_t)(e >> 32), val = (uint32_t)e;
            uint32_t h = (key * 2654435761u) & (uint32_t)(cap - 1);
            while (tab[2 * h] != 0xffffffffu) h = (h + 1) & (uint32_t)(cap - 1);
            tab[2 * h] = key;
            tab[2 * h + 1] = val;
        }
    *mask = (uint32_t)(cap - 1);
    return tab;
}

}  // namespace ncm
