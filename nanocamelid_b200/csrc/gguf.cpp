// GGUF v3 reader (gguf.rs:454-551 semantics) and the synthetic-model writer.
// Host code; built with -ffp-contract=off so the block encoders in synth.h round
// exactly as the device initialiser does.
#include "gguf.h"
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <vector>
#include "../../include/ncm.h"
#include "synth.h"

namespace ncm {

namespace {
struct Rd {
    const uint8_t* p;
    const uint8_t* end;
    bool err = false;
    uint64_t left() const { return (uint64_t)(end - p); }
    bool take(uint64_t n) {   // advance n bytes, or flag a truncated file
        if (err || n > left()) { err = true; return false; }
        p += n;
        return true;
    }
    uint64_t u(int n) {
        if (err || (uint64_t)n > left()) { err = true; return 0; }
        uint64_t v = 0;
        for (int i = 0; i < n; ++i) v |= (uint64_t)p[i] << (8 * i);
        p += n;
        return v;
    }
    std::string str() {
        uint64_t n = u(8);
        if (err || n > left()) { err = true; return {}; }
        std::string s((const char*)p, n);
        p += n;
        return s;
    }
};
int vsize(int t) {
    switch (t) {
        case 0: case 1: case 7: return 1;
        case 2: case 3: return 2;
        case 4: case 5: case 6: return 4;
        case 10: case 11: case 12: return 8;
        default: return -1;
    }
}
// Skips one value of type t; arrays nest at most 4 deep and fixed-size element runs are
// skipped in one bounds-checked step (a corrupt count cannot loop or recurse for long).
void skip(Rd& r, int t, int depth = 0) {
    if (t == 8) { r.str(); return; }
    if (t == 9) {
        int et = (int)r.u(4);
        uint64_t n = r.u(8);
        if (r.err || depth >= 4) { r.err = true; return; }
        const int es = vsize(et);
        if (es > 0) {
            if (n > r.left() / (uint64_t)es) { r.err = true; return; }
            r.take(n * (uint64_t)es);
            return;
        }
        for (uint64_t i = 0; i < n && !r.err; ++i) skip(r, et, depth + 1);
        return;
    }
    int s = vsize(t);
    if (s < 0) { r.err = true; return; }
    r.take((uint64_t)s);
}
}  // namespace

bool GgufFile::open(const char* path, std::string& err) {
    int fd = ::open(path, O_RDONLY);
    if (fd < 0) { err = std::string("cannot open ") + path; return false; }
    struct stat st;
    fstat(fd, &st);
    size = (size_t)st.st_size;
    void* m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) { err = "mmap failed"; return false; }
    map = (const uint8_t*)m;
    Rd r{map, map + size};
    if (size < 24 || memcmp(map, "GGUF", 4) != 0) { err = "not a GGUF file"; return false; }
    r.p += 4;
    uint32_t ver = (uint32_t)r.u(4);
    if (ver < 2 || ver > 3) { err = "unsupported GGUF version"; return false; }
    uint64_t nt = r.u(8), nkv = r.u(8);
    alignment = 32;
    for (uint64_t i = 0; i < nkv && !r.err; ++i) {
        std::string key = r.str();
        int t = (int)r.u(4);
        const uint8_t* vp = r.p;
        if (t == 8) {
            std::string v = r.str();
            if (key == "general.architecture") arch = v;
            continue;
        }
        skip(r, t);
        if (r.err) break;
        uint64_t u = 0;
        float f = 0;
        if (t == 4 || t == 5) { uint32_t x; memcpy(&x, vp, 4); u = x; }
        if (t == 10 || t == 11) memcpy(&u, vp, 8);
        if (t == 6) memcpy(&f, vp, 4);
        if (key == "general.alignment") alignment = u;
        if (key.rfind("llama.", 0) == 0) {
            std::string k = key.substr(6);
            if (k == "context_length") ctx = (int)u;
            else if (k == "embedding_length") emb = (int)u;
            else if (k == "block_count") layers = (int)u;
            else if (k == "feed_forward_length") ffn = (int)u;
            else if (k == "attention.head_count") heads = (int)u;
            else if (k == "attention.head_count_kv") kv_heads = (int)u;
            else if (k == "vocab_size") vocab = (int)u;
            else if (k == "attention.key_length") head_dim = (int)u;
            else if (k == "rope.dimension_count") rope_dim = (int)u;
            else if (k == "rope.freq_base") rope_base = f;
            else if (k == "attention.layer_norm_rms_epsilon") eps = f;
        }
    }
    for (uint64_t i = 0; i < nt && !r.err; ++i) {
        GgufTensor t;
        t.name = r.str();
        int nd = (int)r.u(4);
        if (nd < 1 || nd > 4) { err = "bad tensor rank"; return false; }
        for (int d = 0; d < nd; ++d) t.dims.push_back(r.u(8));
        t.type = (int)r.u(4);
        t.offset = r.u(8);
        tensors.push_back(t);
    }
    if (r.err) { err = "truncated GGUF header"; return false; }
    if (alignment == 0 || (alignment & (alignment - 1))) { err = "bad alignment"; return false; }
    uint64_t pos = (uint64_t)(r.p - map);
    data_start = (pos + alignment - 1) / alignment * alignment;
    // model.rs:48-185 defaults and checks.
    if (arch != "llama") { err = "unsupported architecture: " + arch; return false; }
    if (heads <= 0 || emb % heads) { err = "bad head count"; return false; }
    if (kv_heads <= 0) kv_heads = heads;
    if (heads % kv_heads) { err = "heads not a multiple of kv heads"; return false; }
    if (head_dim <= 0) head_dim = emb / heads;
    if (rope_dim <= 0) rope_dim = head_dim;
    if (vocab <= 0) {
        const GgufTensor* te = find("token_embd.weight");
        if (!te || te->dims.size() != 2) { err = "cannot infer vocab"; return false; }
        vocab = (int)(te->dims[0] == (uint64_t)emb ? te->dims[1] : te->dims[0]);
    }
    if (data_start > size) { err = "truncated GGUF header"; return false; }
    for (auto& t : tensors) {
        int be = ncm_type_block_elems(t.type), bb = ncm_type_block_bytes(t.type);
        if (bb == 0) continue;
        // overflow-safe: the sized types take at least half a byte per element, so no
        // element count in the file exceeds 64 x its size
        const uint64_t lim = (uint64_t)size * 64;
        uint64_t el = 1;
        for (auto d : t.dims) {
            if (d == 0 || d > lim || el > lim / d) { err = "tensor " + t.name + " has bad dimensions"; return false; }
            el *= d;
        }
        t.nbytes = el / (uint64_t)be * (uint64_t)bb;
        const uint64_t room = size - data_start;
        if (t.offset > room || t.nbytes > room - t.offset) { err = "tensor " + t.name + " overruns file"; return false; }
    }
    return true;
}

GgufFile::~GgufFile() {
    if (map) munmap((void*)map, size);
}

const GgufTensor* GgufFile::find(const std::string& name) const {
    for (auto& t : tensors)
        if (t.name == name) return &t;
    return nullptr;
}

// ------------------------------------------------------------------ synthetic writer
std::vector<SynthTensor> synth_tensor_list(const ncm_synth_spec& s) {
    std::vector<SynthTensor> v;
    const int64_t H = s.emb, QW = (int64_t)s.heads * s.head_dim, KW = (int64_t)s.kv_heads * s.head_dim, F = s.ffn;
    v.push_back({"token_embd.weight", s.t_embd, s.vocab, H, false});
    v.push_back({"output_norm.weight", NCM_T_F32, 1, H, true});
    if (!s.tied) v.push_back({"output.weight", s.t_out, s.vocab, H, false});
    for (int i = 0; i < s.layers; ++i) {
        std::string b = "blk." + std::to_string(i) + ".";
        v.push_back({b + "attn_norm.weight", NCM_T_F32, 1, H, true});
        v.push_back({b + "attn_q.weight", s.t_attn, QW, H, false});
        v.push_back({b + "attn_k.weight", s.t_attn, KW, H, false});
        v.push_back({b + "attn_v.weight", s.t_attn, KW, H, false});
        v.push_back({b + "attn_output.weight", s.t_attn, H, QW, false});
        v.push_back({b + "ffn_norm.weight", NCM_T_F32, 1, H, true});
        v.push_back({b + "ffn_gate.weight", s.t_ffn, F, H, false});
        v.push_back({b + "ffn_up.weight", s.t_ffn, F, H, false});
        v.push_back({b + "ffn_down.weight", s.t_down ? s.t_down : s.t_ffn, H, F, false});
    }
    return v;
}

// Encode rows [r0,r1) x cols [c0,c1) of one synthetic tensor into `out` (row-major,
// packed rows), multithreaded over rows.
void synth_encode(const ncm_synth_spec& s, const SynthTensor& t, int64_t r0, int64_t r1, int64_t c0, int64_t c1,
                  uint8_t* out, int threads) {
    const int be = ncm_type_block_elems(t.type), bb = ncm_type_block_bytes(t.type);
    const int64_t bpr = (c1 - c0) / be, rb = bpr * bb;
    if (t.ones) {
        for (int64_t r = r0; r < r1; ++r)
            for (int64_t c = c0; c < c1; ++c) {
                float one = 1.0f;
                memcpy(out + (r - r0) * rb + (c - c0) * 4, &one, 4);
            }
        return;
    }
    const uint64_t key = ncm_synth_key(s.seed, t.name.c_str());
    int nt = threads > 0 ? threads : 1;
    int64_t rows = r1 - r0;
    if (rows < nt) nt = (int)(rows > 0 ? rows : 1);
    std::vector<std::thread> th;
    for (int k = 0; k < nt; ++k) {
        th.emplace_back([&, k]() {
            int64_t a = r0 + rows * k / nt, e = r0 + rows * (k + 1) / nt;
            for (int64_t r = a; r < e; ++r)
                for (int64_t b = 0; b < bpr; ++b)
                    ncm_synth_block(t.type, key, (uint64_t)r, (uint64_t)(c0 + b * be), (uint64_t)t.cols,
                                    out + (r - r0) * rb + b * bb);
        });
    }
    for (auto& x : th) x.join();
}

}  // namespace ncm

using namespace ncm;

static void put_u32(FILE* f, uint32_t v) { fwrite(&v, 4, 1, f); }
static void put_u64(FILE* f, uint64_t v) { fwrite(&v, 8, 1, f); }
static void put_str(FILE* f, const std::string& s) { put_u64(f, s.size()); fwrite(s.data(), 1, s.size(), f); }
static void kv_u32(FILE* f, const char* k, uint32_t v) { put_str(f, k); put_u32(f, 4); put_u32(f, v); }
static void kv_f32(FILE* f, const char* k, float v) { put_str(f, k); put_u32(f, 6); fwrite(&v, 4, 1, f); }

extern "C" ncm_status ncm_gguf_write_synthetic(const char* path, const ncm_synth_spec* spec, int threads) {
    if (!path || !spec) return NCM_EINVAL;
    const ncm_synth_spec& s = *spec;
    if (s.emb % 32 || s.ffn % 32 || s.heads <= 0 || s.kv_heads <= 0 || s.heads % s.kv_heads) return NCM_EINVAL;
    auto list = synth_tensor_list(s);
    for (auto& t : list)   // every row is whole blocks of its type (256 columns for Q4_K)
        if (t.cols % ncm_type_block_elems(t.type)) return NCM_EINVAL;
    FILE* f = fopen(path, "wb");
    if (!f) return NCM_EIO;
    fwrite("GGUF", 1, 4, f);
    put_u32(f, 3);
    put_u64(f, list.size());
    put_u64(f, 12);
    put_str(f, "general.architecture"); put_u32(f, 8); put_str(f, "llama");
    kv_u32(f, "general.alignment", 32);
    kv_u32(f, "llama.context_length", (uint32_t)s.ctx);
    kv_u32(f, "llama.embedding_length", (uint32_t)s.emb);
    kv_u32(f, "llama.block_count", (uint32_t)s.layers);
    kv_u32(f, "llama.feed_forward_length", (uint32_t)s.ffn);
    kv_u32(f, "llama.attention.head_count", (uint32_t)s.heads);
    kv_u32(f, "llama.attention.head_count_kv", (uint32_t)s.kv_heads);
    kv_u32(f, "llama.attention.key_length", (uint32_t)s.head_dim);
    kv_u32(f, "llama.vocab_size", (uint32_t)s.vocab);
    kv_f32(f, "llama.rope.freq_base", s.rope_base);
    kv_f32(f, "llama.attention.layer_norm_rms_epsilon", s.eps);
    uint64_t off = 0;
    std::vector<uint64_t> offs;
    for (auto& t : list) {
        put_str(f, t.name);
        if (t.rows == 1) { put_u32(f, 1); put_u64(f, (uint64_t)t.cols); }
        else { put_u32(f, 2); put_u64(f, (uint64_t)t.cols); put_u64(f, (uint64_t)t.rows); }
        put_u32(f, (uint32_t)t.type);
        put_u64(f, off);
        offs.push_back(off);
        uint64_t nb = (uint64_t)t.rows * (uint64_t)(t.cols / ncm_type_block_elems(t.type)) * ncm_type_block_bytes(t.type);
        off += (nb + 31) / 32 * 32;
    }
    long pos = ftell(f);
    long pad = (32 - pos % 32) % 32;
    static const uint8_t zeros[64] = {0};
    fwrite(zeros, 1, (size_t)pad, f);
    std::vector<uint8_t> buf;
    for (size_t i = 0; i < list.size(); ++i) {
        auto& t = list[i];
        const int64_t rb = t.cols / ncm_type_block_elems(t.type) * ncm_type_block_bytes(t.type);
        int64_t chunk = (64ll << 20) / (rb > 0 ? rb : 1);
        if (chunk < 1) chunk = 1;
        uint64_t written = 0;
        for (int64_t r = 0; r < t.rows; r += chunk) {
            int64_t e = r + chunk < t.rows ? r + chunk : t.rows;
            buf.resize((size_t)((e - r) * rb));
            synth_encode(s, t, r, e, 0, t.cols, buf.data(), threads);
            fwrite(buf.data(), 1, buf.size(), f);
            written += buf.size();
        }
        uint64_t padn = (32 - written % 32) % 32;
        fwrite(zeros, 1, (size_t)padn, f);
    }
    bool ok = ferror(f) == 0;
    fclose(f);
    return ok ? NCM_OK : NCM_EIO;
}

extern "C" ncm_status ncm_synth_tensor_host(const ncm_synth_spec* spec, const char* name, int type, int64_t r0,
                                           int64_t r1, int64_t c0, int64_t c1, int64_t cols, uint8_t* out) {
    if (!spec || !name || !out || r1 < r0 || c1 < c0) return NCM_EINVAL;
    SynthTensor t{name, type, r1, cols, false};
    synth_encode(*spec, t, r0, r1, c0, c1, out, 8);
    return NCM_OK;
}
