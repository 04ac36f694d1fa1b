// Host engine behind the C ABI (include/ncm.h): model load (GGUF or on-device synthetic),
// the per-token decode step captured as CUDA graphs, tensor-parallel plumbing (CUDA IPC
// peer buffers for the fused NVLink reduction, NCCL for the baseline reducer).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <math.h>
#include <string.h>
#include <stdlib.h>
#include <algorithm>
#include <initializer_list>
#include <mutex>
#include <thread>
#include <string>
#include <vector>
#include "../../include/ncm.h"
#include "gguf.h"
#include "common.cuh"
#include "ncm_internal.h"
#include "synth.h"

using namespace ncm;

static thread_local std::string g_err;
static ncm_status fail(ncm_status code, const std::string& msg) {
    g_err = msg;
    return code;
}
#define CK(x)                                                                                   \
    do {                                                                                        \
        cudaError_t e_ = (x);                                                                   \
        if (e_ != cudaSuccess) return fail(NCM_ECUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
    } while (0)
#define CKL(x)                                                                                          \
    do {                                                                                                \
        int e_ = (x);                                                                                   \
        if (e_ != 0) return fail(NCM_ECUDA, std::string(#x) + ": " + cudaGetErrorString((cudaError_t)e_)); \
    } while (0)

extern "C" const char* ncm_last_error(void) { return g_err.c_str(); }
extern "C" int ncm_version(void) { return 1; }

// ------------------------------------------------------------------ NCCL (dlopen'd, baseline only)
namespace {
typedef struct { char internal[128]; } nccl_uid;
typedef void* nccl_comm;
struct Nccl {
    void* h = nullptr;
    int (*GetUniqueId)(nccl_uid*) = nullptr;
    int (*CommInitRank)(nccl_comm*, int, nccl_uid, int) = nullptr;
    int (*AllReduce)(const void*, void*, size_t, int, int, nccl_comm, cudaStream_t) = nullptr;
    int (*AllGather)(const void*, void*, size_t, int, nccl_comm, cudaStream_t) = nullptr;
    int (*CommDestroy)(nccl_comm) = nullptr;
    bool load() {
        static std::mutex mu;
        std::lock_guard<std::mutex> lock(mu);
        if (h) return true;
        const char* names[] = {"libnccl.so.2", "libnccl.so"};
        for (auto n : names) {
            h = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
            if (h) break;
        }
        if (!h) return false;
        GetUniqueId = (int (*)(nccl_uid*))dlsym(h, "ncclGetUniqueId");
        CommInitRank = (int (*)(nccl_comm*, int, nccl_uid, int))dlsym(h, "ncclCommInitRank");
        AllReduce = (int (*)(const void*, void*, size_t, int, int, nccl_comm, cudaStream_t))dlsym(h, "ncclAllReduce");
        AllGather = (int (*)(const void*, void*, size_t, int, nccl_comm, cudaStream_t))dlsym(h, "ncclAllGather");
        CommDestroy = (int (*)(nccl_comm))dlsym(h, "ncclCommDestroy");
        return GetUniqueId && CommInitRank && AllReduce && AllGather;
    }
};
Nccl g_nccl;
constexpr int kNcclFloat = 7;   // ncclFloat32
constexpr int kNcclSum = 0;     // ncclSum
}  // namespace

// ------------------------------------------------------------------ model
struct DevMat {
    int type = 0, rows = 0, cols = 0, pitch = 0;
    uint8_t* d = nullptr;
};
struct Layer {
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    DevMat wq, wk, wv, wo, w1, w3, w2;
};

struct ncm_model {
    int device = 0;
    cudaStream_t stream = nullptr;
    int emb = 0, layers = 0, heads = 0, kv_heads = 0, hd = 0, ffn = 0, vocab = 0, ctx = 0, rope_dim = 0;
    float eps = 1e-5f, base = 10000.0f;
    int nshards = 1, shard = 0;
    int q0 = 0, qh = 0, k0 = 0, kh = 0, f0 = 0, fl = 0, h0 = 0, hr = 0;
    DevMat embd, head;
    float* out_norm = nullptr;
    std::vector<Layer> L;
    float *hidden = nullptr, *q = nullptr, *att = nullptr, *act = nullptr, *logits = nullptr, *kc = nullptr,
          *vc = nullptr, *scores = nullptr, *part = nullptr;
    unsigned* amax_cnt = nullptr;
    float2 *amax_part = nullptr, *rope = nullptr, *head_out = nullptr, *gather = nullptr;
    float* embd_ssq = nullptr;   // per vocab row: sequential f32 sum of squares of the embedding
    // the attention output and silu(gate)*up as Q8_0 blocks, written by their producing
    // kernels, read by the row-parallel projections (wo, w2) of the decode step
    int8_t *att_q = nullptr, *act_q = nullptr;
    float *att_s = nullptr, *act_s = nullptr;
    bool act_quantised = false;   // the gate/up plan allows the quantised hand-off (32-row tiles)
    bool has_q6k = false;         // a Q6_K head or down projection (one GPU, token-by-token prefill)
    int kv_kind = KV_F32;         // KV-cache storage (F32, or the reference's opt-in F16 / Q8_0)
    float *kv_sk = nullptr, *kv_sv = nullptr;   // F16 / Q8_0: staged f32 K / V rows [kMaxBatch][kw]
    int8_t* hx_q = nullptr;       // the normed hidden as Q8_0 for a Q6_K head
    float* hx_s = nullptr;
    int64_t prefetch_bytes = 0;   // per CTA: next kernel's weights streamed into L2 (0: off)
    int cgroups = 4;              // GEMV compute-warp groups (stages worked on at once)
    int av_tma = 1;               // attention V chunks by TMA (f32 cache)
    int attn_sv = -1;             // attention softmax and V accumulation in one launch (-1: by group size)
    int bcgroups = 0;             // multi-row GEMV compute-warp groups (0: the plan's default)
    int tune = 0;                 // measurement knobs
    uint64_t* dbg_ts = nullptr;   // measurement probe buffer [num_sms][8], filled by step-kernel seam launches
    bool dbg_on = false;
    int *state = nullptr, *tokens = nullptr, *err = nullptr;
    int* h_stage = nullptr;   // pinned staging for small transfers
    cudaStream_t ext_stream = nullptr;   // caller stream of the last prefill / decode, until synced
    std::vector<void*> allocs;
    cudaGraphExec_t g_full = nullptr, g_nohead = nullptr;
    bool dirty = true;
    // multi-row verify buffers (allocated on first use): [kMaxBatch][...]
    float *b_hidden = nullptr, *b_q = nullptr, *b_att = nullptr, *b_act = nullptr;
    int8_t* b_xq = nullptr;
    float* b_xs = nullptr;
    int* b_xsum = nullptr;
    float2* b_amax = nullptr;
    unsigned* b_cnt = nullptr;
    int *b_tok = nullptr, *b_arg = nullptr, *b_pos = nullptr;
    float* b_scores = nullptr;
    float* b_part = nullptr;      // tensor parallel: [kMaxBatch][emb] partial rows
    float2* b_pairs = nullptr;    // tensor parallel: [kMaxBatch] head pairs of this shard
    cudaGraphExec_t b_graph[2][kMaxBatch + 1] = {};   // [with head][rows]
    // tensor parallel
    int world = 1, rank = 0, reduce_mode = NCM_REDUCE_FUSED_P2P;
    bool tp_ready = false;
    TpComm comm{};
    uint8_t* comm_base = nullptr;
    size_t comm_bytes = 0, off_flags = 0, off_hx = 0, off_hflags = 0;
    size_t off_rrecv = 0, off_rflags = 0, off_rhx = 0, off_rhflags = 0;
    TpRows rows{};                // multi-row reductions over the peers' areas
    unsigned* rows_ctr = nullptr; // their epochs (this rank's own memory)
    float2* rows_gather = nullptr;   // NCCL variant: [W][kMaxBatch] gathered head pairs
    std::vector<void*> ipc_open;
    nccl_comm nccl = nullptr;
    uint64_t timeout_ns = 10000000000ull;
    ncm_host_reduce_fn host_fn = nullptr;   // NCM_REDUCE_HOST_CALLBACK
    void* host_user = nullptr;
    float* h_red = nullptr;                 // pinned: the partial row / head pair handed to host_fn
};

static ncm_status dalloc(ncm_model* m, void** p, size_t bytes) {
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) return fail(NCM_ECUDA, std::string("cudaMalloc ") + std::to_string(bytes) + ": " + cudaGetErrorString(e));
    m->allocs.push_back(*p);
    return NCM_OK;
}
#define DALLOC(ptr, bytes)                                                   \
    do {                                                                     \
        ncm_status s_ = dalloc(m, (void**)&(ptr), (size_t)(bytes));          \
        if (s_ != NCM_OK) return s_;                                         \
    } while (0)

static bool gemv_type_ok(int t) { return t == NCM_T_Q4_0 || t == NCM_T_Q8_0 || t == NCM_T_Q4_K; }
static int row_bytes(int t, int cols) { return cols / ncm_type_block_elems(t) * ncm_type_block_bytes(t); }

static void free_model(ncm_model* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->g_full) cudaGraphExecDestroy(m->g_full);
    if (m->g_nohead) cudaGraphExecDestroy(m->g_nohead);
    for (auto& row : m->b_graph)
        for (auto& gx : row)
            if (gx) cudaGraphExecDestroy(gx);
    for (void* p : m->ipc_open) cudaIpcCloseMemHandle(p);
    if (m->nccl && g_nccl.CommDestroy) g_nccl.CommDestroy(m->nccl);
    for (void* p : m->allocs) cudaFree(p);
    if (m->h_stage) cudaFreeHost(m->h_stage);
    if (m->h_red) cudaFreeHost(m->h_red);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

// Shard geometry: tp.rs:641-701 validate_shares + shard_geometry.
extern "C" ncm_status ncm_shard_geometry(int heads, int kv_heads, int ffn, int vocab, const int* shares,
                                        int nshards, int shard, int* out) {
    if (!shares || !out || nshards <= 0 || kv_heads <= 0) return fail(NCM_EINVAL, "bad shard arguments");
    long sum = 0;
    for (int i = 0; i < nshards; ++i) {
        if (shares[i] <= 0) return fail(NCM_EINVAL, "every shard needs at least one kv head");
        sum += shares[i];
    }
    if (sum != kv_heads) return fail(NCM_EINVAL, "shares must sum to the kv head count");
    for (int i = 0; i < nshards; ++i)
        if (((long)ffn * shares[i]) % ((long)kv_heads * 32)) return fail(NCM_EINVAL, "ffn not 32-block divisible for a share");
    if (shard < 0 || shard >= nshards) return fail(NCM_EINVAL, "bad shard index");
    const int qpk = heads / kv_heads, unit = ffn / kv_heads;
    int kv_start = 0;
    for (int i = 0; i < shard; ++i) kv_start += shares[i];
    long acc = 0, hs = 0, he = 0;
    for (int i = 0; i < nshards; ++i) {
        if (i == shard) hs = acc;
        acc += ((long)vocab * shares[i] / kv_heads) & ~3L;
        if (i == shard) he = acc;
    }
    out[0] = kv_start * qpk;
    out[1] = shares[shard] * qpk;
    out[2] = kv_start;
    out[3] = shares[shard];
    out[4] = kv_start * unit;
    out[5] = shares[shard] * unit;
    out[6] = (int)hs;
    out[7] = shard + 1 == nshards ? (int)(vocab - hs) : (int)(he - hs);
    return NCM_OK;
}

// Common set-up once the global config is known: shard geometry, activation buffers,
// KV cache, rope table, state.
// The exp exception table (libm_table.cpp) is built once per process and copied once
// per device into the library's fixed device array (no device allocation); every kernel
// that evaluates exp on that device then matches glibc's expf.
static ncm_status ensure_expf_table(int device) {
    static std::mutex mu;
    static std::vector<uint32_t> host_tab;
    static uint32_t mask = 0;
    static int gate = 1;
    static std::vector<int> done;
    std::lock_guard<std::mutex> lk(mu);
    for (int d : done)
        if (d == device) return NCM_OK;
    if (host_tab.empty()) {
        size_t count = 0;
        unsigned hc = std::thread::hardware_concurrency();
        host_tab = build_expf_exceptions(hc ? (int)hc : 8, kExpfTabEntries, &mask, &count, &gate);
        if (host_tab.empty())
            return fail(NCM_EUNSUPPORTED, "this libm's expf has " + std::to_string(count) +
                                              " exceptions, more than the device table holds");
    }
    CKL(expf_table_install(host_tab.data(), host_tab.size() / 2, mask, gate));
    done.push_back(device);
    return NCM_OK;
}

// Bytes of one position's K (or V) row in the cache's storage, and a layer's cache base.
static size_t kv_row_bytes(const ncm_model* m) {
    const size_t kw = (size_t)m->kh * m->hd;
    return m->kv_kind == KV_F16 ? 2 * kw : m->kv_kind == KV_Q8_0 ? kw / 32 * 34 : 4 * kw;
}
static uint8_t* kv_layer(const ncm_model* m, float* cache, int l) {
    return reinterpret_cast<uint8_t*>(cache) + (size_t)l * m->ctx * kv_row_bytes(m);
}

static ncm_status setup_buffers(ncm_model* m, const int* shares, int nshards, int shard) {
    {
        ncm_status s = ensure_expf_table(m->device);
        if (s) return s;
    }
    if (m->heads % m->kv_heads) return fail(NCM_EINVAL, "heads must be a multiple of kv heads");
    if (m->emb % 32) return fail(NCM_EUNSUPPORTED, "embedding length must be a multiple of 32");
    if (m->hd % 32 || m->hd > 256 || m->heads / m->kv_heads > 8)
        return fail(NCM_EUNSUPPORTED, "head_dim must be a multiple of 32 (<= 256), group size <= 8");
    if (nshards > 1) {
        if (nshards > kMaxWorld) return fail(NCM_EINVAL, "at most 8 shards");
        int g[8];
        ncm_status s = ncm_shard_geometry(m->heads, m->kv_heads, m->ffn, m->vocab, shares, nshards, shard, g);
        if (s) return s;
        m->q0 = g[0]; m->qh = g[1]; m->k0 = g[2]; m->kh = g[3]; m->f0 = g[4]; m->fl = g[5]; m->h0 = g[6]; m->hr = g[7];
    } else {
        m->q0 = 0; m->qh = m->heads; m->k0 = 0; m->kh = m->kv_heads; m->f0 = 0; m->fl = m->ffn; m->h0 = 0; m->hr = m->vocab;
    }
    m->nshards = nshards > 1 ? nshards : 1;
    m->shard = nshards > 1 ? shard : 0;
    m->world = m->nshards;
    m->rank = m->shard;
    if (m->fl % 32) return fail(NCM_EUNSUPPORTED, "FFN shard width must be a multiple of 32");
    const int qw = m->qh * m->hd, kw = m->kh * m->hd;
    DALLOC(m->hidden, 4 * m->emb);
    DALLOC(m->q, 4 * qw);
    DALLOC(m->att, 4 * qw);
    DALLOC(m->act, 4 * m->fl);
    DALLOC(m->logits, 4 * (size_t)m->hr);
    DALLOC(m->part, 4 * m->emb);
    DALLOC(m->att_q, qw);
    DALLOC(m->att_s, 4 * (qw / 32));
    DALLOC(m->act_q, m->fl);
    DALLOC(m->act_s, 4 * (m->fl / 32));
    DALLOC(m->dbg_ts, 8 * 16 * (size_t)num_sms());
    DALLOC(m->hx_q, m->emb);
    DALLOC(m->hx_s, 4 * (m->emb / 32));
    DALLOC(m->kc, 4 * (size_t)m->layers * m->ctx * kw);
    DALLOC(m->vc, 4 * (size_t)m->layers * m->ctx * kw);
    DALLOC(m->kv_sk, 4 * (size_t)kMaxBatch * kw);
    DALLOC(m->kv_sv, 4 * (size_t)kMaxBatch * kw);
    DALLOC(m->scores, 4 * (size_t)m->qh * m->ctx);
    DALLOC(m->amax_part, 8 * (size_t)std::max(num_sms(), (m->hr + 31) / 32));   // one per CTA of any head GEMV
    DALLOC(m->amax_cnt, 4);
    DALLOC(m->head_out, 8);
    DALLOC(m->gather, 8 * kMaxWorld);
    DALLOC(m->state, 4 * ST_COUNT);
    DALLOC(m->tokens, 4 * (size_t)m->ctx);
    DALLOC(m->err, 4);
    CK(cudaMemset(m->amax_cnt, 0, 4));
    CK(cudaMemset(m->state, 0, 4 * ST_COUNT));
    CK(cudaMemset(m->tokens, 0, 4 * (size_t)m->ctx));
    CK(cudaMemset(m->err, 0, 4));
    CK(cudaMemset(m->hidden, 0, 4 * m->emb));
    CK(cudaMemset(m->kc, 0, 4 * (size_t)m->layers * m->ctx * kw));
    CK(cudaMemset(m->vc, 0, 4 * (size_t)m->layers * m->ctx * kw));
    CK(cudaMallocHost((void**)&m->h_stage, 4096));
    // inference.rs:860-900 cached_rope_angles with the host libm (the reference calls the
    // same glibc powf / sinf / cosf): table[pos][i] = (sin, cos).
    const int half = m->rope_dim / 2;
    std::vector<float2> rt((size_t)m->ctx * half);
    for (int pos = 0; pos < m->ctx; ++pos)
        for (int i = 0; i < half; ++i) {
            float theta = powf(m->base, -((float)(i * 2)) / (float)m->rope_dim);
            float angle = (float)pos * theta;
            rt[(size_t)pos * half + i] = make_float2(sinf(angle), cosf(angle));
        }
    DALLOC(m->rope, sizeof(float2) * rt.size());
    CK(cudaMemcpy(m->rope, rt.data(), sizeof(float2) * rt.size(), cudaMemcpyHostToDevice));
    if (m->world > 1) {
        // Exchange area, identical layout on every rank:
        // recv[2L][W][H] f32 | flags[2L][grid_max][W] u32 | hx[W] float2 | hflags[W] u32.
        const size_t W = (size_t)m->world, gm = (size_t)num_sms();
        size_t off = 4 * 2 * (size_t)m->layers * W * m->emb;
        off = (off + 255) / 256 * 256;
        m->off_flags = off;
        off += 4 * 2 * (size_t)m->layers * gm * W;
        off = (off + 255) / 256 * 256;
        m->off_hx = off;
        off += 8 * W;
        off = (off + 255) / 256 * 256;
        m->off_hflags = off;
        off += 4 * W;
        // multi-row passes: rrecv[2][W][kMaxBatch * H] f32 | rflags[grid_max][W] u32 |
        // hrecv[2][W][kMaxBatch] float2 | rhflags[W] u32
        off = (off + 255) / 256 * 256;
        m->off_rrecv = off;
        off += 4 * 2 * W * (size_t)kMaxBatch * m->emb;
        off = (off + 255) / 256 * 256;
        m->off_rflags = off;
        off += 4 * gm * W;
        off = (off + 255) / 256 * 256;
        m->off_rhx = off;
        off += 8 * 2 * W * (size_t)kMaxBatch;
        off = (off + 255) / 256 * 256;
        m->off_rhflags = off;
        off += 4 * W;
        m->comm_bytes = (off + 4095) / 4096 * 4096;
        DALLOC(m->comm_base, m->comm_bytes);
        CK(cudaMemset(m->comm_base, 0, m->comm_bytes));
        DALLOC(m->rows_ctr, 16);
        CK(cudaMemset(m->rows_ctr, 0, 16));
        DALLOC(m->rows_gather, sizeof(float2) * W * kMaxBatch);
    }
    return NCM_OK;
}

static ncm_status check_matrix_shape(const DevMat& d, const char* what) {
    if (!gemv_type_ok(d.type)) return fail(NCM_EUNSUPPORTED, std::string(what) + ": tensor type outside Q4_0/Q8_0/Q4_K");
    if (d.cols % 32 || d.cols % ncm_type_block_elems(d.type)) return fail(NCM_EUNSUPPORTED, std::string(what) + ": columns not block aligned");
    if (d.cols > 32768) return fail(NCM_EUNSUPPORTED, std::string(what) + ": more than 32768 columns");
    return NCM_OK;
}

// Shard upload through pinned staging: the mapped file's row slices are packed into one
// of two pinned buffers while the other one's asynchronous copy to HBM runs, so host
// reads and PCIe transfers overlap and only this rank's slice is ever touched.
struct PinnedStager {
    static constexpr size_t kBytes = 64u << 20;
    uint8_t* buf[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int next = 0;
    cudaStream_t s = nullptr;
    bool init(cudaStream_t st) {
        s = st;
        for (int i = 0; i < 2; ++i) {
            if (cudaMallocHost((void**)&buf[i], kBytes) != cudaSuccess) return false;
            if (cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming) != cudaSuccess) return false;
        }
        return true;
    }
    ~PinnedStager() {
        if (s) cudaStreamSynchronize(s);
        for (int i = 0; i < 2; ++i) {
            if (buf[i]) cudaFreeHost(buf[i]);
            if (done[i]) cudaEventDestroy(done[i]);
        }
    }
    // rows of rb bytes from src (stride src_pitch) to dst (stride dst_pitch)
    cudaError_t copy(uint8_t* dst, size_t dst_pitch, const uint8_t* src, size_t src_pitch, size_t rb, size_t rows) {
        const size_t per = std::max<size_t>(1, kBytes / std::max<size_t>(rb, 1));
        for (size_t r0 = 0; r0 < rows; r0 += per) {
            const size_t nr = std::min(per, rows - r0);
            const int i = next;
            next ^= 1;
            cudaError_t e = cudaEventSynchronize(done[i]);   // the buffer's previous copy
            if (e != cudaSuccess) return e;
            uint8_t* b = buf[i];
            if (rb > kBytes) {   // a single row larger than the buffer: plain copy
                e = cudaMemcpy2D(dst + r0 * dst_pitch, dst_pitch, src + r0 * src_pitch, src_pitch, rb, nr,
                                 cudaMemcpyHostToDevice);
                if (e != cudaSuccess) return e;
                continue;
            }
            for (size_t r = 0; r < nr; ++r) memcpy(b + r * rb, src + (r0 + r) * src_pitch, rb);
            e = cudaMemcpy2DAsync(dst + r0 * dst_pitch, dst_pitch, b, rb, rb, nr, cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) return e;
            e = cudaEventRecord(done[i], s);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
};

// Upload rows [r0,r0+nrows) x cols [c0,c0+ncols) of a GGUF tensor (raw blocks unchanged;
// row pitch rounded up to 16 bytes so every row tile is a legal bulk copy).
static ncm_status upload_slice(ncm_model* m, const GgufFile& g, const char* name, int expect_rows, int expect_cols,
                               int r0, int nrows, int c0, int ncols, DevMat& out, PinnedStager* stg = nullptr,
                               uint8_t* dst = nullptr) {
    const GgufTensor* t = g.find(name);
    if (!t) return fail(NCM_EIO, std::string("missing tensor ") + name);
    if (t->dims.size() != 2 || (int)t->dims[0] != expect_cols || (int)t->dims[1] != expect_rows)
        return fail(NCM_EIO, std::string("unexpected shape for ") + name);
    out.type = t->type;
    out.rows = nrows;
    out.cols = ncols;
    const int full_rb = row_bytes(t->type, expect_cols), rb = row_bytes(t->type, ncols);
    out.pitch = (rb + 15) / 16 * 16;
    const int be = ncm_type_block_elems(t->type);
    if (c0 % be || ncols % be) return fail(NCM_EINVAL, std::string("column slice not block aligned: ") + name);
    if (dst) out.d = dst;
    else DALLOC(out.d, (size_t)out.pitch * nrows);
    const uint8_t* src = g.data(*t) + (size_t)r0 * full_rb + (size_t)(c0 / be) * ncm_type_block_bytes(t->type);
    if (stg) CK(stg->copy(out.d, out.pitch, src, full_rb, rb, nrows));
    else CK(cudaMemcpy2D(out.d, out.pitch, src, full_rb, rb, nrows, cudaMemcpyHostToDevice));
    return NCM_OK;
}

// A norm vector: one dimension of exactly n elements, F32 or F16 (the reader has checked
// that the tensor's bytes lie inside the file).
static ncm_status check_norm(const GgufFile& g, const char* name, int n) {
    const GgufTensor* t = g.find(name);
    if (!t) return fail(NCM_EIO, std::string("missing tensor ") + name);
    if (t->type != NCM_T_F32 && t->type != NCM_T_F16)
        return fail(NCM_EUNSUPPORTED, std::string("norm tensor must be F32/F16: ") + name);
    if (t->dims.size() != 1 || t->dims[0] != (uint64_t)n || t->nbytes < (uint64_t)n * (t->type == NCM_T_F32 ? 4 : 2))
        return fail(NCM_EIO, std::string("norm tensor is not ") + std::to_string(n) + " elements long: " + name);
    return NCM_OK;
}

// Host-side check of every tensor the loader reads (names, ranks, shapes), before any
// device work, so that a malformed file fails with NCM_EIO instead of being read past.
static ncm_status check_llama_tensors(const GgufFile& g) {
    const uint64_t H = (uint64_t)g.emb, QW = (uint64_t)g.heads * g.head_dim, KW = (uint64_t)g.kv_heads * g.head_dim,
                   F = (uint64_t)g.ffn, V = (uint64_t)g.vocab;
    auto mat = [&](const std::string& name, uint64_t rows, uint64_t cols, bool required) -> ncm_status {
        const GgufTensor* t = g.find(name);
        if (!t) return required ? fail(NCM_EIO, "missing tensor " + name) : NCM_OK;
        if (t->dims.size() != 2 || t->dims[0] != cols || t->dims[1] != rows)
            return fail(NCM_EIO, "unexpected shape for " + name);
        return NCM_OK;
    };
    ncm_status s;
    if ((s = mat("token_embd.weight", V, H, true))) return s;
    if ((s = mat("output.weight", V, H, false))) return s;
    if ((s = check_norm(g, "output_norm.weight", g.emb))) return s;
    for (int i = 0; i < g.layers; ++i) {
        const std::string b = "blk." + std::to_string(i) + ".";
        if ((s = check_norm(g, (b + "attn_norm.weight").c_str(), g.emb))) return s;
        if ((s = check_norm(g, (b + "ffn_norm.weight").c_str(), g.emb))) return s;
        if ((s = mat(b + "attn_q.weight", QW, H, true)) || (s = mat(b + "attn_k.weight", KW, H, true)) ||
            (s = mat(b + "attn_v.weight", KW, H, true)) || (s = mat(b + "attn_output.weight", H, QW, true)) ||
            (s = mat(b + "ffn_gate.weight", F, H, true)) || (s = mat(b + "ffn_up.weight", F, H, true)) ||
            (s = mat(b + "ffn_down.weight", H, F, true)))
            return s;
    }
    return NCM_OK;
}

static ncm_status upload_f32(ncm_model* m, const GgufFile& g, const char* name, int n, float** out) {
    if (ncm_status s = check_norm(g, name, n)) return s;
    const GgufTensor* t = g.find(name);
    std::vector<float> v(n);
    const uint8_t* d = g.data(*t);
    if (t->type == NCM_T_F32) memcpy(v.data(), d, 4 * (size_t)n);
    else if (t->type == NCM_T_F16) for (int i = 0; i < n; ++i) v[i] = ncm_f16_to_f32((uint16_t)(d[2 * i] | (d[2 * i + 1] << 8)));
    else return fail(NCM_EUNSUPPORTED, std::string("norm tensor must be F32/F16: ") + name);
    DALLOC(*out, 4 * (size_t)n);
    CK(cudaMemcpy(*out, v.data(), 4 * (size_t)n, cudaMemcpyHostToDevice));
    return NCM_OK;
}

// Tied head: Q4_0 requant of token_embd rows [h0, h0+hr) (model.rs:471-508).
static ncm_status build_tied_head(ncm_model* m) {
    m->head.type = NCM_T_Q4_0;
    m->head.rows = m->hr;
    m->head.cols = m->emb;
    m->head.pitch = (row_bytes(NCM_T_Q4_0, m->emb) + 15) / 16 * 16;
    DALLOC(m->head.d, (size_t)m->head.pitch * m->hr);
    CKL(requant_q4_0_launch(m->embd.type, m->embd.d + (size_t)m->h0 * m->embd.pitch, m->hr, m->emb, m->embd.pitch,
                            m->head.d, m->head.pitch, m->stream));
    CK(cudaStreamSynchronize(m->stream));
    return NCM_OK;
}

static GemvParams base_params(ncm_model* m);

// Q6_K (the output.weight / ffn_down type of Q4_K_M files) runs on the row-per-thread
// GEMV, on one GPU, for the head and the down projections only.
static ncm_status check_q6k(ncm_model* m, const DevMat& d, const char* what) {
    if (d.cols % 256 || d.cols > 32768) return fail(NCM_EUNSUPPORTED, std::string(what) + ": Q6_K columns not 256-aligned");
    if (m->world > 1) return fail(NCM_EUNSUPPORTED, std::string(what) + ": Q6_K tensors run on one GPU");
    m->has_q6k = true;
    return NCM_OK;
}

static ncm_status check_all_shapes(ncm_model* m) {
    ncm_status s;
    DALLOC(m->embd_ssq, 4 * (size_t)m->vocab);
    CKL(embed_ssq_launch(m->embd.type, m->embd.d, m->embd.pitch, m->emb, m->vocab, m->embd_ssq, m->stream));
    CK(cudaStreamSynchronize(m->stream));
    if (m->head.type == NCM_T_Q6_K) { if ((s = check_q6k(m, m->head, "output"))) return s; }
    else if ((s = check_matrix_shape(m->head, "output"))) return s;
    for (auto& l : m->L) {
        const DevMat* ms[] = {&l.wq, &l.wk, &l.wv, &l.wo, &l.w1, &l.w3};
        for (auto d : ms)
            if ((s = check_matrix_shape(*d, "layer"))) return s;
        if (l.w2.type == NCM_T_Q6_K) { if ((s = check_q6k(m, l.w2, "ffn_down"))) return s; }
        else if ((s = check_matrix_shape(l.w2, "layer"))) return s;
        if (l.wq.type != l.wk.type || l.wq.type != l.wv.type || l.w1.type != l.w3.type)
            return fail(NCM_EUNSUPPORTED, "q/k/v (and gate/up) must share one quant type");
    }
    int t = m->embd.type;
    if (!(t == NCM_T_Q4_0 || t == NCM_T_Q8_0 || t == NCM_T_Q4_K || t == NCM_T_F32 || t == NCM_T_F16))
        return fail(NCM_EUNSUPPORTED, "token_embd type");
    // gate/up can hand w2 its input as Q8_0 blocks when every tile is one 32-row block
    GemvParams w = base_params(m);
    w.row_align = 32;
    const int g = m->fl % 32 == 0 ? gemv_plan(m->L[0].w1.type, m->emb, m->fl, true, IN_F32_RMS, w) : -1;
    m->act_quantised = g > 0 && w.box_rows == 32;
    // tuning knobs for measurement runs (unset in normal use)
    if (const char* e = getenv("NCM_TUNE_ACTQ")) m->act_quantised = m->act_quantised && atoi(e) != 0;
    if (const char* e = getenv("NCM_TUNE_PREFETCH_KB")) m->prefetch_bytes = (int64_t)atoi(e) * 1024;
    if (const char* e = getenv("NCM_TUNE_CGROUPS")) m->cgroups = atoi(e);
    if (const char* e = getenv("NCM_TUNE_AV_TMA")) m->av_tma = atoi(e);
    if (const char* e = getenv("NCM_TUNE_ATTN_SV")) m->attn_sv = atoi(e);
    // Measured (graph replay, 70 and 1030 positions): one launch for softmax and V is
    // 1-5 % faster per token on the 1B/3B/8B shapes (groups of 3 or 4 query heads); with
    // the 70B shape's 8-head groups the separate softmax launch is 0.6 % faster at 1k.
    if (m->attn_sv < 0) m->attn_sv = m->qh / m->kh < 8 ? 1 : 0;
    if (const char* e = getenv("NCM_TUNE_BCGROUPS")) m->bcgroups = atoi(e);
    if (const char* e = getenv("NCM_TUNE_BITS")) m->tune = atoi(e);
    return NCM_OK;
}

static ncm_status new_model(int device, ncm_model** out) {
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return fail(NCM_ECUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    ncm_model* m = new ncm_model();
    m->device = device;
    e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) { delete m; return fail(NCM_ECUDA, std::string("stream: ") + cudaGetErrorString(e)); }
    *out = m;
    return NCM_OK;
}

extern "C" ncm_status ncm_model_load(const char* path, int ctx_limit, int device, const int* shares, int nshards,
                                    int shard, ncm_model** out) {
    if (!path || !out) return fail(NCM_EINVAL, "null argument");
    GgufFile g;
    std::string err;
    if (!g.open(path, err)) return fail(NCM_EIO, err);
    if (g.emb <= 0 || g.layers <= 0 || g.heads <= 0 || g.kv_heads <= 0 || g.head_dim <= 0 || g.vocab <= 0)
        return fail(NCM_EIO, "incomplete llama metadata");
    if (ncm_status cs = check_llama_tensors(g)) return cs;
    ncm_model* m = nullptr;
    ncm_status s = new_model(device, &m);
    if (s) return s;
    m->emb = g.emb; m->layers = g.layers; m->heads = g.heads; m->kv_heads = g.kv_heads; m->hd = g.head_dim;
    m->ffn = g.ffn; m->vocab = g.vocab; m->rope_dim = g.rope_dim; m->eps = g.eps; m->base = g.rope_base;
    m->ctx = (ctx_limit > 0 && ctx_limit < g.ctx) ? ctx_limit : g.ctx;
    if (m->emb <= 0 || m->layers <= 0 || m->ctx <= 0) { free_model(m); return fail(NCM_EIO, "incomplete llama metadata"); }
    if ((s = setup_buffers(m, shares, nshards, shard))) { free_model(m); return s; }
    PinnedStager stg;
    if (!stg.init(m->stream)) { free_model(m); return fail(NCM_ECUDA, "pinned staging buffers"); }
    const int H = m->emb, QW = m->heads * m->hd, KW = m->kv_heads * m->hd, F = m->ffn;
    const int hd = m->hd;
#define TRY(x) do { if ((s = (x))) { free_model(m); return s; } } while (0)
    TRY(upload_slice(m, g, "token_embd.weight", m->vocab, H, 0, m->vocab, 0, H, m->embd, &stg));
    TRY(upload_f32(m, g, "output_norm.weight", H, &m->out_norm));
    if (g.find("output.weight")) TRY(upload_slice(m, g, "output.weight", m->vocab, H, m->h0, m->hr, 0, H, m->head, &stg));
    else TRY(build_tied_head(m));
    m->L.resize(m->layers);
    char nm[128];
    for (int i = 0; i < m->layers; ++i) {
        Layer& l = m->L[i];
#define NM(s_) (snprintf(nm, sizeof nm, "blk.%d." s_ ".weight", i), nm)
        TRY(upload_f32(m, g, NM("attn_norm"), H, &l.attn_norm));
        TRY(upload_f32(m, g, NM("ffn_norm"), H, &l.ffn_norm));
        // q, k and v rows back to back in one buffer when they share a type (one tensor map)
        uint8_t* qkv = nullptr;
        const GgufTensor *tq = g.find(NM("attn_q")), *tk = g.find(NM("attn_k")), *tv = g.find(NM("attn_v"));
        if (tq && tk && tv && tq->type == tk->type && tq->type == tv->type && ncm_type_block_bytes(tq->type) > 0) {
            const size_t pitch = (row_bytes(tq->type, H) + 15) / 16 * 16;
            TRY(dalloc(m, (void**)&qkv, pitch * (size_t)(m->qh + 2 * m->kh) * hd));
            TRY(upload_slice(m, g, NM("attn_q"), QW, H, m->q0 * hd, m->qh * hd, 0, H, l.wq, &stg, qkv));
            TRY(upload_slice(m, g, NM("attn_k"), KW, H, m->k0 * hd, m->kh * hd, 0, H, l.wk, &stg,
                             qkv + pitch * m->qh * hd));
            TRY(upload_slice(m, g, NM("attn_v"), KW, H, m->k0 * hd, m->kh * hd, 0, H, l.wv, &stg,
                             qkv + pitch * (m->qh + m->kh) * hd));
        } else {
            TRY(upload_slice(m, g, NM("attn_q"), QW, H, m->q0 * hd, m->qh * hd, 0, H, l.wq, &stg));
            TRY(upload_slice(m, g, NM("attn_k"), KW, H, m->k0 * hd, m->kh * hd, 0, H, l.wk, &stg));
            TRY(upload_slice(m, g, NM("attn_v"), KW, H, m->k0 * hd, m->kh * hd, 0, H, l.wv, &stg));
        }
        TRY(upload_slice(m, g, NM("attn_output"), H, QW, 0, H, m->q0 * hd, m->qh * hd, l.wo, &stg));
        TRY(upload_slice(m, g, NM("ffn_gate"), F, H, m->f0, m->fl, 0, H, l.w1, &stg));
        TRY(upload_slice(m, g, NM("ffn_up"), F, H, m->f0, m->fl, 0, H, l.w3, &stg));
        TRY(upload_slice(m, g, NM("ffn_down"), H, F, 0, H, m->f0, m->fl, l.w2, &stg));
#undef NM
    }
    TRY(check_all_shapes(m));
#undef TRY
    *out = m;
    return NCM_OK;
}

static ncm_status synth_mat(ncm_model* m, const ncm_synth_spec& sp, const char* name, int type, int full_cols,
                            int r0, int nrows, int c0, int ncols, DevMat& out, uint8_t* dst = nullptr) {
    out.type = type;
    out.rows = nrows;
    out.cols = ncols;
    out.pitch = (row_bytes(type, ncols) + 15) / 16 * 16;
    if (dst) out.d = dst;
    else DALLOC(out.d, (size_t)out.pitch * nrows);
    CKL(synth_launch(type, ncm_synth_key(sp.seed, name), r0, nrows, c0, ncols, full_cols, out.d, out.pitch, m->stream));
    return NCM_OK;
}
static ncm_status ones(ncm_model* m, int n, float** out) {
    std::vector<float> v(n, 1.0f);
    DALLOC(*out, 4 * (size_t)n);
    CK(cudaMemcpy(*out, v.data(), 4 * (size_t)n, cudaMemcpyHostToDevice));
    return NCM_OK;
}

extern "C" ncm_status ncm_model_create_synthetic(const ncm_synth_spec* spec, int ctx_limit, int device,
                                                const int* shares, int nshards, int shard, ncm_model** out) {
    if (!spec || !out) return fail(NCM_EINVAL, "null argument");
    const ncm_synth_spec& sp = *spec;
    ncm_model* m = nullptr;
    ncm_status s = new_model(device, &m);
    if (s) return s;
    m->emb = sp.emb; m->layers = sp.layers; m->heads = sp.heads; m->kv_heads = sp.kv_heads; m->hd = sp.head_dim;
    m->ffn = sp.ffn; m->vocab = sp.vocab; m->rope_dim = sp.head_dim; m->eps = sp.eps; m->base = sp.rope_base;
    m->ctx = (ctx_limit > 0 && ctx_limit < sp.ctx) ? ctx_limit : sp.ctx;
#define TRY(x) do { if ((s = (x))) { free_model(m); return s; } } while (0)
    TRY(setup_buffers(m, shares, nshards, shard));
    const int H = m->emb, QW = m->heads * m->hd, F = m->ffn, hd = m->hd;
    TRY(synth_mat(m, sp, "token_embd.weight", sp.t_embd, H, 0, m->vocab, 0, H, m->embd));
    TRY(ones(m, H, &m->out_norm));
    if (!sp.tied) TRY(synth_mat(m, sp, "output.weight", sp.t_out, H, m->h0, m->hr, 0, H, m->head));
    else {
        if (cudaStreamSynchronize(m->stream) != cudaSuccess) { free_model(m); return fail(NCM_ECUDA, "synth"); }
        TRY(build_tied_head(m));
    }
    m->L.resize(m->layers);
    char nm[128];
    for (int i = 0; i < m->layers; ++i) {
        Layer& l = m->L[i];
#define NM(s_) (snprintf(nm, sizeof nm, "blk.%d." s_ ".weight", i), nm)
        TRY(ones(m, H, &l.attn_norm));
        TRY(ones(m, H, &l.ffn_norm));
        // q, k and v rows back to back in one buffer (one tensor map for the fused GEMV)
        uint8_t* qkv = nullptr;
        const size_t qkv_pitch = (row_bytes(sp.t_attn, H) + 15) / 16 * 16;
        TRY(dalloc(m, (void**)&qkv, qkv_pitch * (size_t)(m->qh + 2 * m->kh) * hd));
        TRY(synth_mat(m, sp, NM("attn_q"), sp.t_attn, H, m->q0 * hd, m->qh * hd, 0, H, l.wq, qkv));
        TRY(synth_mat(m, sp, NM("attn_k"), sp.t_attn, H, m->k0 * hd, m->kh * hd, 0, H, l.wk,
                      qkv + qkv_pitch * m->qh * hd));
        TRY(synth_mat(m, sp, NM("attn_v"), sp.t_attn, H, m->k0 * hd, m->kh * hd, 0, H, l.wv,
                      qkv + qkv_pitch * (m->qh + m->kh) * hd));
        TRY(synth_mat(m, sp, NM("attn_output"), sp.t_attn, QW, 0, H, m->q0 * hd, m->qh * hd, l.wo));
        TRY(synth_mat(m, sp, NM("ffn_gate"), sp.t_ffn, H, m->f0, m->fl, 0, H, l.w1));
        TRY(synth_mat(m, sp, NM("ffn_up"), sp.t_ffn, H, m->f0, m->fl, 0, H, l.w3));
        TRY(synth_mat(m, sp, NM("ffn_down"), sp.t_down ? sp.t_down : sp.t_ffn, F, 0, H, m->f0, m->fl, l.w2));
#undef NM
    }
    if (cudaStreamSynchronize(m->stream) != cudaSuccess) { free_model(m); return fail(NCM_ECUDA, "synthetic init"); }
    TRY(check_all_shapes(m));
#undef TRY
    *out = m;
    return NCM_OK;
}

extern "C" void ncm_model_free(ncm_model* m) { free_model(m); }

extern "C" ncm_status ncm_model_info(const ncm_model* m, int* out) {
    if (!m || !out) return fail(NCM_EINVAL, "null argument");
    int v[12] = {m->emb, m->layers, m->heads, m->kv_heads, m->hd, m->ffn, m->vocab, m->ctx, m->qh, m->kh, m->fl, m->hr};
    memcpy(out, v, sizeof v);
    return NCM_OK;
}

extern "C" ncm_status ncm_model_reset(ncm_model* m) {
    if (!m) return fail(NCM_EINVAL, "null model");
    CK(cudaSetDevice(m->device));
    const size_t kvn = kv_row_bytes(m) * m->layers * m->ctx;
    CK(cudaMemsetAsync(m->kc, 0, kvn, m->stream));
    CK(cudaMemsetAsync(m->vc, 0, kvn, m->stream));
    // Position and prompt length only: the step counter stays monotonic because the
    // peer flags compare against it.
    CK(cudaMemsetAsync(m->state + ST_POS, 0, 4, m->stream));
    CK(cudaMemsetAsync(m->state + ST_NPROMPT, 0, 4, m->stream));
    CK(cudaStreamSynchronize(m->stream));
    return NCM_OK;
}

// inference.rs:512-531 LlamaKvCache::new: the cache storage the reference selects with
// NANOCAMELID_KV_CACHE_Q8 (Q8_0 blocks, when kv_width is a multiple of 32) or
// NANOCAMELID_KV_CACHE_F16; f32 otherwise.  The cache is cleared and the position reset.
extern "C" ncm_status ncm_model_set_kv_cache(ncm_model* m, int kind) {
    if (!m || kind < KV_F32 || kind > KV_Q8_0) return fail(NCM_EINVAL, "bad KV-cache kind");
    CK(cudaSetDevice(m->device));
    CK(cudaStreamSynchronize(m->stream));
    if (kind == KV_Q8_0 && (m->kh * m->hd) % 32) kind = KV_F32;
    m->kv_kind = kind;   // every kind fits the f32 allocation
    m->dirty = true;
    for (auto& row : m->b_graph)
        for (auto& gx : row)
            if (gx) { cudaGraphExecDestroy(gx); gx = nullptr; }
    return ncm_model_reset(m);
}

// ------------------------------------------------------------------ the decode step
static GemvParams base_params(ncm_model* m) {
    GemvParams p;
    memset(&p, 0, sizeof p);
    p.eps = m->eps;
    p.state = m->state;
    p.rope = m->rope;
    p.rope_half = m->rope_dim / 2;
    p.head_dim = m->hd;
    p.tokens = m->tokens;
    p.ctx = m->ctx;
    p.err = m->err;
    p.tp.world = 1;
    p.tp.timeout_ns = m->timeout_ns;
    p.row_align = 2;
    p.tune = m->tune;
    p.cgroups = m->cgroups;
    p.dbg_ts = m->dbg_on ? m->dbg_ts : nullptr;
    return p;
}

// The next GEMV's weights, for the L2 prefetch a kernel issues once its own loads are
// out: mats share one fused row space (wq/wk/wv), or are a dual pair (w1/w3).
static void set_prefetch(ncm_model* m, GemvParams& p, std::initializer_list<const DevMat*> mats, bool dual) {
    p.pf_nmat = 0;
    int rows = 0;
    for (const DevMat* d : mats) {
        p.pf_base[p.pf_nmat] = d->d;
        p.pf_pitch[p.pf_nmat] = d->pitch;
        p.pf_rows[p.pf_nmat] = d->rows;
        rows = dual ? d->rows : rows + d->rows;
        ++p.pf_nmat;
    }
    p.pf_dual = dual ? 1 : 0;
    p.pf_grid = std::max(1, std::min(num_sms(), rows / 2));
    p.pf_bytes = m->prefetch_bytes;
}

// Plans the launch, encodes one TMA tensor map per weight matrix (box = the planned
// rows x 512 columns) and launches.  mats[i] feeds segment i; `up` is the second matrix
// of the gate/up pair.
static int launch_gemv(std::initializer_list<const DevMat*> mats, const DevMat* up, int in_mode, int epi,
                       GemvParams& p, cudaStream_t s) {
    const DevMat& w0 = **mats.begin();
    const int grid = gemv_plan(w0.type, w0.cols, p.total_rows, up != nullptr, in_mode, p);
    if (grid < 0) return (int)cudaErrorInvalidValue;
    int i = 0;
    for (const DevMat* d : mats) {
        int r = gemv_tensor_map(&p.tm[i++], d->d, d->rows, d->pitch, p.chunk_words, p.box_rows);
        if (r) return r;
    }
    if (up) {
        int r = gemv_tensor_map(&p.tm2, up->d, up->rows, up->pitch, p.chunk_words, p.box_rows);
        if (r) return r;
    }
    return gemv_launch(w0.type, in_mode, epi, p, grid, s, true);
}

static ncm_status check_err(ncm_model* m);
static ncm_status run_rows(ncm_model* m, const int* tokens, int ntok, int pos0, bool with_head, int* argmax_out);
static bool host_mode(const ncm_model* m) { return m->world > 1 && m->reduce_mode == NCM_REDUCE_HOST_CALLBACK; }

// The reference's reduce closure (tp.rs:226-236): n floats of `dev` go to the host
// function, which leaves the global value in place; a non-zero return is the closure's
// Err.  Runs eagerly on the calling thread (synchronous).
static ncm_status host_reduce(ncm_model* m, void* dev, int n, int layer, int phase, cudaStream_t s) {
    CK(cudaMemcpyAsync(m->h_red, dev, 4 * (size_t)n, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    ncm_status st = check_err(m);
    if (st) return st;
    const int rc = m->host_fn(m->h_red, n, layer, phase, m->host_user);
    if (rc != 0)
        return fail(NCM_EPEER, "host reducer returned " + std::to_string(rc) + " at layer " + std::to_string(layer) +
                                   ", phase " + std::to_string(phase));
    CK(cudaMemcpyAsync(dev, m->h_red, 4 * (size_t)n, cudaMemcpyHostToDevice, s));
    return NCM_OK;
}

// Row-parallel projection (wo / w2) with its reduction: one GPU -> hidden += out;
// fused P2P -> NVLink stores + rank-ordered sum in the epilogue; NCCL -> partial,
// ncclAllReduce, residual add; host callback -> partial, host_fn, residual add.
// The input is the f32 vector x, or (xq non-null) its Q8_0 blocks as the producing kernel
// wrote them (bit-identical to quantising x here).  `next` is prefetched into L2.
static ncm_status row_parallel(ncm_model* m, const DevMat& w, const float* x, const int8_t* xq, const float* xs,
                               int slot, const GemvParams* next, cudaStream_t s) {
    if (w.type == NCM_T_Q6_K) {
        // one GPU (checked at load): quantise here unless the producer did, then hidden +=
        if (!xq) {
            CKL(batch_prep_launch(x, w.cols, w.cols, 1, nullptr, m->eps, nullptr, nullptr, m->act_q, m->act_s, nullptr,
                                  s, true));
            xq = m->act_q;
            xs = m->act_s;
        }
        Q6Params q;
        memset(&q, 0, sizeof q);
        q.w = w.d; q.pitch = w.pitch; q.rows = w.rows; q.cols = w.cols; q.xq = xq; q.xs = xs; q.out = m->hidden;
        CKL(q6k_gemv_launch(EPI_RESID, q, s, true));
        return NCM_OK;
    }
    GemvParams p = base_params(m);
    p.nseg = 1;
    p.total_rows = m->emb;
    p.x = x;
    p.xq = xq;
    p.xs = xs;
    const int in = xq ? IN_Q8 : IN_F32;
    if (next) {
        memcpy(p.pf_base, next->pf_base, sizeof p.pf_base);
        memcpy(p.pf_pitch, next->pf_pitch, sizeof p.pf_pitch);
        memcpy(p.pf_rows, next->pf_rows, sizeof p.pf_rows);
        p.pf_nmat = next->pf_nmat; p.pf_grid = next->pf_grid; p.pf_dual = next->pf_dual; p.pf_bytes = next->pf_bytes;
    }
    p.hidden = m->hidden;
    if (m->world == 1) {
        p.seg[0] = {m->hidden, m->emb, 0, SEG_OUT};
        CKL(launch_gemv({&w}, nullptr, in, EPI_RESID, p, s));
    } else if (m->reduce_mode == NCM_REDUCE_FUSED_P2P) {
        p.seg[0] = {nullptr, m->emb, 0, SEG_OUT};
        p.tp = m->comm;
        p.tp_slot = slot;
        CKL(launch_gemv({&w}, nullptr, in, EPI_TP_RESID, p, s));
    } else if (m->reduce_mode == NCM_REDUCE_HOST_CALLBACK) {
        p.seg[0] = {m->part, m->emb, 0, SEG_OUT};
        CKL(launch_gemv({&w}, nullptr, in, EPI_PLAIN, p, s));
        ncm_status st = host_reduce(m, m->part, m->emb, slot / 2, slot % 2, s);
        if (st) return st;
        CKL(resid_add_launch(m->hidden, m->part, m->emb, s, true));
    } else {
        p.seg[0] = {m->part, m->emb, 0, SEG_OUT};
        CKL(launch_gemv({&w}, nullptr, in, EPI_PLAIN, p, s));
        int r = g_nccl.AllReduce(m->part, m->part, (size_t)m->emb, kNcclFloat, kNcclSum, m->nccl, s);
        if (r != 0) return fail(NCM_EPEER, "ncclAllReduce failed");
        CKL(resid_add_launch(m->hidden, m->part, m->emb, s, true));
    }
    return NCM_OK;
}

// Prefetch descriptors of the step's GEMVs (which weights each kernel streams into L2
// for its successor).
static GemvParams pf_of(ncm_model* m, std::initializer_list<const DevMat*> mats, bool dual) {
    GemvParams p;
    memset(&p, 0, sizeof p);
    set_prefetch(m, p, mats, dual);
    return p;
}
static GemvParams pf_qkv(ncm_model* m, int l) { return pf_of(m, {&m->L[l].wq, &m->L[l].wk, &m->L[l].wv}, false); }
static GemvParams pf_w13(ncm_model* m, int l) { return pf_of(m, {&m->L[l].w1, &m->L[l].w3}, true); }
static GemvParams pf_next_after_w2(ncm_model* m, int l) {
    return l + 1 < m->layers ? pf_qkv(m, l + 1) : pf_of(m, {&m->head}, false);
}
static void copy_pf(GemvParams& p, const GemvParams& n) {
    memcpy(p.pf_base, n.pf_base, sizeof p.pf_base);
    memcpy(p.pf_pitch, n.pf_pitch, sizeof p.pf_pitch);
    memcpy(p.pf_rows, n.pf_rows, sizeof p.pf_rows);
    p.pf_nmat = n.pf_nmat; p.pf_grid = n.pf_grid; p.pf_dual = n.pf_dual; p.pf_bytes = n.pf_bytes;
}

// rms_norm -> quantize -> wq/wk/wv -> rope -> store_kv (inference.rs:4521-4646) of layer l.
// It streams wo of the layer into L2 for the output projection after attention.
static int launch_qkv(ncm_model* m, int l, cudaStream_t s) {
    const Layer& L = m->L[l];
    const int qw = m->qh * m->hd, kw = m->kh * m->hd;
    GemvParams p = base_params(m);
    p.nseg = 3;
    p.seg[0] = {m->q, qw, 0, SEG_Q};
    p.seg[1] = {nullptr, kw, qw, SEG_K};
    p.seg[2] = {nullptr, kw, qw + kw, SEG_V};
    p.total_rows = qw + 2 * kw;
    p.x = m->hidden;
    p.norm_w = L.attn_norm;
    p.kcache = m->kc + (size_t)l * m->ctx * kw;
    p.vcache = m->vc + (size_t)l * m->ctx * kw;
    p.kv_width = kw;
    if (m->kv_kind != KV_F32) {
        // F16 / Q8_0 cache: the epilogue stages the f32 row, a store launch converts it
        p.kcache = m->kv_sk;
        p.vcache = m->kv_sv;
        p.kv_stage = 1;
    }
    if (l == 0) p.ssq_tok = m->embd_ssq;
    copy_pf(p, pf_of(m, {&L.wo}, false));
    int r;
    if (L.wk.d == L.wq.d + (size_t)L.wq.pitch * L.wq.rows && L.wv.d == L.wk.d + (size_t)L.wk.pitch * L.wk.rows &&
        L.wq.pitch == L.wk.pitch && L.wq.pitch == L.wv.pitch) {
        // one buffer: one tensor map, tiles across the q / k / v boundaries
        DevMat all = L.wq;
        all.rows = qw + 2 * kw;
        p.fused = 1;
        r = launch_gemv({&all}, nullptr, IN_F32_RMS, EPI_QKV, p, s);
    } else {
        r = launch_gemv({&L.wq, &L.wk, &L.wv}, nullptr, IN_F32_RMS, EPI_QKV, p, s);
    }
    if (!r && m->kv_kind != KV_F32)
        r = kv_store_launch(m->kv_kind, m->kv_sk, m->kv_sv, 1, kw, kv_layer(m, m->kc, l), kv_layer(m, m->vc, l),
                            m->state + ST_POS, s, true);
    return r;
}

// rms_norm -> quantize -> w1, w3 -> silu*mul (inference.rs:4679-4730) of layer l; the
// result also as Q8_0 blocks for w2 when the plan has 32-row tiles.  Streams w2 into L2.
static int launch_w13(ncm_model* m, int l, cudaStream_t s) {
    const Layer& L = m->L[l];
    GemvParams f = base_params(m);
    f.nseg = 1;
    f.seg[0] = {m->act, m->fl, 0, SEG_OUT};
    f.total_rows = m->fl;
    f.x = m->hidden;
    f.norm_w = L.ffn_norm;
    if (m->act_quantised) {
        f.row_align = 32;
        f.qout = m->act_q;
        f.qout_s = m->act_s;
    }
    copy_pf(f, pf_of(m, {&L.w2}, false));
    return launch_gemv({&L.w1}, &L.w3, IN_F32_RMS, EPI_SILU, f, s);
}

static void attn_params(ncm_model* m, int l, AttnParams& a) {
    const int kw = m->kh * m->hd;
    memset(&a, 0, sizeof a);
    a.q = m->q;
    a.kc = m->kc + (size_t)l * m->ctx * kw;
    a.vc = m->vc + (size_t)l * m->ctx * kw;
    a.kv_kind = m->kv_kind;
    a.kc_raw = kv_layer(m, m->kc, l);
    a.vc_raw = kv_layer(m, m->vc, l);
    a.out = m->att;
    a.scores = m->scores;
    a.state = m->state;
    a.pos_override = -1;
    a.heads = m->qh;
    a.kv_heads = m->kh;
    a.hd = m->hd;
    a.kvw = kw;
    a.ctx = m->ctx;
    // one 32-dimension slice per CTA, so each warp's output is one Q8_0 block for wo
    a.out_q = m->att_q;
    a.out_s = m->att_s;
    a.scale = 1.0f / sqrtf((float)m->hd);   // inference.rs:4653
    a.vmap_on = m->av_tma;
    a.sv_on = m->attn_sv;
    a.err = m->err;
}

static ncm_status enqueue_step(ncm_model* m, bool with_head, cudaStream_t s) {
    CKL(embed_launch(m->embd.type, m->embd.d, m->embd.pitch, m->emb, m->tokens, m->state, m->ctx, m->err, m->hidden, s,
                     true));
    for (int l = 0; l < m->layers; ++l) {
        const Layer& L = m->L[l];
        CKL(launch_qkv(m, l, s));
        // attention (inference.rs:4648-4665)
        AttnParams a;
        attn_params(m, l, a);
        CKL(attention_launch(a, s, true));
        // quantize -> wo -> residual (inference.rs:4667-4673), reduce #1 (tp.rs:356-363)
        const GemvParams n1 = pf_w13(m, l);
        ncm_status st = row_parallel(m, L.wo, nullptr, m->att_q, m->att_s, 2 * l, &n1, s);
        if (st) return st;
        CKL(launch_w13(m, l, s));
        // quantize -> w2 -> residual (inference.rs:4732-4748), reduce #2 (tp.rs:416-424)
        const GemvParams n2 = pf_next_after_w2(m, l);
        st = m->act_quantised ? row_parallel(m, L.w2, nullptr, m->act_q, m->act_s, 2 * l + 1, &n2, s)
                              : row_parallel(m, L.w2, m->act, nullptr, nullptr, 2 * l + 1, &n2, s);
        if (st) return st;
    }
    if (!with_head) {
        CKL(advance_launch(m->state, s, true));
        return NCM_OK;
    }
    // output norm -> quantize -> head -> greedy argmax (inference.rs:4783-4845)
    GemvParams h = base_params(m);
    h.nseg = 1;
    h.seg[0] = {m->logits, m->hr, 0, SEG_OUT};
    h.total_rows = m->hr;
    h.x = m->hidden;
    h.norm_w = m->out_norm;
    h.amax_part = m->amax_part;
    h.counter = m->amax_cnt;
    h.head_row0 = m->h0;
    if (m->world > 1 && m->reduce_mode == NCM_REDUCE_FUSED_P2P) h.tp = m->comm;
    if (m->world > 1 && m->reduce_mode != NCM_REDUCE_FUSED_P2P) h.head_out = m->head_out;
    if (m->head.type == NCM_T_Q6_K) {
        // output norm -> quantize (one prep launch), then the Q6_K GEMV with the argmax
        CKL(batch_prep_launch(m->hidden, m->emb, m->emb, 1, m->out_norm, m->eps, nullptr, nullptr, m->hx_q, m->hx_s,
                              nullptr, s, true));
        Q6Params q;
        memset(&q, 0, sizeof q);
        q.w = m->head.d; q.pitch = m->head.pitch; q.rows = m->hr; q.cols = m->emb; q.xq = m->hx_q; q.xs = m->hx_s;
        q.out = m->logits; q.amax_part = m->amax_part; q.counter = m->amax_cnt; q.head_row0 = m->h0;
        q.state = m->state; q.tokens = m->tokens; q.ctx = m->ctx;
        CKL(q6k_gemv_launch(EPI_ARGMAX, q, s, true));
        return NCM_OK;
    }
    CKL(launch_gemv({&m->head}, nullptr, IN_F32_RMS, EPI_ARGMAX, h, s));
    if (h.head_out && host_mode(m)) {
        // this shard's (logit, token); the host merges every shard's pair (strict '>' in
        // rank order, cluster_tp_node.rs:1185-1204) and the merged pair advances the state
        ncm_status st = host_reduce(m, m->head_out, 2, m->layers, NCM_REDUCE_PHASE_HEAD, s);
        if (st) return st;
        CKL(argmax_merge_launch(m->head_out, 1, m->tokens, m->state, m->ctx, s, true));
    } else if (h.head_out) {
        int r = g_nccl.AllGather(m->head_out, m->gather, 2, kNcclFloat, m->nccl, s);
        if (r != 0) return fail(NCM_EPEER, "ncclAllGather failed");
        CKL(argmax_merge_launch(m->gather, m->world, m->tokens, m->state, m->ctx, s, true));
    }
    return NCM_OK;
}

static ncm_status capture(ncm_model* m, bool with_head, cudaGraphExec_t* exec) {
    cudaGraph_t graph;
    CK(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    ncm_status st = enqueue_step(m, with_head, m->stream);
    cudaError_t e = cudaStreamEndCapture(m->stream, &graph);
    if (st) {
        if (e == cudaSuccess) cudaGraphDestroy(graph);
        return st;
    }
    CK(e);
    e = cudaGraphInstantiate(exec, graph, 0);
    cudaGraphDestroy(graph);
    CK(e);
    return NCM_OK;
}

static ncm_status ensure_graphs(ncm_model* m) {
    if (m->world > 1 && !m->tp_ready) return fail(NCM_EINVAL, "tensor-parallel peers not set up (ncm_tp_import / ncm_tp_nccl_init)");
    if (host_mode(m)) return NCM_OK;   // eager steps: the host reducer runs between kernels
    if (!m->dirty && m->g_full) return NCM_OK;
    if (m->g_full) { cudaGraphExecDestroy(m->g_full); m->g_full = nullptr; }
    if (m->g_nohead) { cudaGraphExecDestroy(m->g_nohead); m->g_nohead = nullptr; }
    ncm_status s = capture(m, true, &m->g_full);
    if (s) return s;
    s = capture(m, false, &m->g_nohead);
    if (s) return s;
    m->dirty = false;
    return NCM_OK;
}

static ncm_status check_err(ncm_model* m) {
    int e = 0;
    CK(cudaMemcpy(&e, m->err, 4, cudaMemcpyDeviceToHost));
    if (e) {
        CK(cudaMemset(m->err, 0, 4));
        if (e & NCM_DEVERR_PEER_TIMEOUT) return fail(NCM_ETIMEOUT, "a device-side wait on a peer GPU timed out");
        if (e & NCM_DEVERR_CTX_FULL)
            return fail(NCM_EINVAL, "a decode step ran past the context limit (the position was held at the last slot)");
        return fail(NCM_ECUDA, "device error word " + std::to_string(e));
    }
    return NCM_OK;
}

// One decode step: the captured graph, or eagerly when a host reducer takes part.
static ncm_status run_step(ncm_model* m, bool with_head, cudaStream_t s) {
    if (host_mode(m)) return enqueue_step(m, with_head, s);
    CK(cudaGraphLaunch(with_head ? m->g_full : m->g_nohead, s));
    return NCM_OK;
}

static ncm_status set_pos(ncm_model* m, int pos, int nprompt, cudaStream_t s) {
    m->h_stage[0] = pos;
    m->h_stage[1] = nprompt;
    CK(cudaMemcpyAsync(m->state + ST_POS, &m->h_stage[0], 4, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(m->state + ST_NPROMPT, &m->h_stage[1], 4, cudaMemcpyHostToDevice, s));
    return NCM_OK;
}

extern "C" ncm_status ncm_prefill_tokens(ncm_model* m, const int* prompt, int n_prompt, void* stream) {
    if (!m || !prompt || n_prompt <= 0 || n_prompt > m->ctx) return fail(NCM_EINVAL, "bad prompt");
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->vocab) return fail(NCM_EINVAL, "token id out of range");
    CK(cudaSetDevice(m->device));
    ncm_status s = ensure_graphs(m);
    if (s) return s;
    cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
    if (stream) m->ext_stream = st;
    CK(cudaStreamSynchronize(st));
    if (n_prompt > 1 && !m->has_q6k) {
        // Eight prompt tokens per multi-row pass: every row's K/V and greedy token equal
        // the token-by-token prefill's bit for bit, so the state below is the one that
        // prefill leaves (tokens, position, prompt length, last token).
        int last = 0;
        for (int c0 = 0; c0 < n_prompt; c0 += kMaxBatch) {
            const int nt = std::min(kMaxBatch, n_prompt - c0);
            const bool fin = c0 + nt == n_prompt;
            int out[kMaxBatch];
            if ((s = run_rows(m, prompt + c0, nt, c0, fin, out))) return s;
            if (fin) last = out[nt - 1];
        }
        CK(cudaMemcpy(m->tokens, prompt, 4 * (size_t)n_prompt, cudaMemcpyHostToDevice));
        if (n_prompt < m->ctx) CK(cudaMemcpy(m->tokens + n_prompt, &last, 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(m->state + ST_POS, &n_prompt, 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(m->state + ST_NPROMPT, &n_prompt, 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(m->state + ST_LAST_TOKEN, &last, 4, cudaMemcpyHostToDevice));
        return NCM_OK;
    }
    CK(cudaMemcpyAsync(m->tokens, prompt, 4 * (size_t)n_prompt, cudaMemcpyHostToDevice, st));
    if ((s = set_pos(m, 0, n_prompt, st))) return s;
    for (int i = 0; i + 1 < n_prompt; ++i)
        if ((s = run_step(m, false, st))) return s;
    return run_step(m, true, st);
}

extern "C" ncm_status ncm_decode_steps(ncm_model* m, int n, void* stream) {
    if (!m || n < 0) return fail(NCM_EINVAL, "bad arguments");
    CK(cudaSetDevice(m->device));
    ncm_status s = ensure_graphs(m);
    if (s) return s;
    cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
    if (stream) m->ext_stream = st;
    for (int i = 0; i < n; ++i)
        if ((s = run_step(m, true, st))) return s;
    return NCM_OK;
}

extern "C" ncm_status ncm_sync_tokens(ncm_model* m, int* tokens, int count, int* pos_out) {
    if (!m) return fail(NCM_EINVAL, "null model");
    CK(cudaSetDevice(m->device));
    // this model's streams only: a device-wide sync would also wait on (and fail during)
    // another host thread's graph capture on the same GPU
    CK(cudaStreamSynchronize(m->stream));
    if (m->ext_stream) {
        CK(cudaStreamSynchronize(m->ext_stream));
        m->ext_stream = nullptr;
    }
    ncm_status s = check_err(m);
    if (s) return s;
    if (tokens && count > 0) CK(cudaMemcpy(tokens, m->tokens, 4 * (size_t)(count < m->ctx ? count : m->ctx), cudaMemcpyDeviceToHost));
    if (pos_out) CK(cudaMemcpy(pos_out, m->state + ST_POS, 4, cudaMemcpyDeviceToHost));
    return NCM_OK;
}

extern "C" ncm_status ncm_generate(ncm_model* m, const int* prompt, int n_prompt, int n_gen, int* out_tokens) {
    if (!m || !out_tokens || n_gen < 0) return fail(NCM_EINVAL, "bad arguments");
    if (n_prompt + n_gen > m->ctx) return fail(NCM_EINVAL, "prompt + generation exceeds the context");
    ncm_status s = ncm_prefill_tokens(m, prompt, n_prompt, nullptr);
    if (s) return s;
    if (n_gen > 1 && (s = ncm_decode_steps(m, n_gen - 1, nullptr))) return s;
    CK(cudaStreamSynchronize(m->stream));
    if ((s = check_err(m))) return s;
    if (n_gen > 0) CK(cudaMemcpy(out_tokens, m->tokens + n_prompt, 4 * (size_t)n_gen, cudaMemcpyDeviceToHost));
    return NCM_OK;
}

extern "C" ncm_status ncm_forward_pass(ncm_model* m, int token, int pos, float* logits, int* argmax) {
    if (!m || pos < 0 || pos >= m->ctx || token < 0 || token >= m->vocab) return fail(NCM_EINVAL, "bad token or position");
    CK(cudaSetDevice(m->device));
    ncm_status s = ensure_graphs(m);
    if (s) return s;
    cudaStream_t st = m->stream;
    m->h_stage[2] = token;
    CK(cudaMemcpyAsync(m->tokens + pos, &m->h_stage[2], 4, cudaMemcpyHostToDevice, st));
    if ((s = set_pos(m, pos, pos + 1, st))) return s;
    if ((s = run_step(m, true, st))) return s;
    CK(cudaMemcpyAsync(&m->h_stage[3], m->state + ST_LAST_TOKEN, 4, cudaMemcpyDeviceToHost, st));
    if (logits) CK(cudaMemcpyAsync(logits, m->logits, 4 * (size_t)m->hr, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if ((s = check_err(m))) return s;
    if (argmax) *argmax = m->h_stage[3];
    return NCM_OK;
}

extern "C" ncm_status ncm_debug_read(ncm_model* m, int which, int layer, float* out, int64_t n) {
    if (!m || !out || n < 0) return fail(NCM_EINVAL, "bad arguments");
    CK(cudaSetDevice(m->device));
    CK(cudaStreamSynchronize(m->stream));
    const size_t kw = (size_t)m->kh * m->hd;
    const float* src = nullptr;
    size_t cap = 0;
    switch (which) {
        case 0: src = m->hidden; cap = m->emb; break;
        case 1: src = m->q; cap = (size_t)m->qh * m->hd; break;
        case 2: src = m->att; cap = (size_t)m->qh * m->hd; break;
        case 3: src = m->act; cap = m->fl; break;
        case 4:
            if (m->kv_kind != KV_F32) return fail(NCM_EINVAL, "the K / V caches are not f32");
            src = m->kc + (size_t)layer * m->ctx * kw; cap = (size_t)m->ctx * kw; break;
        case 5:
            if (m->kv_kind != KV_F32) return fail(NCM_EINVAL, "the K / V caches are not f32");
            src = m->vc + (size_t)layer * m->ctx * kw; cap = (size_t)m->ctx * kw; break;
        case 6: src = m->logits; cap = m->hr; break;
        default: return fail(NCM_EINVAL, "unknown buffer");
    }
    if ((size_t)n > cap) return fail(NCM_EINVAL, "read past the buffer");
    CK(cudaMemcpy(out, src, 4 * (size_t)n, cudaMemcpyDeviceToHost));
    return NCM_OK;
}

extern "C" ncm_status ncm_get_hidden(ncm_model* m, float* hidden) {
    if (!m || !hidden) return fail(NCM_EINVAL, "null argument");
    CK(cudaSetDevice(m->device));
    CK(cudaStreamSynchronize(m->stream));
    CK(cudaMemcpy(hidden, m->hidden, 4 * (size_t)m->emb, cudaMemcpyDeviceToHost));
    return NCM_OK;
}

// Measurement seam: one launch of a decode step's GEMV kernel for `layer`, with exactly
// the parameters the captured step uses (so a caller can time the step's dominant kernel
// with events on its own stream).  It overwrites the activations it writes (q and the
// layer's K/V row at the current position, silu*up, or hidden for the row-parallel ones).
extern "C" ncm_status ncm_launch_step_kernel(ncm_model* m, int kind, int layer, void* stream) {
    if (!m || layer < 0 || layer >= m->layers) return fail(NCM_EINVAL, "bad layer");
    CK(cudaSetDevice(m->device));
    cudaStream_t s = stream ? (cudaStream_t)stream : m->stream;
    struct Probe {   // the phase stamps are recorded by these seam launches only
        ncm_model* m;
        Probe(ncm_model* mm) : m(mm) { m->dbg_on = true; }
        ~Probe() { m->dbg_on = false; }
    } probe(m);
    switch (kind) {
        case NCM_STEP_QKV: CKL(launch_qkv(m, layer, s)); return NCM_OK;
        case NCM_STEP_W13: CKL(launch_w13(m, layer, s)); return NCM_OK;
        case NCM_STEP_WO:
            if (m->world > 1) return fail(NCM_EUNSUPPORTED, "row-parallel kernels of a shard wait on their peers");
            return row_parallel(m, m->L[layer].wo, nullptr, m->att_q, m->att_s, 0, nullptr, s);
        case NCM_STEP_W2:
            if (m->world > 1) return fail(NCM_EUNSUPPORTED, "row-parallel kernels of a shard wait on their peers");
            return m->act_quantised ? row_parallel(m, m->L[layer].w2, nullptr, m->act_q, m->act_s, 0, nullptr, s)
                                    : row_parallel(m, m->L[layer].w2, m->act, nullptr, nullptr, 0, nullptr, s);
        default: return fail(NCM_EINVAL, "unknown step kernel");
    }
}

// Measurement seam: the phase stamps (global-timer ns) the last ncm_launch_step_kernel
// launch recorded, [CTA][16] as the GEMV kernel documents them; n = entries to copy.
extern "C" ncm_status ncm_debug_stamps(ncm_model* m, uint64_t* out, int n) {
    if (!m || !out || n < 0 || n > 16 * num_sms()) return fail(NCM_EINVAL, "bad arguments");
    CK(cudaSetDevice(m->device));
    CK(cudaDeviceSynchronize());
    CK(cudaMemcpy(out, m->dbg_ts, 8 * (size_t)n, cudaMemcpyDeviceToHost));
    return NCM_OK;
}

// ------------------------------------------------------------------ multi-row verify
static ncm_status ensure_batch_buffers(ncm_model* m) {
    if (m->b_hidden) return NCM_OK;
    const size_t qw = (size_t)m->qh * m->hd;
    const size_t wmax = std::max((size_t)m->emb, std::max(qw, (size_t)m->fl));
    DALLOC(m->b_hidden, 4 * (size_t)kMaxBatch * m->emb);
    DALLOC(m->b_q, 4 * (size_t)kMaxBatch * qw);
    DALLOC(m->b_att, 4 * (size_t)kMaxBatch * qw);
    DALLOC(m->b_act, 4 * (size_t)kMaxBatch * m->fl);
    DALLOC(m->b_xq, (size_t)kMaxBatch * wmax);
    DALLOC(m->b_xs, 4 * (size_t)kMaxBatch * (wmax / 32));
    DALLOC(m->b_xsum, 4 * (size_t)kMaxBatch * (wmax / 32));
    DALLOC(m->b_amax, sizeof(float2) * kMaxBatch * num_sms());
    DALLOC(m->b_cnt, 4);
    DALLOC(m->b_tok, 4 * kMaxBatch);
    DALLOC(m->b_arg, 4 * kMaxBatch);
    DALLOC(m->b_pos, 4);
    DALLOC(m->b_scores, 4 * (size_t)kMaxBatch * m->qh * m->ctx);
    DALLOC(m->b_part, 4 * (size_t)kMaxBatch * m->emb);
    DALLOC(m->b_pairs, sizeof(float2) * kMaxBatch);
    CK(cudaMemset(m->b_cnt, 0, 4));
    return NCM_OK;
}

static BatchParams batch_base(ncm_model* m, int ntok) {
    BatchParams p;
    memset(&p, 0, sizeof p);
    p.ntok = ntok;
    p.cgroups = m->bcgroups;
    p.rope = m->rope;
    p.rope_half = m->rope_dim / 2;
    p.head_dim = m->hd;
    p.err = m->err;
    p.xq = m->b_xq;
    p.xs = m->b_xs;
    p.xsum = m->b_xsum;
    return p;
}

static int launch_batch(std::initializer_list<const DevMat*> mats, const DevMat* up, int epi, BatchParams& p,
                        cudaStream_t s) {
    const DevMat& w0 = **mats.begin();
    const int grid = batch_plan(w0.type, w0.cols, p.total_rows, up != nullptr, p.ntok, p);
    if (grid < 0) return (int)cudaErrorInvalidValue;
    int i = 0;
    for (const DevMat* d : mats) {
        int r = gemv_tensor_map(&p.tm[i++], d->d, d->rows, d->pitch, p.chunk_words, p.box_rows);
        if (r) return r;
    }
    if (up) {
        int r = gemv_tensor_map(&p.tm2, up->d, up->rows, up->pitch, p.chunk_words, p.box_rows);
        if (r) return r;
    }
    return batch_gemv_launch(w0.type, epi, p, grid, s, true);
}

// Row-parallel wo / w2 of the multi-row pass: one GPU -> hidden rows += out; tensor
// parallel (host-callback reducer) -> partial rows, the host's rank-ordered sum over all
// ntok rows at once (tp.rs:349-363 per row), residual add.
static ncm_status batch_row_parallel(ncm_model* m, const DevMat& w, BatchParams& p, int ntok, int layer, int phase,
                                     cudaStream_t s) {
    if (m->world == 1) {
        CKL(launch_batch({&w}, nullptr, EPI_RESID, p, s));
        return NCM_OK;
    }
    p.seg[0] = {m->b_part, m->emb, 0, SEG_OUT};
    p.out_stride = m->emb;
    CKL(launch_batch({&w}, nullptr, EPI_PLAIN, p, s));
    const int n = ntok * m->emb;
    if (m->reduce_mode == NCM_REDUCE_FUSED_P2P) {
        // every row's partial summed over NVLink in rank order, plus the residual
        CKL(tp_rows_reduce_launch(m->rows, m->b_part, m->b_hidden, n, s));
        return NCM_OK;
    }
    if (m->reduce_mode == NCM_REDUCE_NCCL) {
        int r = g_nccl.AllReduce(m->b_part, m->b_part, (size_t)n, kNcclFloat, kNcclSum, m->nccl, s);
        if (r != 0) return fail(NCM_EPEER, "ncclAllReduce failed");
        CKL(resid_add_launch(m->b_hidden, m->b_part, n, s, true));
        return NCM_OK;
    }
    ncm_status st = host_reduce(m, m->b_part, n, layer, phase, s);
    if (st) return st;
    CKL(resid_add_launch(m->b_hidden, m->b_part, ntok * m->emb, s, true));
    return NCM_OK;
}

// Every GEMV CTA quantises the whole f32 input itself when it is small (saves a launch);
// larger inputs go through one prep launch whose CTAs split the work.
static bool prologue_quant(int ntok, int cols) { return (int64_t)ntok * cols <= 5 * 4096; }

// The multi-row pass (speculative.rs:381-389 prefill_pass_batch, inference.rs:3695-4111,
// then compute_logits_from_hidden + sample_logits(_, 0.0) per row) for tokens b_tok at
// positions *b_pos + t: each weight tile read once for all rows, K/V stored at their
// positions, greedy argmax of every row into b_arg.  Captured once per row count.
static ncm_status enqueue_verify(ncm_model* m, int ntok, cudaStream_t s, bool with_head) {
    const int qw = m->qh * m->hd, kw = m->kh * m->hd;
    CKL(embed_rows_launch(m->embd.type, m->embd.d, m->embd.pitch, m->emb, m->b_tok, ntok, m->b_hidden, s, true));
    for (int l = 0; l < m->layers; ++l) {
        const Layer& L = m->L[l];
        CKL(batch_prep_launch(m->b_hidden, m->emb, m->emb, ntok, L.attn_norm, m->eps, l == 0 ? m->embd_ssq : nullptr,
                              m->b_tok, m->b_xq, m->b_xs, m->b_xsum, s, true));
        BatchParams p = batch_base(m, ntok);
        p.nseg = 3;
        p.seg[0] = {m->b_q, qw, 0, SEG_Q};
        p.seg[1] = {nullptr, kw, qw, SEG_K};
        p.seg[2] = {nullptr, kw, qw + kw, SEG_V};
        p.total_rows = qw + 2 * kw;
        p.out_stride = qw;
        p.pos_dev = m->b_pos;
        p.kcache = m->kc + (size_t)l * m->ctx * kw;
        p.vcache = m->vc + (size_t)l * m->ctx * kw;
        p.kv_width = kw;
        if (m->kv_kind != KV_F32) {
            p.kcache = m->kv_sk;
            p.vcache = m->kv_sv;
            p.kv_stage = 1;
        }
        CKL(launch_batch({&L.wq, &L.wk, &L.wv}, nullptr, EPI_QKV, p, s));
        if (m->kv_kind != KV_F32)
            CKL(kv_store_launch(m->kv_kind, m->kv_sk, m->kv_sv, ntok, kw, kv_layer(m, m->kc, l), kv_layer(m, m->vc, l),
                                m->b_pos, s, true));
        AttnParams a;
        memset(&a, 0, sizeof a);
        a.q = m->b_q;
        a.kc = m->kc + (size_t)l * m->ctx * kw;
        a.vc = m->vc + (size_t)l * m->ctx * kw;
        a.kv_kind = m->kv_kind;
        a.kc_raw = kv_layer(m, m->kc, l);
        a.vc_raw = kv_layer(m, m->vc, l);
        a.out = m->b_att;
        a.scores = m->b_scores;
        a.state = m->b_pos;   // b_pos[0] plays ST_POS (= 0): token z at *b_pos + z
        a.pos_override = -1;
        a.heads = m->qh;
        a.kv_heads = m->kh;
        a.hd = m->hd;
        a.kvw = kw;
        a.ctx = m->ctx;
        a.scale = 1.0f / sqrtf((float)m->hd);
        a.ntok = ntok;
        a.tok_stride = qw;
        a.vmap_on = m->av_tma;
        a.sv_on = m->attn_sv;
        a.err = m->err;
        CKL(attention_launch(a, s, true));
        BatchParams o = batch_base(m, ntok);
        if (prologue_quant(ntok, qw)) {
            o.xf = m->b_att;
            o.xf_stride = qw;
        } else {
            CKL(batch_prep_launch(m->b_att, qw, qw, ntok, nullptr, m->eps, nullptr, nullptr, m->b_xq, m->b_xs, m->b_xsum, s, true));
        }
        o.nseg = 1;
        o.seg[0] = {nullptr, m->emb, 0, SEG_OUT};
        o.total_rows = m->emb;
        o.hidden = m->b_hidden;
        o.hidden_stride = m->emb;
        ncm_status st = batch_row_parallel(m, L.wo, o, ntok, l, NCM_REDUCE_PHASE_ATTENTION, s);
        if (st) return st;
        CKL(batch_prep_launch(m->b_hidden, m->emb, m->emb, ntok, L.ffn_norm, m->eps, nullptr, nullptr, m->b_xq,
                              m->b_xs, m->b_xsum, s, true));
        BatchParams f = batch_base(m, ntok);
        f.nseg = 1;
        f.seg[0] = {m->b_act, m->fl, 0, SEG_OUT};
        f.total_rows = m->fl;
        f.out_stride = m->fl;
        CKL(launch_batch({&L.w1}, &L.w3, EPI_SILU, f, s));
        BatchParams d = batch_base(m, ntok);
        if (prologue_quant(ntok, m->fl)) {
            d.xf = m->b_act;
            d.xf_stride = m->fl;
        } else {
            CKL(batch_prep_launch(m->b_act, m->fl, m->fl, ntok, nullptr, m->eps, nullptr, nullptr, m->b_xq, m->b_xs,
                                  m->b_xsum, s, true));
        }
        d.nseg = 1;
        d.seg[0] = {nullptr, m->emb, 0, SEG_OUT};
        d.total_rows = m->emb;
        d.hidden = m->b_hidden;
        d.hidden_stride = m->emb;
        st = batch_row_parallel(m, L.w2, d, ntok, l, NCM_REDUCE_PHASE_FFN, s);
        if (st) return st;
    }
    if (!with_head) return NCM_OK;   // prompt rows before the last: K/V only
    CKL(batch_prep_launch(m->b_hidden, m->emb, m->emb, ntok, m->out_norm, m->eps, nullptr, nullptr, m->b_xq, m->b_xs,
                          m->b_xsum, s, true));
    BatchParams h = batch_base(m, ntok);
    h.nseg = 1;
    h.seg[0] = {nullptr, m->hr, 0, SEG_OUT};
    h.total_rows = m->hr;
    h.amax_part = m->b_amax;
    h.counter = m->b_cnt;
    h.argmax_out = m->b_arg;
    h.head_row0 = m->h0;
    if (host_mode(m)) {
        // each row's (logit, token) of this vocab shard; the host merges them per row in
        // rank order (cluster_tp_node.rs:1185-1204) and the merged tokens are the result
        h.pair_out = m->b_pairs;
        CKL(launch_batch({&m->head}, nullptr, EPI_ARGMAX, h, s));
        ncm_status st = host_reduce(m, m->b_pairs, 2 * ntok, m->layers, NCM_REDUCE_PHASE_HEAD, s);
        if (st) return st;
        for (int t = 0; t < ntok; ++t) memcpy(m->h_stage + 16 + t, m->h_red + 2 * t + 1, 4);
        return NCM_OK;
    }
    if (m->world > 1) {
        // each row's (logit, token) of this vocab shard, merged per row in rank order
        h.pair_out = m->b_pairs;
        CKL(launch_batch({&m->head}, nullptr, EPI_ARGMAX, h, s));
        if (m->reduce_mode == NCM_REDUCE_FUSED_P2P) {
            CKL(tp_rows_argmax_launch(m->rows, m->b_pairs, ntok, m->b_arg, s));
        } else {
            int r = g_nccl.AllGather(m->b_pairs, m->rows_gather, 2 * (size_t)kMaxBatch, kNcclFloat, m->nccl, s);
            if (r != 0) return fail(NCM_EPEER, "ncclAllGather failed");
            CKL(rows_argmax_merge_launch(m->rows_gather, m->world, ntok, m->b_arg, s));
        }
        return NCM_OK;
    }
    CKL(launch_batch({&m->head}, nullptr, EPI_ARGMAX, h, s));
    return NCM_OK;
}

// One multi-row pass over tokens[0..ntok) at positions pos0 .. pos0+ntok-1 (K/V stored),
// with the head (greedy token of every row into argmax_out) or without it.  Graph per
// (head, rows), captured on first use; eager under the host reducer.
static ncm_status run_rows(ncm_model* m, const int* tokens, int ntok, int pos0, bool with_head, int* argmax_out) {
    CK(cudaSetDevice(m->device));
    ncm_status st = ensure_batch_buffers(m);
    if (st) return st;
    cudaStream_t s = m->stream;
    m->h_stage[4] = pos0;
    memcpy(m->h_stage + 5, tokens, 4 * (size_t)ntok);
    CK(cudaMemcpyAsync(m->b_pos, m->h_stage + 4, 4, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(m->b_tok, m->h_stage + 5, 4 * (size_t)ntok, cudaMemcpyHostToDevice, s));
    if (host_mode(m)) {
        // eager: the host reducer runs between the kernels; the merged tokens are in h_stage
        if ((st = enqueue_verify(m, ntok, s, with_head))) return st;
        CK(cudaStreamSynchronize(s));
        if ((st = check_err(m))) return st;
        if (with_head) memcpy(argmax_out, m->h_stage + 16, 4 * (size_t)ntok);
        return NCM_OK;
    }
    cudaGraphExec_t& gx = m->b_graph[with_head ? 1 : 0][ntok];
    if (gx) {
        CK(cudaGraphLaunch(gx, s));
    } else {
        // first use of this shape: run eagerly (configures the kernels), then capture
        if ((st = enqueue_verify(m, ntok, s, with_head))) return st;
        CK(cudaStreamSynchronize(s));
        cudaGraph_t graph;
        CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        st = enqueue_verify(m, ntok, s, with_head);
        cudaError_t e = cudaStreamEndCapture(s, &graph);
        if (st) {
            if (e == cudaSuccess) cudaGraphDestroy(graph);
            return st;
        }
        CK(e);
        e = cudaGraphInstantiate(&gx, graph, 0);
        cudaGraphDestroy(graph);
        CK(e);
    }
    if (with_head) CK(cudaMemcpyAsync(m->h_stage + 16, m->b_arg, 4 * (size_t)ntok, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if ((st = check_err(m))) return st;
    if (with_head) memcpy(argmax_out, m->h_stage + 16, 4 * (size_t)ntok);
    return NCM_OK;
}

// Every row's greedy token equals the one-token step at that position bit for bit.
extern "C" ncm_status ncm_verify_batch(ncm_model* m, const int* tokens, int ntok, int pos0, int* argmax_out) {
    if (!m || !tokens || !argmax_out || ntok < 1 || ntok > kMaxBatch || pos0 < 0 || pos0 + ntok > m->ctx)
        return fail(NCM_EINVAL, "bad verify batch");
    if (m->has_q6k) return fail(NCM_EUNSUPPORTED, "the multi-row pass has no Q6_K kernel");
    for (int i = 0; i < ntok; ++i)
        if (tokens[i] < 0 || tokens[i] >= m->vocab) return fail(NCM_EINVAL, "token id out of range");
    return run_rows(m, tokens, ntok, pos0, true, argmax_out);
}

// speculative.rs:299-494 speculative_decoding_step at temperature 0, repeated: the
// draft proposes k tokens greedily (its device-resident decode graph), the target
// verifies them in one multi-row pass, the agreeing prefix is accepted and the target's
// own token at the first disagreement (or the trailing token) is emitted.  The output
// equals the target's greedy decode.  stats[0] = drafted, stats[1] = accepted.
//
// The reference runs that last token through both models one token at a time
// (speculative.rs:421-443, 459-484).  Here it stays pending instead and becomes row 0 of
// the next verify and the draft's first step: row 0 gives the target prediction the
// reference takes from its logits, the draft's step gives its first proposal, so every
// accept decision, token and count is the reference's, and a cycle costs k draft steps
// plus one (k+1)-row verify.  When every draft was accepted the draft ingests its last
// proposal (the reference's draft loop already did).  k + 1 > 8 rows falls back to the
// reference's cycle shape.
static ncm_status spec_cycle_reference_shape(ncm_model* target, ncm_model* draft, int k, int n_gen, int* out_tokens,
                                             int* stats, int& n, int& pos, int& tt, int& dt, std::vector<int>& hist) {
    ncm_status st;
    if ((st = ncm_decode_steps(draft, k, nullptr))) return st;
    if ((st = ncm_sync_tokens(draft, hist.data(), pos + k, nullptr))) return st;
    int drafted[kMaxBatch], rows[kMaxBatch];
    for (int i = 0; i < k; ++i) drafted[i] = hist[pos + i];
    if (stats) stats[0] += k;
    if ((st = ncm_verify_batch(target, drafted, k, pos, rows))) return st;
    int i = 0, next = tt;
    while (i < k && drafted[i] == next) {
        if (n < n_gen) out_tokens[n++] = drafted[i];
        if (stats) stats[1] += 1;
        next = rows[i];
        ++i;
    }
    if (n < n_gen) out_tokens[n++] = next;
    const int at = pos + i;
    if ((st = ncm_forward_pass(target, next, at, nullptr, &tt))) return st;
    if ((st = ncm_forward_pass(draft, next, at, nullptr, &dt))) return st;
    pos = at + 1;
    return NCM_OK;
}

extern "C" ncm_status ncm_spec_generate(ncm_model* target, ncm_model* draft, const int* prompt, int n_prompt,
                                       int n_gen, int k, int* out_tokens, int* stats) {
    if (!target || !draft || !prompt || !out_tokens || n_prompt < 1 || n_gen < 0 || k < 1 || k > kMaxBatch)
        return fail(NCM_EINVAL, "bad speculative arguments");
    if (target->vocab != draft->vocab) return fail(NCM_EINVAL, "draft and target vocabularies differ");
    if (n_prompt + n_gen + k + 1 > std::min(target->ctx, draft->ctx))
        return fail(NCM_EINVAL, "prompt + generation + draft window exceeds a context");
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= target->vocab) return fail(NCM_EINVAL, "token id out of range");
    if (stats) stats[0] = stats[1] = 0;
    std::vector<int> hist(std::min(target->ctx, draft->ctx));
    ncm_status st;
    int n = 0;
    if (k + 1 > kMaxBatch) {
        if ((st = ncm_prefill_tokens(target, prompt, n_prompt, nullptr))) return st;
        if ((st = ncm_prefill_tokens(draft, prompt, n_prompt, nullptr))) return st;
        int tt = 0, dt = 0, pos = n_prompt, p0 = 0;
        if ((st = ncm_sync_tokens(target, nullptr, 0, &p0))) return st;
        CK(cudaSetDevice(target->device));
        CK(cudaMemcpy(&tt, target->state + ST_LAST_TOKEN, 4, cudaMemcpyDeviceToHost));
        if ((st = ncm_sync_tokens(draft, nullptr, 0, &p0))) return st;
        CK(cudaSetDevice(draft->device));
        CK(cudaMemcpy(&dt, draft->state + ST_LAST_TOKEN, 4, cudaMemcpyDeviceToHost));
        while (n < n_gen)
            if ((st = spec_cycle_reference_shape(target, draft, k, n_gen, out_tokens, stats, n, pos, tt, dt, hist)))
                return st;
        return NCM_OK;
    }
    // all prompt tokens but the last through both models; the last one is pending
    if (n_prompt > 1) {
        if ((st = ncm_prefill_tokens(target, prompt, n_prompt - 1, nullptr))) return st;
        if ((st = ncm_prefill_tokens(draft, prompt, n_prompt - 1, nullptr))) return st;
    }
    int cur = prompt[n_prompt - 1], q = n_prompt - 1;   // pending token and its position
    while (n < n_gen) {
        // draft: ingest the pending token at q, then propose d0 .. d(k-1) at q+1 .. q+k
        CK(cudaSetDevice(draft->device));
        draft->h_stage[2] = cur;
        CK(cudaMemcpyAsync(draft->tokens + q, &draft->h_stage[2], 4, cudaMemcpyHostToDevice, draft->stream));
        if ((st = set_pos(draft, q, q + 1, draft->stream))) return st;
        if ((st = ncm_decode_steps(draft, k, nullptr))) return st;
        if ((st = ncm_sync_tokens(draft, hist.data(), q + k + 1, nullptr))) return st;
        int rows_in[kMaxBatch], g[kMaxBatch];
        rows_in[0] = cur;
        for (int i = 0; i < k; ++i) rows_in[i + 1] = hist[q + 1 + i];
        if (stats) stats[0] += k;
        // target: the pending token and every proposal in one (k+1)-row pass; row i
        // predicts position q+i+1
        if ((st = ncm_verify_batch(target, rows_in, k + 1, q, g))) return st;
        int i = 0;
        while (i < k && rows_in[i + 1] == g[i]) {
            if (n < n_gen) out_tokens[n++] = rows_in[i + 1];
            if (stats) stats[1] += 1;
            ++i;
        }
        const int next = g[i];   // correction, or the trailing token when all k agreed
        if (n < n_gen) out_tokens[n++] = next;
        if (i == k) {
            // the draft fed d0 .. d(k-2); its cache also needs d(k-1) at q+k
            CK(cudaSetDevice(draft->device));
            draft->h_stage[2] = rows_in[k];
            CK(cudaMemcpyAsync(draft->tokens + q + k, &draft->h_stage[2], 4, cudaMemcpyHostToDevice, draft->stream));
            if ((st = set_pos(draft, q + k, q + k + 1, draft->stream))) return st;
            if ((st = ncm_decode_steps(draft, 1, nullptr))) return st;
            // the pinned staging words are rewritten by the next cycle
            CK(cudaStreamSynchronize(draft->stream));
        }
        cur = next;
        q += i + 1;
    }
    CK(cudaSetDevice(draft->device));
    CK(cudaStreamSynchronize(draft->stream));
    return check_err(draft);
}

// ------------------------------------------------------------------ n-gram speculation
// speculative.rs:80-105 NGramDrafter::draft (host only): the longest suffix n-gram of
// the history (max_ngram down to min_ngram) that occurred earlier, its most recent
// occurrence; the tokens that followed it (up to max_tokens, inside the history).
extern "C" int ncm_ngram_draft(const int* history, int len, int max_tokens, int max_ngram, int min_ngram, int* out) {
    if (!history || !out || len < 0 || max_tokens <= 0 || min_ngram <= 0 || len <= min_ngram) return 0;
    const int max_n = std::min(max_ngram, len - 1);
    for (int n = max_n; n >= min_ngram; --n) {
        const int* pat = history + len - n;
        for (int start = len - n - 1; start >= 0; --start) {
            if (!std::equal(pat, pat + n, history + start)) continue;
            const int cs = start + n, ce = std::min(cs + max_tokens, len);
            if (cs >= ce) break;
            std::copy(history + cs, history + ce, out);
            return ce - cs;
        }
    }
    return 0;
}

// speculative.rs:122-297 ngram_speculative_step at temperature 0, driven as
// main.rs:9720-9760 (k per step = min(k, remaining - 1)): the target's own token t0
// plus the drafts from the history go through one multi-row pass (t0 is row 0); the
// agreeing drafts are emitted, the first disagreement emits the target's token and
// runs the corrective one-token step.  Output = the target's greedy decode.
extern "C" ncm_status ncm_ngram_generate(ncm_model* m, const int* prompt, int n_prompt, int n_gen, int k, int max_ngram,
                                        int min_ngram, int* out_tokens, int* stats) {
    if (!m || !prompt || !out_tokens || n_prompt < 1 || n_gen < 0 || k < 0)
        return fail(NCM_EINVAL, "bad n-gram speculative arguments");
    if (n_prompt + n_gen > m->ctx) return fail(NCM_EINVAL, "prompt + generation exceeds the context");
    if (stats) stats[0] = stats[1] = 0;
    ncm_status st = ncm_prefill_tokens(m, prompt, n_prompt, nullptr);
    if (st) return st;
    int pred = 0, p0 = 0;
    if ((st = ncm_sync_tokens(m, nullptr, 0, &p0))) return st;
    CK(cudaMemcpy(&pred, m->state + ST_LAST_TOKEN, 4, cudaMemcpyDeviceToHost));
    std::vector<int> hist(prompt, prompt + n_prompt), drafts(std::max(k, 1));
    int pos = n_prompt, n = 0;
    while (n < n_gen && pos < m->ctx) {
        const int cur_k = std::min(k, n_gen - n - 1);
        const int t0 = pred;
        hist.push_back(t0);   // the draft sees the history plus t0
        int nd = cur_k > 0 ? ncm_ngram_draft(hist.data(), (int)hist.size(), cur_k, max_ngram, min_ngram, drafts.data()) : 0;
        nd = std::min(nd, std::min(kMaxBatch - 1, m->ctx - (pos + 1)));
        out_tokens[n++] = t0;
        if (nd <= 0) {
            if ((st = ncm_forward_pass(m, t0, pos, nullptr, &pred))) return st;
            pos += 1;
            continue;
        }
        if (stats) stats[0] += nd;
        int rows[kMaxBatch], g[kMaxBatch];
        rows[0] = t0;
        for (int i = 0; i < nd; ++i) rows[i + 1] = drafts[i];
        if ((st = ncm_verify_batch(m, rows, nd + 1, pos, g))) return st;
        int i = 0;
        for (; i < nd; ++i) {
            const int tt = g[i];
            if (drafts[i] == tt && stats) stats[1] += 1;
            if (n < n_gen) out_tokens[n++] = tt;
            hist.push_back(tt);
            if (drafts[i] != tt) {
                // corrective step: replaces the rejected draft's K/V, predicts the next position
                if ((st = ncm_forward_pass(m, tt, pos + i + 1, nullptr, &pred))) return st;
                pos += i + 2;
                break;
            }
        }
        if (i == nd) {
            pred = g[nd];
            pos += nd + 1;
        }
    }
    return NCM_OK;
}

// ------------------------------------------------------------------ tensor parallel
extern "C" ncm_status ncm_tp_export(ncm_model* m, uint8_t* handle_out) {
    if (!m || !handle_out) return fail(NCM_EINVAL, "null argument");
    if (m->world <= 1) return fail(NCM_EINVAL, "model is not sharded");
    CK(cudaSetDevice(m->device));
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, m->comm_base));
    memset(handle_out, 0, NCM_TP_HANDLE_BYTES);
    memcpy(handle_out, &h, sizeof h);
    uint64_t bytes = m->comm_bytes;
    memcpy(handle_out + 128, &bytes, 8);
    return NCM_OK;
}

extern "C" ncm_status ncm_tp_import(ncm_model* m, const uint8_t* handles, int world, int rank) {
    if (!m || !handles) return fail(NCM_EINVAL, "null argument");
    if (world != m->world || rank != m->rank) return fail(NCM_EPEER, "world/rank do not match the shard plan");
    CK(cudaSetDevice(m->device));
    TpComm c{};
    c.world = world;
    c.rank = rank;
    c.H = m->emb;
    c.grid_max = num_sms();
    c.timeout_ns = m->timeout_ns;
    for (int d = 0; d < world; ++d) {
        const uint8_t* hb = handles + (size_t)d * NCM_TP_HANDLE_BYTES;
        uint64_t bytes;
        memcpy(&bytes, hb + 128, 8);
        if (bytes != m->comm_bytes) return fail(NCM_EPEER, "peer exchange area size differs (different model?)");
        uint8_t* base;
        if (d == rank) base = m->comm_base;
        else {
            cudaIpcMemHandle_t h;
            memcpy(&h, hb, sizeof h);
            void* p = nullptr;
            cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) return fail(NCM_EPEER, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
            m->ipc_open.push_back(p);
            base = (uint8_t*)p;
        }
        c.recv[d] = (float*)base;
        c.flags[d] = (unsigned*)(base + m->off_flags);
        c.hx[d] = (float2*)(base + m->off_hx);
        c.hflags[d] = (unsigned*)(base + m->off_hflags);
        m->rows.rrecv[d] = (float*)(base + m->off_rrecv);
        m->rows.rflags[d] = (unsigned*)(base + m->off_rflags);
        m->rows.hrecv[d] = (float2*)(base + m->off_rhx);
        m->rows.hflags[d] = (unsigned*)(base + m->off_rhflags);
    }
    m->rows.world = world;
    m->rows.rank = rank;
    m->rows.grid_max = num_sms();
    m->rows.ctr = m->rows_ctr;
    m->rows.stride = (size_t)kMaxBatch * m->emb;
    m->rows.timeout_ns = m->timeout_ns;
    m->rows.err = m->err;
    m->comm = c;
    m->tp_ready = true;
    m->dirty = true;
    return NCM_OK;
}

extern "C" ncm_status ncm_nccl_unique_id(uint8_t* out) {
    if (!out) return fail(NCM_EINVAL, "null argument");
    if (!g_nccl.load()) return fail(NCM_EUNSUPPORTED, "libnccl.so.2 not found");
    nccl_uid id;
    if (g_nccl.GetUniqueId(&id) != 0) return fail(NCM_EPEER, "ncclGetUniqueId failed");
    memcpy(out, &id, 128);
    return NCM_OK;
}

extern "C" ncm_status ncm_tp_nccl_init(ncm_model* m, const uint8_t* unique_id, int world, int rank) {
    if (!m || !unique_id) return fail(NCM_EINVAL, "null argument");
    if (world != m->world || rank != m->rank) return fail(NCM_EPEER, "world/rank do not match the shard plan");
    if (!g_nccl.load()) return fail(NCM_EUNSUPPORTED, "libnccl.so.2 not found");
    CK(cudaSetDevice(m->device));
    nccl_uid id;
    memcpy(&id, unique_id, 128);
    if (g_nccl.CommInitRank(&m->nccl, world, id, rank) != 0) return fail(NCM_EPEER, "ncclCommInitRank failed");
    return NCM_OK;
}

extern "C" ncm_status ncm_tp_set_reducer(ncm_model* m, int mode) {
    if (!m) return fail(NCM_EINVAL, "null model");
    if (mode != NCM_REDUCE_FUSED_P2P && mode != NCM_REDUCE_NCCL && mode != NCM_REDUCE_HOST_CALLBACK)
        return fail(NCM_EINVAL, "unknown reducer");
    if (mode == NCM_REDUCE_NCCL && m->world > 1 && !m->nccl) return fail(NCM_EINVAL, "NCCL communicator not initialised");
    if (mode == NCM_REDUCE_HOST_CALLBACK && !m->host_fn) return fail(NCM_EINVAL, "no host reducer registered");
    m->reduce_mode = mode;
    m->dirty = true;
    if (m->world > 1)
        m->tp_ready = mode == NCM_REDUCE_NCCL ? m->nccl != nullptr
                      : mode == NCM_REDUCE_HOST_CALLBACK ? true
                                                          : m->comm.world == m->world;
    return NCM_OK;
}

extern "C" ncm_status ncm_tp_set_host_reducer(ncm_model* m, ncm_host_reduce_fn fn, void* user) {
    if (!m || !fn) return fail(NCM_EINVAL, "null argument");
    CK(cudaSetDevice(m->device));
    CK(cudaStreamSynchronize(m->stream));
    if (!m->h_red) CK(cudaMallocHost((void**)&m->h_red, 4 * (size_t)kMaxBatch * std::max(m->emb, 2)));
    m->host_fn = fn;
    m->host_user = user;
    return NCM_OK;
}

extern "C" ncm_status ncm_tp_set_timeout_ns(ncm_model* m, uint64_t ns) {
    if (!m || ns == 0) return fail(NCM_EINVAL, "bad arguments");
    m->timeout_ns = ns;
    m->comm.timeout_ns = ns;
    m->rows.timeout_ns = ns;
    m->dirty = true;
    return NCM_OK;
}

extern "C" ncm_status ncm_test_peer_timeout(int device, uint64_t timeout_ns) {
    CK(cudaSetDevice(device));
    unsigned* flags = nullptr;
    int* err = nullptr;
    CK(cudaMalloc(&flags, 64));
    CK(cudaMalloc(&err, 4));
    CK(cudaMemset(flags, 0, 64));
    CK(cudaMemset(err, 0, 4));
    TpComm c{};
    c.world = 2;
    c.rank = 0;
    c.flags[0] = flags;
    c.flags[1] = flags + 8;
    c.timeout_ns = timeout_ns;
    int r = peer_timeout_test_launch(c, err, nullptr);
    cudaError_t e = cudaDeviceSynchronize();
    int h = 0;
    cudaMemcpy(&h, err, 4, cudaMemcpyDeviceToHost);
    cudaFree(flags);
    cudaFree(err);
    if (r != 0 || e != cudaSuccess) return fail(NCM_ECUDA, "peer timeout test launch failed");
    if (h & NCM_DEVERR_PEER_TIMEOUT) return fail(NCM_ETIMEOUT, "peer wait timed out (expected)");
    return NCM_OK;
}

// ------------------------------------------------------------------ kernel seams
static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

extern "C" ncm_status ncm_quantize_f32_to_q8_0(const float* x, int n, int8_t* x_i8, float* x_scales, void* stream) {
    if (n < 0 || n % 32) return fail(NCM_EINVAL, "n must be a multiple of 32");
    if (n && (!x || !x_i8 || !x_scales)) return fail(NCM_EINVAL, "null pointer");
    CKL(quantize_launch(x, n, x_i8, x_scales, (cudaStream_t)stream));
    return NCM_OK;
}

// Stream-ordered device scratch, freed (stream-ordered) when the scope ends, early
// returns included.
struct AsyncScratch {
    uint8_t* p = nullptr;
    cudaStream_t s = nullptr;
    ~AsyncScratch() {
        if (p) cudaFreeAsync(p, s);
    }
};

// Caller-owned raw block rows as the kernels address them: rows whose byte length is not
// a multiple of `align` (or an unaligned base) are copied into a 16-byte-pitched scratch.
static ncm_status addressable_rows(const void* w, int64_t rows, int rb, int align, cudaStream_t s, AsyncScratch& tmp,
                                   const uint8_t** base, int64_t* pitch) {
    *base = (const uint8_t*)w;
    *pitch = rb;
    if (rb % align == 0 && ((uintptr_t)w % align) == 0) return NCM_OK;
    *pitch = (rb + 15) / 16 * 16;
    tmp.s = s;
    CK(cudaMallocAsync((void**)&tmp.p, (size_t)*pitch * rows, s));
    CK(cudaMemcpy2DAsync(tmp.p, (size_t)*pitch, w, rb, rb, rows, cudaMemcpyDeviceToDevice, s));
    *base = tmp.p;
    return NCM_OK;
}

// Strict GEMV over caller-owned raw blocks (TMA: 16-byte row pitch).
static ncm_status seam_gemv(int qtype, const void* w, int64_t rows, int cols, const int8_t* x_i8,
                            const float* x_scales, float* out, cudaStream_t s) {
    AsyncScratch tmp;
    const uint8_t* base = nullptr;
    int64_t pitch = 0;
    ncm_status st = addressable_rows(w, rows, row_bytes(qtype, cols), 16, s, tmp, &base, &pitch);
    if (st) return st;
    GemvParams p;
    memset(&p, 0, sizeof p);
    p.nseg = 1;
    p.seg[0] = {out, (int)rows, 0, SEG_OUT};
    p.xq = x_i8;
    p.xs = x_scales;
    p.tp.world = 1;
    const int grid = gemv_plan(qtype, cols, (int)rows, false, IN_Q8, p);
    int r = grid < 0 ? (int)cudaErrorInvalidValue
                     : gemv_tensor_map(&p.tm[0], base, rows, (int)pitch, p.chunk_words, p.box_rows);
    if (!r) r = gemv_launch(qtype, IN_Q8, EPI_PLAIN, p, grid, s, false);
    if (r) return fail(NCM_ECUDA, std::string("gemv launch: ") + cudaGetErrorString((cudaError_t)r));
    return NCM_OK;
}

extern "C" ncm_status ncm_matmul_quantized(int qtype, const void* w, int64_t rows, int cols, const int8_t* x_i8,
                                          const float* x_scales, float* out, void* stream) {
    if (qtype == NCM_T_Q6_K) {
        // inference.rs:3045-3087 matmul_q6_k
        if (rows < 0 || rows >= (1ll << 31) || cols <= 0 || cols % 256 || cols > 32768)
            return fail(NCM_EINVAL, "Q6_K: cols must be a positive multiple of 256, at most 32768");
        if (rows == 0) return NCM_OK;
        if (!w || !x_i8 || !x_scales || !out) return fail(NCM_EINVAL, "null pointer");
        cudaStream_t s = (cudaStream_t)stream;
        AsyncScratch tmp;
        const uint8_t* base = nullptr;
        int64_t pitch = 0;
        ncm_status st = addressable_rows(w, rows, row_bytes(qtype, cols), 16, s, tmp, &base, &pitch);
        if (st) return st;
        Q6Params q;
        memset(&q, 0, sizeof q);
        q.w = base; q.pitch = pitch; q.rows = (int)rows; q.cols = cols; q.xq = x_i8; q.xs = x_scales; q.out = out;
        CKL(q6k_gemv_launch(EPI_PLAIN, q, s, false));
        return NCM_OK;
    }
    if (!gemv_type_ok(qtype)) return fail(NCM_EUNSUPPORTED, "quant type outside Q4_0/Q8_0/Q4_K/Q6_K");
    if (rows < 0 || rows >= (1ll << 31) || cols <= 0 || cols % 32 || cols % ncm_type_block_elems(qtype) ||
        cols > 32768)
        return fail(NCM_EINVAL, "cols must be a positive multiple of 32 (256 for Q4_K), at most 32768");
    if (rows == 0) return NCM_OK;
    if (!w || !x_i8 || !x_scales || !out) return fail(NCM_EINVAL, "null pointer");
    if (!aligned16(x_i8) || ((uintptr_t)x_scales & 3)) return fail(NCM_EINVAL, "x_i8 must be 16-byte and x_scales 4-byte aligned");
    return seam_gemv(qtype, w, rows, cols, x_i8, x_scales, out, (cudaStream_t)stream);
}

// inference.rs:1246-1303: every token's row uses the single-token formula; the int8
// tensor-core kernel forms the same integer dots and f32 terms, folded in block order,
// so every row is bit-identical to ncm_matmul_quantized of that row.
extern "C" ncm_status ncm_matmul_quantized_batch(int qtype, const void* w, int64_t rows, int cols, int ntok,
                                                const int8_t* x_i8, const float* x_scales, float* out, void* stream) {
    if (ntok < 1 || ntok > kMaxBatch) return fail(NCM_EINVAL, "1 <= ntok <= 8");
    if (!gemv_type_ok(qtype)) return fail(NCM_EUNSUPPORTED, "quant type outside Q4_0/Q8_0/Q4_K");
    if (rows <= 0 || rows > (1 << 30) || cols <= 0 || cols % ncm_type_block_elems(qtype) || cols % 32)
        return fail(NCM_EINVAL, "bad shape");
    if (!w || !x_i8 || !x_scales || !out) return fail(NCM_EINVAL, "null pointer");
    if ((uintptr_t)x_i8 & 15) return fail(NCM_EINVAL, "x_i8 must be 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    AsyncScratch tmp;
    const uint8_t* base = nullptr;
    int64_t pitch = 0;
    ncm_status s = addressable_rows(w, rows, row_bytes(qtype, cols), 16, st, tmp, &base, &pitch);
    if (s) return s;
    BatchParams p;
    memset(&p, 0, sizeof p);
    p.nseg = 1;
    p.seg[0] = {out, (int)rows, 0, SEG_OUT};
    p.total_rows = (int)rows;
    p.out_stride = (int)rows;
    p.xq = x_i8;
    p.xs = x_scales;
    const int grid = batch_plan(qtype, cols, (int)rows, false, ntok, p);
    if (grid < 0) return fail(NCM_EUNSUPPORTED, "no launch plan for this shape");
    AsyncScratch sums;
    if (p.x_global) {
        // rows read in place: their per-block sums come from a small pass into scratch
        const int64_t nblk = (int64_t)ntok * (cols / 32);
        sums.s = st;
        CK(cudaMallocAsync((void**)&sums.p, 4 * (size_t)nblk, st));
        CKL(block_sums_launch(x_i8, nblk, (int*)sums.p, st));
        p.xsum = (const int*)sums.p;
    }
    int r = gemv_tensor_map(&p.tm[0], base, rows, (int)pitch, p.chunk_words, p.box_rows);
    if (!r) r = batch_gemv_launch(qtype, EPI_PLAIN, p, grid, st, false);
    if (r) return fail(NCM_ECUDA, std::string("batch gemv launch: ") + cudaGetErrorString((cudaError_t)r));
    return NCM_OK;
}

extern "C" ncm_status ncm_block_dots(int qtype, const void* w, int64_t rows, int cols, const int8_t* x_i8,
                                    int32_t* out, void* stream) {
    if (!gemv_type_ok(qtype)) return fail(NCM_EUNSUPPORTED, "quant type outside Q4_0/Q8_0/Q4_K");
    if (rows < 0 || cols <= 0 || cols % 32 || cols % ncm_type_block_elems(qtype)) return fail(NCM_EINVAL, "bad shape");
    if (rows == 0) return NCM_OK;
    if (!w || !x_i8 || !out) return fail(NCM_EINVAL, "null pointer");
    if (((uintptr_t)x_i8 & 3) || ((uintptr_t)w & 3)) return fail(NCM_EINVAL, "w and x_i8 must be 4-byte aligned");
    // The unit code loads 32-bit words: rows of an odd block count (Q4_0 / Q8_0 rows of
    // 18 / 34 bytes per block) are re-pitched to 16 bytes first, as in the GEMV seam.
    cudaStream_t s = (cudaStream_t)stream;
    AsyncScratch tmp;
    const uint8_t* base = nullptr;
    int64_t pitch = 0;
    ncm_status st = addressable_rows(w, rows, row_bytes(qtype, cols), 4, s, tmp, &base, &pitch);
    if (st) return st;
    const int r = block_dots_launch(qtype, base, rows, cols, pitch, x_i8, out, s);
    if (r) return fail(NCM_ECUDA, std::string("block dots launch: ") + cudaGetErrorString((cudaError_t)r));
    return NCM_OK;
}

extern "C" ncm_status ncm_rms_norm(float* out, const float* x, const float* weight, int n, float eps, void* stream) {
    if (!out || !x || !weight || n <= 0 || n > 65536) return fail(NCM_EINVAL, "bad arguments");
    CKL(rms_norm_launch(out, x, weight, n, eps, (cudaStream_t)stream));
    return NCM_OK;
}

extern "C" ncm_status ncm_fused_silu_mul(float* out, const float* gate, const float* up, int n, void* stream) {
    if (n < 0 || (n && (!out || !gate || !up))) return fail(NCM_EINVAL, "bad arguments");
    {
        int dev = 0;
        CK(cudaGetDevice(&dev));
        ncm_status st = ensure_expf_table(dev);
        if (st) return st;
    }
    CKL(silu_mul_launch(out, gate, up, n, (cudaStream_t)stream));
    return NCM_OK;
}

extern "C" ncm_status ncm_attention(float* out, const float* q, const float* k_cache, const float* v_cache, int pos,
                                   int heads, int kv_heads, int head_dim, void* stream) {
    if (!out || !q || !k_cache || !v_cache || pos < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads ||
        heads / kv_heads > 8 || head_dim % 32 || head_dim > 256 || pos >= 16384)
        return fail(NCM_EINVAL, "bad attention arguments");
    cudaStream_t s = (cudaStream_t)stream;
    {
        int dev = 0;
        CK(cudaGetDevice(&dev));
        ncm_status st = ensure_expf_table(dev);
        if (st) return st;
    }
    float* scores = nullptr;
    const int ctx = pos + 1;
    CK(cudaMallocAsync((void**)&scores, 4 * (size_t)heads * ctx, s));
    AttnParams a;
    memset(&a, 0, sizeof a);
    a.q = q; a.kc = k_cache; a.vc = v_cache; a.out = out; a.scores = scores; a.state = nullptr;
    a.pos_override = pos;
    a.heads = heads; a.kv_heads = kv_heads; a.hd = head_dim; a.kvw = kv_heads * head_dim; a.ctx = ctx;
    a.scale = 1.0f / sqrtf((float)head_dim);
    a.vmap_on = 1;
    a.sv_on = 1;
    int r = attention_launch(a, s, false);
    cudaFreeAsync(scores, s);
    CK(cudaStreamSynchronize(s));
    if (r) return fail(NCM_ECUDA, "attention launch failed");
    return NCM_OK;
}

// inference.rs:4142-4458 apply_attention_heads over an F16 (kind 1) or Q8_0 (kind 2) cache
// ([ctx][kv_heads*head_dim] u16, or [ctx][kv_heads*head_dim/32] 34-byte blocks); kind 0
// is ncm_attention.
extern "C" ncm_status ncm_attention_kv(int kind, float* out, const float* q, const void* k_cache, const void* v_cache,
                                      int pos, int heads, int kv_heads, int head_dim, void* stream) {
    if (kind == KV_F32)
        return ncm_attention(out, q, (const float*)k_cache, (const float*)v_cache, pos, heads, kv_heads, head_dim, stream);
    if (kind != KV_F16 && kind != KV_Q8_0) return fail(NCM_EINVAL, "bad KV-cache kind");
    if (!out || !q || !k_cache || !v_cache || pos < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads ||
        heads / kv_heads > 8 || head_dim % 32 || head_dim > 256 || pos >= 16384)
        return fail(NCM_EINVAL, "bad attention arguments");
    cudaStream_t s = (cudaStream_t)stream;
    {
        int dev = 0;
        CK(cudaGetDevice(&dev));
        ncm_status st = ensure_expf_table(dev);
        if (st) return st;
    }
    float* scores = nullptr;
    CK(cudaMallocAsync((void**)&scores, 4 * (size_t)heads * (pos + 1), s));
    AttnParams a;
    memset(&a, 0, sizeof a);
    a.q = q; a.out = out; a.scores = scores; a.pos_override = pos;
    a.kv_kind = kind; a.kc_raw = k_cache; a.vc_raw = v_cache;
    a.heads = heads; a.kv_heads = kv_heads; a.hd = head_dim; a.kvw = kv_heads * head_dim; a.ctx = pos + 1;
    a.scale = 1.0f / sqrtf((float)head_dim);
    int r = attention_launch(a, s, false);
    cudaFreeAsync(scores, s);
    CK(cudaStreamSynchronize(s));
    if (r) return fail(NCM_ECUDA, "attention launch failed");
    return NCM_OK;
}

// ------------------------------------------------------------------ allocation-free attention
// Scores scratch for ncm_attention_noalloc: a fixed array that lives in every GPU that
// loads this library until the process exits (1 MiB per device).
static constexpr int64_t kNoAllocScores = 262144;   // floats: heads * (pos + 1) at most
static __device__ __align__(256) float g_noalloc_scores[kNoAllocScores];

// Host code cannot use g_noalloc_scores directly (the host symbol is only a stand-in for
// the device array); its device address is looked up once per device, with that device
// current, and cached here.
static float* noalloc_scores_ptr(int device, cudaError_t* err) {
    static std::mutex mu;
    static float* ptrs[64] = {nullptr};
    *err = cudaSuccess;
    if (device < 0 || device >= 64) { *err = cudaErrorInvalidDevice; return nullptr; }
    std::lock_guard<std::mutex> lk(mu);
    if (!ptrs[device]) {
        void* p = nullptr;
        *err = cudaGetSymbolAddress(&p, g_noalloc_scores);
        if (*err != cudaSuccess) return nullptr;
        ptrs[device] = (float*)p;
    }
    return ptrs[device];
}

extern "C" ncm_status ncm_attention_noalloc(float* out, const float* q, const float* k_cache, const float* v_cache,
                                           int pos, int heads, int kv_heads, int head_dim, void* stream) {
    if (!out || !q || !k_cache || !v_cache || pos < 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads ||
        heads / kv_heads > 8 || head_dim % 32 || head_dim > 256 || pos >= 16384)
        return fail(NCM_EINVAL, "bad attention arguments");
    if ((int64_t)heads * (pos + 1) > kNoAllocScores)
        return fail(NCM_EINVAL, "ncm_attention_noalloc: heads * (pos + 1) = " + std::to_string((int64_t)heads * (pos + 1)) +
                                    " exceeds the fixed scratch of " + std::to_string(kNoAllocScores) +
                                    " floats; use ncm_attention");
    int dev = 0;
    CK(cudaGetDevice(&dev));
    {
        // glibc-exact exp: the exception table is copied into its own fixed in-library
        // array on the first call on this device (host work plus a copy, no allocation)
        ncm_status st = ensure_expf_table(dev);
        if (st) return st;
    }
    cudaError_t e;
    float* scores = noalloc_scores_ptr(dev, &e);
    if (!scores) return fail(NCM_ECUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    AttnParams a;
    memset(&a, 0, sizeof a);
    a.q = q; a.kc = k_cache; a.vc = v_cache; a.out = out; a.scores = scores; a.state = nullptr;
    a.pos_override = pos;
    a.heads = heads; a.kv_heads = kv_heads; a.hd = head_dim; a.kvw = kv_heads * head_dim; a.ctx = pos + 1;
    a.scale = 1.0f / sqrtf((float)head_dim);
    CKL(attention_launch(a, (cudaStream_t)stream, false));
    return NCM_OK;
}
