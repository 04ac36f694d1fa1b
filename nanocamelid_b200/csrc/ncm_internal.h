// Internal structures shared by kernels.cu (device code + launchers) and engine.cu
// (model, decode graph, tensor parallel plumbing).  Not part of the C ABI.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ncm {

constexpr int kThreads = 256;   // GEMV CTA size (8 warps)
constexpr int kMaxSeg = 3;      // weight matrices fused into one GEMV launch (wq, wk, wv)
constexpr int kMaxWorld = 8;    // GPUs of one NVSwitch box
constexpr int kChunkCols = 512; // columns per TMA chunk: 16 Q4_0/Q8_0 blocks or 2 Q4_K super-blocks
constexpr int kUnits = 8;       // 64-column units per chunk
constexpr int kTStride = 17;    // per-row stride (floats) of the per-block term buffer (conflict-free)
constexpr int kMaxFold = 64;    // fold lanes (rows) per tile
constexpr int kMaxStages = 8;   // GEMV ring stages (one per compute warp)

// Input modes of the GEMV prologue.
enum InMode { IN_F32 = 0, IN_F32_RMS = 1, IN_Q8 = 2 };
// Epilogue modes.
enum EpiMode {
    EPI_PLAIN = 0,   // out[row] = sum
    EPI_RESID = 1,   // hidden[row] += sum              (wo / w2, one GPU)
    EPI_QKV = 2,     // RoPE on q,k; k,v into the KV cache at pos
    EPI_SILU = 3,    // dual matrices: out[row] = silu(g) * u  (w1 / w3)
    EPI_ARGMAX = 4,  // logits + greedy argmax, token appended, position advanced
    EPI_TP_RESID = 5 // partial rows stored into every peer, rank-ordered sum + residual
};
// Per-segment epilogue kinds inside EPI_QKV.
enum SegKind { SEG_Q = 0, SEG_K = 1, SEG_V = 2, SEG_OUT = 3 };

// Device decode state (one int array per model).
enum StateIdx { ST_POS = 0, ST_STEP = 1, ST_NPROMPT = 2, ST_LAST_TOKEN = 3, ST_COUNT = 8 };

struct Seg {
    float* out;         // destination of this segment's rows
    int rows;
    int row_begin;      // first row of the segment in the fused row space
    int kind;           // SegKind
};

// Peer-memory view of the tensor-parallel exchange buffers (identical layout on all ranks).
struct TpComm {
    int world, rank;
    float* recv[kMaxWorld];       // recv[dst] -> rank dst's receive area (this rank's pointer to it)
    unsigned* flags[kMaxWorld];   // flags[dst] -> rank dst's flag area
    float2* hx[kMaxWorld];        // head argmax exchange slots (val, idx-as-float-bits) per rank
    unsigned* hflags[kMaxWorld];
    int H;                        // hidden size (rows of the reduced vectors)
    int grid_max;                 // CTA slots per reduction slot
    uint64_t timeout_ns;
};

// Device-side reduction of a multi-row pass's row-parallel partials and head pairs
// under tensor parallelism (speculative verify, batched prefill): the same rank-order
// sums as the one-row fused reduction, as stand-alone kernels after the batch GEMV.
// Exchange areas (every rank's own, IPC-mapped by its peers):
//   rrecv[dst] -> [2 parities][world][kMaxBatch * H] f32, rflags[dst] -> [grid_max][world]
//   hrecv[dst] -> [2][world][kMaxBatch] float2,           hflags[dst] -> [world]
// The epoch of each use comes from a counter in this rank's own memory (every rank runs
// the same sequence of multi-row reductions): the kernel reads it at the start and the
// last CTA to finish advances it.
struct TpRows {
    int world, rank, grid_max;
    float* rrecv[kMaxWorld];
    unsigned* rflags[kMaxWorld];
    float2* hrecv[kMaxWorld];
    unsigned* hflags[kMaxWorld];
    unsigned* ctr;                // [4]: reduce epoch, reduce CTAs done, head epoch, (unused)
    size_t stride;                // floats per (parity, rank) slot of rrecv: kMaxBatch * H
    uint64_t timeout_ns;
    int* err;
};

struct alignas(64) GemvParams {
    CUtensorMap tm[kMaxSeg];      // weights: dims {pitch/4 words, rows}, box {chunk_words, box_rows}
    CUtensorMap tm2;              // EPI_SILU: the up matrix (same shape as tm[0])
    Seg seg[kMaxSeg];
    int nseg;
    int fused;                    // 1: the segments' matrices are one buffer under tm[0]
    int total_rows;
    int cols, nb, nchunk;         // columns, 32-column blocks per row, 512-column chunks per row
    int chunk_words, chunk_bytes; // TMA box inner extent per row
    int box_rows;                 // rows per tile (TMA box outer extent)
    int stage_bytes, nstages;
    int xq_off, xs_off, xsum_off, xf_off, nw_off, t_off, stage_off, smem_bytes;
    // input
    const float* x;               // IN_F32 / IN_F32_RMS
    const float* norm_w;
    float eps;
    const float* ssq_tok;         // layer 0: sequential sum of squares per vocab row (or null)
    const int8_t* xq;             // IN_Q8
    const float* xs;
    // epilogue context
    float* hidden;                // EPI_TP_RESID target
    int* state;                   // StateIdx array
    const float2* rope;           // [ctx][rope_half] (sin, cos)
    int rope_half, head_dim;
    float* kcache; float* vcache; // this layer's [ctx][kv_width] caches
    int kv_width;
    int* tokens;                  // token history [ctx]
    float2* amax_part;            // [grid] (val, idx bits)
    unsigned* counter;
    int head_row0;                // global vocab row of this shard's first head row
    float2* head_out;             // NCCL baseline: local (logit, token) only, no state update
    int ctx;
    TpComm tp;
    int tp_slot;                  // layer*2 + phase
    int* err;
    int kv_stage;                 // 1: K / V rows go to kcache / vcache as given (staging for an
                                  //    F16 / Q8_0 cache), 0: the f32 cache rows at pos
    int row_align;                // CTA row ranges start at multiples of this (2, or 32 with qout)
    int tune;                     // measurement knobs (0 in normal use; 16: full-width rows on short tiles)
    int cgroups;                  // compute-warp groups (1, 2 or 4; 0: 4): stages worked on at once

    uint64_t* dbg_ts;             // measurement probe: per-CTA phase stamps [grid][8] (null in normal use)
    int8_t* qout;                 // EPI_SILU: the output rows also as Q8_0 blocks (box_rows == 32) ...
    float* qout_s;                //   ... and their scales: the next projection's quantised input
    // L2 prefetch of the next kernel's weights once this CTA has issued its own loads:
    // up to pf_bytes of this CTA's share (rows [b*pf_rows/pf_grid, ...)) of each matrix.
    const uint8_t* pf_base[kMaxSeg + 1];
    int64_t pf_pitch[kMaxSeg + 1];
    int pf_rows[kMaxSeg + 1];
    int pf_nmat, pf_grid, pf_dual;
    int64_t pf_bytes;
};

struct alignas(64) AttnParams {
    CUtensorMap vmap;        // optional: this layer's f32 V cache [ctx][kvw], box 32 x kAvChunk (vmap_on)
    const float* q;          // [heads_local * hd] roped
    const float* kc;         // layer cache [ctx][kvw]
    const float* vc;
    float* scores;           // [heads_local][ctx] scratch
    float* out;              // [heads_local * hd]
    const int* state;
    int pos_override;        // >= 0: use instead of state[ST_POS]
    int heads, kv_heads, hd, kvw, ctx;
    float scale;
    int ntok;                // rows in one launch (grid z): token z at position pos + z, q / out at
    int tok_stride;          //   + z * tok_stride floats, scores at + z * heads * ctx
    int8_t* out_q;           // when set (one row): the output also as Q8_0
    float* out_s;            //   blocks (quantize_f32_to_q8_0), the next projection's input
    int kv_kind;             // cache storage: 0 f32 (kc / vc), 1 F16, 2 Q8_0 (kc_raw / vc_raw)
    const void* kc_raw;
    const void* vc_raw;
    int vmap_on;             // V chunks by TMA through vmap (f32 cache)
    int sv_on;               // with vmap_on: softmax and V accumulation in one launch
    int* err;                // device error word for bounded waits (may be null)
};

// KV-cache storage kinds (inference.rs:505-599; NANOCAMELID_KV_CACHE_F16 / _Q8).
enum KvKind { KV_F32 = 0, KV_F16 = 1, KV_Q8_0 = 2 };

// Multi-row (speculative verify) GEMV: ntok activation rows share every weight tile;
// int8 tensor-core MMA forms the block dots (16 weight rows x 8 token rows per
// instruction), each (row, token) chain is folded in block order as in the one-row GEMV.
constexpr int kMaxBatch = 8;
struct alignas(64) BatchParams {
    CUtensorMap tm[kMaxSeg];
    CUtensorMap tm2;              // EPI_SILU: the up matrix
    Seg seg[kMaxSeg];             // seg.out: token 0's destination (token t at + t * out_stride)
    int nseg, total_rows;
    int cols, nb, nchunk, chunk_words, chunk_bytes, box_rows, stage_bytes, nstages;
    int xq_off, xs_off, xsum_off, stage_off, smem_bytes, xq_pitch;
    int nslab;                    // 16-row slabs per tile (one fold warp each)
    int cgroups;                  // compute-warp groups (1, 2, or 4 with one slab; 0: 2)
    int t_off;                    // term ring (one slot per stage)
    int ntok;
    const int8_t* xq;             // [ntok][cols] quantised rows
    const float* xs;              // [ntok][cols / 32]
    const int* xsum;              // [ntok][cols / 32] per-block sums of xq (read when x_global)
    int x_global;                 // 1: rows too wide for shared memory, read from xq / xs / xsum
    const float* xf;              // when set: f32 rows [ntok][xf_stride], quantised in the prologue
    int xf_stride;
    int out_stride;
    float* hidden;                // EPI_RESID: hidden[t * hidden_stride + row] += sum
    int hidden_stride;
    int pos0;                     // EPI_QKV: position of token 0 (token t at pos0 + t) ...
    const int* pos_dev;           // ... or read from device memory when set (graph replay)
    const float2* rope;
    int rope_half, head_dim;
    float* kcache; float* vcache;
    int kv_width;
    int kv_stage;                 // 1: token t's K / V row at kcache / vcache + t * kv_width (staging)
    float2* amax_part;            // EPI_ARGMAX: [grid][kMaxBatch]
    unsigned* counter;
    int* argmax_out;              // [ntok] global vocab rows
    float2* pair_out;             // or, when set: [ntok] (logit, token bits) of this vocab shard
    int head_row0;
    int* err;
};

// Q6_K GEMV (q8.rs:2092-2150 dot_q8_scaled, inference.rs:3045-3087 matmul_q6_k): one
// thread per output row folds the row's 256 products per super-block in the reference's
// order.  Input: Q8_0 activation in global memory.  Epilogues EPI_PLAIN, EPI_RESID,
// EPI_ARGMAX (one GPU, or head_out for a vocab shard).
struct Q6Params {
    const uint8_t* w;             // raw Q6_K rows, 16-byte aligned pitch
    int64_t pitch;
    int rows, cols;
    const int8_t* xq;             // [cols]
    const float* xs;              // [cols / 32]
    float* out;                   // EPI_PLAIN: out[row]; EPI_RESID: out[row] += ; EPI_ARGMAX: logits (or null)
    float2* amax_part;            // EPI_ARGMAX: [grid]
    unsigned* counter;
    int head_row0;
    float2* head_out;             // set: this shard's (logit, token) only, state untouched
    int* state;
    int* tokens;
    int ctx;
};


// Launchers (kernels.cu).
int q6k_gemv_launch(int epi, const Q6Params& p, cudaStream_t s, bool pdl);
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled_fn();
// Fills the layout fields of p for a (qtype, cols) matrix set with `rows` total rows; returns the grid.
int gemv_plan(int qtype, int cols, int rows, bool dual, int in_mode, GemvParams& p);
int gemv_tensor_map(CUtensorMap* tm, const void* base, int64_t rows, int pitch, int chunk_words, int box_rows);
int gemv_launch(int qtype, int in_mode, int epi, const GemvParams& p, int grid, cudaStream_t s, bool pdl);
int attention_launch(const AttnParams& a, cudaStream_t s, bool pdl);
// store_kv (inference.rs:539-568) of ntok staged f32 K / V rows [ntok][kw] into an F16 or
// Q8_0 cache (layer base kc / vc) at positions pos + t, pos = pos_dev[0] (+ pos_add).
int kv_store_launch(int kind, const float* sk, const float* sv, int ntok, int kw, void* kc, void* vc,
                    const int* pos_dev, cudaStream_t s, bool pdl);
int embed_ssq_launch(int type, const uint8_t* table, int64_t pitch, int emb, int vocab, float* out, cudaStream_t s);
int embed_launch(int type, const uint8_t* table, int64_t pitch, int emb, const int* tokens, int* state, int ctx,
                 int* err, float* hidden, cudaStream_t s, bool pdl);
int resid_add_launch(float* hidden, const float* part, int n, cudaStream_t s, bool pdl);
int tp_rows_reduce_launch(const TpRows& t, const float* part, float* hidden, int n, cudaStream_t s);
int tp_rows_argmax_launch(const TpRows& t, const float2* pairs, int ntok, int* argmax_out, cudaStream_t s);
int rows_argmax_merge_launch(const float2* gathered, int world, int ntok, int* argmax_out, cudaStream_t s);
int argmax_merge_launch(const float2* gathered, int world, int* tokens, int* state, int ctx, cudaStream_t s, bool pdl);
int advance_launch(int* state, cudaStream_t s, bool pdl);
int quantize_launch(const float* x, int n, int8_t* xq, float* xs, cudaStream_t s);
int block_dots_launch(int qtype, const uint8_t* w, int64_t rows, int cols, int64_t pitch, const int8_t* xq,
                      int32_t* out, cudaStream_t s);
int rms_norm_launch(float* out, const float* x, const float* w, int n, float eps, cudaStream_t s);
int silu_mul_launch(float* out, const float* g, const float* u, int n, cudaStream_t s);
int synth_launch(int type, uint64_t key, int64_t r0, int64_t nrows, int64_t c0, int64_t ncols, int64_t full_cols,
                 uint8_t* out, int64_t pitch, cudaStream_t s);
int requant_q4_0_launch(int src_type, const uint8_t* src, int64_t rows, int cols, int64_t src_pitch, uint8_t* dst,
                        int64_t dst_pitch, cudaStream_t s);
int peer_timeout_test_launch(TpComm c, int* err, cudaStream_t s);
int batch_plan(int qtype, int cols, int rows, bool dual, int ntok, BatchParams& p);
int batch_gemv_launch(int qtype, int epi, const BatchParams& p, int grid, cudaStream_t s, bool pdl);
int batch_prep_launch(const float* x, int x_stride, int n, int ntok, const float* norm_w, float eps,
                      const float* ssq_tab, const int* toks, int8_t* xq, float* xs, int* xsum, cudaStream_t s,
                      bool pdl);
int block_sums_launch(const int8_t* xq, int64_t nblocks, int* xsum, cudaStream_t s);
int embed_rows_launch(int type, const uint8_t* table, int64_t pitch, int emb, const int* toks, int ntok,
                      float* hidden, cudaStream_t s, bool pdl);
int num_sms();
// The glibc expf exception table: at most kExpfTabEntries {key, value} pairs, kept in a
// fixed in-library device array.
constexpr uint32_t kExpfTabEntries = 1u << 20;
int expf_table_install(const uint32_t* host_tab, size_t entries, uint32_t mask, int gate);
// libm_table.cpp
}  // namespace ncm
#include <vector>
namespace ncm {
// *gate = 0 when some exception lies outside the near-midpoint window the device checks
// first (then the device probes the table for every value).
std::vector<uint32_t> build_expf_exceptions(int threads, uint32_t max_entries, uint32_t* mask, size_t* count,
                                            int* gate);

}  // namespace ncm
