/*
 * ncm.h -- C ABI of the B200 decode hot path (libncm.so).
 *
 * The reference (timtoole02/NanoCamelid) is a Rust crate with no FFI; its seams are
 * Rust function signatures.  Each entry point below replaces one of them and says
 * which (file:line within the reference project).  Conventions:
 *   - plain pointers and sizes only; no torch or CUDA types (streams are `void*`
 *     holding a cudaStream_t, NULL = the legacy default stream);
 *   - every call returns an ncm_status; ncm_last_error() gives the message of the
 *     most recent failure on the calling thread;
 *   - "device" pointers are CUDA device memory owned by the caller; the library
 *     never frees them.  Execution is stream ordered;
 *   - a model handle is not re-entrant: one host thread drives one handle.
 * The library has no CPU fallback: every compute entry point runs CUDA kernels
 * built for sm_100a and fails with NCM_ECUDA where they cannot run.
 */
#ifndef NCM_H
#define NCM_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef int ncm_status;
#define NCM_OK 0
#define NCM_EINVAL 1       /* bad argument / shape (reference: panics, assert!) */
#define NCM_ECUDA 2        /* CUDA runtime error, or no usable device */
#define NCM_ETIMEOUT 3     /* a bounded device wait on a peer expired */
#define NCM_EPEER 4        /* peer setup failed (IPC open, share list) */
#define NCM_EIO 5          /* file / GGUF format error */
#define NCM_EUNSUPPORTED 6 /* tensor type or shape outside the path */

/* GGUF tensor type ids (gguf.rs:84-116). */
#define NCM_TYPE_F32 0
#define NCM_TYPE_F16 1
#define NCM_TYPE_Q4_0 2
#define NCM_TYPE_Q8_0 8
#define NCM_TYPE_Q4_K 12
#define NCM_TYPE_Q6_K 14

const char* ncm_last_error(void);
int ncm_version(void);

/* ---------------------------------------------------------------- kernels
 * inference.rs:935-947 quantize_f32_to_q8_0(x, x_i8, x_scales): per 32 values
 * scale = max|x|/127 (stored f32), q = round-half-away(x * (1/scale)), clamp +-127.
 * n must be a multiple of 32.  All pointers device. */
ncm_status ncm_quantize_f32_to_q8_0(const float* x, int n, int8_t* x_i8, float* x_scales, void* stream);

/* inference.rs:1201-1244 matmul_quantized(out, x_i8, x_scales, w, rows, cols, _):
 * out[r] = sum_b d_w[r,b] * s_x[b] * dot_b over the raw GGUF blocks of `w`
 * (row-major, rows x cols, type Q4_0 / Q8_0 / Q4_K / Q6_K, row pitch = raw row bytes);
 * Q6_K is inference.rs:3045-3087 matmul_q6_k over q8.rs:2092-2150 dot_q8_scaled.
 * `out` is overwritten.  All pointers device. */
ncm_status ncm_matmul_quantized(int qtype, const void* w, int64_t rows, int cols, const int8_t* x_i8,
                                const float* x_scales, float* out, void* stream);

/* inference.rs:1246-1303 matmul_quantized_batch(out, x_i8, x_scales, w, shape{batch,rows,cols}, _):
 * ntok activation rows (x_i8[ntok][cols], x_scales[ntok][cols/32]) -> out[ntok][rows],
 * 1 <= ntok <= 8, every row bit-identical to ncm_matmul_quantized of that row.  The
 * block dots run on int8 tensor-core MMA; x_i8 16-byte aligned; rows whose byte length
 * is not a multiple of 16 are re-pitched into a scratch first. */
ncm_status ncm_matmul_quantized_batch(int qtype, const void* w, int64_t rows, int cols, int ntok,
                                      const int8_t* x_i8, const float* x_scales, float* out, void* stream);

/* Debug seam for the bit-exact gate (q8.rs:2699-2702 dot_q4_0_q8_0_scalar,
 * q8.rs:505 Q8_0Block::dot_i32, q8.rs:1338-1376 integer sums of Q4_K):
 * Q4_0 / Q8_0 -> out[rows][cols/32] int32 block dots;
 * Q4_K -> out[rows][cols/32][2] = {sum q*x, sum x} per 32-sub-block. */
ncm_status ncm_block_dots(int qtype, const void* w, int64_t rows, int cols, const int8_t* x_i8,
                          int32_t* out, void* stream);

/* inference.rs:697-706 rms_norm(out, x, weight, eps). n <= 65536. Device pointers. */
ncm_status ncm_rms_norm(float* out, const float* x, const float* weight, int n, float eps, void* stream);

/* inference.rs:3367-3390 fused_silu_mul(gate_up, gate, up). Device pointers. */
ncm_status ncm_fused_silu_mul(float* out, const float* gate, const float* up, int n, void* stream);

/* inference.rs:4142-4292 apply_attention_heads for one token at `pos` over an f32
 * cache laid out [ctx][kv_heads*head_dim] (inference.rs:540-547); q already roped.
 * out[heads*head_dim] is overwritten.  Device pointers. */
ncm_status ncm_attention(float* out, const float* q, const float* k_cache, const float* v_cache, int pos,
                         int heads, int kv_heads, int head_dim, void* stream);

/* inference.rs:4319-4458 apply_attention_head_q8_0 / _f16: the same attention over an F16
 * cache (kind 1: u16 [ctx][kv_heads*head_dim], exact decode then the f32 path) or a
 * Q8_0 cache (kind 2: 34-byte blocks [ctx][kv_heads*head_dim/32]; q quantised like the
 * store, scores from integer block dots scaled (s_q * s_k), V decoded as q * s).  Kind 0
 * is ncm_attention.  Device pointers. */
ncm_status ncm_attention_kv(int kind, float* out, const float* q, const void* k_cache, const void* v_cache, int pos,
                            int heads, int kv_heads, int head_dim, void* stream);

/* No counterpart in the reference.  The same computation as ncm_attention, for callers
 * that must not allocate device memory on the call path: hosts that hand all device
 * memory to their own pool at start-up and forbid allocation afterwards (a fixed memory
 * budget shared with other work), and latency-critical loops where a cudaMalloc, which
 * can synchronise the device, would stall the stream.  The
 * softmax-score scratch is a fixed 1 MiB array (262144 floats) compiled into the
 * library, held by every GPU that loads it until the process exits; calls with
 * pos >= 16384 (the limit ncm_attention has too) or heads * (pos + 1) > 262144 are
 * rejected with NCM_EINVAL.  The first call on a device does that device's set-up: it
 * looks up the device's copy of the array (cudaGetSymbolAddress) and copies the glibc
 * expf exception table (built on the host, once per process, about two seconds) into
 * its own fixed in-library array, so that exp matches the host glibc bit for bit; make
 * that first call once on each device before any stream capture.  All calls on a device
 * share the one scratch array: calls that can overlap on the GPU race, so serialise them
 * (one stream, or events).  Nothing in it needs clearing, because each call writes every
 * score it reads.  The launch is stream ordered and does not synchronise. */
ncm_status ncm_attention_noalloc(float* out, const float* q, const float* k_cache, const float* v_cache, int pos,
                                 int heads, int kv_heads, int head_dim, void* stream);

/* ---------------------------------------------------------------- fixtures
 * Random-init model spec (the five BASELINE configs are random-init shapes). */
typedef struct {
    int32_t emb, layers, heads, kv_heads, head_dim, ffn, vocab, ctx;
    float rope_base, eps;
    int32_t tied;                       /* 1: no output.weight (head = Q4_0 requant of token_embd) */
    int32_t t_embd, t_attn, t_ffn, t_out; /* GGUF type ids */
    uint64_t seed;
    int32_t t_down;                     /* ffn_down type id (0: t_ffn) */
} ncm_synth_spec;

/* Writes a GGUF v3 file with llama metadata (keys read at model.rs:55-153) and the
 * synthetic weights.  The reference has no GGUF writer; this one is new. Host only. */
ncm_status ncm_gguf_write_synthetic(const char* path, const ncm_synth_spec* spec, int threads);

/* Encodes rows [r0,r1) x cols [c0,c1) of synthetic tensor `name` into host memory
 * (row-major raw blocks) -- lets tests compare device bytes with file bytes. */
ncm_status ncm_synth_tensor_host(const ncm_synth_spec* spec, const char* name, int type, int64_t r0, int64_t r1,
                                 int64_t c0, int64_t c1, int64_t cols, uint8_t* out);

/* ---------------------------------------------------------------- tensor parallel plan
 * tp.rs:641-701 validate_shares + shard_geometry.  out[8] = {q_start, q_heads,
 * kv_start, kv_heads, ffn_start, ffn_len, head_row_start, head_rows}. Host only. */
ncm_status ncm_shard_geometry(int heads, int kv_heads, int ffn, int vocab, const int* shares, int nshards,
                              int shard, int* out);

/* ---------------------------------------------------------------- model / decode */
typedef struct ncm_model ncm_model;

/* model.rs:461-545 LlamaWeights::load + tp.rs:916-1075 load_tp_shard_direct: reads a
 * GGUF file and uploads this shard's raw quant blocks to HBM unchanged (column
 * slices gathered per row).  shares == NULL / nshards <= 1 loads the whole model.
 * The tied head is rebuilt on device as the reference's Q4_0 requant (model.rs:471-508).
 * ctx_limit > 0 caps the KV cache length.  `device` is the CUDA ordinal. */
ncm_status ncm_model_load(const char* gguf_path, int ctx_limit, int device, const int* shares, int nshards,
                          int shard, ncm_model** out);

/* Same model as ncm_gguf_write_synthetic + ncm_model_load, generated directly on the
 * device (bit-identical blocks; no file). */
ncm_status ncm_model_create_synthetic(const ncm_synth_spec* spec, int ctx_limit, int device, const int* shares,
                                      int nshards, int shard, ncm_model** out);

void ncm_model_free(ncm_model* m);

/* out[12] = {emb, layers, heads, kv_heads, head_dim, ffn, vocab, ctx, local q heads,
 * local kv heads, local ffn, local head rows}. */
ncm_status ncm_model_info(const ncm_model* m, int* out);

/* Clears the KV cache and the decode position (new session, cluster_tp_node.rs:987-996). */
ncm_status ncm_model_reset(ncm_model* m);

/* inference.rs:505-531 LlamaKvCache::new storage selection (NANOCAMELID_KV_CACHE_F16 /
 * NANOCAMELID_KV_CACHE_Q8): kind 0 f32, 1 F16 (truncating f32 -> f16 per value on store),
 * 2 Q8_0 (quantize_row_to_q8_0_blocks on store, inference.rs:4298-4317).  Clears the
 * cache and the position; call before prefill. */
ncm_status ncm_model_set_kv_cache(ncm_model* m, int kind);

/* inference.rs:3649-3670 forward_pass + 4834-4845 sample_logits(_, 0.0) for ONE token
 * at `pos`, host buffers: copies the token in, runs the step, copies the greedy
 * argmax (and the logits when logits != NULL; for a shard, its local head rows) out.
 * Synchronous. */
ncm_status ncm_forward_pass(ncm_model* m, int token, int pos, float* logits, int* argmax);

/* bin/cluster_tp_node.rs:808-875 run_reference loop: the prompt (eight tokens per
 * multi-row pass, with the same K/V and state as token by token), then
 * n_gen greedy tokens.  Host buffers; the decode loop runs device-resident (CUDA
 * graph replays, no per-token host sync).  out_tokens[n_gen]. */
ncm_status ncm_generate(ncm_model* m, const int* prompt, int n_prompt, int n_gen, int* out_tokens);

/* Device-resident decode: run `n` more greedy steps from the current position on
 * `stream` without host synchronisation (bench path).  ncm_sync_tokens waits for the
 * model's stream and for the last caller stream given to prefill / decode (which must
 * stay valid until then), copies the token history [0, count) to host and checks the
 * device error word.  The position lives on the device, so a step that would start at or
 * past the context limit is held at the last slot (nothing is stored past the K/V cache)
 * and the next checking call returns NCM_EINVAL. */
ncm_status ncm_decode_steps(ncm_model* m, int n, void* stream);
ncm_status ncm_prefill_tokens(ncm_model* m, const int* prompt, int n_prompt, void* stream);
ncm_status ncm_sync_tokens(ncm_model* m, int* tokens, int count, int* pos_out);

/* Copies the device hidden state (after the last step) to host: float[emb]. */
ncm_status ncm_get_hidden(ncm_model* m, float* hidden);

/* Debug seam for layer-level parity: copies n floats of an activation buffer to host.
 * which: 0 hidden, 1 q (roped, last layer), 2 attention output, 3 silu(gate)*up,
 * 4 / 5 K / V cache of `layer` ([ctx][local kv width]), 6 logits (local head rows). */
ncm_status ncm_debug_read(ncm_model* m, int which, int layer, float* out, int64_t n);

/* Measurement seam (no reference counterpart; the reference times whole tokens): one
 * launch, on `stream`, of the decode step's GEMV kernel of kind NCM_STEP_* for `layer`,
 * with the parameters the captured step uses, so that a caller can time the step's
 * dominant kernel with events.  It overwrites the activations that kernel writes.
 * NCM_STEP_WO / NCM_STEP_W2 run on unsharded models only. */
enum { NCM_STEP_QKV = 0, NCM_STEP_W13 = 1, NCM_STEP_WO = 2, NCM_STEP_W2 = 3 };
ncm_status ncm_launch_step_kernel(ncm_model* m, int kind, int layer, void* stream);

/* Measurement seam (no reference counterpart): per-CTA global-timer stamps (ns) of the
 * GEMV pipeline phases recorded by the last ncm_launch_step_kernel launch: out[16 * cta +
 * i], i = 0 entry, 1 after the dependent-launch wait, 2 prologue done, 3 last weight load
 * issued, 4 last fold done, 5 time in tile epilogues, 6 exit, 7 / 8 compute warp 0 time
 * waiting for weights / for a free term slot, 9 fold time waiting for terms, 10 producer
 * time waiting for a free stage, 11 compute warp 0 done.  n entries (<= 16 per SM). */
ncm_status ncm_debug_stamps(ncm_model* m, uint64_t* out, int n);

/* ---------------------------------------------------------------- speculative decoding
 * speculative.rs:381-389 prefill_pass_batch + compute_logits_from_hidden +
 * sample_logits(_, 0.0) per row: tokens[ntok] (1 <= ntok <= 8) at positions
 * pos0 .. pos0+ntok-1 through the target in one multi-row pass (each weight tile read
 * once for all rows; int8 tensor-core block dots), K/V stored at those positions;
 * argmax_out[t] = greedy token after row t.  Each row equals the one-token step at its
 * position bit for bit.  The model's decode position is not changed.  On a shard,
 * every rank calls it with the same arguments: the rows' partial sums and head pairs
 * are reduced by the model's reducer (fused NVLink, NCCL or the host callback) and every
 * rank gets the same tokens. */
ncm_status ncm_verify_batch(ncm_model* m, const int* tokens, int ntok, int pos0, int* argmax_out);

/* speculative.rs:299-494 speculative_decoding_step at temperature 0, from a prompt:
 * the draft proposes k (<= 8) tokens, the target verifies them with ncm_verify_batch,
 * the agreeing prefix plus the target's next token are emitted.  out_tokens[n_gen]
 * equals the target's greedy decode; stats[2] = {drafted, accepted} (may be NULL). */
ncm_status ncm_spec_generate(ncm_model* target, ncm_model* draft, const int* prompt, int n_prompt, int n_gen, int k,
                             int* out_tokens, int* stats);

/* speculative.rs:80-105 NGramDrafter::draft, host only (no GPU): up to max_tokens
 * tokens that followed the most recent earlier occurrence of the longest suffix
 * n-gram of history[0..len) (n from max_ngram down to min_ngram; the reference's
 * defaults are 4 and 3).  Returns the count written to out. */
int ncm_ngram_draft(const int* history, int len, int max_tokens, int max_ngram, int min_ngram, int* out);

/* speculative.rs:122-297 ngram_speculative_step at temperature 0, repeated as
 * main.rs:9720-9760 (prompt-lookup speculation, the reference's default draft source):
 * n_gen tokens into out_tokens, equal to the greedy decode; stats = {drafted,
 * accepted}.  Up to 7 drafts per multi-row pass (row 0 = the target's own token). */
ncm_status ncm_ngram_generate(ncm_model* m, const int* prompt, int n_prompt, int n_gen, int k, int max_ngram,
                              int min_ngram, int* out_tokens, int* stats);

/* ---------------------------------------------------------------- multi-GPU (one process per GPU)
 * Replaces the TCP star reducer (bin/cluster_tp_node.rs:505-550, 1042-1056, 1154-1180)
 * feeding tp.rs:226-428 tp_forward_token_reduced.
 * 1) ncm_tp_export: bytes describing this rank's receive buffers (CUDA IPC handle);
 * 2) the caller all-gathers them (torch.distributed on the host side);
 * 3) ncm_tp_import: opens every peer's buffers;  mode selects the reducer:
 *    NCM_REDUCE_FUSED_P2P -- partial rows written into every peer's slot by NVLink
 *        stores from the o_proj / down GEMV epilogue, rank-ordered sum on each GPU;
 *    NCM_REDUCE_NCCL -- ncclAllReduce(sum) between GEMV and residual (baseline);
 *    NCM_REDUCE_HOST_CALLBACK -- the reference's `reduce` closure (tp.rs:226-236):
 *        the partial row goes to a host function registered with
 *        ncm_tp_set_host_reducer, which leaves the global sum in place (any transport:
 *        the reference's TCP star, a host collective, a test harness); steps run
 *        eagerly, synchronously, on the calling thread. */
#define NCM_REDUCE_FUSED_P2P 0
#define NCM_REDUCE_NCCL 1
#define NCM_REDUCE_HOST_CALLBACK 2
/* Phases passed to the host reducer: tp.rs:203-206 ReducePhase::{Attention, Ffn}
 * (buf = n = emb floats, this rank's partial; leave the sum over ranks, added in rank
 * order from 0.0f), and the head merge (buf = 2 floats {logit, token bits} of this
 * shard's first maximum; leave the merged pair: strict '>' in rank order,
 * cluster_tp_node.rs:1185-1204).  Return 0, or non-zero for the closure's Err ->
 * NCM_EPEER from the step. */
#define NCM_REDUCE_PHASE_ATTENTION 0
#define NCM_REDUCE_PHASE_FFN 1
#define NCM_REDUCE_PHASE_HEAD 2
typedef int (*ncm_host_reduce_fn)(float* buf, int n, int layer, int phase, void* user);
ncm_status ncm_tp_set_host_reducer(ncm_model* m, ncm_host_reduce_fn fn, void* user);
#define NCM_TP_HANDLE_BYTES 256
ncm_status ncm_tp_export(ncm_model* m, uint8_t* handle_out /* NCM_TP_HANDLE_BYTES */);
ncm_status ncm_tp_import(ncm_model* m, const uint8_t* handles /* world x NCM_TP_HANDLE_BYTES */, int world,
                         int rank);
ncm_status ncm_nccl_unique_id(uint8_t* out /* 128 bytes */);
ncm_status ncm_tp_nccl_init(ncm_model* m, const uint8_t* unique_id, int world, int rank);
ncm_status ncm_tp_set_reducer(ncm_model* m, int mode);
/* Bound (ns) on every device-side wait for a peer; expiry -> NCM_ETIMEOUT. */
ncm_status ncm_tp_set_timeout_ns(ncm_model* m, uint64_t ns);

/* Test seam for the bounded peer wait: runs the fused reduction's wait on flags
 * nobody sets (world=2, peer = a local buffer) and returns NCM_ETIMEOUT after
 * about timeout_ns; the context stays usable. */
ncm_status ncm_test_peer_timeout(int device, uint64_t timeout_ns);

#ifdef __cplusplus
}
#endif
#endif
