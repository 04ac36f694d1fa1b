"""nanocamelid_b200 -- B200 decode hot path of NanoCamelid behind a C ABI (libncm.so).

Python mirror of the reference's seams (same names and argument meaning):
  quantize_f32_to_q8_0   inference.rs:935
  matmul_quantized       inference.rs:1201
  matmul_quantized_batch inference.rs:1246
  Model.forward_pass     inference.rs:3649 (+ sample_logits 4834)
  Model.generate         bin/cluster_tp_node.rs:808 run_reference loop
  shard_geometry         tp.rs:662
Device tensors are passed as raw pointers (`int`, e.g. torch's data_ptr()).  There is
no CPU fallback: if libncm.so is missing the import of `lib()` raises.
"""
import ctypes
import os
from dataclasses import dataclass, field

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libncm.so")

Q4_0, Q8_0, Q4_K, Q6_K, F32, F16 = 2, 8, 12, 14, 0, 1
REDUCE_FUSED_P2P, REDUCE_NCCL, REDUCE_HOST_CALLBACK = 0, 1, 2
STEP_QKV, STEP_W13, STEP_WO, STEP_W2 = 0, 1, 2, 3
PHASE_ATTENTION, PHASE_FFN, PHASE_HEAD = 0, 1, 2   # tp.rs:203-206 ReducePhase, + the head merge
HOST_REDUCE_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_void_p)
TP_HANDLE_BYTES = 256

STATUS = {0: "OK", 1: "EINVAL", 2: "ECUDA", 3: "ETIMEOUT", 4: "EPEER", 5: "EIO", 6: "EUNSUPPORTED"}


class NcmError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


class SynthSpec(ctypes.Structure):
    """ncm_synth_spec: a random-init llama model (BASELINE configs are random-init)."""
    _fields_ = [("emb", ctypes.c_int32), ("layers", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("ffn", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("ctx", ctypes.c_int32), ("rope_base", ctypes.c_float),
                ("eps", ctypes.c_float), ("tied", ctypes.c_int32), ("t_embd", ctypes.c_int32),
                ("t_attn", ctypes.c_int32), ("t_ffn", ctypes.c_int32), ("t_out", ctypes.c_int32),
                ("seed", ctypes.c_uint64), ("t_down", ctypes.c_int32)]

    def replace(self, **kw):
        s = SynthSpec()
        ctypes.pointer(s)[0] = self
        for k, v in kw.items():
            setattr(s, k, v)
        return s

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


def spec(emb, layers, heads, kv_heads, head_dim, ffn, vocab=128256, ctx=2048, tied=True, t_embd=Q4_0,
         t_attn=Q4_0, t_ffn=Q4_0, t_out=Q4_0, seed=0, rope_base=500000.0, eps=1e-5, t_down=0):
    return SynthSpec(emb, layers, heads, kv_heads, head_dim, ffn, vocab, ctx, rope_base, eps, int(tied), t_embd,
                     t_attn, t_ffn, t_out, seed, t_down)


# BASELINE.json configs (shapes; random-init N(0, 0.02) weights, seeded).
CONFIGS = {
    "cfg1_1b_q4_0": spec(2048, 16, 32, 8, 64, 8192, tied=True),
    "cfg2_3b_q4_0": spec(3072, 28, 24, 8, 128, 8192, tied=True),
    # 8B: attention Q8_0, FFN Q4_K; output.weight type unspecified upstream -> Q8_0, token_embd Q8_0.
    "cfg3_8b_mixed": spec(4096, 32, 32, 8, 128, 14336, tied=False, t_embd=Q8_0, t_attn=Q8_0, t_ffn=Q4_K,
                          t_out=Q8_0),
    "cfg4_70b_q4_0": spec(8192, 80, 64, 8, 128, 28672, tied=False),
    # speculative target: config-3 shape, all Q4_0, separate seed
    "cfg5_target_q4_0": spec(4096, 32, 32, 8, 128, 14336, tied=False, seed=1),
}

_lib = None


def lib():
    """Loads libncm.so (fails loudly if it has not been built).  NCM_LIBRARY, when set,
    names another build of the same library to load instead."""
    global _lib
    if _lib is not None:
        return _lib
    path = os.environ.get("NCM_LIBRARY") or LIB_PATH
    if not os.path.exists(path):
        raise ImportError(f"{path} missing: run `python -m nanocamelid_b200.build` (or __graft_entry__.build())")
    L = ctypes.CDLL(os.path.abspath(path))
    c_int, c_i64, c_p, c_f, c_u64 = ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_float, ctypes.c_uint64
    pint = ctypes.POINTER(ctypes.c_int)
    pu8 = ctypes.POINTER(ctypes.c_uint8)
    sigs = {
        "ncm_last_error": (ctypes.c_char_p, []),
        "ncm_version": (c_int, []),
        "ncm_quantize_f32_to_q8_0": (c_int, [c_p, c_int, c_p, c_p, c_p]),
        "ncm_matmul_quantized": (c_int, [c_int, c_p, c_i64, c_int, c_p, c_p, c_p, c_p]),
        "ncm_matmul_quantized_batch": (c_int, [c_int, c_p, c_i64, c_int, c_int, c_p, c_p, c_p, c_p]),
        "ncm_block_dots": (c_int, [c_int, c_p, c_i64, c_int, c_p, c_p, c_p]),
        "ncm_rms_norm": (c_int, [c_p, c_p, c_p, c_int, c_f, c_p]),
        "ncm_fused_silu_mul": (c_int, [c_p, c_p, c_p, c_int, c_p]),
        "ncm_attention": (c_int, [c_p, c_p, c_p, c_p, c_int, c_int, c_int, c_int, c_p]),
        "ncm_attention_kv": (c_int, [c_int, c_p, c_p, c_p, c_p, c_int, c_int, c_int, c_int, c_p]),
        "ncm_model_set_kv_cache": (c_int, [c_p, c_int]),
        "ncm_gguf_write_synthetic": (c_int, [ctypes.c_char_p, ctypes.POINTER(SynthSpec), c_int]),
        "ncm_synth_tensor_host": (c_int, [ctypes.POINTER(SynthSpec), ctypes.c_char_p, c_int, c_i64, c_i64, c_i64,
                                          c_i64, c_i64, c_p]),
        "ncm_shard_geometry": (c_int, [c_int, c_int, c_int, c_int, pint, c_int, c_int, pint]),
        "ncm_model_load": (c_int, [ctypes.c_char_p, c_int, c_int, pint, c_int, c_int, ctypes.POINTER(c_p)]),
        "ncm_model_create_synthetic": (c_int, [ctypes.POINTER(SynthSpec), c_int, c_int, pint, c_int, c_int,
                                               ctypes.POINTER(c_p)]),
        "ncm_model_free": (None, [c_p]),
        "ncm_model_info": (c_int, [c_p, pint]),
        "ncm_model_reset": (c_int, [c_p]),
        "ncm_forward_pass": (c_int, [c_p, c_int, c_int, c_p, pint]),
        "ncm_generate": (c_int, [c_p, pint, c_int, c_int, pint]),
        "ncm_decode_steps": (c_int, [c_p, c_int, c_p]),
        "ncm_prefill_tokens": (c_int, [c_p, pint, c_int, c_p]),
        "ncm_sync_tokens": (c_int, [c_p, pint, c_int, pint]),
        "ncm_get_hidden": (c_int, [c_p, c_p]),
        "ncm_debug_read": (c_int, [c_p, c_int, c_int, c_p, c_i64]),
        "ncm_launch_step_kernel": (c_int, [c_p, c_int, c_int, c_p]),
        "ncm_debug_stamps": (c_int, [c_p, c_p, c_int]),
        "ncm_tp_export": (c_int, [c_p, pu8]),
        "ncm_tp_import": (c_int, [c_p, pu8, c_int, c_int]),
        "ncm_nccl_unique_id": (c_int, [pu8]),
        "ncm_tp_nccl_init": (c_int, [c_p, pu8, c_int, c_int]),
        "ncm_tp_set_reducer": (c_int, [c_p, c_int]),
        "ncm_tp_set_host_reducer": (c_int, [c_p, HOST_REDUCE_FN, c_p]),
        "ncm_tp_set_timeout_ns": (c_int, [c_p, c_u64]),
        "ncm_verify_batch": (c_int, [c_p, pint, c_int, c_int, pint]),
        "ncm_spec_generate": (c_int, [c_p, c_p, pint, c_int, c_int, c_int, pint, pint]),
        "ncm_ngram_draft": (c_int, [pint, c_int, c_int, c_int, c_int, pint]),
        "ncm_ngram_generate": (c_int, [c_p, pint, c_int, c_int, c_int, c_int, c_int, pint, pint]),
        "ncm_test_peer_timeout": (c_int, [c_int, c_u64]),
    }
    for name, (res, args) in sigs.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def _ck(status):
    if status != 0:
        raise NcmError(status, lib().ncm_last_error().decode())


def _ints(v):
    v = list(v)
    return (ctypes.c_int * max(1, len(v)))(*v)


def _stream(stream):
    return ctypes.c_void_p(stream if stream else None)


# ---------------------------------------------------------------- kernel seams (device pointers)
def quantize_f32_to_q8_0(x_ptr, n, x_i8_ptr, x_scales_ptr, stream=0):
    """inference.rs:935 quantize_f32_to_q8_0 on device buffers."""
    _ck(lib().ncm_quantize_f32_to_q8_0(x_ptr, n, x_i8_ptr, x_scales_ptr, _stream(stream)))


def matmul_quantized(out_ptr, x_i8_ptr, x_scales_ptr, w_ptr, rows, cols, qtype, stream=0):
    """inference.rs:1201 matmul_quantized(out, x_i8, x_scales, w, rows, cols, _)."""
    _ck(lib().ncm_matmul_quantized(qtype, w_ptr, rows, cols, x_i8_ptr, x_scales_ptr, out_ptr, _stream(stream)))


def matmul_quantized_batch(out_ptr, x_i8_ptr, x_scales_ptr, w_ptr, batch_size, rows, cols, qtype, stream=0):
    """inference.rs:1246 matmul_quantized_batch with BatchMatmulShape{batch_size, rows, cols}."""
    _ck(lib().ncm_matmul_quantized_batch(qtype, w_ptr, rows, cols, batch_size, x_i8_ptr, x_scales_ptr, out_ptr,
                                         _stream(stream)))


def block_dots(out_ptr, x_i8_ptr, w_ptr, rows, cols, qtype, stream=0):
    _ck(lib().ncm_block_dots(qtype, w_ptr, rows, cols, x_i8_ptr, out_ptr, _stream(stream)))


def rms_norm(out_ptr, x_ptr, w_ptr, n, eps, stream=0):
    _ck(lib().ncm_rms_norm(out_ptr, x_ptr, w_ptr, n, eps, _stream(stream)))


def fused_silu_mul(out_ptr, gate_ptr, up_ptr, n, stream=0):
    _ck(lib().ncm_fused_silu_mul(out_ptr, gate_ptr, up_ptr, n, _stream(stream)))


def attention(out_ptr, q_ptr, k_cache_ptr, v_cache_ptr, pos, heads, kv_heads, head_dim, stream=0):
    _ck(lib().ncm_attention(out_ptr, q_ptr, k_cache_ptr, v_cache_ptr, pos, heads, kv_heads, head_dim,
                            _stream(stream)))


KV_F32, KV_F16, KV_Q8_0 = 0, 1, 2   # inference.rs:505-531 cache storage kinds


def attention_kv(kind, out_ptr, q_ptr, k_cache_ptr, v_cache_ptr, pos, heads, kv_heads, head_dim, stream=0):
    """inference.rs:4319-4458: attention over an F16 (KV_F16) or Q8_0 (KV_Q8_0) cache."""
    _ck(lib().ncm_attention_kv(kind, out_ptr, q_ptr, k_cache_ptr, v_cache_ptr, pos, heads, kv_heads, head_dim,
                               _stream(stream)))


# ---------------------------------------------------------------- host helpers
def write_synthetic_gguf(path, spec_, threads=None):
    threads = threads or os.cpu_count() or 4
    _ck(lib().ncm_gguf_write_synthetic(str(path).encode(), ctypes.byref(spec_), threads))


def synth_tensor_bytes(spec_, name, qtype, r0, r1, c0, c1, cols):
    be = 256 if qtype in (Q4_K, Q6_K) else 32
    bb = {Q4_0: 18, Q8_0: 34, Q4_K: 144, Q6_K: 210}[qtype]
    buf = (ctypes.c_uint8 * ((r1 - r0) * ((c1 - c0) // be) * bb))()
    _ck(lib().ncm_synth_tensor_host(ctypes.byref(spec_), name.encode(), qtype, r0, r1, c0, c1, cols, buf))
    return bytes(buf)


def shard_geometry(heads, kv_heads, ffn, vocab, shares, shard):
    """tp.rs:662 shard_geometry -> dict (raises NcmError like validate_shares' Err)."""
    out = (ctypes.c_int * 8)()
    _ck(lib().ncm_shard_geometry(heads, kv_heads, ffn, vocab, _ints(shares), len(shares), shard, out))
    keys = ["q_start", "q_heads", "kv_start", "kv_heads", "ffn_start", "ffn_len", "head_row_start", "head_rows"]
    return dict(zip(keys, list(out)))


@dataclass
class ModelInfo:
    emb: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    ctx: int
    local_q_heads: int
    local_kv_heads: int
    local_ffn: int
    local_head_rows: int


class Model:
    """A model resident on one GPU (one shard of it under tensor parallelism)."""

    def __init__(self, handle):
        self._h = ctypes.c_void_p(handle)

    @classmethod
    def load(cls, path, ctx_limit=0, device=0, shares=None, shard=0):
        h = ctypes.c_void_p()
        sh = list(shares) if shares else []
        _ck(lib().ncm_model_load(str(path).encode(), ctx_limit, device, _ints(sh) if sh else None, len(sh), shard,
                                 ctypes.byref(h)))
        return cls(h.value)

    @classmethod
    def synthetic(cls, spec_, ctx_limit=0, device=0, shares=None, shard=0):
        h = ctypes.c_void_p()
        sh = list(shares) if shares else []
        _ck(lib().ncm_model_create_synthetic(ctypes.byref(spec_), ctx_limit, device, _ints(sh) if sh else None,
                                             len(sh), shard, ctypes.byref(h)))
        return cls(h.value)

    def close(self):
        if self._h and self._h.value:
            lib().ncm_model_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def info(self):
        out = (ctypes.c_int * 12)()
        _ck(lib().ncm_model_info(self._h, out))
        return ModelInfo(*list(out))

    def reset(self):
        _ck(lib().ncm_model_reset(self._h))

    def set_kv_cache(self, kind):
        """KV_F32 / KV_F16 / KV_Q8_0 cache storage (NANOCAMELID_KV_CACHE_F16 / _Q8); clears it."""
        _ck(lib().ncm_model_set_kv_cache(self._h, kind))

    def forward_pass(self, token, pos, want_logits=False):
        """inference.rs:3649 forward_pass + sample_logits(_, 0.0): returns (argmax, logits|None)."""
        import numpy as np
        am = ctypes.c_int()
        logits = None
        ptr = None
        if want_logits:
            logits = np.empty(self.info.local_head_rows, dtype=np.float32)
            ptr = logits.ctypes.data_as(ctypes.c_void_p)
        _ck(lib().ncm_forward_pass(self._h, token, pos, ptr, ctypes.byref(am)))
        return am.value, logits

    def generate(self, prompt, n_gen):
        out = (ctypes.c_int * max(1, n_gen))()
        _ck(lib().ncm_generate(self._h, _ints(prompt), len(prompt), n_gen, out))
        return list(out)[:n_gen]

    def prefill(self, prompt, stream=0):
        _ck(lib().ncm_prefill_tokens(self._h, _ints(prompt), len(prompt), _stream(stream)))

    def decode_steps(self, n, stream=0):
        _ck(lib().ncm_decode_steps(self._h, n, _stream(stream)))

    def sync_tokens(self, count):
        out = (ctypes.c_int * max(1, count))()
        pos = ctypes.c_int()
        _ck(lib().ncm_sync_tokens(self._h, out, count, ctypes.byref(pos)))
        return list(out)[:count], pos.value

    def launch_step_kernel(self, kind, layer, stream=0):
        """One launch of the decode step's GEMV of `kind` (STEP_*) for `layer` (timing)."""
        _ck(lib().ncm_launch_step_kernel(self._h, kind, layer, _stream(stream)))

    def debug_stamps(self, n):
        """Phase stamps of the last launch_step_kernel (uint64[n]); see include/ncm.h."""
        import numpy as np
        out = np.zeros(n, dtype=np.uint64)
        _ck(lib().ncm_debug_stamps(self._h, out.ctypes.data_as(ctypes.c_void_p), n))
        return out

    def hidden(self):
        import numpy as np
        h = np.empty(self.info.emb, dtype=np.float32)
        _ck(lib().ncm_get_hidden(self._h, h.ctypes.data_as(ctypes.c_void_p)))
        return h

    def debug_read(self, which, n, layer=0):
        """Activation buffer readback (0 hidden, 1 q, 2 attn out, 3 silu*up, 4/5 K/V cache, 6 logits)."""
        import numpy as np
        out = np.empty(n, dtype=np.float32)
        _ck(lib().ncm_debug_read(self._h, which, layer, out.ctypes.data_as(ctypes.c_void_p), n))
        return out

    def verify_batch(self, tokens, pos0):
        """speculative.rs:381 prefill_pass_batch + per-row greedy argmax (one pass)."""
        out = (ctypes.c_int * len(tokens))()
        _ck(lib().ncm_verify_batch(self._h, _ints(tokens), len(tokens), pos0, out))
        return list(out)

    def spec_generate(self, draft, prompt, n_gen, k=4):
        """speculative.rs:299-494 greedy speculative decoding with `draft`; returns
        (tokens, (drafted, accepted))."""
        out = (ctypes.c_int * max(1, n_gen))()
        stats = (ctypes.c_int * 2)()
        _ck(lib().ncm_spec_generate(self._h, draft._h, _ints(prompt), len(prompt), n_gen, k, out, stats))
        return list(out)[:n_gen], (stats[0], stats[1])

    def ngram_generate(self, prompt, n_gen, k=4, max_ngram=4, min_ngram=3):
        """speculative.rs:122-297 prompt-lookup (n-gram) speculative decoding; returns
        (tokens, (drafted, accepted))."""
        out = (ctypes.c_int * max(1, n_gen))()
        stats = (ctypes.c_int * 2)()
        _ck(lib().ncm_ngram_generate(self._h, _ints(prompt), len(prompt), n_gen, k, max_ngram, min_ngram, out, stats))
        return list(out)[:n_gen], (stats[0], stats[1])

    # tensor parallel
    def tp_export(self):
        buf = (ctypes.c_uint8 * TP_HANDLE_BYTES)()
        _ck(lib().ncm_tp_export(self._h, buf))
        return bytes(buf)

    def tp_import(self, handles, world, rank):
        blob = b"".join(handles)
        buf = (ctypes.c_uint8 * len(blob)).from_buffer_copy(blob)
        _ck(lib().ncm_tp_import(self._h, buf, world, rank))

    def tp_nccl_init(self, unique_id, world, rank):
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id)
        _ck(lib().ncm_tp_nccl_init(self._h, buf, world, rank))

    def tp_set_reducer(self, mode):
        _ck(lib().ncm_tp_set_reducer(self._h, mode))

    def tp_set_host_reducer(self, fn):
        """Registers fn(buf, layer, phase) -> int (0 = ok) as this rank's reduce closure
        (tp.rs:226-236).  buf is a float32 numpy view of the partial row (PHASE_ATTENTION /
        PHASE_FFN) or of {logit, token bits} (PHASE_HEAD); fn leaves the global value in
        it.  Then tp_set_reducer(REDUCE_HOST_CALLBACK)."""
        import numpy as np

        def tramp(ptr, n, layer, phase, _user):
            try:
                buf = np.ctypeslib.as_array(ptr, shape=(n,))
                rc = fn(buf, layer, phase)
                return int(rc or 0)
            except Exception:   # an exception is the closure's Err
                return -1

        self._host_reducer = HOST_REDUCE_FN(tramp)   # kept alive with the model
        _ck(lib().ncm_tp_set_host_reducer(self._h, self._host_reducer, None))

    def tp_set_timeout_ns(self, ns):
        _ck(lib().ncm_tp_set_timeout_ns(self._h, int(ns)))


def ngram_draft(history, max_tokens, max_ngram=4, min_ngram=3):
    """speculative.rs:80-105 NGramDrafter::draft (host only)."""
    out = (ctypes.c_int * max(1, max_tokens))()
    n = lib().ncm_ngram_draft(_ints(history), len(history), max_tokens, max_ngram, min_ngram, out)
    return list(out)[:n]


def nccl_unique_id():
    buf = (ctypes.c_uint8 * 128)()
    _ck(lib().ncm_nccl_unique_id(buf))
    return bytes(buf)


def peer_timeout_selftest(device=0, timeout_ns=100_000_000):
    """Runs the bounded peer wait on flags nobody sets; returns the status code."""
    return lib().ncm_test_peer_timeout(device, timeout_ns)
