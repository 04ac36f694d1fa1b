"""ctypes wrapper of the CPU oracle (oracle.c) -- TEST INFRASTRUCTURE ONLY.

Loaded by tests/, __graft_entry__.smoke() and bench.py's CPU arms as the checker / the
timed CPU restatement of the reference's portable path.  Never imported by the
nanocamelid_b200 package.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
_lib = None


class SynthSpec(ctypes.Structure):
    """orc_synth_spec: a random-init llama model (the BASELINE configs' weights)."""
    _fields_ = [("emb", ctypes.c_int32), ("layers", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("ffn", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("ctx", ctypes.c_int32), ("rope_base", ctypes.c_float),
                ("eps", ctypes.c_float), ("tied", ctypes.c_int32), ("t_embd", ctypes.c_int32),
                ("t_attn", ctypes.c_int32), ("t_ffn", ctypes.c_int32), ("t_out", ctypes.c_int32),
                ("seed", ctypes.c_uint64), ("t_down", ctypes.c_int32)]

    @classmethod
    def of(cls, spec):
        """From any object with the same field names (e.g. the product's spec)."""
        return cls(*[getattr(spec, k) for k, _ in cls._fields_])


def build():
    r = subprocess.run(["make", "-C", HERE, "-s"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)
    return LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    src = os.path.join(HERE, "oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(src) > os.path.getmtime(LIB_PATH):
        build()
    L = ctypes.CDLL(LIB_PATH)
    P, I, F, L64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_long
    sigs = {
        "orc_f16_to_f32": (F, [ctypes.c_uint16]),
        "orc_f32_to_f16": (ctypes.c_uint16, [F]),
        "orc_quantize_q8_0": (None, [P, I, P, P]),
        "orc_quantize_matrix_q8_0": (None, [P, L64, I, P]),
        "orc_quantize_matrix_q4_0": (None, [P, L64, I, P]),
        "orc_matmul_quantized": (None, [I, P, L64, I, P, P, P]),
        "orc_matmul_quantized_batch": (None, [I, P, L64, I, I, P, P, P]),
        "orc_block_dots": (None, [I, P, L64, I, P, P]),
        "orc_block_dot": (ctypes.c_int32, [I, P, P]),
        "orc_q4_k_dot": (F, [P, P, P]),
        "orc_q6_k_dot": (F, [P, P, P]),
        "orc_q6_k_dequant": (None, [P, P]),
        "orc_q4_0_unpack": (None, [P, P]),
        "orc_dequant_row": (None, [I, P, I, P]),
        "orc_rms_norm": (None, [P, P, P, I, F]),
        "orc_apply_rope": (None, [P, I, I, I, I, F]),
        "orc_silu_mul": (None, [P, P, P, I]),
        "orc_attention": (None, [P, P, P, P, I, I, I, I, I]),
        "orc_attention_kv": (None, [I, P, P, P, P, I, I, I, I, I]),
        "orc_kv_quantize_row_q8_0": (None, [P, I, P]),
        "orc_kv_store_f16": (None, [P, I, P]),
        "orc_argmax": (I, [P, L64]),
        "orc_model_load": (P, [ctypes.c_char_p, I]),
        "orc_model_create_synthetic": (P, [ctypes.POINTER(SynthSpec), I]),
        "orc_model_fill_kv": (None, [P, I, ctypes.c_uint64]),
        "orc_model_set_kv_kind": (I, [P, I]),
        "orc_synth_key": (ctypes.c_uint64, [ctypes.c_uint64, ctypes.c_char_p]),
        "orc_synth_tensor": (None, [I, ctypes.c_uint64, L64, L64, L64, L64, L64, P]),
        "orc_generate_batched": (I, [P, P, I, I, I, P, P]),
        "orc_model_info": (I, [P, P]),
        "orc_model_reset": (None, [P]),
        "orc_model_head_blocks": (P, [P]),
        "orc_forward_pass": (I, [P, I, I, P]),
        "orc_generate": (I, [P, P, I, I, P, P]),
        "orc_prefill_batch": (None, [P, P, I, I, P]),
        "orc_compute_logits": (None, [P, P, P]),
        "orc_spec_generate": (I, [P, P, P, I, I, I, P, P]),
        "orc_ngram_draft": (I, [P, I, I, I, I, P]),
        "orc_ngram_generate": (I, [P, P, I, I, I, I, I, I, P, P]),
        "orc_model_buf": (P, [P, I, I]),
        "orc_shard_geometry": (I, [I, I, I, I, P, I, I, P]),
        "orc_tp_build": (P, [P, P, I]),
        "orc_tp_reset": (None, [P]),
        "orc_tp_forward": (I, [P, I, I, P]),
        "orc_tp_generate": (I, [P, P, I, I, P]),
    }
    for n, (r, a) in sigs.items():
        f = getattr(L, n)
        f.restype = r
        f.argtypes = a
    _lib = L
    return L


def ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


BLOCK_BYTES = {2: 18, 8: 34, 12: 144, 14: 210}
BLOCK_ELEMS = {2: 32, 8: 32, 12: 256, 14: 256}


def quantize_q8_0(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.zeros(x.size, dtype=np.int8)
    s = np.zeros(x.size // 32, dtype=np.float32)
    lib().orc_quantize_q8_0(ptr(x), x.size, ptr(q), ptr(s))
    return q, s


def matmul(qtype, w, rows, cols, xq, xs):
    out = np.zeros(rows, dtype=np.float32)
    lib().orc_matmul_quantized(qtype, ptr(w), rows, cols, ptr(xq), ptr(xs), ptr(out))
    return out


def matmul_batch(qtype, w, rows, cols, ntok, xq, xs):
    out = np.zeros(ntok * rows, dtype=np.float32)
    lib().orc_matmul_quantized_batch(qtype, ptr(w), rows, cols, ntok, ptr(xq), ptr(xs), ptr(out))
    return out.reshape(ntok, rows)


def block_dots(qtype, w, rows, cols, xq):
    n = rows * (cols // 32) * (2 if qtype == 12 else 1)
    out = np.zeros(n, dtype=np.int32)
    lib().orc_block_dots(qtype, ptr(w), rows, cols, ptr(xq), ptr(out))
    return out


def synth_tensor(spec, name, qtype, r0, r1, c0, c1, cols):
    """Raw blocks of rows [r0, r1) x columns [c0, c1) of a synthetic tensor (the oracle's
    own generator)."""
    be = 256 if qtype in (12, 14) else (32 if qtype in (2, 8) else 1)
    bb = {2: 18, 8: 34, 12: 144, 14: 210, 0: 4, 1: 2}[qtype]
    out = np.zeros((r1 - r0) * ((c1 - c0) // be) * bb, dtype=np.uint8)
    sp = SynthSpec.of(spec)
    key = lib().orc_synth_key(sp.seed, name.encode())
    lib().orc_synth_tensor(qtype, key, r0, r1 - r0, c0, c1 - c0, cols, ptr(out))
    return out.tobytes()


class OracleModel:
    def __init__(self, path=None, ctx_limit=0, spec=None):
        """From a GGUF file, or (spec=...) the synthetic model of that spec built in host
        memory by the oracle's own generator."""
        if spec is not None:
            self._spec = SynthSpec.of(spec)
            self.h = lib().orc_model_create_synthetic(ctypes.byref(self._spec), ctx_limit)
        else:
            self.h = lib().orc_model_load(str(path).encode(), ctx_limit)
        if not self.h:
            raise RuntimeError(f"oracle could not build the model ({path or 'synthetic'})")
        info = np.zeros(10, dtype=np.int32)
        lib().orc_model_info(self.h, ptr(info))
        (self.emb, self.layers, self.ffn, self.heads, self.kv_heads, self.head_dim, self.vocab, self.rope_dim,
         self.ctx, self.head_type) = [int(v) for v in info]

    def reset(self):
        lib().orc_model_reset(self.h)

    def forward_pass(self, token, pos, want_logits=False):
        lg = np.zeros(self.vocab, dtype=np.float32) if want_logits else None
        t = lib().orc_forward_pass(self.h, token, pos, ptr(lg) if want_logits else None)
        return t, lg

    def generate(self, prompt, n_gen, want_last_logits=False):
        p = np.asarray(prompt, dtype=np.int32)
        out = np.zeros(max(1, n_gen), dtype=np.int32)
        lg = np.zeros(self.vocab, dtype=np.float32) if want_last_logits else None
        lib().orc_generate(self.h, ptr(p), len(p), n_gen, ptr(out), ptr(lg) if want_last_logits else None)
        return [int(v) for v in out[:n_gen]], lg

    def generate_batched(self, prompt, n_gen, chunk=64, want_last_logits=False):
        """orc_generate with the prompt ingested `chunk` rows per batched pass (bit-identical
        to token-by-token, inference.rs:6866-6913)."""
        p = np.asarray(prompt, dtype=np.int32)
        out = np.zeros(max(1, n_gen), dtype=np.int32)
        lg = np.zeros(self.vocab, dtype=np.float32) if want_last_logits else None
        lib().orc_generate_batched(self.h, ptr(p), len(p), n_gen, chunk, ptr(out), ptr(lg) if want_last_logits else None)
        return [int(v) for v in out[:n_gen]], lg

    def set_kv_cache(self, kind):
        """inference.rs:512-531: 0 f32, 1 F16 (NANOCAMELID_KV_CACHE_F16), 2 Q8_0
        (NANOCAMELID_KV_CACHE_Q8); returns the kind in use.  Clears the cache."""
        return lib().orc_model_set_kv_kind(self.h, kind)

    def fill_kv(self, npos, seed=0):
        lib().orc_model_fill_kv(self.h, npos, seed)

    def buf(self, which, n, layer=0):
        p = lib().orc_model_buf(self.h, which, layer)
        return np.ctypeslib.as_array((ctypes.c_float * n).from_address(p)).copy()

    def head_blocks(self):
        return lib().orc_model_head_blocks(self.h)


def spec_generate(target, draft, prompt, n_gen, k):
    p = np.asarray(prompt, dtype=np.int32)
    out = np.zeros(n_gen, dtype=np.int32)
    stats = np.zeros(2, dtype=np.int32)
    n = lib().orc_spec_generate(target.h, draft.h, ptr(p), len(p), n_gen, k, ptr(out), ptr(stats))
    return [int(v) for v in out[:n]], (int(stats[0]), int(stats[1]))


def ngram_draft(history, max_tokens, max_ngram=4, min_ngram=3):
    h = np.asarray(history, dtype=np.int32)
    out = np.zeros(max(1, max_tokens), dtype=np.int32)
    n = lib().orc_ngram_draft(ptr(h), len(h), max_tokens, max_ngram, min_ngram, ptr(out))
    return [int(v) for v in out[:n]]


def ngram_generate(target, prompt, n_gen, k=4, max_ngram=4, min_ngram=3, max_batch=8):
    p = np.asarray(prompt, dtype=np.int32)
    out = np.zeros(max(1, n_gen), dtype=np.int32)
    stats = np.zeros(2, dtype=np.int32)
    n = lib().orc_ngram_generate(target.h, ptr(p), len(p), n_gen, k, max_ngram, min_ngram, max_batch, ptr(out),
                                 ptr(stats))
    return [int(v) for v in out[:n]], (int(stats[0]), int(stats[1]))


class OracleTP:
    def __init__(self, model, shares):
        sh = np.asarray(shares, dtype=np.int32)
        self.model = model
        self.h = lib().orc_tp_build(model.h, ptr(sh), len(sh))
        if not self.h:
            raise RuntimeError("oracle TP build failed (bad shares?)")

    def forward_pass(self, token, pos, want_logits=False):
        lg = np.zeros(self.model.vocab, dtype=np.float32) if want_logits else None
        return lib().orc_tp_forward(self.h, token, pos, ptr(lg) if want_logits else None), lg

    def generate(self, prompt, n_gen):
        p = np.asarray(prompt, dtype=np.int32)
        out = np.zeros(max(1, n_gen), dtype=np.int32)
        lib().orc_tp_generate(self.h, ptr(p), len(p), n_gen, ptr(out))
        return [int(v) for v in out[:n_gen]]
