"""Host-side checks that need no GPU: the C-ABI surface, the tensor-parallel plan, the
synthetic GGUF writer against the oracle's loader, and the oracle's own tensor-parallel
and speculative paths (tp.rs, speculative.rs semantics)."""
import os
import re
import struct

import numpy as np
import pytest

from conftest import ROOT, TINY

pytestmark = pytest.mark.cpu


def test_library_exports_every_declared_symbol(ncm):
    """Every function include/ncm.h declares is exported by libncm.so."""
    text = open(os.path.join(ROOT, "include", "ncm.h")).read()
    names = sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_ \*]*?\b(ncm_[a-z0-9_]+)\s*\(", text, re.M)))
    assert len(names) >= 30
    L = ncm.lib()
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


SHAPES = [(32, 8, 14336, 128256), (24, 8, 8192, 128256), (32, 8, 8192, 128256), (64, 8, 28672, 128256)]
SHARES = [[8], [4, 4], [2, 3, 3], [1] * 8, [2, 2, 2, 2]]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("shares", SHARES)
def test_shard_geometry_matches_oracle_and_covers(ncm, orc, shape, shares):
    """tp.rs:641-701: q_start = kv_start*(Hq/Hkv), ffn_start = kv_start*F/Hkv, head rows
    (V*s/Hkv) & !3 with the remainder on the last shard; shards tile every range."""
    heads, kvh, ffn, vocab = shape
    sh = np.asarray(shares, dtype=np.int32)
    ends = {"q": 0, "kv": 0, "ffn": 0, "head": 0}
    for i in range(len(shares)):
        g = ncm.shard_geometry(heads, kvh, ffn, vocab, shares, i)
        ref = np.zeros(8, dtype=np.int32)
        assert orc.lib().orc_shard_geometry(heads, kvh, ffn, vocab, orc.ptr(sh), len(sh), i, orc.ptr(ref)) == 0
        assert list(g.values()) == [int(v) for v in ref]
        assert g["q_start"] == ends["q"] and g["kv_start"] == ends["kv"] and g["ffn_start"] == ends["ffn"]
        assert g["head_row_start"] == ends["head"] and g["head_row_start"] % 4 == 0
        ends["q"] += g["q_heads"]; ends["kv"] += g["kv_heads"]
        ends["ffn"] += g["ffn_len"]; ends["head"] += g["head_rows"]
    assert (ends["q"], ends["kv"], ends["ffn"], ends["head"]) == (heads, kvh, ffn, vocab)


@pytest.mark.parametrize("shares", [[3, 3], [0, 8], [1, 1, 1]])
def test_shard_geometry_rejects_bad_shares(ncm, shares):
    """tp.rs:641-660 validate_shares: sum must equal the KV heads, no empty shard."""
    with pytest.raises(ncm.NcmError):
        ncm.shard_geometry(32, 8, 14336, 128256, shares, 0)


def test_even_shares():
    from nanocamelid_b200 import tp
    assert tp.even_shares(8, 4) == [2, 2, 2, 2]
    with pytest.raises(ValueError):
        tp.even_shares(8, 3)


def test_default_shares_even_or_remainder_last(ncm):
    from nanocamelid_b200 import tp
    assert tp.default_shares(8, 3) == [2, 3, 3]
    assert tp.default_shares(8, 8) == [1] * 8 and tp.default_shares(8, 2) == [4, 4]
    assert tp.default_shares(8, 5) == [1, 1, 2, 2, 2]
    for world in range(1, 9):   # every default plan is one validate_shares accepts
        sh = tp.default_shares(8, world)
        for i in range(world):
            ncm.shard_geometry(32, 8, 14336, 128256, sh, i)
    with pytest.raises(ValueError):
        tp.default_shares(8, 9)


# ---------------------------------------------------------------- GGUF
GGUF_SCALAR = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}


def _gguf_value(f, t):
    if t in GGUF_SCALAR:
        f.read(GGUF_SCALAR[t])
    elif t == 8:
        (n,) = struct.unpack("<Q", f.read(8))
        f.read(n)
    elif t == 9:
        et, n = struct.unpack("<IQ", f.read(12))
        for _ in range(n):
            _gguf_value(f, et)
    else:
        raise ValueError(f"GGUF value type {t}")


DIMS_AT = {}


def read_gguf_tensors(path):
    """Minimal GGUF v3 reader (gguf.rs:454-551): {name: (type, dims, data offset)}."""
    with open(path, "rb") as f:
        assert f.read(4) == b"GGUF"
        ver, nt, nkv = struct.unpack("<IQQ", f.read(20))
        align = 32
        for _ in range(nkv):
            (kl,) = struct.unpack("<Q", f.read(8))
            key = f.read(kl).decode()
            (t,) = struct.unpack("<I", f.read(4))
            if key == "general.alignment" and t == 4:
                (align,) = struct.unpack("<I", f.read(4))
            else:
                _gguf_value(f, t)
        infos = {}
        for _ in range(nt):
            (nl,) = struct.unpack("<Q", f.read(8))
            name = f.read(nl).decode()
            (nd,) = struct.unpack("<I", f.read(4))
            dims_at = f.tell()
            dims = struct.unpack("<" + "Q" * nd, f.read(8 * nd))
            t, off = struct.unpack("<IQ", f.read(12))
            infos[name] = (t, dims, off)
            DIMS_AT[(str(path), name)] = dims_at
        base = (f.tell() + align - 1) // align * align
    return {k: (t, d, base + o) for k, (t, d, o) in infos.items()}


def tiny(ncm, **kw):
    d = dict(TINY)
    d.update(kw)
    return ncm.spec(d["emb"], d["layers"], d["heads"], d["kv_heads"], d["head_dim"], d["ffn"], vocab=d["vocab"],
                    ctx=d["ctx"], tied=d.get("tied", True), t_embd=d.get("t_embd", ncm.Q4_0),
                    t_attn=d.get("t_attn", ncm.Q4_0), t_ffn=d.get("t_ffn", ncm.Q4_0), t_out=d.get("t_out", ncm.Q4_0),
                    seed=d.get("seed", 7), t_down=d.get("t_down", 0))


def test_gguf_writer_blocks_equal_host_generator(ncm, tmp_path):
    """The synthetic GGUF's tensor bytes equal ncm_synth_tensor_host (the same generator
    the on-device initialiser runs), including column slices."""
    sp = tiny(ncm, tied=False, t_embd=ncm.Q8_0, t_attn=ncm.Q8_0, t_ffn=ncm.Q4_K, t_out=ncm.Q4_0, emb=512, ffn=1024)
    path = tmp_path / "m.gguf"
    ncm.write_synthetic_gguf(path, sp)
    tens = read_gguf_tensors(path)
    raw = open(path, "rb").read()
    bb = {ncm.Q4_0: (18, 32), ncm.Q8_0: (34, 32), ncm.Q4_K: (144, 256)}
    for name in ["blk.0.attn_q.weight", "blk.1.ffn_down.weight", "blk.0.ffn_gate.weight", "output.weight"]:
        t, dims, off = tens[name]
        cols, rows = dims[0], dims[1]
        b, e = bb[t]
        row_bytes = cols // e * b
        want = ncm.synth_tensor_bytes(sp, name, t, 0, rows, 0, cols, cols)
        assert raw[off:off + rows * row_bytes] == want, name
        c0, c1 = e, 3 * e
        part = ncm.synth_tensor_bytes(sp, name, t, 1, 3, c0, c1, cols)
        exp = b"".join(raw[off + r * row_bytes + c0 // e * b: off + r * row_bytes + c1 // e * b] for r in (1, 2))
        assert part == exp, name


@pytest.mark.parametrize("qtype", ["Q4_0", "Q8_0", "Q4_K", "Q6_K"])
def test_oracle_generator_equals_product_generator(ncm, orc, qtype):
    """The oracle's own restatement of the synthetic-weight generator (used by the CPU
    baseline, which loads no product code) gives the product's bytes, slices included."""
    t = getattr(ncm, qtype)
    sp = tiny(ncm, emb=512, ffn=1024, seed=23)
    for name, rows, cols in [("blk.0.ffn_gate.weight", 5, 512), ("blk.1.ffn_down.weight", 3, 1024)]:
        assert orc.synth_tensor(sp, name, t, 0, rows, 0, cols, cols) == \
            ncm.synth_tensor_bytes(sp, name, t, 0, rows, 0, cols, cols), name
        e = 256 if t in (ncm.Q4_K, ncm.Q6_K) else 32
        assert orc.synth_tensor(sp, name, t, 1, 3, e, 3 * e, cols) == \
            ncm.synth_tensor_bytes(sp, name, t, 1, 3, e, 3 * e, cols), name


@pytest.mark.parametrize("kw", [dict(tied=True), dict(tied=False, t_embd=8, t_attn=8, t_ffn=12, t_out=8, ffn=768),
                                dict(tied=False, t_embd=8, t_attn=8, t_ffn=12, t_out=14, t_down=14, ffn=768)])
def test_oracle_synthetic_model_equals_gguf_model(ncm, orc, tmp_path, kw):
    """orc_model_create_synthetic builds in memory exactly the model orc_model_load reads
    from the synthetic GGUF file; the batched prefill decodes like the token-by-token one."""
    sp = tiny(ncm, **kw)
    path = tmp_path / "m.gguf"
    ncm.write_synthetic_gguf(path, sp)
    prompt = _prompt(7, sp.vocab, 3)
    a = orc.OracleModel(path).generate(prompt, 6, want_last_logits=True)
    b = orc.OracleModel(spec=sp).generate(prompt, 6, want_last_logits=True)
    c = orc.OracleModel(spec=sp).generate_batched(prompt, 6, chunk=3, want_last_logits=True)
    assert a[0] == b[0] == c[0]
    assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))
    assert np.array_equal(a[1].view(np.uint32), c[1].view(np.uint32))


def test_gguf_writer_is_deterministic_and_loads(ncm, orc, tmp_path):
    sp = tiny(ncm)
    a, b = tmp_path / "a.gguf", tmp_path / "b.gguf"
    ncm.write_synthetic_gguf(a, sp, threads=1)
    ncm.write_synthetic_gguf(b, sp, threads=4)
    assert open(a, "rb").read() == open(b, "rb").read()
    m = orc.OracleModel(a)
    assert (m.emb, m.layers, m.heads, m.kv_heads, m.head_dim, m.ffn, m.vocab) == (
        TINY["emb"], TINY["layers"], TINY["heads"], TINY["kv_heads"], TINY["head_dim"], TINY["ffn"], TINY["vocab"])


# ---------------------------------------------------------------- oracle TP / speculative
def _prompt(n, vocab, seed):
    return [int(v) for v in np.random.default_rng(seed).integers(0, vocab, size=n)]


@pytest.mark.parametrize("kvh,heads,shares", [(2, 4, [1, 1]), (8, 8, [2, 3, 3]), (8, 8, [1] * 8)])
def test_oracle_tp_matches_single_node(ncm, orc, tmp_path, kvh, heads, shares):
    """bin/cluster_tp_split_smoke.rs:101-165 semantics: TP greedy tokens identical to the
    single-node path, logits within 1e-3 relative."""
    hd = TINY["emb"] // heads
    sp = tiny(ncm, kv_heads=kvh, heads=heads, head_dim=hd, ffn=2048 if kvh == 8 else 512)
    path = tmp_path / "m.gguf"
    ncm.write_synthetic_gguf(path, sp)
    full = orc.OracleModel(path)
    tp = orc.OracleTP(orc.OracleModel(path), shares)
    prompt = _prompt(5, sp.vocab, 3)
    ref = full.generate(prompt, 12)[0]
    assert tp.generate(prompt, 12) == ref
    full.reset()
    tp = orc.OracleTP(orc.OracleModel(path), shares)
    for pos, t in enumerate(prompt):
        _, la = full.forward_pass(t, pos, want_logits=True)
        _, lb = tp.forward_pass(t, pos, want_logits=True)
        assert float(np.max(np.abs(la - lb))) <= 1e-3 * float(np.max(np.abs(la)))


def test_oracle_speculative_equals_greedy(ncm, orc, tmp_path):
    """speculative.rs:299-494: greedy speculative decoding emits the target's greedy tokens."""
    tgt_spec = tiny(ncm, seed=11)
    draft_spec = tiny(ncm, seed=12, layers=1)
    pt, pd = tmp_path / "t.gguf", tmp_path / "d.gguf"
    ncm.write_synthetic_gguf(pt, tgt_spec)
    ncm.write_synthetic_gguf(pd, draft_spec)
    prompt = _prompt(6, tgt_spec.vocab, 4)
    greedy = orc.OracleModel(pt).generate(prompt, 16)[0]
    for k in (1, 4):
        toks, stats = orc.spec_generate(orc.OracleModel(pt), orc.OracleModel(pd), prompt, 16, k)
        assert toks == greedy, k


def test_oracle_regression_fixture(ncm, orc, tmp_path):
    """tests/golden/tiny_oracle.json (made by tests/golden/make_golden.py): greedy tokens and
    a logit checksum of the oracle on a tiny synthetic model -- pins the writer + oracle
    against silent drift."""
    import json
    g = json.load(open(os.path.join(ROOT, "tests", "golden", "tiny_oracle.json")))
    sp = tiny(ncm, **g["spec_overrides"])
    path = tmp_path / "m.gguf"
    ncm.write_synthetic_gguf(path, sp)
    m = orc.OracleModel(path)
    toks, lg = m.generate(g["prompt"], g["n_gen"], want_last_logits=True)
    assert toks == g["tokens"]
    assert lg.view(np.uint32)[: len(g["logit_bits_head"])].tolist() == g["logit_bits_head"]


def test_rank_ordered_sum_and_per_row_head_merge():
    """tp.rank_ordered: f32 sum from 0.0f in rank order (tp.rs:349-363); head pairs
    merged per row by strict '>' in rank order, token bits copied unchanged."""
    from nanocamelid_b200 import PHASE_FFN, PHASE_HEAD
    from nanocamelid_b200 import tp
    rng = np.random.default_rng(5)
    parts = [(rng.standard_normal(64) * 10.0 ** rng.integers(-4, 4, 64)).astype(np.float32) for _ in range(3)]
    want = np.float32(0.0) + parts[0]
    want = (want + parts[1]).astype(np.float32)
    want = (want + parts[2]).astype(np.float32)
    assert np.array_equal(tp.rank_ordered(parts, PHASE_FFN).view(np.uint32), want.view(np.uint32))
    pairs = []
    for r, logits in enumerate(([1.0, 5.0, 2.0], [3.0, 5.0, 2.0], [3.0, 4.0, 9.0])):
        a = np.zeros(6, dtype=np.float32)
        a[0::2] = logits
        a.view(np.int32)[1::2] = [100 * r + 1, 100 * r + 2, 100 * r + 3]   # denormal bit patterns
        pairs.append(a)
    got = tp.rank_ordered(pairs, PHASE_HEAD)
    assert got[0::2].tolist() == [3.0, 5.0, 9.0]
    assert got.view(np.int32)[1::2].tolist() == [101, 2, 203]


# ---------------------------------------------------------------- n-gram drafter
NGRAM_KATS = [   # speculative.rs:561-595: (history, max_tokens, max_ngram, min_ngram, draft)
    ([1, 2, 3, 4, 5, 6, 9, 9, 1, 2, 3, 4], 3, 4, 3, [5, 6, 9]),
    ([3, 4, 7, 0, 3, 4, 8, 0, 3, 4], 2, 4, 3, [8, 0]),
    ([1, 2, 3, 4, 5], 4, 4, 3, []),
    ([1, 2], 4, 4, 3, []),
    ([], 4, 4, 3, []),
    ([1, 2, 9, 8, 7, 6, 1, 2], 2, 3, 2, [9, 8]),
    ([1, 2, 9, 8, 7, 6, 1, 2], 10, 3, 2, [9, 8, 7, 6, 1, 2]),
]


@pytest.mark.parametrize("kat", NGRAM_KATS)
def test_ngram_draft_reference_vectors(ncm, orc, kat):
    """NGramDrafter::draft (speculative.rs:80-105) on the reference's own test vectors,
    for the library's host drafter and the oracle's restatement."""
    history, max_tokens, max_n, min_n, want = kat
    assert ncm.ngram_draft(history, max_tokens, max_n, min_n) == want
    assert orc.ngram_draft(history, max_tokens, max_n, min_n) == want


def test_ngram_draft_matches_oracle_on_random_histories(ncm, orc):
    rng = np.random.default_rng(11)
    for trial in range(400):
        h = [int(v) for v in rng.integers(0, int(rng.integers(2, 6)), size=int(rng.integers(0, 40)))]
        max_tokens, max_n = int(rng.integers(1, 9)), int(rng.integers(1, 6))
        min_n = int(rng.integers(1, max_n + 1))
        assert ncm.ngram_draft(h, max_tokens, max_n, min_n) == orc.ngram_draft(h, max_tokens, max_n, min_n), trial


def test_oracle_ngram_generate_equals_greedy(ncm, orc, tmp_path):
    """ngram_speculative_step (speculative.rs:122-297): the emitted stream is the plain
    greedy loop's."""
    sp = tiny(ncm, seed=13)
    path = tmp_path / "m.gguf"
    ncm.write_synthetic_gguf(path, sp)
    prompt = [5, 9, 2, 7, 5, 9, 2, 7, 5, 9]
    greedy = orc.OracleModel(path).generate(prompt, 20)[0]
    for k in (1, 4):
        toks, (drafted, accepted) = orc.ngram_generate(orc.OracleModel(path), prompt, 20, k)
        assert toks == greedy, k
        assert 0 <= accepted <= drafted


def _header_prototypes():
    """{name: parameter count} for every function include/ncm.h declares."""
    text = open(os.path.join(ROOT, "include", "ncm.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    protos = {}
    for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_ \*]*?\b(ncm_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text,
                         re.M | re.S):
        args = m.group(2).strip()
        protos[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return protos


def test_python_bindings_match_header_arity(ncm):
    """The ctypes mirror declares every header function with the header's parameter
    count (guards the C ABI against drift)."""
    protos = _header_prototypes()
    assert len(protos) >= 30
    L = ncm.lib()
    for name, n in protos.items():
        fn = getattr(L, name)
        if fn.argtypes is None:
            continue   # not used from Python
        assert len(fn.argtypes) == n, (name, len(fn.argtypes), n)


_FUZZ = r'''
import ctypes, sys
import numpy as np
import nanocamelid_b200 as ncm
raw = open(sys.argv[1], "rb").read()
L = ncm.lib()
def load(b):
    open(sys.argv[2], "wb").write(b)
    h = ctypes.c_void_p()
    # device -1: parsing runs in full, then device selection fails before any allocation
    return L.ncm_model_load(sys.argv[2].encode(), 0, -1, None, 0, 0, ctypes.byref(h))
rng = np.random.default_rng(0)
hdr = int(sys.argv[3])
bad = []
for cut in sorted(set(int(v) for v in np.linspace(0, len(raw) - 1, 60)) | set(range(0, hdr, max(1, hdr // 40)))):
    s = load(raw[:cut])
    if s != 5:
        bad.append(("truncated", cut, s))
for trial in range(300):
    b = bytearray(raw[:hdr + 64])
    for _ in range(int(rng.integers(1, 6))):
        b[int(rng.integers(0, hdr))] = int(rng.integers(0, 256))
    s = load(bytes(b) + raw[hdr + 64:])
    if s not in (0, 1, 2, 5, 6):
        bad.append(("corrupt", trial, s))
print("BAD", bad)
'''


def test_gguf_reader_rejects_truncated_and_corrupt_files(ncm, tmp_path):
    """The GGUF reader (gguf.rs:454-551 semantics) on hostile files: every truncation is
    NCM_EIO, and random byte corruption of the header and tensor table ends in a status
    (parse error, or a parse that then stops at device selection), never a crash."""
    import subprocess
    import sys
    sp = tiny(ncm)
    path = tmp_path / "m.gguf"
    ncm.write_synthetic_gguf(path, sp)
    hdr = min(read_gguf_tensors(path).values(), key=lambda v: v[2])[2]   # first tensor's data offset
    r = subprocess.run([sys.executable, "-c", _FUZZ, str(path), str(tmp_path / "x.gguf"), str(hdr)],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, (r.returncode, r.stderr[-2000:])
    assert "BAD []" in r.stdout, r.stdout[-2000:]


@pytest.mark.parametrize("name,dim", [("blk.1.attn_norm.weight", 224), ("output_norm.weight", 128),
                                      ("blk.0.ffn_norm.weight", 512)])
def test_model_load_rejects_misshapen_norm_tensors(ncm, tmp_path, name, dim):
    """A norm tensor whose length is not the embedding width (shorter ones could read past
    the mapped file) is rejected with NCM_EIO by the host-side tensor check, before any
    device is touched (device -1 here)."""
    import ctypes
    sp = tiny(ncm)
    path = tmp_path / "m.gguf"
    ncm.write_synthetic_gguf(path, sp)
    read_gguf_tensors(path)
    raw = bytearray(open(path, "rb").read())
    at = DIMS_AT[(str(path), name)]
    raw[at:at + 8] = struct.pack("<Q", dim)
    bad = tmp_path / "bad.gguf"
    open(bad, "wb").write(bytes(raw))
    h = ctypes.c_void_p()
    st = ncm.lib().ncm_model_load(str(bad).encode(), 0, -1, None, 0, 0, ctypes.byref(h))
    assert st == 5, (st, ncm.lib().ncm_last_error())
    assert name.encode() in ncm.lib().ncm_last_error()
