"""Speculative verify on the GPU: the multi-row (tensor-core) GEMV, the multi-row target
pass and greedy speculative decoding (speculative.rs:299-494, inference.rs:6866-6913:
every batch row equals the one-row result; the speculative output equals the target's
greedy decode)."""
import numpy as np
import pytest

from conftest import TINY

pytestmark = pytest.mark.gpu

BB = {2: 18, 8: 34, 12: 144}
BE = {2: 32, 8: 32, 12: 256}


def random_blocks(qtype, rows, cols, seed):
    rng = np.random.default_rng(seed)
    nb = rows * (cols // BE[qtype])
    raw = rng.integers(0, 256, size=(nb, BB[qtype]), dtype=np.uint8)
    scales = (rng.standard_normal(nb) * 0.01).astype(np.float16).view(np.uint16)
    raw[:, 0], raw[:, 1] = scales & 0xFF, scales >> 8
    if qtype == 12:
        dmin = (np.abs(rng.standard_normal(nb)) * 0.003).astype(np.float16).view(np.uint16)
        raw[:, 2], raw[:, 3] = dmin & 0xFF, dmin >> 8
    return raw.reshape(-1)


@pytest.mark.parametrize("qtype", [2, 8, 12])
@pytest.mark.parametrize("rows,cols", [(300, 4096), (37, 512), (2100, 3072), (64, 14336), (45, 96), (130, 288)])
@pytest.mark.parametrize("ntok", [1, 5, 8])
def test_batch_rows_bit_equal_single_rows(ncm, orc, cuda, qtype, rows, cols, ntok):
    torch = cuda
    if cols % BE[qtype]:
        pytest.skip("Q4_K needs 256-aligned columns")
    w = random_blocks(qtype, rows, cols, seed=rows + cols + qtype)
    x = np.random.default_rng(ntok + rows).standard_normal((ntok, cols)).astype(np.float32)
    qs = [orc.quantize_q8_0(x[t]) for t in range(ntok)]
    xq = np.concatenate([q for q, _ in qs])
    xs = np.concatenate([s for _, s in qs])
    keep = [torch.from_numpy(a).cuda() for a in (xq, xs, w)]
    out = torch.full((ntok * rows,), float("nan"), dtype=torch.float32, device="cuda")
    ncm.matmul_quantized_batch(out.data_ptr(), keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), ntok,
                               rows, cols, qtype)
    single = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
    got = out.cpu().numpy().reshape(ntok, rows)
    ref = orc.matmul_batch(qtype, w, rows, cols, ntok, xq, xs)
    for t in range(ntok):
        ncm.matmul_quantized(single.data_ptr(), keep[0].data_ptr() + t * cols, keep[1].data_ptr() + t * cols // 8,
                             keep[2].data_ptr(), rows, cols, qtype)
        torch.cuda.synchronize()
        assert np.array_equal(got[t].view(np.uint32), single.cpu().numpy().view(np.uint32)), t
    assert float(np.max(np.abs(got - ref))) <= 1e-4 * float(np.max(np.abs(ref)))


def tiny(ncm, **kw):
    d = dict(TINY)
    d.update(kw)
    return ncm.spec(d["emb"], d["layers"], d["heads"], d["kv_heads"], d["head_dim"], d["ffn"], vocab=d["vocab"],
                    ctx=d["ctx"], tied=d.get("tied", True), t_embd=d.get("t_embd", ncm.Q4_0),
                    t_attn=d.get("t_attn", ncm.Q4_0), t_ffn=d.get("t_ffn", ncm.Q4_0), t_out=d.get("t_out", ncm.Q4_0),
                    seed=d.get("seed", 7))


VARIANTS = {
    "q4_0_tied": {},
    "mixed_q8attn_q4kffn": dict(tied=False, t_embd=8, t_attn=8, t_ffn=12, t_out=8, emb=512, ffn=1024),
    "q4_0_hd128": dict(tied=False, heads=4, kv_heads=1, head_dim=128, emb=512, ffn=768),
    "q8_0_odd_blocks": dict(tied=False, t_embd=8, t_attn=8, t_ffn=8, t_out=2, heads=9, kv_heads=3, head_dim=32,
                            emb=288, ffn=800),
}


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_verify_rows_equal_sequential_steps(ncm, cuda, variant):
    """Each verify row's greedy token equals the one-token step at that position, and the
    K/V written by the multi-row pass equal the one-token steps' (inference.rs:3695)."""
    sp = tiny(ncm, **VARIANTS[variant])
    a = ncm.Model.synthetic(sp, device=0)
    b = ncm.Model.synthetic(sp, device=0)
    prompt = [int(v) for v in np.random.default_rng(3).integers(0, sp.vocab, size=6)]
    a.generate(prompt, 1)
    b.generate(prompt, 1)
    toks = [int(v) for v in np.random.default_rng(4).integers(0, sp.vocab, size=5)]
    rows = a.verify_batch(toks, len(prompt))
    seq = [b.forward_pass(t, len(prompt) + i)[0] for i, t in enumerate(toks)]
    assert rows == seq
    kw = sp.kv_heads * sp.head_dim
    for layer in (0, sp.layers - 1):
        for which in (4, 5):
            ka = a.debug_read(which, (len(prompt) + len(toks)) * kw, layer)
            kb = b.debug_read(which, (len(prompt) + len(toks)) * kw, layer)
            assert np.array_equal(ka.view(np.uint32), kb.view(np.uint32)), (layer, which)


@pytest.mark.parametrize("k", [1, 4, 8])
def test_spec_generate_equals_target_greedy(ncm, orc, cuda, tmp_path, k):
    tsp = tiny(ncm, seed=11)
    dsp = tiny(ncm, seed=12, layers=1)
    prompt = [int(v) for v in np.random.default_rng(5).integers(0, tsp.vocab, size=7)]
    n_gen = 30
    target = ncm.Model.synthetic(tsp, device=0)
    draft = ncm.Model.synthetic(dsp, device=0)
    greedy = ncm.Model.synthetic(tsp, device=0).generate(prompt, n_gen)
    toks, (drafted, accepted) = target.spec_generate(draft, prompt, n_gen, k=k)
    assert toks == greedy
    assert 0 <= accepted <= drafted
    # and the oracle's speculative restatement agrees
    pt, pd = tmp_path / "t.gguf", tmp_path / "d.gguf"
    ncm.write_synthetic_gguf(pt, tsp)
    ncm.write_synthetic_gguf(pd, dsp)
    ref, ref_stats = orc.spec_generate(orc.OracleModel(pt), orc.OracleModel(pd), prompt, n_gen, k)
    assert toks == ref
    assert (drafted, accepted) == tuple(ref_stats)


def test_spec_self_draft_accepts_everything(ncm, cuda):
    """Draft == target: every drafted token is accepted (speculative.rs:418-433)."""
    sp = tiny(ncm, seed=21)
    prompt = [3, 14, 15, 92]
    target = ncm.Model.synthetic(sp, device=0)
    draft = ncm.Model.synthetic(sp, device=0)
    toks, (drafted, accepted) = target.spec_generate(draft, prompt, 25, k=4)
    assert toks == ncm.Model.synthetic(sp, device=0).generate(prompt, 25)
    assert accepted == drafted


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_batched_prefill_equals_token_by_token(ncm, cuda, variant):
    """The prompt is ingested eight rows per multi-row pass (the verify kernels): the K/V
    of every prompt position, the first generated token and the decode after it equal a
    token-by-token ingestion (one-token steps) bit for bit."""
    sp = tiny(ncm, **VARIANTS[variant])
    prompt = [int(v) for v in np.random.default_rng(8).integers(0, sp.vocab, size=19)]   # 8 + 8 + 3 rows
    a = ncm.Model.synthetic(sp, device=0)
    b = ncm.Model.synthetic(sp, device=0)
    ga = a.generate(prompt, 6)
    for pos, t in enumerate(prompt):
        nxt = b.forward_pass(t, pos)[0]
    assert ga[0] == nxt
    kw = sp.kv_heads * sp.head_dim
    for layer in range(sp.layers):
        for which in (4, 5):
            ka = a.debug_read(which, len(prompt) * kw, layer)
            kb = b.debug_read(which, len(prompt) * kw, layer)
            assert np.array_equal(ka.view(np.uint32), kb.view(np.uint32)), (layer, which)
    for i in range(1, len(ga)):   # the decode after the prompt continues identically
        assert b.forward_pass(ga[i - 1], len(prompt) + i - 1)[0] == ga[i], i


@pytest.mark.parametrize("k", [1, 4, 8])
def test_ngram_generate_equals_greedy_and_oracle(ncm, orc, cuda, tmp_path, k):
    """Prompt-lookup speculation (speculative.rs:122-297, main.rs:9720-9760): t0 and the
    history drafts verified in one multi-row pass; tokens equal the greedy decode, and
    tokens and drafted / accepted counts equal the oracle's restatement."""
    sp = tiny(ncm, seed=21)
    prompt = [308, 799, 395, 620, 308, 799, 395, 620, 308, 799, 395, 620, 308]
    n_gen = 40
    greedy = ncm.Model.synthetic(sp, device=0).generate(prompt, n_gen)
    toks, stats = ncm.Model.synthetic(sp, device=0).ngram_generate(prompt, n_gen, k=k)
    assert toks == greedy
    path = tmp_path / "m.gguf"
    ncm.write_synthetic_gguf(path, sp)
    ref, ref_stats = orc.ngram_generate(orc.OracleModel(path), prompt, n_gen, k)
    assert toks == ref
    assert stats == ref_stats
    assert stats[0] > stats[1] > 0   # drafts accepted and one rejected (corrective step)
