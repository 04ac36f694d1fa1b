"""End-to-end decode on the GPU vs the CPU oracle.

Gates (the reference's own parity rule, README.md:107-115): greedy tokens identical to
the single-node reference path; logits within 1e-3 relative (max |diff| <= 1e-3 *
max |logit|)."""
import os

import numpy as np
import pytest

from conftest import TINY

pytestmark = pytest.mark.gpu


def tiny_spec(ncm, **kw):
    d = dict(TINY)
    d.update(kw)
    return ncm.spec(d["emb"], d["layers"], d["heads"], d["kv_heads"], d["head_dim"], d["ffn"], vocab=d["vocab"],
                    ctx=d["ctx"], tied=d.get("tied", True), t_embd=d.get("t_embd", ncm.Q4_0),
                    t_attn=d.get("t_attn", ncm.Q4_0), t_ffn=d.get("t_ffn", ncm.Q4_0), t_out=d.get("t_out", ncm.Q4_0),
                    seed=d.get("seed", 7), t_down=d.get("t_down", 0))


def prompt_ids(n, vocab, seed=0):
    rng = np.random.default_rng(seed)
    return [int(v) for v in rng.integers(0, vocab, size=n)]


VARIANTS = {
    "q4_0_tied": {},
    "q8_0_untied": dict(tied=False, t_embd=8, t_attn=8, t_ffn=8, t_out=8),
    "mixed_q8attn_q4kffn": dict(tied=False, t_embd=8, t_attn=8, t_ffn=12, t_out=8, emb=512, ffn=1024),
    "q4_0_untied_hd128": dict(tied=False, heads=4, kv_heads=1, head_dim=128, emb=512, ffn=768),
    "q4_0_hd32_mha": dict(heads=8, kv_heads=8, head_dim=32, ffn=2048),
    # widths with an odd number of 32-value blocks (emb 288 = 9 blocks, ffn 800 = 25)
    "q8_0_odd_blocks": dict(tied=False, t_embd=8, t_attn=8, t_ffn=8, t_out=2, heads=9, kv_heads=3,
                            head_dim=32, emb=288, ffn=800),
    # the Q4_K_M layout: Q6_K output.weight and ffn_down (inference.rs:3045-3087)
    "q4k_ffn_q6k_head_down": dict(tied=False, t_embd=8, t_attn=8, t_ffn=12, t_out=14, t_down=14, emb=512,
                                  ffn=1024),
}


@pytest.mark.parametrize("variant", list(VARIANTS))
def test_greedy_decode_matches_oracle(ncm, orc, cuda, tmp_path, variant):
    sp = tiny_spec(ncm, **VARIANTS[variant])
    path = tmp_path / "m.gguf"
    ncm.write_synthetic_gguf(path, sp)
    ref = orc.OracleModel(path)
    prompt = prompt_ids(6, sp.vocab, seed=1)
    n_gen = 24
    ref_tokens, ref_logits = ref.generate(prompt, n_gen, want_last_logits=True)
    m = ncm.Model.load(path, device=0)
    got = m.generate(prompt, n_gen)
    assert got == ref_tokens
    # logits of one more forward pass at the next position
    pos = len(prompt) + n_gen - 1
    t_ref, lg_ref = ref.forward_pass(ref_tokens[-1], pos, want_logits=True)
    t_got, lg_got = m.forward_pass(ref_tokens[-1], pos, want_logits=True)
    assert t_got == t_ref
    assert float(np.max(np.abs(lg_got - lg_ref))) <= 1e-3 * float(np.max(np.abs(lg_ref)))
    # the strict-order kernels give the oracle's bits
    assert np.array_equal(lg_got.view(np.uint32), lg_ref.view(np.uint32))
    m.close()


def test_device_synthetic_equals_gguf_file(ncm, orc, cuda, tmp_path):
    """On-device random init == GGUF writer + load (same blocks), checked through decode."""
    sp = tiny_spec(ncm, tied=False, t_embd=8, t_attn=8, t_ffn=12, t_out=2, emb=512, ffn=1024)
    path = tmp_path / "m.gguf"
    ncm.write_synthetic_gguf(path, sp)
    a = ncm.Model.load(path, device=0)
    b = ncm.Model.synthetic(sp, device=0)
    prompt = prompt_ids(5, sp.vocab, seed=2)
    assert a.generate(prompt, 12) == b.generate(prompt, 12)
    _, la = a.forward_pass(3, 20, want_logits=True)
    _, lb = b.forward_pass(3, 20, want_logits=True)
    assert np.array_equal(la, lb)


def test_forward_pass_host_seam_and_reset(ncm, orc, cuda, tmp_path):
    sp = tiny_spec(ncm)
    path = tmp_path / "m.gguf"
    ncm.write_synthetic_gguf(path, sp)
    ref = orc.OracleModel(path)
    m = ncm.Model.load(path, device=0)
    toks = prompt_ids(10, sp.vocab, seed=5)
    for pos, t in enumerate(toks):
        r, lr = ref.forward_pass(t, pos, want_logits=True)
        g, lg = m.forward_pass(t, pos, want_logits=True)
        assert g == r
        assert float(np.max(np.abs(lg - lr))) <= 1e-3 * float(np.max(np.abs(lr)))
    m.reset()
    ref.reset()
    assert m.generate(toks[:3], 8) == ref.generate(toks[:3], 8)[0]


def test_bad_arguments_fail_loudly(ncm, cuda, tmp_path):
    sp = tiny_spec(ncm)
    m = ncm.Model.synthetic(sp, device=0)
    with pytest.raises(ncm.NcmError):
        m.forward_pass(sp.vocab + 5, 0)
    with pytest.raises(ncm.NcmError):
        m.generate([1, 2, 3], sp.ctx)
    with pytest.raises(ncm.NcmError):
        ncm.Model.load(tmp_path / "missing.gguf")


def test_decode_past_the_context_is_an_error_not_an_overrun(ncm, cuda):
    """Graph-replayed steps read the position on the device, so the host cannot stop a
    caller that decodes more tokens than the context holds.  The step's first kernel holds
    the position at the last slot (no K/V row is stored past the cache) and the error
    word makes the next synchronising call fail; the model stays usable."""
    sp = tiny_spec(ncm, ctx=16)
    m = ncm.Model.synthetic(sp, device=0)
    p = prompt_ids(4, sp.vocab, seed=3)
    first = m.generate(p, 8)
    m.reset()
    m.generate(p, 12)                      # positions 0..15: the context is full
    m.decode_steps(6)                      # past the context
    with pytest.raises(ncm.NcmError, match="context limit"):
        m.sync_tokens(sp.ctx)
    _, pos = m.sync_tokens(sp.ctx)          # the error word was cleared
    assert pos <= sp.ctx
    m.reset()
    assert m.generate(p, 8) == first


@pytest.mark.slow
def test_config1_full_size_token_parity(ncm, orc, cuda, tmp_path):
    """Llama-3.2-1B shape, Q4_0, tied head, 16-token prompt, 32 greedy tokens."""
    sp = ncm.CONFIGS["cfg1_1b_q4_0"]
    path = tmp_path / "cfg1.gguf"
    ncm.write_synthetic_gguf(path, sp)
    prompt = prompt_ids(16, sp.vocab, seed=0)
    ref = orc.OracleModel(path, ctx_limit=64)
    ref_tokens, ref_logits = ref.generate(prompt, 32, want_last_logits=True)
    m = ncm.Model.load(path, ctx_limit=64, device=0)
    got = m.generate(prompt, 32)
    assert got == ref_tokens
    _, lg = m.forward_pass(ref_tokens[-1], 16 + 31, want_logits=True)
    assert float(np.max(np.abs(lg - ref_logits))) <= 1e-3 * float(np.max(np.abs(ref_logits)))


@pytest.mark.parametrize("kind", [1, 2])
def test_greedy_decode_with_f16_q8_kv_cache(ncm, orc, cuda, kind):
    """The reference's opt-in KV caches (NANOCAMELID_KV_CACHE_F16 / _Q8, inference.rs:505-599,
    4319-4458) through the whole decode, batched prefill and verify included: tokens and
    logits equal the oracle's with the same cache, bit for bit."""
    sp = tiny_spec(ncm, tied=False, heads=8, kv_heads=2, head_dim=64, emb=512, ffn=1024, seed=21)
    ref = orc.OracleModel(spec=sp)
    assert ref.set_kv_cache(kind) == kind
    prompt = prompt_ids(11, sp.vocab, seed=4)
    n_gen = 16
    ref_tokens, ref_logits = ref.generate(prompt, n_gen, want_last_logits=True)
    m = ncm.Model.synthetic(sp, device=0)
    m.set_kv_cache(kind)
    got = m.generate(prompt, n_gen)
    assert got == ref_tokens
    _, lg = m.forward_pass(got[-1], len(prompt) + n_gen - 1, want_logits=True)
    assert np.array_equal(lg.view(np.uint32), ref_logits.view(np.uint32))
    # one multi-row pass over the stored cache: each row's greedy token is the decode's
    rows = m.verify_batch(got[:4], len(prompt))
    assert rows == got[1:5]
    m.close()
