"""Greedy token parity at full size on the BASELINE configs.

The CPU oracle's decode of each config (random-init synthetic model, seeded prompt) is
stored once in tests/golden/parity_<config>.json by tests/golden/make_parity_fixtures.py.
Each test builds the same model on the GPU, runs the configured prompt and greedy
decode through the C ABI (batched prefill, then the graphed decode steps), and checks:
  * every greedy token equals the oracle's (the gate of bin/cluster_tp_split_smoke.rs:
    101-165 and inference.rs:3649-3670);
  * the last step's logits: the top 32 within 1e-3 of the largest |logit| (the
    north-star tolerance), and all 128256 values bit-identical (their SHA-256), which is
    what the strict-order kernels promise.
"""
import hashlib
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CONFIGS = ["cfg1_1b_q4_0", "cfg2_3b_q4_0", "cfg3_8b_mixed", "cfg5_target_q4_0", "cfg4_70b_q4_0"]


def _fixture(name):
    path = os.path.join(GOLDEN, f"parity_{name}.json")
    if not os.path.exists(path):
        pytest.fail(f"missing fixture {path}: run tests/golden/make_parity_fixtures.py {name}")
    with open(path) as f:
        return json.load(f)


@pytest.mark.parametrize("name", CONFIGS)
def test_full_size_greedy_parity(ncm, cuda, name):
    fx = _fixture(name)
    sp = ncm.CONFIGS[name]
    assert all(getattr(sp, k) == type(getattr(sp, k))(v) for k, v in fx["spec"].items()), "config drifted"
    rng = np.random.default_rng(fx["prompt_seed"])
    prompt = [int(v) for v in rng.integers(0, sp.vocab, size=fx["n_prompt"])]
    n_gen = fx["n_gen"]
    m = ncm.Model.synthetic(sp, ctx_limit=fx["n_prompt"] + n_gen + 1, device=0)
    try:
        got = m.generate(prompt, n_gen)
        first_bad = next((i for i, (a, b) in enumerate(zip(got, fx["tokens"])) if a != b), None)
        assert got == fx["tokens"], f"{name}: first differing greedy token at step {first_bad}"
        _, lg = m.forward_pass(got[-1], fx["n_prompt"] + n_gen - 1, want_logits=True)
    finally:
        m.close()
    d = fx["last_logits"]
    top = np.asarray(d["top_idx"])
    want = np.asarray(d["top_bits"], dtype=np.uint32).view(np.float32)
    err = float(np.max(np.abs(lg[top] - want)))
    assert err <= 1e-3 * d["max_abs"], f"{name}: top-32 logits differ by {err}"
    assert hashlib.sha256(np.ascontiguousarray(lg, dtype=np.float32).tobytes()).hexdigest() == d["sha256"], \
        f"{name}: logits within tolerance (max top-32 diff {err}) but not bit-identical"
