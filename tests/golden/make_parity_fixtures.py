"""Regenerates tests/golden/parity_<config>.json: the CPU oracle's greedy decode of the
BASELINE configs at full size (random-init synthetic models, seeded prompts), used by the
GPU token-parity tests so that the oracle's cost is paid once.  Run from the repository
root (hours of CPU time for the 70B shape):
    python tests/golden/make_parity_fixtures.py [config ...]
Each fixture holds the prompt recipe, the greedy tokens, and the logits of the last
decode step as a SHA-256 of their f32 bytes plus the top 32 (index, f32 bits).
"""
import hashlib
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

import nanocamelid_b200 as ncm  # noqa: E402  (the config table only; no library load)
from oracle import oracle as orc  # noqa: E402

# config -> (prompt tokens, greedy tokens).  cfg1 16/32, cfg2 64/128,
# cfg3 512/256, cfg5 target 128/256; cfg4 (70B, 1024-token context) is checked on a
# bounded decode subset of 8 tokens after its full 1024-token context.
RUNS = {
    "cfg1_1b_q4_0": (16, 32),
    "cfg2_3b_q4_0": (64, 128),
    "cfg3_8b_mixed": (512, 256),
    "cfg5_target_q4_0": (128, 256),
    "cfg4_70b_q4_0": (1024, 8),
}
PROMPT_SEED = 0
TOPK = 32


def prompt_ids(n, vocab, seed=PROMPT_SEED):
    rng = np.random.default_rng(seed)
    return [int(v) for v in rng.integers(0, vocab, size=n)]


def logits_digest(lg):
    lg = np.ascontiguousarray(lg, dtype=np.float32)
    top = np.argsort(-lg, kind="stable")[:TOPK]
    return {"sha256": hashlib.sha256(lg.tobytes()).hexdigest(), "top_idx": [int(i) for i in top],
            "top_bits": [int(b) for b in lg[top].view(np.uint32)], "max_abs": float(np.max(np.abs(lg)))}


def make(name):
    sp = ncm.CONFIGS[name]
    n_prompt, n_gen = RUNS[name]
    prompt = prompt_ids(n_prompt, sp.vocab)
    t0 = time.time()
    ref = orc.OracleModel(spec=sp, ctx_limit=n_prompt + n_gen + 1)
    t1 = time.time()
    toks, lg = ref.generate_batched(prompt, n_gen, chunk=64, want_last_logits=True)
    t2 = time.time()
    out = {"config": name, "spec": {k: (float(v) if isinstance(v, float) else int(v)) for k, v in sp.as_dict().items()},
           "prompt_seed": PROMPT_SEED, "n_prompt": n_prompt, "n_gen": n_gen, "tokens": toks,
           "last_logits": logits_digest(lg),
           "oracle_seconds": {"build": round(t1 - t0, 1), "decode": round(t2 - t1, 1)}}
    path = os.path.join(HERE, f"parity_{name}.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print(f"wrote {path}: {toks[:8]}... ({t2 - t0:.0f} s)", flush=True)


if __name__ == "__main__":
    for n in (sys.argv[1:] or list(RUNS)):
        make(n)
