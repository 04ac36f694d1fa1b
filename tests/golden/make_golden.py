"""Regenerates tests/golden/tiny_oracle.json: the CPU oracle's greedy decode of a tiny
synthetic model (writer + oracle regression pin).  Run from the repository root:
    python tests/golden/make_golden.py
"""
import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import numpy as np  # noqa: E402

import nanocamelid_b200 as ncm  # noqa: E402
from conftest import TINY  # noqa: E402
from oracle import oracle as orc  # noqa: E402

OVERRIDES = {"tied": True, "seed": 5}
PROMPT = [17, 400, 3, 999, 512, 8]
N_GEN = 10


def main():
    d = dict(TINY)
    d.update(OVERRIDES)
    sp = ncm.spec(d["emb"], d["layers"], d["heads"], d["kv_heads"], d["head_dim"], d["ffn"], vocab=d["vocab"],
                  ctx=d["ctx"], tied=d["tied"], seed=d["seed"])
    with tempfile.TemporaryDirectory() as t:
        path = os.path.join(t, "m.gguf")
        ncm.write_synthetic_gguf(path, sp)
        toks, lg = orc.OracleModel(path).generate(PROMPT, N_GEN, want_last_logits=True)
    out = {"spec_overrides": OVERRIDES, "prompt": PROMPT, "n_gen": N_GEN, "tokens": toks,
           "logit_bits_head": lg.view(np.uint32)[:16].tolist()}
    with open(os.path.join(HERE, "tiny_oracle.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", os.path.join(HERE, "tiny_oracle.json"), toks)


if __name__ == "__main__":
    main()
