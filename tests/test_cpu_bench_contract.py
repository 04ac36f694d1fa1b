"""bench.py's reference arm on the host cores: the JSON line the driver reads (impl,
metric, cpu_baseline, e2e with zero host<->device bytes), and that ranks other than 0
exit cleanly without work under torchrun."""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.cpu


def _run(extra_env, *args):
    env = dict(os.environ, **extra_env)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          env=env, timeout=600, cwd=ROOT)


def test_reference_arm_json_line():
    r = _run({}, "--impl", "reference", "--config", "cfg1_1b_q4_0", "--steps", "2", "--warmup", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == "bs1 decode tok/s" and line["unit"] == "tok/s"
    assert line["higher_is_better"] is True and line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"] and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_do_no_work():
    r = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, "--impl", "reference", "--gpus", "2",
             "--steps", "2", "--warmup", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_decode_phases_stay_inside_the_context():
    """Every phase of the decode bench (fused timed steps, then the NCCL baseline, which
    restarts with one forward_pass and two untimed steps) writes positions below ctx."""
    sys.path.insert(0, ROOT)
    import bench
    for prompt in (64, 1024):
        for warmup in (0, 1, 3, 5, 8):
            for steps in (1, 20, 60, 120, 500):
                ctx = bench.decode_context(prompt, warmup, steps)
                assert prompt + warmup + steps <= ctx          # fused phase: last step at pos - 1
                start = bench.nccl_phase_start(prompt, warmup)
                assert start >= prompt
                assert start + 1 + 2 + steps <= ctx          # NCCL phase
                if warmup >= 3:                               # the same timed positions
                    assert start + 3 == prompt + warmup
