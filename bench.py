"""Decode benchmark: bs1 greedy decode tok/s on BASELINE.json configs[1] (Llama-3.2-3B
shape, Q4_0, tied head, random-init N(0, 0.02), 64-token seeded prompt) at N GPUs of one
node (tensor parallel over KV-head shares -- even, or --shares such as 2,3,3 -- with the
fused NVLink reduction).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {b200,reference}]
                  [--reducer {p2p,nccl}] [--config NAME]

A step is one decode token (one full forward + greedy argmax at the next position).
`value` = K / (device time of K steps, max over ranks) with all weights resident in HBM;
`e2e` = the same through the C-ABI forward_pass with host token in / argmax out per step.
The reference arm times the CPU restatement of the reference's portable path (the
reference is Rust and cannot be built here) on a bounded sample of the same workload.
"""
import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "bs1 decode tok/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=120)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--reducer", default="p2p", choices=["p2p", "nccl"])
    ap.add_argument("--shares", default="", help="KV-head shares per rank, e.g. 2,3,3 (default: even, remainder last)")
    ap.add_argument("--config", default="cfg2_3b_q4_0")
    ap.add_argument("--prompt", type=int, default=64)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--spec", action="store_true",
                    help="BASELINE config 5: greedy speculative decoding, draft = config 1, target = config-3 "
                         "shape all Q4_0, k = 4, 128-token prompt, 256 tokens (one GPU)")
    ap.add_argument("--verify-only", action="store_true",
                    help="config 5 target: time the multi-row verify pass (1/4/5/8 rows) and one graphed step")
    ap.add_argument("--verify-rows", default="1,4,5,8")
    ap.add_argument("--gemv-only", action="store_true",
                    help="only the roofline GEMV (head-shaped Q4_0 matrix): the small case for ncu captures")
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    def __init__(self, index):
        self.index, self.samples, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 7:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for s in self.samples for n, v in zip(names, s[3:7]) if v.lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": float(self.samples[0][1]),
                "reasons": reasons}


def weight_bytes(sp, world, shares=None):
    """Algorithmic weight bytes read per decoded token, per GPU (the largest shard: its
    KV-head fraction of every sharded matrix and of the vocab rows)."""
    bpw = {2: 18 / 32, 8: 34 / 32, 12: 144 / 256}
    H, F, hd = sp.emb, sp.ffn, sp.head_dim
    qw, kw = sp.heads * hd, sp.kv_heads * hd
    layer = (qw * H + 2 * kw * H + H * qw) * bpw[sp.t_attn] + 3 * F * H * bpw[sp.t_ffn]
    head = sp.vocab * H * (bpw[2] if sp.tied else bpw[sp.t_out])
    frac = max(shares) / sp.kv_heads if shares else 1.0 / world
    return (sp.layers * layer + head) * frac


class OracleRun:
    """The CPU restatement of the reference's portable path (oracle/) on the same model."""

    def __init__(self, sp):
        import numpy as np
        import nanocamelid_b200 as ncm
        from oracle import oracle as orc
        self.tmp = tempfile.TemporaryDirectory()
        path = os.path.join(self.tmp.name, "m.gguf")
        ncm.write_synthetic_gguf(path, sp)
        self.ref = orc.OracleModel(path, ctx_limit=64)
        rng = np.random.default_rng(0)
        self.pos, self.tok = 0, 0
        for t in [int(v) for v in rng.integers(0, sp.vocab, 4)]:
            self.step(t)

    def step(self, tok=None):
        self.tok, _ = self.ref.forward_pass(self.tok if tok is None else tok, self.pos)
        self.pos += 1

    def timed(self, n, budget_s):
        k, t0 = 0, time.perf_counter()
        while k < n and time.perf_counter() - t0 < budget_s and self.pos < 63:
            self.step()
            k += 1
        return k, time.perf_counter() - t0


def cpu_sample(sp, budget_s=20.0):
    run = OracleRun(sp)
    run.step()
    n, dt = run.timed(32, budget_s)
    return {"value": round(n / dt, 3), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} greedy decode tokens after a 4-token prompt on the same model: CPU restatement of the "
                      f"reference x86 portable path (oracle/, OpenMP over {os.cpu_count()} threads)"}


def run_reference(args, sp, rank):
    if rank != 0:
        return
    run = OracleRun(sp)
    for _ in range(min(args.warmup, 3)):
        run.step()
    n, dt = run.timed(args.steps, 30.0)
    v = n / dt
    cpu = {"value": round(v, 3), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
           "sample": f"{n} greedy decode tokens after a 4-token prompt (+{min(args.warmup, 3)} warm-up tokens), "
                     f"CPU restatement of the reference x86 portable path, OpenMP over {os.cpu_count()} threads"}
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tok/s",
                      "n_gpus": args.gpus, "steps": n, "warmup": min(args.warmup, 3), "higher_is_better": True,
                      "dtype": "int8 dot / f32", "data": "synthetic", "config": {"workload": args.config, "prompt": 4},
                      "cpu_baseline": cpu, "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                                                   "d2h_bytes_per_step": 0}}), flush=True)


def gemv_roofline(torch, ncm, sp, peak):
    """Times the strict Q4_0 GEMV on the workload's largest Q4_0 matrix (the tied LM head,
    vocab x hidden, > L2) with CUDA events on its launch stream."""
    import numpy as np
    rows, cols = sp.vocab, sp.emb
    nbytes = rows * cols // 32 * 18
    w = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    w.view(-1)[:] = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda")
    blocks = w.view(rows * cols // 32, 18)
    blocks[:, 1] = 0x20   # f16 scales ~1e-2: finite, normal
    xq = torch.randint(-127, 128, (cols,), dtype=torch.int8, device="cuda")
    xs = torch.full((cols // 32,), 0.01, dtype=torch.float32, device="cuda")
    out = torch.empty(rows, dtype=torch.float32, device="cuda")
    s = torch.cuda.current_stream()
    for _ in range(3):
        ncm.matmul_quantized(out.data_ptr(), xq.data_ptr(), xs.data_ptr(), w.data_ptr(), rows, cols, ncm.Q4_0,
                             s.cuda_stream)
    n = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(s)
    for _ in range(n):
        ncm.matmul_quantized(out.data_ptr(), xq.data_ptr(), xs.data_ptr(), w.data_ptr(), rows, cols, ncm.Q4_0,
                             s.cuda_stream)
    e1.record(s)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / n
    algo = nbytes + cols + cols // 32 * 4 + rows * 4
    gbs = algo / sec / 1e9
    traffic = None
    prof = os.path.join(ROOT, "profiles", "gemv_q4_0_head_3b.traffic.json")
    if os.path.exists(prof):
        try:
            traffic = json.load(open(prof)).get("dram_bytes_per_launch")
        except Exception:
            traffic = None
    return {"bound": "hbm", "kernel": "gemv_kernel<Q4_0,IN_Q8,PLAIN> (tied head 128256x3072)", "achieved": round(gbs, 1),
            "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4), "traffic": traffic,
            "algorithmic_bytes_per_launch": algo, "launch_us": round(sec * 1e6, 2), "peak_source": "measured"}


def run_b200(args, sp):
    import numpy as np
    import torch
    import torch.distributed as dist
    import nanocamelid_b200 as ncm
    from nanocamelid_b200 import tp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    if world > 1:
        shares = [int(v) for v in args.shares.split(",")] if args.shares else tp.default_shares(sp.kv_heads, world)
        if len(shares) != world:
            raise SystemExit(f"--shares lists {len(shares)} ranks for {world} processes")
    else:
        shares = None
    ctx = args.prompt + args.warmup + args.steps + 8
    m = ncm.Model.synthetic(sp, ctx_limit=ctx, device=local, shares=shares, shard=rank)
    if world > 1:
        tp.connect(m, rank, world, ncm.REDUCE_NCCL if args.reducer == "nccl" else ncm.REDUCE_FUSED_P2P)
    rng = np.random.default_rng(0)
    prompt = [int(v) for v in rng.integers(0, sp.vocab, args.prompt)]
    stream = torch.cuda.Stream()
    m.prefill(prompt, stream.cuda_stream)
    m.decode_steps(args.warmup, stream.cuda_stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0.record(stream)
        m.decode_steps(args.steps, stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    toks, pos = m.sync_tokens(ctx)
    tok_s = args.steps / (ms / 1e3)
    # end to end through the C-ABI forward_pass: host token in, argmax out, per step
    e2e = None
    if not args.no_e2e:
        cur = toks[pos]
        for _ in range(3):
            cur, _ = m.forward_pass(cur, pos - 4)   # warm (rewrites an already-decoded slot)
        if world > 1:
            dist.barrier()
        ne = min(args.steps, 64)
        p0 = pos - ne - 1 if pos - ne - 1 > args.prompt else args.prompt
        t0 = time.perf_counter()
        cur = toks[p0]
        for i in range(ne):
            cur, _ = m.forward_pass(cur, p0 + i)
        el = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([el], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            el = float(t.item())
        e2e = {"value": round(ne / el, 2), "unit": "tok/s", "h2d_bytes_per_step": 12, "d2h_bytes_per_step": 4,
               "api": "ncm_forward_pass (host token -> device step -> host argmax, synchronous)"}
    if rank == 0:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))) if os.path.exists(
            os.path.join(ROOT, "MEASURED_PEAKS.json")) else {"hbm_gbs": 6650.0}
        peak = float(peaks.get("hbm_gbs", 6650.0))
        roof = gemv_roofline(torch, ncm, sp, peak)
        bpt = weight_bytes(sp, world, shares)
        whole = {"bytes_per_token_per_gpu": int(bpt), "achieved_gbs": round(bpt * tok_s / 1e9, 1),
                 "frac_of_measured_hbm": round(bpt * tok_s / 1e9 / peak, 4)}
        cpu = None if (args.no_cpu or world > 1) else cpu_sample(sp)
        launches_per_step = 2 + 6 * sp.layers + (0 if world == 1 or args.reducer == "p2p" else 2 * sp.layers + 1)
        line = {"metric": METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int8 dot / f32", "data": "synthetic",
                "config": {"workload": args.config, "prompt": args.prompt, "decode_positions":
                           f"{args.prompt + args.warmup}..{args.prompt + args.warmup + args.steps - 1}",
                           "parallelism": f"tp{world}", "reducer": args.reducer if world > 1 else None,
                           "shares": shares,
                           "l2": "inputs larger than L2 (weights %.2f GB/token/GPU)" % (bpt / 1e9)},
                "roofline": roof, "decode_roofline": whole, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": launches_per_step * args.steps, "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    m.close()
    if world > 1:
        dist.destroy_process_group()


def run_spec(args, ncm):
    """Config 5 on one GPU: tokens emitted per second by ncm_spec_generate (host-driven
    draft/verify loop, synchronous), next to the target's plain greedy decode."""
    import numpy as np
    import torch
    target_sp, draft_sp = ncm.CONFIGS["cfg5_target_q4_0"], ncm.CONFIGS["cfg1_1b_q4_0"]
    n_prompt, n_gen, k = 128, 256, 4
    ctx = n_prompt + n_gen + 2 * k + 2
    prompt = [int(v) for v in np.random.default_rng(0).integers(0, target_sp.vocab, n_prompt)]
    target = ncm.Model.synthetic(target_sp, ctx_limit=ctx, device=0)
    draft = ncm.Model.synthetic(draft_sp, ctx_limit=ctx, device=0)
    target.spec_generate(draft, prompt, 8, k=k)                     # warm-up (graphs, buffers)
    target.reset(); draft.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    toks, (drafted, accepted) = target.spec_generate(draft, prompt, n_gen, k=k)
    torch.cuda.synchronize()
    dt_spec = time.perf_counter() - t0
    ref = ncm.Model.synthetic(target_sp, ctx_limit=ctx, device=0)
    ref.generate(prompt, 8)
    ref.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    greedy = ref.generate(prompt, n_gen)
    torch.cuda.synchronize()
    dt_greedy = time.perf_counter() - t0
    # prompt-lookup drafting (the reference's default draft source) on the same target
    target.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ng_toks, (ng_drafted, ng_accepted) = target.ngram_generate(prompt, n_gen, k=k)
    torch.cuda.synchronize()
    dt_ngram = time.perf_counter() - t0
    vms, step_ms = verify_times(ncm, target, n_prompt)
    print(json.dumps({"metric": "bs1 speculative decode tok/s", "value": round(n_gen / dt_spec, 2), "unit": "tok/s",
                      "n_gpus": 1, "higher_is_better": True, "data": "synthetic",
                      "config": {"workload": "cfg5: draft cfg1_1b_q4_0, target cfg5_target_q4_0 (8B shape, Q4_0)",
                                 "k": k, "prompt": n_prompt, "tokens": n_gen},
                      "acceptance": round(accepted / max(1, drafted), 4), "drafted": drafted, "accepted": accepted,
                      "target_greedy_tok_s": round(n_gen / dt_greedy, 2), "tokens_equal_greedy": toks == greedy,
                      "verify_ms_by_rows": vms, "target_step_ms": step_ms,
                      "ngram": {"tok_s": round(n_gen / dt_ngram, 2), "drafted": ng_drafted, "accepted": ng_accepted,
                                "tokens_equal_greedy": ng_toks == greedy},
                      "timing": "wall clock around the call (prefill included), synchronous"}))


def verify_times(ncm, target, n_prompt, reps=10, rows=(1, 4, 5, 8)):
    """Wall time of one synchronous ncm_verify_batch call per row count, and of one
    graphed single-token step, at position n_prompt (the verify graphs are warm)."""
    import torch
    out = {}
    for ntok in rows:
        toks = [5 + i for i in range(ntok)]
        for _ in range(3):
            target.verify_batch(toks, n_prompt)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(reps):
            target.verify_batch(toks, n_prompt)
        out[str(ntok)] = round((time.perf_counter() - t0) / reps * 1e3, 3)
    for i in range(3):
        target.forward_pass(7, n_prompt + i)
    t0 = time.perf_counter()
    for i in range(reps):
        target.forward_pass(7, n_prompt + i)
    return out, round((time.perf_counter() - t0) / reps * 1e3, 3)


def run_verify(args, ncm):
    """The config-5 target's multi-row verify pass alone (a small, repeatable command
    for launch lists and captures)."""
    import numpy as np
    sp = ncm.CONFIGS["cfg5_target_q4_0"]
    n_prompt = args.prompt
    prompt = [int(v) for v in np.random.default_rng(0).integers(0, sp.vocab, n_prompt)]
    reps = max(1, args.steps)
    target = ncm.Model.synthetic(sp, ctx_limit=n_prompt + 16 + reps, device=0)   # verify rows + timed steps
    target.generate(prompt, 1)
    rows = tuple(int(v) for v in args.verify_rows.split(","))
    vms, step_ms = verify_times(ncm, target, n_prompt, reps=reps, rows=rows)
    print(json.dumps({"workload": f"cfg5_target_q4_0 verify pass at position {n_prompt}", "verify_ms_by_rows": vms,
                      "single_step_ms": step_ms, "timing": "wall clock per synchronous call"}))


def main():
    args = parse()
    import nanocamelid_b200 as ncm
    sp = ncm.CONFIGS[args.config]
    rank = int(os.environ.get("RANK", "0"))
    if args.spec:
        run_spec(args, ncm)
    elif args.verify_only:
        run_verify(args, ncm)
    elif args.gemv_only:
        import torch
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        print(json.dumps({"roofline": gemv_roofline(torch, ncm, sp, peaks["hbm_gbs"])}))
    elif args.impl == "reference":
        run_reference(args, sp, rank)
    else:
        run_b200(args, sp)


if __name__ == "__main__":
    main()
