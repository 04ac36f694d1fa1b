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
    ap.add_argument("--config", default="cfg4_70b_q4_0")
    ap.add_argument("--prompt", type=int, default=None, help="context length (default: the config's, BASELINE.json)")
    ap.add_argument("--layers", type=int, default=0, help="small case for profiler captures: fewer layers")
    ap.add_argument("--vocab", type=int, default=0, help="small case for profiler captures: smaller vocab")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-prefill", action="store_true",
                    help="profiler captures: one decode step at the last prompt position instead of the prefill "
                         "(the earlier K/V rows stay zero; the step's work is the same)")
    ap.add_argument("--spec", action="store_true",
                    help="BASELINE config 5: greedy speculative decoding, draft = config 1, target = config-3 "
                         "shape all Q4_0, k = 4, 128-token prompt, 256 tokens (one GPU)")
    ap.add_argument("--verify-only", action="store_true",
                    help="config 5 target: time the multi-row verify pass (1/4/5/8 rows) and one graphed step")
    ap.add_argument("--verify-rows", default="1,4,5,8")
    ap.add_argument("--kernels", action="store_true",
                    help="per-kernel CUDA-event times of the decode step's GEMVs (one launch per layer in turn)")
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


# BASELINE.json prompt (context) length per config
PROMPTS = {"cfg1_1b_q4_0": 16, "cfg2_3b_q4_0": 64, "cfg3_8b_mixed": 512, "cfg4_70b_q4_0": 1024, "cfg5_target_q4_0": 128}


def bench_config(args, world, shares):
    """The `config` object both arms print (identical, so the two lines are comparable)."""
    first = args.prompt + args.warmup
    return {"workload": args.config, "prompt": args.prompt,
            "decode_positions": f"{first}..{first + args.steps - 1}", "parallelism": f"tp{world}",
            "reducer": args.reducer if world > 1 else None, "shares": shares}


class OracleRun:
    """The CPU restatement of the reference's portable path (oracle/) on the same model,
    built in host memory by the oracle's own generator (no product code is loaded).  The
    K/V cache of the first `ctx_pos` positions is filled with seeded values instead of
    being prefilled (a 1024-token prefill of the 70B shape is hours of CPU time), so a
    step at position p does the reference's full per-token work at that position."""

    def __init__(self, sp, ctx_pos, ctx_limit):
        from oracle import oracle as orc
        self.ref = orc.OracleModel(spec=sp, ctx_limit=ctx_limit)
        self.ref.fill_kv(ctx_pos)
        self.pos, self.tok = ctx_pos, 0

    def step(self):
        self.tok, _ = self.ref.forward_pass(self.tok, self.pos)
        self.pos += 1

    def timed(self, n, budget_s):
        k, t0 = 0, time.perf_counter()
        while k < n and time.perf_counter() - t0 < budget_s and self.pos < self.ref.ctx:
            self.step()
            k += 1
        return k, time.perf_counter() - t0


def oracle_sample(args, sp, warmup, n, budget_s):
    """(tok/s, tokens timed, the sample's description): decode steps of the CPU oracle at
    the GPU arm's timed positions, OpenMP over every host core."""
    first = args.prompt + args.warmup
    run = OracleRun(sp, first - warmup, first + args.steps + 8)
    for _ in range(warmup):
        run.step()
    k, dt = run.timed(n, budget_s)
    desc = (f"{k} greedy decode steps at positions {first}..{first + k - 1} of {args.config} ({warmup} untimed "
            f"before them); K/V of the earlier positions seeded instead of prefilled; CPU restatement of the "
            f"reference x86 portable path (oracle/), OpenMP over {os.cpu_count()} threads")
    return k / dt, k, desc


def cpu_sample(args, sp, budget_s=20.0):
    v, _, desc = oracle_sample(args, sp, 1, args.steps, budget_s)
    return {"value": round(v, 3), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port", "sample": desc}


def run_reference(args, sp, rank):
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    shares = None
    if world > 1:
        from nanocamelid_b200 import tp
        shares = [int(v) for v in args.shares.split(",")] if args.shares else tp.default_shares(sp.kv_heads, world)
    w = min(args.warmup, 2)
    v, n, desc = oracle_sample(args, sp, w, args.steps, 30.0)
    cpu = {"value": round(v, 3), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port", "sample": desc}
    print(json.dumps({"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tok/s",
                      "n_gpus": args.gpus, "steps": n, "warmup": w, "higher_is_better": True,
                      "dtype": "int8 dot / f32", "data": "synthetic", "config": bench_config(args, world, shares),
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
    prof = os.path.join(ROOT, "profiles", f"gemv_q4_0_head_{rows}x{cols}.traffic.json")
    if os.path.exists(prof):
        try:
            traffic = json.load(open(prof)).get("dram_bytes_per_launch")
        except Exception:
            traffic = None
    return {"bound": "hbm", "kernel": f"ncm_qgemv_kernel<Q4_0,IN_Q8,PLAIN> (head-shaped {rows}x{cols}, microbench)",
            "achieved": round(gbs, 1),
            "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4), "traffic": traffic,
            "algorithmic_bytes_per_launch": algo, "launch_us": round(sec * 1e6, 2), "peak_source": "measured"}


def step_kernel_roofline(torch, ncm, m, sp, kind, peak, stream, world=1):
    """CUDA-event time of the decode step's own GEMV of `kind` (same kernel, same launch
    parameters as inside the captured step, PDL included), one launch per layer in turn so
    that every launch streams weights that are not in L2."""
    bpw = {2: 18 / 32, 8: 34 / 32, 12: 144 / 256}
    tn = {2: "Q4_0", 8: "Q8_0", 12: "Q4_K"}
    H, F = sp.emb, sp.ffn // world
    qw, kw = sp.heads * sp.head_dim // world, sp.kv_heads * sp.head_dim // world
    if kind in (ncm.STEP_WO, ncm.STEP_W2):
        name, wbytes = "row-parallel", (H * (qw if kind == ncm.STEP_WO else F)) * bpw[sp.t_attn if kind == ncm.STEP_WO else sp.t_ffn]
        io = 0
    elif kind == ncm.STEP_W13:
        name, wbytes = f"ncm_qgemv_kernel<{tn[sp.t_ffn]},IN_F32_RMS,EPI_SILU> (ffn_gate+ffn_up {F}x{H} x2)", 2 * F * H * bpw[sp.t_ffn]
        io = H * 4 * 2 + F * 4
    else:
        name, wbytes = f"ncm_qgemv_kernel<{tn[sp.t_attn]},IN_F32_RMS,EPI_QKV> (attn_q/k/v {qw + 2 * kw}x{H})", (qw + 2 * kw) * H * bpw[sp.t_attn]
        io = H * 4 * 2 + (qw + 2 * kw) * 4
    n = max(8, min(sp.layers, 40))
    for i in range(4):
        m.launch_step_kernel(kind, i % sp.layers, stream.cuda_stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(n):
        m.launch_step_kernel(kind, i % sp.layers, stream.cuda_stream)
    e1.record(stream)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / n
    algo = int(wbytes + io)
    traffic = None
    prof = os.path.join(ROOT, "profiles", f"{args_config_key(sp)}_w13.traffic.json")
    if kind == ncm.STEP_W13 and os.path.exists(prof):
        try:
            traffic = json.load(open(prof)).get("dram_bytes_per_launch")
        except Exception:
            traffic = None
    return {"bound": "hbm", "kernel": name, "achieved": round(algo / sec / 1e9, 1), "peak": peak, "unit": "GB/s",
            "frac": round(algo / sec / 1e9 / peak, 4), "traffic": traffic, "algorithmic_bytes_per_launch": algo,
            "launch_us": round(sec * 1e6, 2), "launches_timed": n, "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)"}


def args_config_key(sp):
    return "gemv_q4_0_70b" if sp.emb == 8192 else f"gemv_emb{sp.emb}"


def decode_context(prompt, warmup, steps):
    """Context slots the decode bench needs: the prompt, the warm-up and timed steps, and a
    margin (the e2e and NCCL-baseline phases rewrite positions inside this range)."""
    return prompt + warmup + steps + 8


def nccl_phase_start(prompt, warmup):
    """Position the NCCL-baseline phase restarts from: one forward_pass there and two
    untimed steps bring it to the fused phase's first timed position (prompt + warmup)."""
    return max(prompt, prompt + warmup - 3)


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
    ctx = decode_context(args.prompt, args.warmup, args.steps)
    m = ncm.Model.synthetic(sp, ctx_limit=ctx, device=local, shares=shares, shard=rank)
    if world > 1:
        # peers' exchange areas and an NCCL communicator: the fused reducer is timed first,
        # then the NCCL-allreduce baseline on the same shards
        tp.connect(m, rank, world, ncm.REDUCE_NCCL)
        m.tp_set_reducer(ncm.REDUCE_FUSED_P2P if args.reducer == "p2p" else ncm.REDUCE_NCCL)
    rng = np.random.default_rng(0)
    prompt = [int(v) for v in rng.integers(0, sp.vocab, args.prompt)]
    stream = torch.cuda.Stream()
    if args.no_prefill:
        m.forward_pass(prompt[-1], len(prompt) - 1)
    else:
        m.prefill(prompt, stream.cuda_stream)
    m.decode_steps(args.warmup, stream.cuda_stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    def timed_steps(n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0.record(stream)
        m.decode_steps(n, stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t = e0.elapsed_time(e1)
        if world > 1:
            tt = torch.tensor([t], device="cuda")
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    with ClockSampler(local) as clk:
        ms = timed_steps(args.steps)
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
    nccl = None
    if world > 1 and args.reducer == "p2p":
        # the NCCL-allreduce baseline of the same decode (same shards): back to the fused
        # run's start, so that it rewrites the same positions and stays inside the context
        m.tp_set_reducer(ncm.REDUCE_NCCL)
        p_start = nccl_phase_start(args.prompt, args.warmup)
        m.forward_pass(toks[p_start], p_start)
        m.decode_steps(2, stream.cuda_stream)
        torch.cuda.synchronize()
        n_ms = timed_steps(args.steps)
        nccl = {"value": round(args.steps / (n_ms / 1e3), 2), "unit": "tok/s", "ms_per_step": round(n_ms / args.steps, 4),
                "reducer": "ncclAllReduce(sum) of the wo/w2 partial rows + residual add, ncclAllGather argmax merge"}
        m.tp_set_reducer(ncm.REDUCE_FUSED_P2P)
    if args.kernels and world == 1:
        peak = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"])
        import numpy as np
        out = {}
        for name, kind in (("qkv", ncm.STEP_QKV), ("wo", ncm.STEP_WO), ("w13", ncm.STEP_W13), ("w2", ncm.STEP_W2)):
            r = step_kernel_roofline(torch, ncm, m, sp, kind, peak, stream)
            out[name] = {"us": r["launch_us"], "GBps": r["achieved"], "frac": r["frac"]} if kind in (
                ncm.STEP_QKV, ncm.STEP_W13) else {"us": r["launch_us"]}
            # one more launch alone, with its phase stamps (relative to the earliest entry)
            torch.cuda.synchronize()
            m.launch_step_kernel(kind, min(1, sp.layers - 1), stream.cuda_stream)
            torch.cuda.synchronize()
            ts = m.debug_stamps(16 * 148).reshape(148, 16).astype(np.int64)
            t0 = ts[:, 0].min()
            rel = lambda i: ts[:, i] - t0
            us = lambda a: round(float(a) / 1e3, 2)
            out[name]["stamps_us"] = {
                "pdl_max": us(rel(1).max()), "prologue_avg": us((ts[:, 2] - ts[:, 1]).mean()),
                "prologue_max": us((ts[:, 2] - ts[:, 1]).max()), "last_issue_avg": us(rel(3).mean()),
                "compute_end_avg": us(rel(11).mean()), "fold_end_avg": us(rel(4).mean()),
                "fold_end_max": us(rel(4).max()), "exit_max": us(rel(6).max()),
                "epilogue_avg": us(ts[:, 5].mean()), "c_wait_data_avg": us(ts[:, 7].mean()),
                "c_wait_slot_avg": us(ts[:, 8].mean()), "f_wait_terms_avg": us(ts[:, 9].mean()),
                "p_wait_stage_avg": us(ts[:, 10].mean()),
                "stage_x_avg": us((ts[:, 12] - ts[:, 1]).mean()) if ts[:, 12].max() > 0 else None,
                "seq_sum_avg": us((ts[:, 13] - ts[:, 12]).mean()) if ts[:, 13].max() > 0 else None}
        print(json.dumps({"kernels": out, "tok_s": round(tok_s, 2), "ms_per_step": round(ms / args.steps, 4),
                          "env": {k: v for k, v in os.environ.items() if k.startswith("NCM_TUNE")}}), flush=True)
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peaks = json.load(open(peaks_path)) if os.path.exists(peaks_path) else {"hbm_gbs": 6650.0}
    peak = float(peaks.get("hbm_gbs", 6650.0))
    # the decode step's dominant kernel, timed live (rank 0's shard under TP)
    roof = step_kernel_roofline(torch, ncm, m, sp, ncm.STEP_W13, peak, stream, world=world)
    if world > 1:
        dist.barrier()
    if rank == 0:
        head = gemv_roofline(torch, ncm, sp, peak)
        bpt = weight_bytes(sp, world, shares)
        whole = {"bytes_per_token_per_gpu": int(bpt), "achieved_gbs": round(bpt * tok_s / 1e9, 1),
                 "frac_of_measured_hbm": round(bpt * tok_s / 1e9 / peak, 4)}
        cpu = None if (args.no_cpu or world > 1) else cpu_sample(args, sp)
        # per layer: q/k/v, attention (scores + softmax + V, or scores + one softmax·V launch
        # for GQA groups under 8 heads), wo, gate/up, down; plus embed and head
        attn = 3 if sp.heads // sp.kv_heads >= 8 else 2
        launches_per_step = 2 + (4 + attn) * sp.layers + (0 if world == 1 or args.reducer == "p2p" else 2 * sp.layers + 1)
        cfg = bench_config(args, world, shares)
        cfg["l2"] = "inputs larger than L2 (weights %.2f GB/token/GPU)" % (bpt / 1e9)
        line = {"metric": METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int8 dot / f32", "data": "synthetic",
                "config": cfg, "roofline": roof, "head_gemv_roofline": head, "decode_roofline": whole,
                "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches_per_step * args.steps,
                "clocks": clk.summary()}
        if nccl:
            line["nccl_baseline"] = nccl
        print(json.dumps(line), flush=True)
    m.close()
    if world > 1:
        dist.destroy_process_group()


def run_spec(args, ncm):
    """Config 5: tokens emitted per second by ncm_spec_generate (host-driven draft/verify
    loop, synchronous), next to the target's plain greedy decode.  Under torchrun the
    target is tensor parallel over the ranks (KV-head shares, the fused NVLink reducer for
    both the one-row steps and the multi-row verify); every rank runs its own full draft."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from nanocamelid_b200 import tp
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    target_sp, draft_sp = ncm.CONFIGS["cfg5_target_q4_0"], ncm.CONFIGS["cfg1_1b_q4_0"]
    n_prompt, n_gen, k = 128, 256, 4
    ctx = n_prompt + n_gen + 2 * k + 2
    prompt = [int(v) for v in np.random.default_rng(0).integers(0, target_sp.vocab, n_prompt)]
    shares = (([int(v) for v in args.shares.split(",")] if args.shares else tp.default_shares(target_sp.kv_heads, world))
              if world > 1 else None)
    target = ncm.Model.synthetic(target_sp, ctx_limit=ctx, device=local, shares=shares, shard=rank)
    if world > 1:
        tp.connect(target, rank, world, ncm.REDUCE_FUSED_P2P)
    draft = ncm.Model.synthetic(draft_sp, ctx_limit=ctx, device=local)

    def timed(fn):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        r = fn()
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([dt], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
        return r, dt

    target.spec_generate(draft, prompt, 8, k=k)                     # warm-up (graphs, buffers)
    target.reset(); draft.reset()
    (toks, (drafted, accepted)), dt_spec = timed(lambda: target.spec_generate(draft, prompt, n_gen, k=k))
    target.reset()
    target.generate(prompt, 8)
    target.reset()
    greedy, dt_greedy = timed(lambda: target.generate(prompt, n_gen))
    # prompt-lookup drafting (the reference's default draft source) on the same target
    target.reset()
    (ng_toks, (ng_drafted, ng_accepted)), dt_ngram = timed(lambda: target.ngram_generate(prompt, n_gen, k=k))
    vms, step_ms = verify_times(ncm, target, n_prompt) if world == 1 else (None, None)
    if rank == 0:
        print(json.dumps({"metric": "bs1 speculative decode tok/s", "value": round(n_gen / dt_spec, 2), "unit": "tok/s",
                          "n_gpus": world, "higher_is_better": True, "data": "synthetic",
                          "config": {"workload": "cfg5: draft cfg1_1b_q4_0, target cfg5_target_q4_0 (8B shape, Q4_0)",
                                     "k": k, "prompt": n_prompt, "tokens": n_gen,
                                     "parallelism": f"tp{world}" if world > 1 else "tp1", "shares": shares},
                          "acceptance": round(accepted / max(1, drafted), 4), "drafted": drafted, "accepted": accepted,
                          "target_greedy_tok_s": round(n_gen / dt_greedy, 2), "tokens_equal_greedy": toks == greedy,
                          "verify_ms_by_rows": vms, "target_step_ms": step_ms,
                          "ngram": {"tok_s": round(n_gen / dt_ngram, 2), "drafted": ng_drafted, "accepted": ng_accepted,
                                    "tokens_equal_greedy": ng_toks == greedy},
                          "timing": "wall clock around the call (prefill included), synchronous, max over ranks"}),
              flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


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
    if args.layers:
        sp = sp.replace(layers=args.layers)
    if args.vocab:
        sp = sp.replace(vocab=args.vocab)
    if args.prompt is None:
        args.prompt = PROMPTS.get(args.config, 64)
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
