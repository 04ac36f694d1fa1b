"""Tensor parallel on 2+ GPUs (one process per GPU), and the host-callback reducer.

The reference's TP path (tp.rs:226-428 with the fixed-order reducer,
cluster_tp_node.rs:1154-1180) is restated by the oracle's TP (OracleTP).  The fused NVLink
peer-store reduction sums in the same rank order, so its greedy tokens equal the oracle
TP's and its logits agree to 1e-5 relative.  The NCCL baseline sums in ring order: its
prompt logits agree with the oracle TP's to 1e-3 relative.  (TP against the single-node
path is a property of the model, not of this code: bin/cluster_tp_split_smoke.rs:101-165
reports it; the oracle tests it on CPU.)  A rank that stops stepping is detected by the
others' bounded waits (NCM_ETIMEOUT), with no GPU fault: the silent rank stays alive (its
memory stays mapped) and only skips the step."""
import json
import os
import socket
import threading

import numpy as np
import pytest

from conftest import TINY

pytestmark = [pytest.mark.gpu]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ngpus():
    import torch
    return torch.cuda.device_count()


def _spec(ncm, kv_heads, heads):
    d = dict(TINY)
    return ncm.spec(d["emb"], d["layers"], heads, kv_heads, d["emb"] // heads, 256 * kv_heads,
                    vocab=d["vocab"], ctx=d["ctx"], tied=True, seed=9)


def _worker(rank, world, port, path, shares, reducer, prompt, n_gen, out_dir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    # a file rendezvous in the test's own directory: no TCP port to race for
    dist.init_process_group("gloo", init_method="file://" + os.path.join(out_dir, "pg_store"), rank=rank, world_size=world)
    try:
        import nanocamelid_b200 as ncm
        from nanocamelid_b200 import tp
        m = ncm.Model.load(path, device=rank, shares=shares, shard=rank)
        mode = {"p2p": ncm.REDUCE_FUSED_P2P, "nccl": ncm.REDUCE_NCCL, "host": ncm.REDUCE_HOST_CALLBACK}[reducer]
        tp.connect(m, rank, world, mode)
        lgs = [m.forward_pass(t, pos, want_logits=True)[1] for pos, t in enumerate(prompt)]
        np.save(os.path.join(out_dir, f"lg{rank}.npy"), np.stack(lgs))
        m.reset()
        toks = m.generate(prompt, n_gen)
        json.dump({"tokens": toks}, open(os.path.join(out_dir, f"r{rank}.json"), "w"))
        dist.barrier()
        m.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.multigpu
@pytest.mark.parametrize("reducer", ["p2p", "nccl", "host"])
@pytest.mark.parametrize("kvh,heads,shares", [(2, 4, [1, 1]), (4, 4, [1, 3]), (8, 8, [4, 4]), (8, 8, [2, 3, 3])])
def test_tp_decode_matches_oracle_tp(ncm, orc, tmp_path, reducer, kvh, heads, shares):
    world = len(shares)
    if _ngpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    sp = _spec(ncm, kvh, heads)
    path = str(tmp_path / "m.gguf")
    ncm.write_synthetic_gguf(path, sp)
    prompt = [int(v) for v in np.random.default_rng(2).integers(0, sp.vocab, size=6)]
    n_gen = 20
    ref_tokens = orc.OracleTP(orc.OracleModel(path), shares).generate(prompt, n_gen)
    rtp = orc.OracleTP(orc.OracleModel(path), shares)
    ref_lg = np.stack([rtp.forward_pass(t, pos, want_logits=True)[1] for pos, t in enumerate(prompt)])
    mp.spawn(_worker, args=(world, _free_port(), path, shares, reducer, prompt, n_gen, str(tmp_path)),
             nprocs=world, join=True)
    toks = [json.load(open(tmp_path / f"r{r}.json"))["tokens"] for r in range(world)]
    lg = np.concatenate([np.load(tmp_path / f"lg{r}.npy") for r in range(world)], axis=1)
    assert lg.shape == ref_lg.shape
    gap = float(np.max(np.abs(lg - ref_lg))) / float(np.max(np.abs(ref_lg)))
    assert all(t == toks[0] for t in toks), toks
    if reducer in ("p2p", "host"):   # both sum in rank order from 0.0f
        assert toks[0] == ref_tokens and gap <= 1e-5, (toks[0], ref_tokens, gap)
    else:
        assert gap <= 1e-3, gap


def _silent_worker(rank, world, port, path, out_dir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    # a file rendezvous in the test's own directory: no TCP port to race for
    dist.init_process_group("gloo", init_method="file://" + os.path.join(out_dir, "pg_store"), rank=rank, world_size=world)
    try:
        import nanocamelid_b200 as ncm
        from nanocamelid_b200 import tp
        m = ncm.Model.load(path, device=rank, shares=[1, 1], shard=rank)
        tp.connect(m, rank, world, ncm.REDUCE_FUSED_P2P)
        m.tp_set_timeout_ns(300_000_000)
        result = "stepped"
        if rank == 0:
            # rank 1 never launches this step: every wait on its flags must give up
            try:
                m.forward_pass(5, 0)
            except ncm.NcmError as e:
                result = f"error {e}"
        dist.barrier()          # rank 1 stays alive (memory mapped) until rank 0 is done
        json.dump({"result": result}, open(os.path.join(out_dir, f"s{rank}.json"), "w"))
        m.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.multigpu
def test_tp_missing_rank_times_out(ncm, tmp_path):
    if _ngpus() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    sp = _spec(ncm, 2, 4)
    path = str(tmp_path / "m.gguf")
    ncm.write_synthetic_gguf(path, sp)
    mp.spawn(_silent_worker, args=(2, _free_port(), path, str(tmp_path)), nprocs=2, join=True)
    r0 = json.load(open(tmp_path / "s0.json"))["result"]
    assert r0.startswith("error") and "TIMEOUT" in r0.upper(), r0


def _thread_reducers(world, fail_at=None):
    """One reduce closure per shard for shards driven by threads of one process: each
    publishes its buffer, waits for the others, and takes the rank-ordered value
    (tp.rank_ordered).  fail_at = (layer, phase): every closure returns an error there."""
    from nanocamelid_b200 import tp
    slots = [None] * world
    bar = threading.Barrier(world)

    def make(rank):
        def fn(buf, layer, phase):
            if fail_at == (layer, phase):
                return 7
            slots[rank] = buf.copy()
            bar.wait(timeout=30)
            out = tp.rank_ordered(slots, phase)
            bar.wait(timeout=30)   # every shard has read the slots before they are reused
            buf[:] = out
            return 0
        return fn
    return [make(r) for r in range(world)]


def _run_shards(models, fn):
    res = [None] * len(models)

    def go(r):
        try:
            res[r] = fn(r, models[r])
        except Exception as e:   # reported to the test thread
            res[r] = e
    th = [threading.Thread(target=go, args=(r,)) for r in range(len(models))]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    return res


def test_tp_host_callback_reducer_on_one_gpu(ncm, orc, cuda, tmp_path):
    """NCM_REDUCE_HOST_CALLBACK (the reference's reduce closure, tp.rs:226-236): two
    shards of one model on one GPU, driven by two threads, reduced on the host; greedy
    tokens equal the oracle's TP restatement and the logits agree to 1e-5.  Then every
    closure fails at layer 1 (tp.rs's Err path): each step returns NCM_EPEER, and the
    same models decode correctly afterwards."""
    sp = _spec(ncm, 2, 4)
    path = str(tmp_path / "m.gguf")
    ncm.write_synthetic_gguf(path, sp)
    shares = [1, 1]
    prompt = [int(v) for v in np.random.default_rng(2).integers(0, sp.vocab, size=6)]
    n_gen = 16
    ref_tokens = orc.OracleTP(orc.OracleModel(path), shares).generate(prompt, n_gen)
    rtp = orc.OracleTP(orc.OracleModel(path), shares)
    ref_lg = np.stack([rtp.forward_pass(t, pos, want_logits=True)[1] for pos, t in enumerate(prompt)])
    models = [ncm.Model.load(path, device=0, shares=shares, shard=r) for r in range(2)]
    try:
        for m, fn in zip(models, _thread_reducers(2)):
            m.tp_set_host_reducer(fn)
            m.tp_set_reducer(ncm.REDUCE_HOST_CALLBACK)
        lgs = _run_shards(models, lambda r, m: np.stack(
            [m.forward_pass(t, pos, want_logits=True)[1] for pos, t in enumerate(prompt)]))
        assert not any(isinstance(x, Exception) for x in lgs), lgs
        lg = np.concatenate(lgs, axis=1)
        gap = float(np.max(np.abs(lg - ref_lg))) / float(np.max(np.abs(ref_lg)))
        assert gap <= 1e-5, gap
        for m in models:
            m.reset()
        toks = _run_shards(models, lambda r, m: m.generate(prompt, n_gen))
        assert toks[0] == toks[1] == ref_tokens, (toks, ref_tokens)

        # the closure's Err at layer 1, FFN phase: a step error, no device wait involved
        for m, fn in zip(models, _thread_reducers(2, fail_at=(1, ncm.PHASE_FFN))):
            m.tp_set_host_reducer(fn)
        errs = _run_shards(models, lambda r, m: m.forward_pass(prompt[0], 0))
        for e in errs:
            assert isinstance(e, ncm.NcmError) and e.status == 4 and "layer 1" in str(e), errs
        for m, fn in zip(models, _thread_reducers(2)):
            m.tp_set_host_reducer(fn)
            m.reset()
        toks = _run_shards(models, lambda r, m: m.generate(prompt, n_gen))
        assert toks[0] == toks[1] == ref_tokens, (toks, ref_tokens)
    finally:
        for m in models:
            m.close()


@pytest.mark.parametrize("k", [4, 8])
def test_tp_speculative_with_host_reducer_on_one_gpu(ncm, orc, cuda, tmp_path, k):
    """Config 5 with a tensor-parallel target (two shards of one GPU, threads, host
    reducer): every rank runs the same speculative loop with its own full draft; the
    multi-row verify reduces all rows through the host closure and merges each row's
    head pair.  The output equals the oracle TP's greedy decode (k = 4: the pending-token
    cycle with 5-row verifies; k = 8: the reference-shaped cycle)."""
    sp = _spec(ncm, 2, 4)
    d = dict(TINY)
    dsp = ncm.spec(d["emb"], 1, 4, 2, d["emb"] // 4, 512, vocab=d["vocab"], ctx=d["ctx"], tied=True, seed=12)
    path = str(tmp_path / "m.gguf")
    ncm.write_synthetic_gguf(path, sp)
    shares = [1, 1]
    prompt = [int(v) for v in np.random.default_rng(4).integers(0, sp.vocab, size=7)]
    n_gen = 24
    ref = orc.OracleTP(orc.OracleModel(path), shares).generate(prompt, n_gen)
    models = [ncm.Model.load(path, device=0, shares=shares, shard=r) for r in range(2)]
    drafts = [ncm.Model.synthetic(dsp, device=0) for _ in range(2)]
    for dm in drafts:   # capture every graph the drafts use (decode; 6- and 7-row prefill) up front
        dm.generate(prompt[:-1], 2)
        dm.generate(prompt, 2)
        dm.reset()
    try:
        for m, fn in zip(models, _thread_reducers(2)):
            m.tp_set_host_reducer(fn)
            m.tp_set_reducer(ncm.REDUCE_HOST_CALLBACK)
        out = _run_shards(models, lambda r, m: m.spec_generate(drafts[r], prompt, n_gen, k=k))
        assert not any(isinstance(x, Exception) for x in out), out
        (t0, s0), (t1, s1) = out
        assert t0 == t1 == ref, (t0, t1, ref)
        assert s0 == s1
    finally:
        for m in models + drafts:
            m.close()


def _rows_worker(rank, world, port, path, dpath, shares, reducer, prompt, n_gen, out_dir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method="file://" + os.path.join(out_dir, "pg_store"), rank=rank, world_size=world)
    try:
        import nanocamelid_b200 as ncm
        from nanocamelid_b200 import tp
        m = ncm.Model.load(path, device=rank, shares=shares, shard=rank)
        draft = ncm.Model.load(dpath, device=rank)
        mode = {"p2p": ncm.REDUCE_FUSED_P2P, "nccl": ncm.REDUCE_NCCL}[reducer]
        tp.connect(m, rank, world, mode)
        greedy = m.generate(prompt, n_gen)          # 13-token prompt: 8- and 5-row prefill passes
        m.reset()
        spec, stats = m.spec_generate(draft, prompt, n_gen, k=4)   # 5-row verify passes
        json.dump({"greedy": greedy, "spec": spec}, open(os.path.join(out_dir, f"r{rank}.json"), "w"))
        dist.barrier()
        m.close()
        draft.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.multigpu
@pytest.mark.parametrize("reducer", ["p2p", "nccl"])
@pytest.mark.parametrize("kvh,heads,shares", [(2, 4, [1, 1]), (8, 8, [2, 3, 3])])
def test_tp_multirow_passes_on_device_reducers(ncm, orc, tmp_path, reducer, kvh, heads, shares):
    """Multi-row passes of a sharded target with the device reducers, one process per
    GPU: the batched prefill (8 + 5 rows) and the speculative verify (k = 4, 5 rows) sum
    every row's row-parallel partials over NVLink in rank order (p2p) or with
    ncclAllReduce (nccl), and merge every row's head pair across the vocab shards.  The
    p2p reducer's greedy and speculative tokens both equal the oracle TP's greedy decode
    (tp.rs:349-363 per row, speculative.rs:365-373); the NCCL reducer's ranks agree."""
    world = len(shares)
    if _ngpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    sp = _spec(ncm, kvh, heads)
    d = dict(TINY)
    dsp = ncm.spec(d["emb"], 1, 4, 2, d["emb"] // 4, 512, vocab=d["vocab"], ctx=d["ctx"], tied=True, seed=12)
    path, dpath = str(tmp_path / "m.gguf"), str(tmp_path / "d.gguf")
    ncm.write_synthetic_gguf(path, sp)
    ncm.write_synthetic_gguf(dpath, dsp)
    prompt = [int(v) for v in np.random.default_rng(5).integers(0, sp.vocab, size=13)]
    n_gen = 20
    ref = orc.OracleTP(orc.OracleModel(path), shares).generate(prompt, n_gen)
    mp.spawn(_rows_worker, args=(world, _free_port(), path, dpath, shares, reducer, prompt, n_gen, str(tmp_path)),
             nprocs=world, join=True)
    out = [json.load(open(tmp_path / f"r{r}.json")) for r in range(world)]
    assert all(o == out[0] for o in out), out
    assert len(out[0]["greedy"]) == n_gen and len(out[0]["spec"]) == n_gen
    if reducer == "p2p":
        assert out[0]["greedy"] == ref and out[0]["spec"] == ref, (out[0], ref)
