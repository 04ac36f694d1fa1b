"""Tensor parallel on 2+ GPUs (one process per GPU): greedy tokens identical to the
single-node oracle and logits within 1e-3 relative, for the fused NVLink peer-store
reduction and the NCCL all-reduce baseline (bin/cluster_tp_split_smoke.rs:101-165
semantics: token identity, max |dlogit|); and a rank that stops stepping is detected by
the others' bounded waits (NCM_ETIMEOUT), with no GPU fault: the silent rank stays alive
(its memory stays mapped) and only skips the step."""
import json
import os
import socket

import numpy as np
import pytest

from conftest import TINY

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ngpus():
    import torch
    return torch.cuda.device_count()


def _spec(ncm, kv_heads, heads):
    d = dict(TINY)
    return ncm.spec(d["emb"], d["layers"], heads, kv_heads, d["emb"] // heads, 2048 if kv_heads == 8 else 512,
                    vocab=d["vocab"], ctx=d["ctx"], tied=True, seed=9)


def _worker(rank, world, port, path, shares, reducer, prompt, n_gen, out_dir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import nanocamelid_b200 as ncm
        from nanocamelid_b200 import tp
        m = ncm.Model.load(path, device=rank, shares=shares, shard=rank)
        tp.connect(m, rank, world, ncm.REDUCE_NCCL if reducer == "nccl" else ncm.REDUCE_FUSED_P2P)
        toks = m.generate(prompt, n_gen)
        am, lg = m.forward_pass(toks[-1], len(prompt) + n_gen - 1, want_logits=True)
        np.save(os.path.join(out_dir, f"lg{rank}.npy"), lg)
        json.dump({"tokens": toks, "argmax": am}, open(os.path.join(out_dir, f"r{rank}.json"), "w"))
        dist.barrier()
        m.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("reducer", ["p2p", "nccl"])
@pytest.mark.parametrize("kvh,heads,shares", [(2, 4, [1, 1]), (8, 8, [2, 3, 3])])
def test_tp_decode_matches_single_node(ncm, orc, tmp_path, reducer, kvh, heads, shares):
    world = len(shares)
    if _ngpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    sp = _spec(ncm, kvh, heads)
    path = str(tmp_path / "m.gguf")
    ncm.write_synthetic_gguf(path, sp)
    prompt = [int(v) for v in np.random.default_rng(2).integers(0, sp.vocab, size=6)]
    n_gen = 20
    ref = orc.OracleModel(path)
    ref_tokens = ref.generate(prompt, n_gen)[0]
    _, ref_lg = ref.forward_pass(ref_tokens[-1], len(prompt) + n_gen - 1, want_logits=True)
    mp.spawn(_worker, args=(world, _free_port(), path, shares, reducer, prompt, n_gen, str(tmp_path)),
             nprocs=world, join=True)
    lgs = []
    for r in range(world):
        res = json.load(open(tmp_path / f"r{r}.json"))
        assert res["tokens"] == ref_tokens, (r, res["tokens"], ref_tokens)
        lgs.append(np.load(tmp_path / f"lg{r}.npy"))
    lg = np.concatenate(lgs)
    assert lg.shape == ref_lg.shape
    assert float(np.max(np.abs(lg - ref_lg))) <= 1e-3 * float(np.max(np.abs(ref_lg)))


def _silent_worker(rank, world, port, path, out_dir):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
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
