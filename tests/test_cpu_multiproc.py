"""World-size-2 gloo runs of the multi-process host logic (CPU only): the shard-plan
exchange that every tensor-parallel rank performs before loading, and the max-over-ranks
reduction bench.py uses for its timings."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.cpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shares, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # a file rendezvous in the test's own directory: no TCP port to race for
    dist.init_process_group("gloo", init_method="file://" + os.path.join(result_dir, "pg_store"), rank=rank, world_size=world)
    try:
        import nanocamelid_b200 as ncm
        from nanocamelid_b200 import tp
        sp = ncm.CONFIGS["cfg3_8b_mixed"]
        plans = tp.check_plan(sp, shares, world, rank)
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
            f.write(f"{len(plans)} {plans[rank]['kv_start']} {t.item()}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shares", [[4, 4], [3, 5]])
def test_two_rank_plan_exchange(tmp_path, shares):
    mp.spawn(_worker, args=(2, _free_port(), shares, str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        n, kv0, mx = open(tmp_path / f"r{r}").read().split()
        assert int(n) == 2 and float(mx) == 2.0
        assert int(kv0) == (0 if r == 0 else shares[0])


def _bad_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # a file rendezvous in the test's own directory: no TCP port to race for
    dist.init_process_group("gloo", init_method="file://" + os.path.join(result_dir, "pg_store"), rank=rank, world_size=world)
    try:
        import nanocamelid_b200 as ncm
        from nanocamelid_b200 import tp
        sp = ncm.CONFIGS["cfg2_3b_q4_0"]
        # ranks disagree on the shares: the exchanged plans do not tile the model
        shares = [4, 4] if rank == 0 else [2, 6]
        try:
            tp.check_plan(sp, shares, world, rank)
            msg = "accepted"
        except RuntimeError as e:
            msg = "rejected: " + str(e)
        with open(os.path.join(result_dir, f"r{rank}"), "w") as f:
            f.write(msg)
    finally:
        dist.destroy_process_group()


def test_two_rank_plan_mismatch_is_rejected(tmp_path):
    mp.spawn(_bad_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert open(tmp_path / f"r{r}").read().startswith("rejected"), r


def _reducer_worker(rank, world, port, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # a file rendezvous in the test's own directory: no TCP port to race for
    dist.init_process_group("gloo", init_method="file://" + os.path.join(result_dir, "pg_store"), rank=rank, world_size=world)
    try:
        import numpy as np
        import nanocamelid_b200 as ncm
        from nanocamelid_b200 import tp
        fn = tp.host_reducer(world)
        rng = np.random.default_rng(rank)
        part = (rng.standard_normal(300) * 10.0 ** rng.integers(-3, 3, 300)).astype(np.float32)
        buf = part.copy()
        assert fn(buf, 3, ncm.PHASE_FFN) == 0
        np.save(os.path.join(result_dir, f"p{rank}.npy"), part)
        np.save(os.path.join(result_dir, f"s{rank}.npy"), buf)
        # head pairs: equal logits on both ranks -> rank 0's token (strict '>')
        tok = np.array([0.0, 0.0], dtype=np.float32)
        tok.view(np.int32)[1] = 1000 + rank
        tok[0] = 2.5
        assert fn(tok, 3, ncm.PHASE_HEAD) == 0
        np.save(os.path.join(result_dir, f"h{rank}.npy"), tok)
    finally:
        dist.destroy_process_group()


def test_host_reducer_rank_ordered_sum_and_head_merge(tmp_path):
    """tp.host_reducer over gloo: both ranks hold ((0 + p0) + p1) in f32 and the same
    merged head pair (rank 0 wins a tie)."""
    import numpy as np
    mp.spawn(_reducer_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    p = [np.load(tmp_path / f"p{r}.npy") for r in range(2)]
    want = (np.float32(0.0) + p[0]).astype(np.float32) + p[1]
    for r in range(2):
        got = np.load(tmp_path / f"s{r}.npy")
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), r
        h = np.load(tmp_path / f"h{r}.npy")
        assert h[0] == 2.5 and h.view(np.int32)[1] == 1000, r
