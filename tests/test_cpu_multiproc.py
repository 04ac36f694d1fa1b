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
    dist.init_process_group("gloo", rank=rank, world_size=world)
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
    dist.init_process_group("gloo", rank=rank, world_size=world)
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
