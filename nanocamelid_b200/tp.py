"""Tensor-parallel set-up over torch.distributed (host plumbing only).

One process per GPU.  The data path never goes through torch: each rank's model shard
exports a CUDA IPC handle of its exchange area (receive slots + flags), the handles are
all-gathered with torch.distributed, and every rank opens its peers' areas so that the
row-parallel GEMV epilogues can store partial rows straight into peer HBM over NVLink
(replacing the reference's TCP star allreduce, bin/cluster_tp_node.rs:1154-1180).
For the NCCL baseline reducer, rank 0's ncclUniqueId is broadcast the same way.
"""
import torch.distributed as dist

from . import (PHASE_HEAD, REDUCE_FUSED_P2P, REDUCE_HOST_CALLBACK, REDUCE_NCCL, Model, nccl_unique_id,
               shard_geometry)


def even_shares(kv_heads, world):
    if kv_heads % world:
        raise ValueError(f"{kv_heads} kv heads cannot be split evenly over {world} ranks")
    return [kv_heads // world] * world


def default_shares(kv_heads, world):
    """Even KV-head shares where world divides the KV heads, else the remainder on the
    last ranks (8 heads over 3 ranks -> [2, 3, 3], the reference's uneven plan)."""
    if world < 1 or world > kv_heads:
        raise ValueError(f"{world} ranks for {kv_heads} kv heads")
    base, rem = divmod(kv_heads, world)
    return [base + (1 if r >= world - rem else 0) for r in range(world)]


def exchange(obj, world, group=None):
    """All-gather of one picklable object per rank, in rank order (handles, plans)."""
    out = [None] * world
    dist.all_gather_object(out, obj, group=group)
    return out


def check_plan(spec_, shares, world, rank, group=None):
    """Every rank computes its own shard geometry (tp.rs:662-701); the ranks exchange them
    and check that together they tile the Q heads, KV heads, FFN columns and head rows
    in rank order.  Returns the list of all ranks' geometries."""
    mine = shard_geometry(spec_.heads, spec_.kv_heads, spec_.ffn, spec_.vocab, shares, rank)
    plans = exchange(mine, world, group)
    q = kv = f = h = 0
    for r, g in enumerate(plans):
        if (g["q_start"], g["kv_start"], g["ffn_start"], g["head_row_start"]) != (q, kv, f, h):
            raise RuntimeError(f"rank {r}: shard plan does not continue the previous rank's")
        q += g["q_heads"]; kv += g["kv_heads"]; f += g["ffn_len"]; h += g["head_rows"]
    if (q, kv, f, h) != (spec_.heads, spec_.kv_heads, spec_.ffn, spec_.vocab):
        raise RuntimeError("shard plans do not cover the model")
    return plans


def rank_ordered(parts, phase):
    """The global value from every rank's buffer, in rank order: the f32 sum from 0.0f
    (tp.rs:349-363, the master's fixed-order sum in cluster_tp_node.rs:1154-1180), or for
    the head the first maximum of every row's pair by strict '>'
    (cluster_tp_node.rs:1185-1204; the token slot is copied, never computed on)."""
    import numpy as np
    if phase == PHASE_HEAD:
        # one (logit, token bits) pair per row: merged row by row
        best = np.array(parts[0], dtype=np.float32, copy=True).reshape(-1, 2)
        for p in parts[1:]:
            p = np.asarray(p, dtype=np.float32).reshape(-1, 2)
            take = p[:, 0] > best[:, 0]
            best[take] = p[take]
        return best.reshape(-1)
    acc = np.zeros(len(parts[0]), dtype=np.float32)
    for p in parts:
        acc = acc + p
    return acc


def host_reducer(world, group=None):
    """A reduce closure (tp.rs:226-236) over a torch.distributed group of CPU ranks
    (gloo or any backend): all-gathers this rank's buffer and leaves rank_ordered() of
    all of them in place.  For Model.tp_set_host_reducer."""
    import numpy as np
    import torch

    def fn(buf, layer, phase):
        mine = torch.from_numpy(np.array(buf, dtype=np.float32, copy=True))
        outs = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(outs, mine, group=group)
        buf[:] = rank_ordered([o.numpy() for o in outs], phase)
        return 0

    return fn


def connect(model: Model, rank, world, reducer=REDUCE_FUSED_P2P, group=None):
    """Exchanges peer handles (and an NCCL id for the baseline) and selects the reducer.
    REDUCE_HOST_CALLBACK uses host_reducer over `group` (no device buffers are shared)."""
    if world <= 1:
        return
    if reducer == REDUCE_HOST_CALLBACK:
        model.tp_set_host_reducer(host_reducer(world, group))
        model.tp_set_reducer(reducer)
        return
    handles = exchange(model.tp_export(), world, group)
    model.tp_import(handles, world, rank)
    if reducer == REDUCE_NCCL:
        uid = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0, group=group)
        model.tp_nccl_init(uid[0], world, rank)
    model.tp_set_reducer(reducer)
