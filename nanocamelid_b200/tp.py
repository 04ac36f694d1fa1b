"""Tensor-parallel set-up over torch.distributed (host plumbing only).

One process per GPU.  The data path never goes through torch: each rank's model shard
exports a CUDA IPC handle of its exchange area (receive slots + flags), the handles are
all-gathered with torch.distributed, and every rank opens its peers' areas so that the
row-parallel GEMV epilogues can store partial rows straight into peer HBM over NVLink
(replacing the reference's TCP star allreduce, bin/cluster_tp_node.rs:1154-1180).
For the NCCL baseline reducer, rank 0's ncclUniqueId is broadcast the same way.
"""
import torch.distributed as dist

from . import REDUCE_FUSED_P2P, REDUCE_NCCL, Model, nccl_unique_id, shard_geometry


def even_shares(kv_heads, world):
    if kv_heads % world:
        raise ValueError(f"{kv_heads} kv heads cannot be split evenly over {world} ranks")
    return [kv_heads // world] * world


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


def connect(model: Model, rank, world, reducer=REDUCE_FUSED_P2P, group=None):
    """Exchanges peer handles (and an NCCL id for the baseline) and selects the reducer."""
    if world <= 1:
        return
    handles = exchange(model.tp_export(), world, group)
    model.tp_import(handles, world, rank)
    if reducer == REDUCE_NCCL:
        uid = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0, group=group)
        model.tp_nccl_init(uid[0], world, rank)
    model.tp_set_reducer(reducer)
