"""Tensor-parallel set-up over torch.distributed (host plumbing only).

One process per GPU.  The data path never goes through torch: each rank's model shard
exports a CUDA IPC handle of its exchange area (receive slots + flags), the handles are
all-gathered with torch.distributed, and every rank opens its peers' areas so that the
row-parallel GEMV epilogues can store partial rows straight into peer HBM over NVLink
(replacing the reference's TCP star allreduce, bin/cluster_tp_node.rs:1154-1180).
For the NCCL baseline reducer, rank 0's ncclUniqueId is broadcast the same way.
"""
import torch.distributed as dist

from . import REDUCE_FUSED_P2P, REDUCE_NCCL, Model, nccl_unique_id


def even_shares(kv_heads, world):
    if kv_heads % world:
        raise ValueError(f"{kv_heads} kv heads cannot be split evenly over {world} ranks")
    return [kv_heads // world] * world


def connect(model: Model, rank, world, reducer=REDUCE_FUSED_P2P, group=None):
    """Exchanges peer handles (and an NCCL id for the baseline) and selects the reducer."""
    if world <= 1:
        return
    handles = [None] * world
    dist.all_gather_object(handles, model.tp_export(), group=group)
    model.tp_import(handles, world, rank)
    if reducer == REDUCE_NCCL:
        uid = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0, group=group)
        model.tp_nccl_init(uid[0], world, rank)
    model.tp_set_reducer(reducer)
