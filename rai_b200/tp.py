"""Tensor-parallel setup across processes (one process per GPU).

Each rank loads its shard with `RaiModel(blob, device, tp_rank, tp_size)`;
`connect` then swaps the ranks' exchange-arena handles through
torch.distributed (any backend that carries Python objects: gloo or nccl),
maps them, and ends with a barrier so that no rank creates a decoder (whose
first forward may write into a peer's arena) before every rank is mapped.
"""
from typing import Optional


def connect(model, group: Optional[object] = None) -> None:
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world != model.tp_size:
        raise ValueError(f"process group has {world} ranks, the model shard expects {model.tp_size}")
    if dist.get_rank(group) != model.tp_rank:
        raise ValueError("process-group rank and model tensor-parallel rank differ")
    mine = model.tp_handle()
    handles = [None] * world
    dist.all_gather_object(handles, mine, group=group)
    model.tp_connect(handles)
    dist.barrier(group=group)
