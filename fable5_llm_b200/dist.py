"""Row-sharded decode across GPUs: the host-side handshake.

One process and one ``DecodeModel(world_size=G, rank=r)`` per GPU.  Every
rank holds its ``split_rows`` share of each matrix (ref/seq_format.py:
1177-1189); the persistent kernel's GEMV epilogues store their output rows
into every rank's buffers, so before the first step the ranks exchange the
CUDA IPC handles of those buffers.  This module does the exchange over any
``torch.distributed`` process group (gloo or nccl).
"""
from __future__ import annotations


def gather_handles(handle: bytes, group=None):
    """All-gather one 64-byte handle per rank -> list in rank order."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    for i, h in enumerate(out):
        if not isinstance(h, (bytes, bytearray)) or len(h) != 64:
            raise RuntimeError(f"rank {i} sent a malformed IPC handle")
    return [bytes(h) for h in out]


def connect(model, group=None):
    """Exchange IPC handles among the group's ranks and attach the peers."""
    model.attach_peers(gather_handles(model.ipc_handle(), group))
