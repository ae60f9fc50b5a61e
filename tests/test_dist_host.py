"""Host logic of row-sharded decode on CPU (gloo, world size 2): the IPC
handle exchange every rank performs before its first step."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ws, port, bad, q):
    import torch.distributed as dist
    from fable5_llm_b200 import dist as F
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        h = bytes([rank]) * 64 if not (bad and rank == 1) else b"short"
        try:
            q.put((rank, F.gather_handles(h)))
        except RuntimeError as e:
            q.put((rank, str(e)))
    finally:
        dist.destroy_process_group()


def _run(bad):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, bad, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    return out


def test_gather_handles_rank_order():
    out = _run(bad=False)
    for r in range(2):
        assert out[r] == [bytes([0]) * 64, bytes([1]) * 64]


def test_gather_handles_rejects_malformed():
    out = _run(bad=True)
    for r in range(2):
        assert "malformed" in out[r]
