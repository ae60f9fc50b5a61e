"""Row-sharded decode on 2 GPUs (persistent engine): every rank streams its
split_rows share of each matrix and the GEMV epilogues store their output
rows into both GPUs' buffers; tokens, max logits and the replicated
DeltaNet / KV state must equal the oracle's bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
SEED = 2026
TOKS = [5, 4095, 77, 1000, 3, 3, 2048]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ws, port, q):
    import torch.distributed as dist
    from fable5_llm_b200 import dist as F
    from fable5_llm_b200.config import Geometry
    from fable5_llm_b200.model import DecodeModel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        m = DecodeModel(Geometry(4, 4096), max_T=128, device=rank, world_size=ws, rank=rank)
        m.load_synthetic(SEED)
        m.reset()
        F.connect(m)
        dist.barrier()
        res = [m.decode_step(tok, t) for t, tok in enumerate(TOKS)]
        st = {i: (m.get_dn_state(i, len(TOKS))["S"] if lt != "full_attention" else m.get_kv(i, len(TOKS)))
              for i, lt in enumerate(m.geom.layer_types)}
        dist.barrier()
        q.put((rank, res, st if rank == 0 else None))
        m.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_row_sharded_2gpu_vs_oracle():
    import oracle as O
    from oracle.model import OracleModel
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = {}
    for _ in ps:
        r, res, st = q.get(timeout=600)
        out[r] = (res, st)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    r = O.OracleRunner(OracleModel(SEED, O.Geometry(4, 4096)), max_T=128)
    for t, tok in enumerate(TOKS):
        ref_tok, y = r.step(tok, t)
        for rank in (0, 1):
            assert out[rank][0][t] == (ref_tok, int(y.max())), f"rank {rank} step {t}"
    st = out[0][1]
    for i, c in enumerate(r.caches):
        if hasattr(c, "S"):
            assert np.array_equal(st[i], c.S), f"layer {i} S"
        else:
            for tt in range(len(TOKS)):
                for h in range(4):
                    assert np.array_equal(st[i]["k"][tt][h][0], c.k8[h, tt]) and st[i]["k"][tt][h][1] == c.ke[h, tt]
