"""Tensor-parallel decode on 2, 4 and 8 GPUs equals single-GPU decode.

One process per GPU builds its shard of the same seeded 4-layer model,
exchanges an NCCL id over gloo (the communicator also carries the CUDA IPC
handles of the exchange regions) and takes three greedy steps through the
peer-memory exchange; GPU 0 also runs the whole model alone.  Logits agree
within 1e-4 of max |logit| (only the order of the row-parallel sums differs),
the tokens are identical and no bounded wait gave up.  Each world size is
skipped when the box has fewer GPUs.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=4, attn_every=4, vocab=4096, ctx=512, seed=7)
START = dict(token=321, pos=100, kv_seed=5)
STEPS = 3


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from qwen382743090_b200 import runtime as rt

    try:
        torch.cuda.set_device(rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        rt.Context(rank)
        uid = [rt.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = rt.Comm(world, rank, uid[0])
        m = rt.Model(**CFG, tp_rank=rank, tp_size=world)
        m.set_comm(comm)
        m.set_position(**START)
        s = torch.cuda.Stream()
        toks = []
        for _ in range(STEPS):
            m.step(s.cuda_stream)
            s.synchronize()
            toks.append(m.position())
        logits = m.download("logits")[1].view(np.float32).copy()
        info = rt.shard_info(**CFG, tp_rank=rank, tp_size=world)
        got = [None] * world
        dist.all_gather_object(got, (toks, info.vocab0, logits, rt.fault_status()))
        m.close()
        comm.close()
        if rank == 0:
            ref = rt.Model(**CFG)
            ref.set_position(**START)
            ref_toks = []
            for _ in range(STEPS):
                ref.step(s.cuda_stream)
                s.synchronize()
                ref_toks.append(ref.position())
            ref_logits = ref.download("logits")[1].view(np.float32).copy()
            ref.close()
            q.put(dict(got=got, ref_toks=ref_toks, ref_logits=ref_logits))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put(dict(error=f"rank {rank}: {e!r}"))
        raise


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decode_matches_single_gpu(world):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
    assert "error" not in res, res.get("error")
    for p in procs:
        assert p.exitcode == 0
    got = res["got"]
    toks = [g[0] for g in got]
    assert all(t == res["ref_toks"] for t in toks), (toks, res["ref_toks"])
    full = np.zeros_like(res["ref_logits"])
    for toks_r, v0, lg, fault in got:
        assert fault == 0
        full[v0: v0 + lg.size] = lg
    ref = res["ref_logits"].astype(np.float64)
    err = np.abs(full - ref).max() / np.abs(ref).max()
    assert err <= 1e-4, err
