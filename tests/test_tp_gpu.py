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


# the pack case: uneven ffn_down K (12 super-blocks) and replicated KV heads at 4 ranks
PACK_CFG = dict(n_layers=4, attn_every=4, hidden=2048, ffn=3072, vocab=4096, gdn_qk_heads=8, gdn_v_heads=16,
                attn_q_heads=24, attn_kv_heads=4, ctx=512, seed=7)
SHARD_TENSORS = ("attn_norm", "post_attention_norm", "ffn_gate", "ffn_up", "ffn_down", "attn_qkvz", "ssm_ba",
                 "ssm_out", "ssm_conv1d", "ssm_dt", "ssm_a", "ssm_norm", "conv_state0", "ssm_state")
ATTN_TENSORS = ("attn_norm", "post_attention_norm", "ffn_gate", "ffn_up", "ffn_down", "attn_q", "attn_k", "attn_v",
                "attn_output", "attn_q_norm", "attn_k_norm")


def _load_from_pack(rt, cfg, rank, world, pack_path, dist):
    """Rank 0 writes the seeded model as a pack; every rank loads its shard
    from it and checks each tensor against the seeded shard, byte for byte."""
    from qwen382743090_b200 import q38pack

    if rank == 0:
        with rt.Model(**cfg) as whole:
            q38pack.export_model_pack(whole, pack_path)
    dist.barrier()
    m = rt.Model(pack=pack_path, **cfg, tp_rank=rank, tp_size=world)
    bad = []
    with rt.Model(**cfg, tp_rank=rank, tp_size=world) as seeded:
        names = ["token_embd", "output", "output_norm"]
        for L in range(cfg["n_layers"]):
            attn = L % cfg["attn_every"] == cfg["attn_every"] - 1
            names += [f"blk.{L}.{t}" for t in (ATTN_TENSORS if attn else SHARD_TENSORS)]
        for n in names:
            if not np.array_equal(seeded.download(n)[1], m.download(n)[1]):
                bad.append(n)
    return m, bad


def _worker(rank, world, port, q, cfg=CFG, pack_path=None):
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
        bad = []
        if pack_path:
            m, bad = _load_from_pack(rt, cfg, rank, world, pack_path, dist)
        else:
            m = rt.Model(**cfg, tp_rank=rank, tp_size=world)
        m.set_comm(comm)
        m.set_position(**START)
        s = torch.cuda.Stream()
        toks = []
        for _ in range(STEPS):
            m.step(s.cuda_stream)
            s.synchronize()
            toks.append(m.position())
        logits = m.download("logits")[1].view(np.float32).copy()
        info = rt.shard_info(**cfg, tp_rank=rank, tp_size=world)
        got = [None] * world
        dist.all_gather_object(got, (toks, info.vocab0, logits, rt.fault_status(), bad))
        m.close()
        comm.close()
        if rank == 0:
            ref = rt.Model(**cfg)
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


def _run(world, cfg=CFG, pack_path=None):
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
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, cfg, pack_path)) for r in range(world)]
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
    for toks_r, v0, lg, fault, bad in got:
        assert fault == 0
        assert not bad, f"pack-loaded shard tensors differ from the seeded shard: {bad}"
        full[v0: v0 + lg.size] = lg
    ref = res["ref_logits"].astype(np.float64)
    err = np.abs(full - ref).max() / np.abs(ref).max()
    assert err <= 1e-4, err


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decode_matches_single_gpu(world):
    _run(world)


@pytest.mark.parametrize("world", [2, 4])
def test_tp_decode_from_pack(world, tmp_path):
    """Each rank loads its shard from one Q38PACK (row windows of the tensors,
    residue-class GDN heads, uneven ffn_down K): byte-equal to the seeded
    shard, and the decode equals the single-GPU model."""
    _run(world, PACK_CFG, str(tmp_path / "model.q38pack"))
