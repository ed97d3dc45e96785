"""Tensor-parallel shard plans (host side, no GPU): at every tp_size the ranks'
slices partition the model exactly, and the row-parallel K slices fall on
whole super-blocks.  The second test runs the plan exchange as two gloo ranks.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from qwen382743090_b200 import runtime as rt

HQ, HV, AQ, AK, F, VOCAB = 16, 48, 24, 4, 17408, 151936


def plans(n):
    return [rt.shard_info(tp_rank=r, tp_size=n) for r in range(n)]


def check_partition(ps, n):
    qk = [h for p in ps for h in range(p.qk_head0, p.qk_head0 + p.qk_heads)]
    assert sorted(qk) == list(range(HQ))
    vh = [h for p in ps for h in p.v_head[: p.v_heads]]
    assert sorted(vh) == list(range(HV))
    for p in ps:
        local = list(p.v_head[: p.v_heads])
        # local value head j uses local q/k head j % qk_heads, i.e. global h % 16
        for j, h in enumerate(local):
            assert h % HQ == p.qk_head0 + j % p.qk_heads
        # ssm_out K slice: consecutive local heads pair into whole 256-blocks
        for j in range(0, len(local), 2):
            assert local[j] % 2 == 0 and local[j + 1] == local[j] + 1
    rows = sorted((p.ffn_row0, p.ffn_row1) for p in ps)
    assert rows[0][0] == 0 and rows[-1][1] == F
    assert all(a[1] == b[0] for a, b in zip(rows, rows[1:]))
    assert all((r1 - r0) % 256 == 0 for r0, r1 in rows)
    assert max(r1 - r0 for r0, r1 in rows) - min(r1 - r0 for r0, r1 in rows) <= 256
    qh = [h for p in ps for h in range(p.q_head0, p.q_head0 + p.q_heads)]
    assert sorted(qh) == list(range(AQ))
    for p in ps:  # every local query head's KV head is local
        for h in range(p.q_head0, p.q_head0 + p.q_heads):
            assert p.kv_head0 <= h // (AQ // AK) < p.kv_head0 + p.kv_heads
    voc = sorted((p.vocab0, p.vocab1) for p in ps)
    assert voc[0][0] == 0 and voc[-1][1] == VOCAB and all(a[1] == b[0] for a, b in zip(voc, voc[1:]))


@pytest.mark.parametrize("n", [1, 2, 4, 8])
def test_shard_plans_partition_the_model(n):
    check_partition(plans(n), n)


def test_unsupported_tp_size_is_rejected():
    with pytest.raises(rt.Q38Error):
        rt.shard_info(tp_rank=0, tp_size=3)


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    mine = rt.shard_info(tp_rank=rank, tp_size=world)
    got = [None] * world
    dist.all_gather_object(got, (mine.qk_head0, mine.qk_heads, list(mine.v_head[: mine.v_heads]), mine.ffn_row0,
                                 mine.ffn_row1, mine.q_head0, mine.q_heads, mine.vocab0, mine.vocab1))
    dist.destroy_process_group()
    if rank == 0:
        q.put(got)


def test_two_gloo_ranks_agree_on_a_partition():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    heads = sorted(h for g in got for h in g[2])
    assert heads == list(range(HV))
    assert got[0][4] == got[1][3] and got[1][4] == F
