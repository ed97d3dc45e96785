"""The tensor-parallel exchange (q38_tp_exchange) on one GPU.

The peers' side is played by the host: their partials are written into this
rank's exchange region as the 16-byte units {x[2i], epoch, x[2i+1], epoch} a
peer's kernel would store, so only one kernel runs and nothing waits on
another launch.  Checked: x_out is x_in plus every rank's partial added in
rank order (bit-exact float32), this rank's partial lands in every peer's
region in the same unit format, the x-fragments decode to RMSNorm(x_out) * w,
and a partial that never arrives ends the bounded wait with fault site 5
instead of a hang (after which calls skip their waits until the fault word is
cleared).
"""
from __future__ import annotations

import time

import numpy as np
import pytest

from qwen382743090_b200 import runtime as rt

from xfrag_format import unpack_values

pytestmark = pytest.mark.gpu

N = 5120
KMAX = 8  # slots per parity in a region


def _units(p: np.ndarray, epoch: int) -> np.ndarray:
    u = np.zeros((p.size // 2, 4), np.uint32)
    u[:, 0] = p[0::2].view(np.uint32)
    u[:, 1] = epoch
    u[:, 2] = p[1::2].view(np.uint32)
    u[:, 3] = epoch
    return u


def _slot_offset(par: int, sender: int) -> int:
    return (par * KMAX + sender) * (N // 2) * 16


class Setup:
    def __init__(self, ctx, size, rank, step, seed):
        rng = np.random.default_rng(seed)
        self.size, self.rank, self.step = size, rank, step
        self.x_in = rng.standard_normal(N).astype(np.float32) * np.float32(30.0)
        self.parts = [rng.standard_normal(N).astype(np.float32) for _ in range(size)]
        self.w = (1.0 + 0.1 * rng.standard_normal(N)).astype(np.float32)
        nbytes = rt.tp_exchange_bytes(N)
        assert nbytes == 2 * KMAX * (N // 2) * 16 + 2048  # slots + this rank's scratch
        self.regions = [ctx.alloc(nbytes) for _ in range(size)]
        for r in self.regions:
            r.fill(0)
        self.xd = ctx.upload(self.x_in)
        self.xo = ctx.alloc(4 * N)
        self.pd = ctx.upload(self.parts[rank])
        self.wd = ctx.upload(self.w)
        self.xf = ctx.alloc(rt.xfrag_bytes(N))
        self.sd = ctx.upload(np.array([step, 0, 0, 0], np.uint32))

    def epoch(self, instance):
        return ((self.step << 9) + instance + 1) & 0xFFFFFFFF

    def run(self, instance, eps=1e-6):
        rt.tp_exchange(self.xd.ptr, self.xo.ptr, self.pd.ptr, [r.ptr for r in self.regions], self.sd.ptr, N,
                       self.rank, self.size, instance, self.wd.ptr, self.xf.ptr, eps)

    def free(self):
        for b in self.regions + [self.xd, self.xo, self.pd, self.wd, self.xf, self.sd]:
            b.free()


@pytest.mark.parametrize("size,rank,instance", [(2, 0, 7), (2, 1, 0), (4, 2, 125), (8, 5, 38), (8, 0, 510)])
def test_exchange_sums_in_rank_order_and_packs(ctx, size, rank, instance):
    s = Setup(ctx, size, rank, step=3, seed=size * 10 + rank)
    E, par = s.epoch(instance), instance & 1
    mine = s.regions[rank]
    for j in range(size):
        if j != rank:
            mine.upload(_units(s.parts[j], E), offset=_slot_offset(par, j))
    s.run(instance)
    rt.synchronize()
    assert rt.fault_status() == 0
    ref = s.x_in.copy()
    for j in range(size):
        ref = (ref + s.parts[j]).astype(np.float32)  # float32, rank order
    got = s.xo.download(np.float32, N)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
    # this rank's partial, as units, in every peer's region
    want = _units(s.parts[rank], E)
    for j in range(size):
        if j == rank:
            continue
        units = s.regions[j].download(np.uint32, (N // 2) * 4, offset=_slot_offset(par, rank)).reshape(-1, 4)
        np.testing.assert_array_equal(units, want)
    # x-fragments of the normalised row
    x64 = ref.astype(np.float64)
    inv = 1.0 / np.sqrt(np.mean(x64 * x64) + 1e-6)
    v = x64 * inv * s.w.astype(np.float64)
    dec = unpack_values(s.xf.download(np.uint8, rt.xfrag_bytes(N)), N // 256)
    for b in range(N // 256):
        blk = slice(256 * b, 256 * b + 256)
        assert np.abs(dec[blk] - v[blk]).max() <= 1e-6 * np.abs(v[blk]).max()
    s.free()


def test_exchange_wait_is_bounded(ctx):
    """No peer ever sends: every poll gives up after its bound, the kernel
    finishes and the host reads fault site 5; with the fault word set the next
    exchange returns without waiting."""
    rt.fault_clear()
    s = Setup(ctx, size=2, rank=0, step=1, seed=5)
    t0 = time.time()
    s.run(4)
    rt.synchronize()
    first = time.time() - t0
    assert rt.fault_status() == 5
    assert first < 60.0
    t0 = time.time()
    s.run(5)
    rt.synchronize()
    assert time.time() - t0 < 0.5
    rt.fault_clear()
    assert rt.fault_status() == 0
    s.free()


def test_exchange_rejects_bad_arguments(ctx):
    s = Setup(ctx, size=2, rank=0, step=0, seed=1)
    regions = [r.ptr for r in s.regions]
    with pytest.raises(rt.Q38Error):  # x_out aliases x_in
        rt.tp_exchange(s.xd.ptr, s.xd.ptr, s.pd.ptr, regions, s.sd.ptr, N, 0, 2, 0)
    with pytest.raises(rt.Q38Error):  # rank >= size
        rt.tp_exchange(s.xd.ptr, s.xo.ptr, s.pd.ptr, regions, s.sd.ptr, N, 2, 2, 0)
    with pytest.raises(rt.Q38Error):  # n not a multiple of 256
        rt.tp_exchange(s.xd.ptr, s.xo.ptr, s.pd.ptr, regions, s.sd.ptr, N - 128, 0, 2, 0)
    with pytest.raises(rt.Q38Error):  # instance out of range
        rt.tp_exchange(s.xd.ptr, s.xo.ptr, s.pd.ptr, regions, s.sd.ptr, N, 0, 2, 511)
    with pytest.raises(rt.Q38Error):  # a missing region
        rt.tp_exchange(s.xd.ptr, s.xo.ptr, s.pd.ptr, regions[:1] + [0], s.sd.ptr, N, 0, 2, 0)
    s.free()
