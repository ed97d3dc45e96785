"""The tcgen05 batched GEMM (q38_gemm_f32_tc: kind::i8 MMAs, accumulators in
tensor memory) against the FP64 oracle, row by row, with the GEMV tolerance (a
row fails only beyond 1e-4 absolute and 1e-3 relative); shapes that take one
CTA per row block and shapes whose K range is split across CTAs."""
from __future__ import annotations

import numpy as np
import pytest

from qwen382743090_b200 import runtime as rt
from qwen382743090_b200 import synth

pytestmark = pytest.mark.gpu


def close_rows(y, ref, what):
    err = np.abs(np.asarray(y, np.float64) - ref)
    bad = (err > 1e-4) & (err > 1e-3 * np.abs(ref))
    assert not bad.any(), f"{what}: {bad.sum()} outputs out of tolerance (max err {err.max():.3g})"


@pytest.mark.parametrize("ggml_type", [13, 12])
@pytest.mark.parametrize("batch", [2, 3, 4, 5, 8, 11])
@pytest.mark.parametrize("rows,cols", [(6144, 5120), (17408, 5120), (5120, 17408), (297, 2048), (8, 1024),
                                       (13, 512)])
def test_tc_gemm_matches_oracle(ctx, port, ggml_type, batch, rows, cols):
    if rows * cols > 6144 * 5120 and batch not in (4, 8):
        pytest.skip("large shapes at batch 4 and 8 only")
    blocks = synth.gen_blocks(ggml_type, rows, cols, seed=rows + cols + batch + 1)
    wd = ctx.upload(synth.repack_tiled(ggml_type, blocks, rows, cols))
    x = synth.gen_x(cols, seed=batch * 37 + cols, batch=batch)
    xd = ctx.upload(x)
    yd = ctx.alloc(4 * rows * batch)
    yd.fill(0xFF)
    rt.gemm_f32_tc(rt.weight_desc(ggml_type, 2, rows, cols, wd.ptr), xd.ptr, batch, yd.ptr)
    y = yd.download(np.float32, rows * batch).reshape(batch, rows)
    assert rt.fault_status() == 0
    ref = port.gemv(ggml_type, blocks, x, rows, cols, threads=16)
    for b in range(batch):
        close_rows(y[b], ref[b], f"batch {b} of {batch}, {rows}x{cols}")
    for buf in (wd, xd, yd):
        buf.free()


def test_tc_gemm_many_waves(ctx, port):
    """151936 rows: 1187 row blocks, one CTA per SM at a time, so later CTAs
    allocate tensor memory on SMs whose earlier CTAs have freed it."""
    rows, cols, batch = 151936, 5120, 3
    blocks = synth.gen_blocks(12, rows, cols, seed=123)
    wd = ctx.upload(synth.repack_tiled(12, blocks, rows, cols))
    x = synth.gen_x(cols, seed=124, batch=batch)
    xd = ctx.upload(x)
    yd = ctx.alloc(4 * rows * batch)
    yd.fill(0xFF)
    rt.gemm_f32_tc(rt.weight_desc(12, 2, rows, cols, wd.ptr), xd.ptr, batch, yd.ptr)
    y = yd.download(np.float32, rows * batch).reshape(batch, rows)
    assert rt.fault_status() == 0
    ref = port.gemv(12, blocks, x, rows, cols, threads=16)
    for b in range(batch):
        close_rows(y[b], ref[b], f"batch row {b}")
    for buf in (wd, xd, yd):
        buf.free()


def test_tc_gemm_repeatable_and_agrees_with_mma_sync(ctx):
    """Two calls give the same bits (fixed split-K order, counters re-zeroed by
    every call), and the result agrees with the mma.sync GEMM within the GEMV
    tolerance."""
    rows, cols, batch = 6144, 5120, 8
    blocks = synth.gen_blocks(13, rows, cols, seed=99)
    wd = ctx.upload(synth.repack_tiled(13, blocks, rows, cols))
    desc = rt.weight_desc(13, 2, rows, cols, wd.ptr)
    xd = ctx.upload(synth.gen_x(cols, seed=98, batch=batch))
    ya, yb, yc = (ctx.alloc(4 * rows * batch) for _ in range(3))
    rt.gemm_f32_tc(desc, xd.ptr, batch, ya.ptr)
    rt.gemm_f32_tc(desc, xd.ptr, batch, yb.ptr)
    rt.gemm_f32(desc, xd.ptr, batch, yc.ptr)
    a, b, c = (buf.download(np.float32, rows * batch) for buf in (ya, yb, yc))
    assert rt.fault_status() == 0
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    close_rows(a, c.astype(np.float64), "tcgen05 vs mma.sync")
    for buf in (wd, xd, ya, yb, yc):
        buf.free()


def test_tc_gemm_rejects_other_layouts(ctx):
    blocks = synth.gen_blocks(13, 64, 512, seed=3)
    wd = ctx.upload(blocks)
    xd, yd = ctx.alloc(4 * 512 * 2), ctx.alloc(4 * 64 * 2)
    with pytest.raises(rt.Q38Error):
        rt.gemm_f32_tc(rt.weight_desc(13, 0, 64, 512, wd.ptr), xd.ptr, 2, yd.ptr)
    for buf in (wd, xd, yd):
        buf.free()


@pytest.mark.parametrize("batch", [2, 8])
def test_tc_gemm_back_to_back_calls(ctx, port, batch):
    """Sixty calls queued on one stream without a synchronisation (each launch
    may start while its predecessor drains): every call's rows stay correct and
    no bounded wait gives up."""
    rows, cols = 6144, 5120
    blocks = [synth.gen_blocks(13, rows, cols, seed=40 + i) for i in range(3)]
    wds = [ctx.upload(synth.repack_tiled(13, b, rows, cols)) for b in blocks]
    descs = [rt.weight_desc(13, 2, rows, cols, wd.ptr) for wd in wds]
    x = synth.gen_x(cols, seed=batch + 500, batch=batch)
    xd = ctx.upload(x)
    ys = [ctx.alloc(4 * rows * batch) for _ in range(3)]
    for i in range(60):
        rt.gemm_f32_tc(descs[i % 3], xd.ptr, batch, ys[i % 3].ptr)
    rt.synchronize()
    assert rt.fault_status() == 0
    for i in range(3):
        y = ys[i].download(np.float32, rows * batch).reshape(batch, rows)
        ref = port.gemv(13, blocks[i], x, rows, cols, threads=16)
        for b in range(batch):
            close_rows(y[b], ref[b], f"copy {i} batch row {b}")
    for buf in (*wds, xd, *ys):
        buf.free()
