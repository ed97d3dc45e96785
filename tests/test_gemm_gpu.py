"""Batched (multi-token verify / prefill) Q5_K / Q4_K GEMM on the tensor cores against
the FP64 oracle, row by row, with the GEMV tolerance (a row fails only beyond
1e-4 absolute and 1e-3 relative)."""
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
@pytest.mark.parametrize("batch", [2, 4, 8])
@pytest.mark.parametrize("rows,cols", [(6144, 5120), (5120, 17408), (297, 2048), (8, 1024), (13, 512)])
def test_tiled_mma_gemm_matches_oracle(ctx, port, ggml_type, batch, rows, cols):
    blocks = synth.gen_blocks(ggml_type, rows, cols, seed=rows + cols + batch)
    wd = ctx.upload(synth.repack_tiled(ggml_type, blocks, rows, cols))
    x = synth.gen_x(cols, seed=batch * 31 + cols, batch=batch)
    xd = ctx.upload(x)
    yd = ctx.alloc(4 * rows * batch)
    yd.fill(0xFF)
    rt.gemm_f32(rt.weight_desc(ggml_type, 2, rows, cols, wd.ptr), xd.ptr, batch, yd.ptr)
    y = yd.download(np.float32, rows * batch).reshape(batch, rows)
    ref = port.gemv(ggml_type, blocks, x, rows, cols, threads=16)
    for b in range(batch):
        close_rows(y[b], ref[b], f"batch {b} of {batch}, {rows}x{cols}")
    assert rt.fault_status() == 0
    for buf in (wd, xd, yd):
        buf.free()


def test_batched_other_types_loop_rows(ctx, port):
    rows, cols, batch = 512, 2048, 3
    blocks = synth.gen_blocks(14, rows, cols, seed=5)
    wd = ctx.upload(blocks)
    x = synth.gen_x(cols, seed=6, batch=batch)
    xd, yd = ctx.upload(x), ctx.alloc(4 * rows * batch)
    rt.gemm_f32(rt.weight_desc(14, 0, rows, cols, wd.ptr), xd.ptr, batch, yd.ptr)
    y = yd.download(np.float32, rows * batch).reshape(batch, rows)
    ref = port.gemv(14, blocks, x, rows, cols, threads=8)
    for b in range(batch):
        close_rows(y[b], ref[b], f"Q6_K batch {b}")
    for buf in (wd, xd, yd):
        buf.free()


@pytest.mark.parametrize("ggml_type", [13, 12])
@pytest.mark.parametrize("rows,cols,batch", [(6144, 5120, 8), (1000, 6144, 3), (6144, 5120, 11)])
def test_batched_rows_equal_batch1_gemv(ctx, ggml_type, rows, cols, batch):
    """Each row of the batched GEMM is bit-identical to the batch-1 GEMV of
    that activation row (same tiles, same CTA split, same arithmetic order);
    batch 11 runs as 8 + 3."""
    blocks = synth.gen_blocks(ggml_type, rows, cols, seed=rows * 3 + batch)
    wd = ctx.upload(synth.repack_tiled(ggml_type, blocks, rows, cols))
    desc = rt.weight_desc(ggml_type, 2, rows, cols, wd.ptr)
    x = synth.gen_x(cols, seed=batch + 77, batch=batch)
    xd, yd, y1 = ctx.upload(x), ctx.alloc(4 * rows * batch), ctx.alloc(4 * rows)
    rt.gemm_f32(desc, xd.ptr, batch, yd.ptr)
    Y = yd.download(np.float32, rows * batch).reshape(batch, rows)
    for b in range(batch):
        rt.gemv_f32(desc, xd.ptr + 4 * cols * b, y1.ptr)
        np.testing.assert_array_equal(Y[b].view(np.uint32), y1.download(np.float32, rows).view(np.uint32))
    assert rt.fault_status() == 0
    for buf in (wd, xd, yd, y1):
        buf.free()
