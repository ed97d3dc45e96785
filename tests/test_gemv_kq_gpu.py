"""GPU parity of the layout-0 (GGUF-native) K-quant GEMVs against the FP64 oracle.

Covers Q4_K, Q5_K, Q6_K and IQ4_XS with F32 activations (packed inside each
CTA, or through the workspace x-pack for wide K) and Q8_K activations, at the
reference's projection shapes plus ragged ones: odd row counts, K not a
multiple of 1024 (partial 4-block chunks), a single row.  Tolerance as the
reference's check (src/driver.cpp:6966-6975): a row fails only when it is off
by more than 1e-4 absolute AND 1e-3 relative.
"""
from __future__ import annotations

import numpy as np
import pytest

from qwen382743090_b200 import runtime as rt
from qwen382743090_b200 import synth

pytestmark = pytest.mark.gpu

TYPES = {12: "Q4_K", 13: "Q5_K", 14: "Q6_K", 23: "IQ4_XS"}


def assert_close(got, ref, what):
    got = np.asarray(got, dtype=np.float64)
    err = np.abs(got - ref)
    bad = (err > 1e-4) & (err > 1e-3 * np.abs(ref))
    i = int(np.argmax(err / (np.abs(ref) + 1e-4)))
    assert not bad.any(), f"{what}: {bad.sum()} rows out of tolerance; row {i} got {got[i]} ref {ref[i]}"


SHAPES = [(6144, 5120), (48, 5120), (1024, 5120), (5120, 6144), (5120, 17408), (297, 1280), (7, 768), (1, 256),
          (33, 2048)]


@pytest.mark.parametrize("ggml_type", list(TYPES))
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_layout0_f32_matches_fp64_oracle(ctx, port, ggml_type, rows, cols):
    blocks = synth.gen_blocks(ggml_type, rows, cols, seed=ggml_type * 1000 + rows + cols)
    wd = ctx.upload(blocks)
    x = synth.gen_x(cols, seed=cols + ggml_type)[0]
    xd = ctx.upload(x)
    yd = ctx.alloc(4 * rows)
    yd.fill(0xFF)
    rt.gemv_f32(rt.weight_desc(ggml_type, 0, rows, cols, wd.ptr), xd.ptr, yd.ptr)
    rt.synchronize()
    y = yd.download(np.float32, rows)
    ref = port.gemv(ggml_type, blocks, x, rows, cols, threads=8)[0]
    assert_close(y, ref, f"{TYPES[ggml_type]} f32 {rows}x{cols}")
    assert rt.fault_status() == 0
    for b in (wd, xd, yd):
        b.free()


@pytest.mark.parametrize("ggml_type", list(TYPES))
@pytest.mark.parametrize("rows,cols", [(6144, 5120), (5120, 17408), (297, 1280)])
def test_layout0_q8k_matches_oracle(ctx, port, ggml_type, rows, cols):
    blocks = synth.gen_blocks(ggml_type, rows, cols, seed=ggml_type * 7 + rows)
    wd = ctx.upload(blocks)
    x = synth.gen_x(cols, seed=cols * 3 + ggml_type)[0]
    xq = port.quantize_q8k(x)
    xqd = ctx.upload(xq)
    yd = ctx.alloc(4 * rows)
    rt.gemv_q8k(rt.weight_desc(ggml_type, 0, rows, cols, wd.ptr), xqd.ptr, yd.ptr)
    rt.synchronize()
    y = yd.download(np.float32, rows)
    ref = port.gemv_q8k(ggml_type, blocks, xq, rows, cols, threads=8)[0]
    assert_close(y, ref, f"{TYPES[ggml_type]} x Q8_K {rows}x{cols}")
    for b in (wd, xqd, yd):
        b.free()


@pytest.mark.parametrize("ggml_type", list(TYPES))
def test_layout0_activation_paths_agree_and_are_deterministic(ctx, port, ggml_type):
    """In-CTA f32 packing, a staged x-pack and the reference-named entry give
    the same bits, run after run."""
    rows, cols = 2050, 4096
    blocks = synth.gen_blocks(ggml_type, rows, cols, seed=ggml_type + 77)
    wd = ctx.upload(blocks)
    x = synth.gen_x(cols, seed=78)[0]
    xd = ctx.upload(x)
    xp = ctx.alloc(rt.xpack_bytes(3, cols))
    ys = [ctx.alloc(4 * rows) for _ in range(4)]
    desc = rt.weight_desc(ggml_type, 0, rows, cols, wd.ptr)
    rt.gemv_f32(desc, xd.ptr, ys[0].ptr)
    rt.xpack_f32(xd.ptr, cols, 1, xp.ptr)
    rt.gemv_packed(desc, xp.ptr, 3, 1, ys[1].ptr)
    rt.reference_gemv_f32(ggml_type, wd.ptr, xd.ptr, ys[2].ptr, cols, rows)
    rt.gemv_f32(desc, xd.ptr, ys[3].ptr)
    out = [b.download(np.float32, rows).view(np.uint32) for b in ys]
    for o in out[1:]:
        np.testing.assert_array_equal(o, out[0])
    assert_close(out[0].view(np.float32), port.gemv(ggml_type, blocks, x, rows, cols, threads=8)[0], "paths")
    for b in (wd, xd, xp, *ys):
        b.free()


def test_q5k_q8k_dp4a_entry_matches_oracle(ctx, port):
    rows, cols = 5120, 6144
    blocks = synth.gen_blocks(13, rows, cols, seed=5)
    wd = ctx.upload(blocks)
    xq = port.quantize_q8k(synth.gen_x(cols, seed=6)[0])
    xqd = ctx.upload(xq)
    yd = ctx.alloc(4 * rows)
    rt.q5k_q8k_dp4a_gemv(wd.ptr, xqd.ptr, yd.ptr, cols, rows)
    y = yd.download(np.float32, rows)
    assert_close(y, port.gemv_q8k(13, blocks, xq, rows, cols, threads=8)[0], "q38_q5k_q8k_dp4a_gemv")
    for b in (wd, xqd, yd):
        b.free()


def test_layout0_nan_and_zero_activations(ctx):
    rows, cols = 64, 1024
    for t in TYPES:
        blocks = synth.gen_blocks(t, rows, cols, seed=t)
        wd = ctx.upload(blocks)
        yd = ctx.alloc(4 * rows)
        xd = ctx.upload(np.zeros(cols, np.float32))
        rt.gemv_f32(rt.weight_desc(t, 0, rows, cols, wd.ptr), xd.ptr, yd.ptr)
        assert np.all(yd.download(np.float32, rows) == 0.0)
        x = synth.gen_x(cols, seed=1)[0]
        x[700] = np.nan
        xd2 = ctx.upload(x)
        rt.gemv_f32(rt.weight_desc(t, 0, rows, cols, wd.ptr), xd2.ptr, yd.ptr)
        assert np.isnan(yd.download(np.float32, rows)).all()
        for b in (wd, yd, xd, xd2):
            b.free()


@pytest.mark.parametrize("rows,cols", [(151936, 5120), (40961, 2048)])
def test_q6k_vocab_projection_wide_launch(ctx, port, rows, cols):
    """The lm_head shape (config 2: 5120 -> 151936, Q6_K) and an odd-row wide
    matrix through a four-limb x-pack (as the decode engine feeds it): the
    20-warp launch for very large Q6_K matrices."""
    blocks = synth.gen_blocks(14, rows, cols, seed=rows + cols)
    wd = ctx.upload(blocks)
    x = synth.gen_x(cols, seed=cols + 5)[0]
    xd = ctx.upload(x)
    xp = ctx.alloc(rt.xpack_bytes(4, cols))
    yd = ctx.alloc(4 * rows)
    yd.fill(0xFF)
    rt.xpack_f32_limbs(xd.ptr, cols, 1, 4, xp.ptr)
    rt.gemv_packed(rt.weight_desc(14, 0, rows, cols, wd.ptr), xp.ptr, 4, 1, yd.ptr)
    y = yd.download(np.float32, rows)
    ref = port.gemv(14, blocks, x, rows, cols, threads=16)[0]
    assert_close(y, ref, f"Q6_K wide {rows}x{cols}")
    assert rt.fault_status() == 0
    for b in (wd, xd, xp, yd):
        b.free()
