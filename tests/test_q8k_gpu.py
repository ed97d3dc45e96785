"""Q8_K activations made on the device (q38_quantize_q8k, q38_rmsnorm_q8k)
against the reference's CPU quantiser: the golden blocks made by the
reference's own quantize_q8_k_cpu (tests/golden/kquant_golden.npz) bit for
bit, the oracle port on ties, zero and negative-maximum blocks, and the fused
RMSNorm's blocks equal to the CPU quantisation of its own f32 output."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from qwen382743090_b200 import runtime as rt

pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).parent / "golden" / "kquant_golden.npz")


def _quantize(ctx, x):
    xd = ctx.upload(x.astype(np.float32))
    out = ctx.alloc(292 * (x.size // 256))
    rt.quantize_q8k(xd.ptr, x.size, out.ptr)
    rt.synchronize()
    got = out.download(np.uint8, 292 * (x.size // 256))
    xd.free()
    out.free()
    return got


def test_quantize_matches_reference_golden_blocks(ctx):
    got = _quantize(ctx, GOLDEN["q8k_x"])
    np.testing.assert_array_equal(got, GOLDEN["q8k_blocks"])


def test_quantize_edge_blocks_match_oracle(ctx, port):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(256 * 6).astype(np.float32)
    x[0:256] = 0.0                                      # all zero: d = 0
    x[256 + 17] = -9.0                                  # negative maximum
    x[512 + 3], x[512 + 200] = 7.5, -7.5                # tie: the first one wins
    x[768:1024] = np.round(x[768:1024] * 4) / 4         # many exact halves after scaling
    x[1024:1280] *= np.float32(1e-30)                   # tiny values
    x[1280:1536] = 1.0                                  # constant block
    np.testing.assert_array_equal(_quantize(ctx, x), port.quantize_q8k(x))


def test_rmsnorm_q8k_quantises_its_own_output(ctx, port):
    rng = np.random.default_rng(11)
    n = 5120
    x = (rng.standard_normal(n) * 3.0).astype(np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    xd, wd = ctx.upload(x), ctx.upload(w)
    yd, out = ctx.alloc(4 * n), ctx.alloc(292 * (n // 256))
    for _ in range(2):
        rt.rmsnorm_q8k(xd.ptr, wd.ptr, n, 1e-6, out.ptr, y=yd.ptr)
    rt.synchronize()
    y = yd.download(np.float32, n)
    np.testing.assert_array_equal(out.download(np.uint8, 292 * (n // 256)), port.quantize_q8k(y))
    ref = port.rmsnorm(x, w, 1e-6)
    assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()
    with pytest.raises(rt.Q38Error):
        rt.rmsnorm_q8k(xd.ptr, wd.ptr, n + 128, 1e-6, out.ptr)
    for b in (xd, wd, yd, out):
        b.free()


def test_q8_1_blocks_bit_exact_to_the_reference(ctx):
    """q38_quantize_q8_1 against the reference's own quantize_q8_1_cpu blocks
    (zero block, negative maximum, ties, tiny values)."""
    x = GOLDEN["q81_x"].astype(np.float32)
    xd, out = ctx.upload(x), ctx.alloc(36 * (x.size // 32))
    rt.quantize_q8_1(xd.ptr, x.size, out.ptr)
    rt.synchronize()
    np.testing.assert_array_equal(out.download(np.uint8, 36 * (x.size // 32)), GOLDEN["q81_blocks"])
    xd.free()
    out.free()


@pytest.mark.parametrize("rows,cols", [(6144, 5120), (17408, 5120), (5120, 17408), (37, 256)])
def test_iq4xs_q8_1_gemv_matches_fp64_of_dequantised_operands(ctx, port, rows, cols):
    """The IQ4_XS x Q8_1 GEMV against the FP64 dot of the dequantised weights
    with the dequantised Q8_1 values (the reference's check, src/driver.cpp:
    2835-2875), with the GEMV tolerance."""
    from qwen382743090_b200 import synth

    w = synth.gen_blocks(23, rows, cols, seed=rows + cols)
    x = synth.gen_x(cols, seed=cols + 1)[0]
    wd, xd = ctx.upload(w), ctx.upload(x)
    xq, y = ctx.alloc(36 * (cols // 32)), ctx.alloc(4 * rows)
    rt.quantize_q8_1(xd.ptr, cols, xq.ptr)
    rt.iq4xs_q8_1_gemv(wd.ptr, xq.ptr, y.ptr, cols, rows)
    rt.synchronize()
    blocks = xq.download(np.uint8, 36 * (cols // 32))
    np.testing.assert_array_equal(blocks, port.quantize_q8_1(x))
    ref = port.gemv(23, w, port.dequant_q8_1(blocks), rows, cols, threads=16)[0]
    err = np.abs(y.download(np.float32, rows).astype(np.float64) - ref)
    assert not ((err > 1e-4) & (err > 1e-3 * np.abs(ref))).any(), err.max()
    assert rt.fault_status() == 0
    for b in (wd, xd, xq, y):
        b.free()
