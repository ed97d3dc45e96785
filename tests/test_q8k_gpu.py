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
