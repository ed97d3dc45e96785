"""The device reference rows (q38_check_rows) against the golden vectors made
by the reference's own quant.cpp (tests/golden/kquant_golden.npz): the
dequantised weights bit for bit, the FP64 dots up to summation order.  These
are what the C++ facade's smoke entries check the fast GEMVs against."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from qwen382743090_b200 import runtime as rt

pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).parent / "golden" / "kquant_golden.npz")
TYPES = {"q4k": 12, "q5k": 13, "q6k": 14, "iq4xs": 23}


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_matches_reference_bits(ctx, name):
    blocks = GOLDEN[f"{name}_blocks"]
    ref = GOLDEN[f"{name}_deq"]
    nblk = ref.size // 256
    wd = ctx.upload(blocks)
    out = ctx.alloc(4 * ref.size)
    rt.check_rows(rt.weight_desc(TYPES[name], 0, nblk, 256, wd.ptr), nblk, deq=out.ptr)
    rt.synchronize()
    np.testing.assert_array_equal(out.download(np.float32, ref.size).view(np.uint32), ref.view(np.uint32))
    wd.free()
    out.free()


def test_soa_dequant_matches_reference_bits(ctx):
    rec = GOLDEN["q5k_soa_rec"].reshape(-1, 180)
    ref = GOLDEN["q5k_soa_deq"]
    nblk = rec.shape[0]
    planes = np.concatenate([rec[:, :20].ravel(), rec[:, 20:52].ravel(), rec[:, 52:].ravel()])
    wd = ctx.upload(planes)
    out = ctx.alloc(4 * ref.size)
    desc = rt.weight_desc(13, 1, nblk, 256, wd.ptr, wd.ptr + 20 * nblk, wd.ptr + 52 * nblk)
    rt.check_rows(desc, nblk, deq=out.ptr)
    rt.synchronize()
    np.testing.assert_array_equal(out.download(np.float32, ref.size).view(np.uint32), ref.view(np.uint32))
    wd.free()
    out.free()


@pytest.mark.parametrize("name", list(TYPES))
def test_fp64_rows_match_reference(ctx, name):
    w = GOLDEN[f"gemv_{name}_w"]
    x = GOLDEN["gemv_x"][0]
    ref = GOLDEN[f"gemv_{name}_y"]
    rows, cols = ref.size, x.size
    wd = ctx.upload(w)
    xd = ctx.upload(x)
    yd = ctx.alloc(8 * rows)
    rt.check_rows(rt.weight_desc(TYPES[name], 0, rows, cols, wd.ptr), rows, x=xd.ptr, y64=yd.ptr)
    rt.synchronize()
    got = yd.download(np.float64, rows)
    np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12 * np.abs(ref).max())
    for b in (wd, xd, yd):
        b.free()


def test_check_rows_rejects_bad_arguments(ctx):
    w = ctx.alloc(176 * 4)
    with pytest.raises(rt.Q38Error):  # no output requested
        rt.check_rows(rt.weight_desc(13, 0, 4, 256, w.ptr), 4)
    with pytest.raises(rt.Q38Error):  # more rows than the matrix
        rt.check_rows(rt.weight_desc(13, 0, 4, 256, w.ptr), 5, deq=w.ptr)
    with pytest.raises(rt.Q38Error):  # layout 2 is not covered
        rt.check_rows(rt.weight_desc(13, 2, 8, 512, w.ptr), 1, deq=w.ptr)
    w.free()
