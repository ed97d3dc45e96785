"""Resident model placement on the B200: a pack uploaded once through VMM
(q38_pack_upload) serves every GEMV through descriptors derived from its
records, in all three layouts, and matches the FP64 oracle; the GEMV CLIs
report PASS."""
from __future__ import annotations

import io
from contextlib import redirect_stdout

import numpy as np
import pytest

from qwen382743090_b200 import cli, q38pack, runtime as rt, synth

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layout", [1, 2])
def test_uploaded_pack_gemvs_match_oracle(ctx, port, tmp_path, layout):
    path = tmp_path / f"m{layout}.q38pack"
    q38pack.synthetic_pack(path, seed=3, hidden=2048, layers=1, q5k_layout=layout, version=2)
    with q38pack.open_pack(path) as p:
        base = p.upload(ctx)
        st, off = p.plan()
        assert base % (2 << 20) == 0
        for i, t in enumerate(p.tensors):
            if t.ggml_type not in (12, 13, 14, 23):
                continue
            rows, cols = int(t.dims[1]), int(t.dims[0])
            d = p.weight_desc(i, base)
            assert d.data == base + int(off[i]) and d.layout == t.layout
            x = synth.gen_x(cols, seed=i)[0]
            xd = ctx.upload(x)
            yd = ctx.alloc(4 * rows)
            rt.gemv_f32(d, xd.ptr, yd.ptr)
            y = yd.download(np.float32, rows).astype(np.float64)
            ref = port.gemv(t.ggml_type, p.blocks(i), x, rows, cols, threads=8)[0]
            err = np.abs(y - ref)
            assert np.all((err <= 1e-4) | (err <= 1e-3 * np.abs(ref))), t.name
            xd.free()
            yd.free()
        rt.check(rt.lib().q38_free(ctx.handle, base))


def test_gemv_cli_passes(tmp_path):
    buf = io.StringIO()
    with redirect_stdout(buf):
        rc = cli.main(["q38-q5k-sm86-gemv", "--synthetic", "--seed", "7", "--rows", "6144", "--cols", "5120",
                       "--iters", "20"])
    out = buf.getvalue()
    assert rc == 0 and out.strip().endswith("q5_k_sm86: PASS"), out
    path = tmp_path / "m.q38pack"
    q38pack.synthetic_pack(path, seed=4, hidden=1024, layers=1, q5k_layout=1)
    buf = io.StringIO()
    with redirect_stdout(buf):
        rc = cli.main(["q38-gemv", "--model", str(path), "--tensor", "blk.0.ffn_gate.weight", "--iters", "10"])
    assert rc == 0 and "iq4_xs: PASS" in buf.getvalue(), buf.getvalue()
