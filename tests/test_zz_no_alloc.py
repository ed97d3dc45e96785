"""q38_q5k_sm86_soa_gemv_vec_noalloc: the Q5_K SoA GEMV whose x-pack lives in a
fixed device array of the library instead of a cudaMalloc'd workspace.

It must give exactly the results of q38_q5k_sm86_soa_gemv_vec (same pack and
GEMV kernels), on back-to-back calls that reuse the one scratch, without the
device's free memory moving, and reject inputs wider than the scratch.  This
file sorts last so the GPU tests also run after every other test has used the
workspace entry points in the same process.
"""
from __future__ import annotations

import numpy as np
import pytest

from qwen382743090_b200 import runtime as rt
from qwen382743090_b200 import synth

NOALLOC_MAX_COLS = 32768


def _soa(ctx, rows, cols, seed):
    blocks = synth.gen_blocks(13, rows, cols, seed)
    buf, qh_off, qs_off = synth.repack_q5k_soa(blocks)
    dev = ctx.upload(buf)
    return blocks, dev, (dev.ptr, dev.ptr + qh_off, dev.ptr + qs_off)


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_on_back_to_back_calls(ctx, port):
    # widest first, then narrower: the second matrix's x-pack must not read
    # anything the first one left in the scratch
    cases = [(5120, 17408, 1), (6144, 5120, 2)]
    for rows, cols, seed in cases:
        blocks, wdev, planes = _soa(ctx, rows, cols, seed=rows + seed)
        xs = [synth.gen_x(cols, seed=cols + 100 * k + seed)[0] for k in range(2)]
        xd = [ctx.upload(x) for x in xs]
        y_ws = [ctx.alloc(4 * rows) for _ in xs]
        y_na = [ctx.alloc(4 * rows) for _ in xs]
        for b in y_na:
            b.fill(0xFF)
        for k in range(2):
            rt.q5k_soa_gemv(*planes, xd[k].ptr, y_ws[k].ptr, cols, rows)
        # two no-alloc calls in a row on one stream, no synchronisation between them
        rt.q5k_soa_gemv_noalloc(*planes, xd[0].ptr, y_na[0].ptr, cols, rows)
        rt.q5k_soa_gemv_noalloc(*planes, xd[1].ptr, y_na[1].ptr, cols, rows)
        rt.synchronize()
        assert rt.fault_status() == 0
        for k in range(2):
            a = y_ws[k].download(np.float32, rows)
            b = y_na[k].download(np.float32, rows)
            np.testing.assert_array_equal(b.view(np.uint32), a.view(np.uint32))
        ref = port.gemv(13, blocks, xs[1], rows, cols, threads=8)[0]
        err = np.abs(y_na[1].download(np.float32, rows).astype(np.float64) - ref)
        assert not ((err > 1e-4) & (err > 1e-3 * np.abs(ref))).any()
        for buf in (wdev, *xd, *y_ws, *y_na):
            buf.free()


@pytest.mark.gpu
def test_noalloc_calls_leave_device_memory_unchanged(ctx):
    torch = pytest.importorskip("torch")
    rows, cols = 256, NOALLOC_MAX_COLS
    _, wdev, planes = _soa(ctx, rows, cols, seed=77)
    xd = ctx.upload(synth.gen_x(cols, seed=78)[0])
    yd = ctx.alloc(4 * rows)
    torch.cuda.mem_get_info(0)  # torch's own CUDA start-up happens before the measurement
    rt.q5k_soa_gemv_noalloc(*planes, xd.ptr, yd.ptr, cols, rows)  # loads the kernels
    rt.synchronize()
    free0 = torch.cuda.mem_get_info(0)[0]
    for c in (1024, 5120, cols):
        rt.q5k_soa_gemv_noalloc(*planes, xd.ptr, yd.ptr, c, rows)
    rt.synchronize()
    assert torch.cuda.mem_get_info(0)[0] == free0
    assert rt.fault_status() == 0
    for buf in (wdev, xd, yd):
        buf.free()


_FRESH_PROCESS = r"""
import json, sys
import torch
from qwen382743090_b200 import runtime as rt, synth
rows, cols = 256, int(sys.argv[1])
ctx = rt.Context(0)
blocks = synth.gen_blocks(13, rows, cols, 77)
buf, qh, qs = synth.repack_q5k_soa(blocks)
w, x, y = ctx.upload(buf), ctx.upload(synth.gen_x(cols, 78)[0]), ctx.alloc(4 * rows)
planes = (w.ptr, w.ptr + qh, w.ptr + qs)
torch.cuda.mem_get_info(0)
out = {"scratch_start": rt.scratch_bytes(0)}
rt.q5k_soa_gemv_noalloc(*planes, x.ptr, y.ptr, cols, rows)
rt.synchronize()
out["free_after_first"] = torch.cuda.mem_get_info(0)[0]
for c in (1024, 5120, cols):
    rt.q5k_soa_gemv_noalloc(*planes, x.ptr, y.ptr, c, rows)
rt.synchronize()
out["free_after_noalloc"] = torch.cuda.mem_get_info(0)[0]
out["scratch_after_noalloc"] = rt.scratch_bytes(0)
rt.q5k_soa_gemv(*planes, x.ptr, y.ptr, cols, rows)  # control: the workspace entry point
rt.synchronize()
out["scratch_after_workspace_call"] = rt.scratch_bytes(0)
out["fault"] = rt.fault_status()
print(json.dumps(out))
"""


@pytest.mark.gpu
def test_noalloc_allocates_nothing_in_a_fresh_process():
    """In a process where no call has grown the library's workspace yet, the
    no-alloc calls leave its lazily grown scratch at 0 bytes and the device's
    free memory unchanged, while one call of the workspace entry point (the
    control) does grow the scratch: a regression of the no-alloc entry to the
    workspace would fail here."""
    import json
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    res = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, str(NOALLOC_MAX_COLS)], cwd=root,
                         capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    out = json.loads(res.stdout.strip().splitlines()[-1])
    assert out["fault"] == 0
    assert out["scratch_start"] == 0
    assert out["scratch_after_noalloc"] == 0
    assert out["free_after_noalloc"] == out["free_after_first"]
    assert out["scratch_after_workspace_call"] > 0


def test_noalloc_rejects_cols_beyond_the_scratch():
    """Checked on the host before any device call, so this runs without a GPU."""
    cols = NOALLOC_MAX_COLS + 1024
    with pytest.raises(rt.Q38Error) as e:
        rt.q5k_soa_gemv_noalloc(256, 512, 768, 1024, 1280, cols, 4)
    assert e.value.code == 1
    assert "exceeds the fixed x-pack scratch" in str(e.value)
