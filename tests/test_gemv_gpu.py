"""GPU parity of the Q5_K SoA GEMV against the FP64 oracle, through the C ABI.

Tolerance: each output within 1e-3 relative OR 1e-4
absolute of the FP64 dot of the dequantised weights -- a row fails only when
both bounds are exceeded, the same rule as the reference's own check
(src/driver.cpp:6966-6975).
"""
from __future__ import annotations

import numpy as np
import pytest

from qwen382743090_b200 import runtime as rt
from qwen382743090_b200 import synth

pytestmark = pytest.mark.gpu

ABS_TOL = 1e-4
REL_TOL = 1e-3


def assert_gemv_close(got, ref, what=""):
    got = np.asarray(got, dtype=np.float64)
    err = np.abs(got - ref)
    bad = (err > ABS_TOL) & (err > REL_TOL * np.abs(ref))
    assert not bad.any(), (f"{what}: {bad.sum()} rows out of tolerance; worst row {int(np.argmax(err))} "
                           f"got {got[np.argmax(err)]} ref {ref[np.argmax(err)]}")


class SoaMatrix:
    """A Q5_K matrix uploaded in the SoA plane layout (one device buffer)."""

    def __init__(self, ctx, rows, cols, seed):
        self.rows, self.cols = rows, cols
        self.blocks = synth.gen_blocks(13, rows, cols, seed)
        self.buf, self.qh_off, self.qs_off = synth.repack_q5k_soa(self.blocks)
        self.dev = ctx.upload(self.buf)

    @property
    def planes(self):
        return self.dev.ptr, self.dev.ptr + self.qh_off, self.dev.ptr + self.qs_off

    def desc(self):
        m, h, s = self.planes
        return rt.weight_desc(13, 1, self.rows, self.cols, m, h, s)


def run_f32(ctx, mat, x):
    xd = ctx.upload(x.astype(np.float32))
    yd = ctx.alloc(4 * mat.rows)
    yd.fill(0xFF)
    m, h, s = mat.planes
    rt.q5k_soa_gemv(m, h, s, xd.ptr, yd.ptr, mat.cols, mat.rows)
    rt.synchronize()
    y = yd.download(np.float32, mat.rows)
    xd.free()
    yd.free()
    return y


SHAPES = [
    (6144, 5120),   # config 1: attn_gate
    (48, 5120),     # beta / alpha projections
    (5120, 6144),   # ssm_out
    (5120, 17408),  # ffn_down
    (1, 1024),
    (3, 1024),
    (297, 2048),    # odd rows, ragged CTA ranges
]


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_q5k_soa_f32_matches_fp64_oracle(ctx, port, rows, cols):
    mat = SoaMatrix(ctx, rows, cols, seed=rows * 31 + cols)
    x = synth.gen_x(cols, seed=cols + 5)[0]
    y = run_f32(ctx, mat, x)
    ref = port.gemv(13, mat.blocks, x, rows, cols, threads=8)[0]
    assert_gemv_close(y, ref, f"Q5_K SoA f32 {rows}x{cols}")
    assert rt.fault_status() == 0
    mat.dev.free()


def test_q5k_soa_unaligned_x(ctx, port):
    """x that is not 16-byte aligned takes the x-pack path; same tolerance."""
    rows, cols = 640, 5120
    mat = SoaMatrix(ctx, rows, cols, seed=41)
    x = synth.gen_x(cols, seed=42)[0]
    xd = ctx.alloc(4 * cols + 64)
    rt.check(rt.lib().q38_memcpy_h2d(xd.ptr + 4, x.ctypes.data, 4 * cols, None))
    yd = ctx.alloc(4 * rows)
    m, h, s = mat.planes
    rt.q5k_soa_gemv(m, h, s, xd.ptr + 4, yd.ptr, cols, rows)
    rt.synchronize()
    assert_gemv_close(yd.download(np.float32, rows), port.gemv(13, mat.blocks, x, rows, cols)[0], "unaligned x")
    for b in (mat.dev, xd, yd):
        b.free()


def test_q5k_soa_q8k_matches_oracle(ctx, port):
    rows, cols = 6144, 5120
    mat = SoaMatrix(ctx, rows, cols, seed=99)
    x = synth.gen_x(cols, seed=100)[0]
    xq = port.quantize_q8k(x)
    xqd = ctx.upload(xq)
    yd = ctx.alloc(4 * rows)
    m, h, s = mat.planes
    rt.q5k_soa_q8k_gemv(m, h, s, xqd.ptr, yd.ptr, cols, rows)
    rt.synchronize()
    y = yd.download(np.float32, rows)
    ref = port.gemv_q8k(13, mat.blocks, xq, rows, cols, threads=8)[0]
    assert_gemv_close(y, ref, "Q5_K SoA x Q8_K")
    for b in (mat.dev, xqd, yd):
        b.free()


def test_packed_x_reused_across_gemvs_and_deterministic(ctx, port):
    """One x-pack feeds several projections (qkv, z, beta, alpha share the
    normed x); results are bit-identical run to run (no atomics)."""
    cols = 5120
    mats = [SoaMatrix(ctx, r, cols, seed=r) for r in (10240, 6144, 48)]
    x = synth.gen_x(cols, seed=3)[0]
    xd = ctx.upload(x)
    xp = ctx.alloc(rt.xpack_bytes(3, cols))
    rt.xpack_f32(xd.ptr, cols, 1, xp.ptr)
    for mat in mats:
        yd = ctx.alloc(4 * mat.rows)
        rt.gemv_packed(mat.desc(), xp.ptr, 3, 1, yd.ptr)
        y1 = yd.download(np.float32, mat.rows)
        rt.gemv_packed(mat.desc(), xp.ptr, 3, 1, yd.ptr)
        y2 = yd.download(np.float32, mat.rows)
        np.testing.assert_array_equal(y1.view(np.uint32), y2.view(np.uint32))
        ref = port.gemv(13, mat.blocks, x, mat.rows, cols, threads=8)[0]
        assert_gemv_close(y1, ref, f"packed {mat.rows}x{cols}")
        yd.free()
        mat.dev.free()
    xd.free()
    xp.free()


def test_activation_edge_cases(ctx, port):
    rows, cols = 256, 2048
    mat = SoaMatrix(ctx, rows, cols, seed=5)
    # zeros -> exact zeros
    y = run_f32(ctx, mat, np.zeros(cols, dtype=np.float32))
    assert np.all(y == 0.0)
    # one large outlier per block next to tiny values (limb precision)
    x = synth.gen_x(cols, seed=6)[0] * 1e-3
    x[::256] = 1000.0
    y = run_f32(ctx, mat, x)
    assert_gemv_close(y, port.gemv(13, mat.blocks, x, rows, cols)[0], "outliers")
    # large dynamic range across blocks
    x = synth.gen_x(cols, seed=7)[0] * np.repeat(np.exp2(np.arange(-20, 12, 4)), 256)[:cols].astype(np.float32)
    y = run_f32(ctx, mat, x)
    assert_gemv_close(y, port.gemv(13, mat.blocks, x, rows, cols)[0], "dynamic range")
    # NaN in x poisons every row, as an FP32 dot would
    x = synth.gen_x(cols, seed=8)[0]
    x[300] = np.nan
    y = run_f32(ctx, mat, x)
    assert np.isnan(y).all()
    mat.dev.free()


def test_shape_errors_are_reported(ctx):
    with pytest.raises(rt.Q38Error) as e:
        rt.q5k_soa_gemv(256, 256, 256, 256, 256, 1000, 4)
    assert e.value.code == 1
    with pytest.raises(rt.Q38Error) as e:
        rt.q5k_soa_gemv(256, 256, 256, 256, 256, 768, 4)  # 3 super-blocks: not a multiple of 4
    assert e.value.code == 3


# ---- B200 fragment tiles (Q38PACK layout 2, Q5_K and Q4_K) -------------------------
TILED_SHAPES = [(6144, 5120), (48, 5120), (5120, 6144), (5120, 17408), (1, 512), (3, 1024), (297, 2048),
                (10240, 5120), (13, 1536), (151, 512)]


@pytest.mark.parametrize("ggml_type", [13, 12, 14, 23])
@pytest.mark.parametrize("rows,cols", TILED_SHAPES)
def test_tiled_f32_matches_fp64_oracle(ctx, port, ggml_type, rows, cols):
    blocks = synth.gen_blocks(ggml_type, rows, cols, seed=rows * 7 + cols + ggml_type)
    tiles = synth.repack_tiled(ggml_type, blocks, rows, cols)
    assert tiles.nbytes == rt.tiled_bytes(ggml_type, cols, rows)
    wd = ctx.upload(tiles)
    x = synth.gen_x(cols, seed=cols + 11)[0]
    xd = ctx.upload(x)
    yd = ctx.alloc(4 * rows)
    yd.fill(0xFF)
    rt.gemv_f32(rt.weight_desc(ggml_type, 2, rows, cols, wd.ptr), xd.ptr, yd.ptr)
    rt.synchronize()
    y = yd.download(np.float32, rows)
    ref = port.gemv(ggml_type, blocks, x, rows, cols, threads=8)[0]
    assert_gemv_close(y, ref, f"type {ggml_type} tiled f32 {rows}x{cols}")
    assert rt.fault_status() == 0
    for b in (wd, xd, yd):
        b.free()


def test_q5k_tiled_entry_point(ctx, port):
    """q38_q5k_tiled_gemv (the layout-2 drop-in of q38_q5k_sm86_soa_gemv_vec)."""
    rows, cols = 6144, 5120
    blocks = synth.gen_blocks(13, rows, cols, seed=5)
    wd = ctx.upload(synth.repack_q5k_tiled(blocks, rows, cols))
    x = synth.gen_x(cols, seed=6)[0]
    xd = ctx.upload(x)
    yd = ctx.alloc(4 * rows)
    rt.q5k_tiled_gemv(wd.ptr, xd.ptr, yd.ptr, cols, rows)
    assert_gemv_close(yd.download(np.float32, rows), port.gemv(13, blocks, x, rows, cols, threads=8)[0],
                      "q38_q5k_tiled_gemv")
    for b in (wd, xd, yd):
        b.free()


@pytest.mark.parametrize("ggml_type", [13, 12, 14, 23])
def test_tiled_q8k_and_determinism(ctx, port, ggml_type):
    rows, cols = 6144, 5120
    blocks = synth.gen_blocks(ggml_type, rows, cols, seed=21)
    wd = ctx.upload(synth.repack_tiled(ggml_type, blocks, rows, cols))
    x = synth.gen_x(cols, seed=22)[0]
    xq = port.quantize_q8k(x)
    xqd = ctx.upload(xq)
    yd = ctx.alloc(4 * rows)
    desc = rt.weight_desc(ggml_type, 2, rows, cols, wd.ptr)
    rt.gemv_q8k(desc, xqd.ptr, yd.ptr)
    y1 = yd.download(np.float32, rows)
    rt.gemv_q8k(desc, xqd.ptr, yd.ptr)
    y2 = yd.download(np.float32, rows)
    np.testing.assert_array_equal(y1.view(np.uint32), y2.view(np.uint32))
    ref = port.gemv_q8k(ggml_type, blocks, xq, rows, cols, threads=8)[0]
    assert_gemv_close(y1, ref, f"type {ggml_type} tiled x Q8_K")
    for b in (wd, xqd, yd):
        b.free()


@pytest.mark.parametrize("rows,cols", [(6144, 5120), (5120, 17408), (777, 4096)])
def test_tiled_xfrag_paths_agree(ctx, port, rows, cols):
    """q38_gemv_f32 on layout 2 (x-fragments built in the workspace) and an
    explicit q38_xfrag_f32 + q38_gemv_xfrag compute the same bits; the two
    x-fragment placements (shared memory up to K = 6144 at this ring size,
    L1 above) both match FP64."""
    blocks = synth.gen_blocks(13, rows, cols, seed=rows + cols)
    wd = ctx.upload(synth.repack_q5k_tiled(blocks, rows, cols))
    x = synth.gen_x(cols, seed=cols)[0]
    xd = ctx.upload(x)
    xf = ctx.alloc(rt.xfrag_bytes(cols))
    y1 = ctx.alloc(4 * rows)
    y2 = ctx.alloc(4 * rows)
    desc = rt.weight_desc(13, 2, rows, cols, wd.ptr)
    rt.gemv_f32(desc, xd.ptr, y1.ptr)
    rt.xfrag_f32(xd.ptr, cols, 1, xf.ptr)
    rt.gemv_xfrag(desc, xf.ptr, y2.ptr)
    a = y1.download(np.float32, rows)
    b = y2.download(np.float32, rows)
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    assert_gemv_close(a, port.gemv(13, blocks, x, rows, cols, threads=8)[0], f"tiled paths {rows}x{cols}")
    for buf in (wd, xd, xf, y1, y2):
        buf.free()


def test_tiled_argument_errors(ctx):
    desc = rt.weight_desc(13, 2, 64, 768, 256)  # cols not a multiple of 512
    with pytest.raises(rt.Q38Error) as e:
        rt.gemv_xfrag(desc, 256, 256)
    assert e.value.code == 1
    with pytest.raises(rt.Q38Error) as e:
        rt.gemv_xfrag(rt.weight_desc(14, 2, 64, 1024, 256), 256, 256)  # Q6_K tiles read Q6 x-fragments
    assert e.value.code == 3
    with pytest.raises(rt.Q38Error) as e:
        rt.gemv_packed(rt.weight_desc(13, 2, 64, 1024, 256), 256, 3, 1, 256)  # layout 2 takes x-fragments
    assert e.value.code == 3
    assert rt.tiled_bytes(13, 768, 8) == 0 and rt.tiled_bytes(14, 1024, 8) == 2 * 3360
    assert rt.tiled_bytes(23, 1024, 8) == 2 * 2208 and rt.tiled_bytes(23, 768, 8) == 0


def test_xfrag_bytes_match_restatement(ctx):
    """q38_xfrag_f32 writes exactly the x-fragment bytes of the NumPy
    restatement (tests/xfrag_format.py): limbs, units and group sums, over
    ordinary, tiny, subnormal, zero, mixed-range and non-finite blocks."""
    from xfrag_format import BLOCK_BYTES, pack

    rng = np.random.default_rng(21)
    nb = 12
    x = rng.standard_normal(nb * 256).astype(np.float32)
    x[256:512] *= np.float32(1e-30)           # tiny normals (slow scaling path)
    x[512:768] = np.float32(1e-40) * rng.standard_normal(256).astype(np.float32)  # subnormals
    x[768:1024] = 0.0
    x[1024:1280] *= np.float32(1e6)
    x[1280] = np.float32(3.5e4)               # one large value, the rest small
    x[1536] = np.float32(1.5)                 # unit 2^-29: exact ties at the rounding step
    x[1537:1600] = ((np.arange(63) + 0.5) * 2.0 ** -29).astype(np.float32)
    x[2048:2304] *= np.float32(1e30)
    x[2560] = np.float32(np.inf)              # poison block
    xd = ctx.upload(x)
    xf = ctx.alloc(rt.xfrag_bytes(nb * 256))
    rt.xfrag_f32(xd.ptr, nb * 256, 1, xf.ptr)
    rt.synchronize()
    got = xf.download(np.uint8, nb * BLOCK_BYTES)
    ref = pack(x)
    for b in range(nb):
        g = got[b * BLOCK_BYTES:(b + 1) * BLOCK_BYTES]
        r = ref[b * BLOCK_BYTES:(b + 1) * BLOCK_BYTES]
        if b == 10:  # non-finite: zero limbs, NaN records
            assert not g[:1024].any()
            assert np.isnan(g[1024:].view(np.float64)[::2]).all()
            continue
        np.testing.assert_array_equal(g, r, err_msg=f"super-block {b}")
    xd.free()
    xf.free()


@pytest.mark.parametrize("ggml_type,layout,rows,cols", [(13, 2, 6144, 5120), (12, 2, 777, 4096), (14, 2, 1000, 2048),
                                                       (23, 2, 640, 2048), (14, 0, 1000, 2048)])
def test_host_buffer_gemv_equals_device_path(ctx, ggml_type, layout, rows, cols):
    """q38_gemv_f32_host (x and y in page-locked host memory: layout 2 packs x
    into x-fragments while reading it and stores y from the GEMV, other
    layouts copy both) computes the same bits as q38_gemv_f32 on device
    buffers; pageable host memory is rejected before anything is launched."""
    torch = pytest.importorskip("torch")
    blocks = synth.gen_blocks(ggml_type, rows, cols, seed=rows)
    data = synth.repack_tiled(ggml_type, blocks, rows, cols) if layout == 2 else blocks
    wd = ctx.upload(data)
    desc = rt.weight_desc(ggml_type, layout, rows, cols, wd.ptr)
    x = synth.gen_x(cols, seed=cols)[0]
    xd = ctx.upload(x)
    yd = ctx.alloc(4 * rows)
    rt.gemv_f32(desc, xd.ptr, yd.ptr)
    xh = torch.from_numpy(x.copy()).pin_memory()
    yh = torch.full((rows,), float("nan"), dtype=torch.float32).pin_memory()
    for fn in (rt.gemv_f32_host, rt.gemv_f32_host_fed, rt.gemv_f32_host):  # the staging buffer is reused
        yh.fill_(float("nan"))
        fn(desc, xh.data_ptr(), yh.data_ptr())
        rt.synchronize()
        np.testing.assert_array_equal(yh.numpy().view(np.uint32), yd.download(np.float32, rows).view(np.uint32))
    pageable = np.zeros(cols, np.float32)
    with pytest.raises(rt.Q38Error):
        rt.gemv_f32_host(desc, pageable.ctypes.data, yh.data_ptr())
    for b in (wd, xd, yd):
        b.free()


@pytest.mark.parametrize("ta,rows_a,tb,rows_b,cols", [
    (13, 16384, 12, 96, 5120),    # qkv+z with beta+alpha (16 warps)
    (12, 2720, 13, 2720, 5120),   # ffn_gate with ffn_up of a TP8 shard (12 warps)
    (12, 8704, 13, 8704, 5120),   # the same at TP2 (16 warps)
    (13, 777, 12, 300, 4096),     # ragged rows
])
def test_xfrag_pair_equals_two_launches(ctx, ta, rows_a, tb, rows_b, cols):
    """q38_gemv_xfrag_pair gives each output the bits of its own
    q38_gemv_xfrag, for both type orders and both launch shapes."""
    x = synth.gen_x(cols, seed=cols + 1)[0]
    xd = ctx.upload(x)
    xf = ctx.alloc(rt.xfrag_bytes(cols))
    rt.xfrag_f32(xd.ptr, cols, 1, xf.ptr)
    mats, descs, outs = [], [], []
    for t, rows, seed in ((ta, rows_a, 1), (tb, rows_b, 2)):
        blocks = synth.gen_blocks(t, rows, cols, seed=rows + seed)
        wd = ctx.upload(synth.repack_tiled(t, blocks, rows, cols))
        mats.append(wd)
        descs.append(rt.weight_desc(t, 2, rows, cols, wd.ptr))
        outs.append((ctx.alloc(4 * rows), ctx.alloc(4 * rows)))
    for d, (single, _) in zip(descs, outs):
        rt.gemv_xfrag(d, xf.ptr, single.ptr)
    for _ in range(2):
        rt.gemv_xfrag_pair(descs[0], descs[1], xf.ptr, outs[0][1].ptr, outs[1][1].ptr)
    rt.synchronize()
    for (single, paired), rows in zip(outs, (rows_a, rows_b)):
        np.testing.assert_array_equal(paired.download(np.float32, rows).view(np.uint32),
                                      single.download(np.float32, rows).view(np.uint32))
    with pytest.raises(rt.Q38Error):  # two matrices of one type have no pair kernel
        rt.gemv_xfrag_pair(descs[0], descs[0], xf.ptr, outs[0][1].ptr, outs[0][1].ptr)
    for b in mats + [xd, xf] + [o for pair in outs for o in pair]:
        b.free()


def test_q6k_tiles_repacked_on_device_equal_host_repack(ctx, port):
    """The engine's device repack of GGUF Q6_K blocks gives the host's tile
    bytes: a one-layer model's tiled vocabulary projection, read back and
    un-tiled, is GGUF Q6_K whose GEMV matches the model's own logits."""
    cfg = dict(n_layers=1, attn_every=4, hidden=1024, ffn=2048, vocab=1000, gdn_qk_heads=4, gdn_v_heads=8,
               attn_q_heads=12, attn_kv_heads=4, ctx=64, seed=3)
    with rt.Model(**cfg) as m:
        d, raw = m.download("output")
        assert (d.ggml_type, d.layout, d.rows, d.cols) == (14, 2, 1000, 1024)
        blocks = synth.untile(14, raw, d.rows, d.cols)
        np.testing.assert_array_equal(synth.repack_tiled(14, blocks, d.rows, d.cols), raw)
        x = synth.gen_x(1024, seed=4)[0]
        xd, yd = ctx.upload(x), ctx.alloc(4 * 1000)
        rt.gemv_f32(d, xd.ptr, yd.ptr)
        assert_gemv_close(yd.download(np.float32, 1000), port.gemv(14, blocks, x, 1000, 1024)[0], "engine lm_head tiles")
        for b in (xd, yd):
            b.free()


def test_host_buffer_gemvs_chain_through_host_memory(ctx):
    """One host-buffer GEMV's y as the next one's x, queued back to back on
    one stream without a synchronisation: q38_gemv_f32_host reads x only after
    the earlier GEMV has stored it, so the chain equals the device path."""
    torch = pytest.importorskip("torch")
    n = 5120
    ws = [ctx.upload(synth.repack_tiled(13, synth.gen_blocks(13, n, n, seed=70 + i), n, n)) for i in range(3)]
    descs = [rt.weight_desc(13, 2, n, n, w.ptr) for w in ws]
    x = synth.gen_x(n, seed=71)[0]
    xd, ya, yb = ctx.upload(x), ctx.alloc(4 * n), ctx.alloc(4 * n)
    rt.gemv_f32(descs[0], xd.ptr, ya.ptr)
    rt.gemv_f32(descs[1], ya.ptr, yb.ptr)
    rt.gemv_f32(descs[2], yb.ptr, ya.ptr)
    want = ya.download(np.float32, n)
    h = [torch.from_numpy(x.copy()).pin_memory()] + [torch.empty(n, dtype=torch.float32).pin_memory() for _ in range(3)]
    for i in range(3):
        rt.gemv_f32_host(descs[i], h[i].data_ptr(), h[i + 1].data_ptr())
    rt.synchronize()
    np.testing.assert_array_equal(h[3].numpy().view(np.uint32), want.view(np.uint32))
    for b in (*ws, xd, ya, yb):
        b.free()
