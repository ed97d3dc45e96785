"""Pin the CPU oracle (oracle/q38_oracle.c) before trusting it.

1. Against the committed golden vectors (tests/golden/kquant_golden.npz, made
   from the reference's own src/quant.cpp by tests/golden/make_golden.py).
2. Against the reference's test fixture: the one Q5_K block of
   tests/test_q38pack.py:70-79 and its expected SoA META/QH/QS (:128-158).
3. Against the reference's compiled quant.cpp itself (oracle/_ref), on fresh
   seeded blocks, when that library was built here.
Dequantised weights and Q8_K bytes must match bit for bit; the FP64 GEMV
reference must match exactly (same summation order).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle
from qwen382743090_b200 import synth

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "kquant_golden.npz")
TYPES = {"q4k": 12, "q5k": 13, "q6k": 14, "iq4xs": 23}


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_matches_golden(port, name):
    got = port.dequant(TYPES[name], GOLD[f"{name}_blocks"])
    np.testing.assert_array_equal(bits(got), bits(GOLD[f"{name}_deq"]))


def test_q5k_soa_repack_and_dequant_match_golden(port):
    q5 = GOLD["q5k_blocks"].reshape(-1, 176)
    recs = np.stack([port.repack_q5k_soa_block(b) for b in q5]).reshape(-1)
    np.testing.assert_array_equal(recs, GOLD["q5k_soa_rec"])
    np.testing.assert_array_equal(bits(port.dequant(1013, recs)), bits(GOLD["q5k_soa_deq"]))
    # lossless: SoA dequant == standard dequant, bit for bit
    np.testing.assert_array_equal(bits(GOLD["q5k_soa_deq"]), bits(GOLD["q5k_deq"]))


def test_reference_test_block(port):
    """tests/test_q38pack.py:128-158: META = d,dmin + unpacked (scale, min)
    pairs; QH and QS copied byte for byte."""
    blk = GOLD["q5k_test_block"]
    soa = port.repack_q5k_soa_block(blk)
    np.testing.assert_array_equal(soa, GOLD["q5k_test_soa"])
    assert bytes(soa[:4]) == bytes(blk[:4])
    sc, mn = synth.unpack_scale_min_k4(blk[4:16].reshape(1, 12))
    expect = bytes(blk[:4]) + bytes(np.stack([sc[0], mn[0]], axis=1).reshape(-1))
    assert bytes(soa[:20]) == expect
    assert bytes(soa[20:52]) == bytes(blk[16:48])
    assert bytes(soa[52:180]) == bytes(blk[48:176])
    np.testing.assert_array_equal(bits(port.dequant(13, blk)), bits(GOLD["q5k_test_deq"]))
    # the same block through the package's vectorised repack (converter path)
    buf, qh_off, qs_off = synth.repack_q5k_soa(blk)
    assert bytes(buf[:20]) == expect
    assert bytes(buf[qh_off:qh_off + 32]) == bytes(blk[16:48])
    assert bytes(buf[qs_off:qs_off + 128]) == bytes(blk[48:176])


def test_q8k_quantize_matches_golden(port):
    np.testing.assert_array_equal(port.quantize_q8k(GOLD["q8k_x"]), GOLD["q8k_blocks"])


def test_q8_1_quantize_matches_golden(port):
    np.testing.assert_array_equal(port.quantize_q8_1(GOLD["q81_x"]), GOLD["q81_blocks"])
    with pytest.raises(ValueError):
        port.quantize_q8_1(np.ones(40, dtype=np.float32))


def test_q8k_rejects_ragged(port):
    with pytest.raises(ValueError):
        port.quantize_q8k(np.ones(300, dtype=np.float32))


@pytest.mark.parametrize("name", list(TYPES))
def test_gemv_fp64_matches_golden(port, name):
    y = port.gemv(TYPES[name], GOLD[f"gemv_{name}_w"], GOLD["gemv_x"], 24, 512)[0]
    np.testing.assert_array_equal(y, GOLD[f"gemv_{name}_y"])


def test_gemv_q8k_matches_golden(port):
    y = port.gemv_q8k(13, GOLD["gemv_q5k_w"], GOLD["gemv_xq8"], 24, 512)[0]
    np.testing.assert_array_equal(y, GOLD["gemv_q5k_q8k_y"])


def test_fp16_conversions_match_golden(port):
    f = np.array([port.fp16_to_fp32(h) for h in range(65536)], dtype=np.float32)
    np.testing.assert_array_equal(bits(f), GOLD["fp16_to_fp32"])
    h = np.array([port.fp32_to_fp16(float(v)) for v in GOLD["fp32_to_fp16_in"]], dtype=np.uint16)
    np.testing.assert_array_equal(h, GOLD["fp32_to_fp16_out"])


def test_soa_gemv_equals_standard_gemv(port):
    rows, cols = 16, 1024
    w = synth.gen_blocks(13, rows, cols, 7)
    x = synth.gen_x(cols, 8)
    buf, qh, qs = synth.repack_q5k_soa(w)
    n = rows * cols // 256
    y_soa = port.gemv_q5k_soa(buf[: n * 20], buf[qh: qh + n * 32], buf[qs: qs + n * 128], x, rows, cols)
    y_std = port.gemv(13, w, x, rows, cols)
    np.testing.assert_array_equal(y_soa, y_std)


def test_threaded_gemv_equals_single_thread(port):
    rows, cols = 37, 768
    w = synth.gen_blocks(14, rows, cols, 11)
    x = synth.gen_x(cols, 12)
    np.testing.assert_array_equal(port.gemv(14, w, x, rows, cols, threads=4), port.gemv(14, w, x, rows, cols))


# ---- against the reference's compiled quant.cpp (only where it was built) ----
ref = oracle.ref()
needs_ref = pytest.mark.skipif(ref is None, reason="oracle/_ref not built (reference tree absent)")


@needs_ref
@pytest.mark.parametrize("t", [12, 13, 14, 23])
def test_dequant_bit_exact_vs_reference(port, t):
    blocks = synth.gen_blocks(t, 64, 1024, 1000 + t)
    np.testing.assert_array_equal(bits(port.dequant(t, blocks)), bits(ref.dequant(t, blocks)))
    raw = np.random.default_rng(t).integers(0, 256, size=64 * oracle.BLOCK_BYTES[t], dtype=np.uint8)
    a, b = port.dequant(t, raw), ref.dequant(t, raw)
    np.testing.assert_array_equal(bits(a), bits(b))


@needs_ref
def test_q5k_soa_bit_exact_vs_reference(port):
    blocks = synth.gen_blocks(13, 32, 1024, 77).reshape(-1, 176)
    for b in blocks:
        r1, r2 = port.repack_q5k_soa_block(b), ref.repack_q5k_soa_block(b)
        np.testing.assert_array_equal(r1, r2)
        np.testing.assert_array_equal(bits(port.dequant(1013, r1)), bits(ref.dequant(1013, r2)))


@needs_ref
def test_q8k_bit_exact_vs_reference(port):
    rng = np.random.default_rng(5)
    for scale in (1e-3, 1.0, 1e3):
        x = (rng.standard_normal(256 * 8) * scale).astype(np.float32)
        np.testing.assert_array_equal(port.quantize_q8k(x), ref.quantize_q8k(x))


@needs_ref
def test_q8_1_bit_exact_vs_reference(port):
    rng = np.random.default_rng(7)
    for scale in (1e-4, 1.0, 1e4):
        x = (rng.standard_normal(32 * 64) * scale).astype(np.float32)
        x[:32] = 0.0
        np.testing.assert_array_equal(port.quantize_q8_1(x), ref.quantize_q8_1(x))


@needs_ref
def test_fp32_to_fp16_vs_reference(port):
    rng = np.random.default_rng(6)
    v = (rng.standard_normal(5000) * np.exp2(rng.integers(-40, 25, 5000))).astype(np.float32)
    for f in v:
        assert port.fp32_to_fp16(float(f)) == ref.fp32_to_fp16(float(f))


@needs_ref
@pytest.mark.parametrize("t", [12, 13, 14, 23])
def test_gemv_exact_vs_reference(port, t):
    rows, cols = 40, 1536
    w = synth.gen_blocks(t, rows, cols, 300 + t)
    x = synth.gen_x(cols, 301, batch=2)
    np.testing.assert_array_equal(port.gemv(t, w, x, rows, cols), ref.gemv(t, w, x, rows, cols))
