"""Generate tests/golden/kquant_golden.npz from the reference's own CPU code.

    make -C oracle && python tests/golden/make_golden.py

The vectors are computed by oracle/_ref/libq38ref.so, i.e. the reference's
src/quant.cpp compiled unmodified from the reference tree, so the committed
fixture pins the C restatement (oracle/q38_oracle.c) and the GPU kernels to
the reference's behaviour even where the reference tree is absent.

Contents (all inputs are seeded; seeds are stored in the file):
  q4k/q5k/q6k/iq4xs_blocks, *_deq   8 synthetic + 4 raw-random blocks per type
                                     and their dequantised floats
  q5k_soa_rec, q5k_soa_deq           the same Q5_K blocks repacked to the
                                     180-B SoA record and dequantised
  q5k_test_block, q5k_test_soa       the one golden block of the reference's
                                     tests/test_q38pack.py:70-79 and its repack
  q8k_x, q8k_blocks                  Q8_K quantisation of seeded vectors with
                                     edge cases (zeros, negative max, ties)
  q81_x, q81_blocks                  Q8_1 quantisation of the same vector
  gemv_<type>_w/_x/_y                small GEMVs (rows 24, cols 512), FP64 dot
  gemv_q5k_q8k_y                     Q5_K x Q8_K GEMV (FP64 of dequantised operands)
  fp16_to_fp32                       all 65536 half values as float32 bits
  fp32_to_fp16_in/_out               special and random floats -> half bits
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from qwen382743090_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "kquant_golden.npz"
TYPES = {"q4k": 12, "q5k": 13, "q6k": 14, "iq4xs": 23}
SEED = 20261201


def q5k_test_block() -> np.ndarray:
    """The reference test's block: dm = fp16(0.5), fp16(0.25); scales[i] =
    (17i+3)&255; qh[i] = (11i+5)&255; qs[i] = (7i+9)&255."""
    dm = np.array([0.5, 0.25], dtype=np.float16).view(np.uint8)
    scales = np.array([(i * 17 + 3) & 0xFF for i in range(12)], dtype=np.uint8)
    qh = np.array([(i * 11 + 5) & 0xFF for i in range(32)], dtype=np.uint8)
    qs = np.array([(i * 7 + 9) & 0xFF for i in range(128)], dtype=np.uint8)
    return np.concatenate([dm, scales, qh, qs])


def main() -> None:
    ref = oracle.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libq38ref.so is missing: run `make -C oracle` with the reference tree present")
    rng = np.random.default_rng(SEED)
    out: dict[str, np.ndarray] = {"seed": np.array([SEED])}

    for name, t in TYPES.items():
        bb = oracle.BLOCK_BYTES[t]
        syn = synth.gen_blocks(t, 8, 256, SEED + t)
        raw = rng.integers(0, 256, size=4 * bb, dtype=np.uint8)
        # keep the fp16 scale fields finite in the raw blocks
        raw = raw.reshape(4, bb)
        if t == 14:
            raw[:, 208:210] = np.array([0x20, 0x1C], dtype=np.uint8)
        else:
            raw[:, 0:2] = np.array([0x20, 0x1C], dtype=np.uint8)
            if t in (12, 13):
                raw[:, 2:4] = np.array([0x80, 0x1A], dtype=np.uint8)
        blocks = np.concatenate([syn, raw.reshape(-1)])
        out[f"{name}_blocks"] = blocks
        out[f"{name}_deq"] = ref.dequant(t, blocks)

    q5 = out["q5k_blocks"].reshape(-1, 176)
    recs = np.stack([ref.repack_q5k_soa_block(b) for b in q5])
    out["q5k_soa_rec"] = recs.reshape(-1)
    out["q5k_soa_deq"] = ref.dequant(1013, recs.reshape(-1))

    tb = q5k_test_block()
    out["q5k_test_block"] = tb
    out["q5k_test_soa"] = ref.repack_q5k_soa_block(tb)
    out["q5k_test_deq"] = ref.dequant(13, tb)

    x = rng.standard_normal(256 * 6).astype(np.float32)
    x[256:512] = 0.0                                   # all-zero block
    x[512:768] *= 0.01
    x[600] = -5.0                                      # negative maximum
    x[768:1024] = np.round(x[768:1024] * 4) / 4        # many exact ties
    x[1024 + 7] = 3.0
    x[1024 + 9] = -3.0                                 # |max| tie: first one wins
    out["q8k_x"] = x
    out["q8k_blocks"] = ref.quantize_q8k(x)

    # Q8_1 (the rejected IQ4_XS x Q8_1 path): the same edge cases in 32-value blocks
    out["q81_x"] = x
    out["q81_blocks"] = ref.quantize_q8_1(x)

    rows, cols = 24, 512
    xg = synth.gen_x(cols, SEED + 1)
    out["gemv_x"] = xg
    for name, t in TYPES.items():
        w = synth.gen_blocks(t, rows, cols, SEED + 100 + t)
        out[f"gemv_{name}_w"] = w
        out[f"gemv_{name}_y"] = ref.gemv(t, w, xg, rows, cols)[0]
    xq = ref.quantize_q8k(xg)
    out["gemv_xq8"] = xq
    out["gemv_q5k_q8k_y"] = ref.gemv_q8k(13, out["gemv_q5k_w"], xq, rows, cols)[0]

    halves = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f = np.array([ref.fp16_to_fp32(int(h)) for h in halves], dtype=np.float32)
    out["fp16_to_fp32"] = f.view(np.uint32)
    specials = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65520.0, 65519.99, 1e-8, 5.96e-8, 2.98e-8, 2.99e-8,
                         6.1e-5, 6.097e-5, np.inf, -np.inf, np.nan, 3.14159, 1.0009765625, 1.00048828125,
                         1.00146484375], dtype=np.float32)
    rnd = (rng.standard_normal(2000) * np.exp2(rng.integers(-30, 20, 2000))).astype(np.float32)
    fin = np.concatenate([specials, rnd])
    out["fp32_to_fp16_in"] = fin
    out["fp32_to_fp16_out"] = np.array([ref.fp32_to_fp16(float(v)) for v in fin], dtype=np.uint16)

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
