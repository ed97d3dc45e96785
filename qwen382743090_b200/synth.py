"""Seeded synthetic K-quant tensors and activations.

The reference benchmarks only real model weights (not available here); the
synthetic generators below follow the value distributions of the benchmark
configurations:

* d, dmin   fp16(|N(0,1)| * 2^-8)
* Q4_K/Q5_K scales[12]: eight 6-bit scales and eight 6-bit mins, each uniform
  0..63, packed with the inverse of get_scale_min_k4 (src/quant.cpp:89-97)
* qh, qs, ql bytes uniform 0..255
* Q6_K int8 scales uniform -128..127, IQ4_XS scales_h/scales_l uniform
* x   f32 N(0,1)

Every array is a pure function of (seed, shape) through numpy's PCG64, so the
same seed always gives the same bytes.
"""
from __future__ import annotations

import numpy as np

QK = 256
BLOCK_BYTES = {12: 144, 13: 176, 14: 210, 23: 136}


def _rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(np.random.PCG64(int(seed) & ((1 << 63) - 1)))


def _half_scale(rng: np.random.Generator, n: int) -> np.ndarray:
    return (np.abs(rng.standard_normal(n)) * 2.0 ** -8).astype(np.float16).view(np.uint16)


def pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Inverse of get_scale_min_k4: (n, 8) 6-bit scales and mins -> (n, 12) bytes."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.zeros((sc.shape[0], 12), dtype=np.uint8)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return out


def unpack_scale_min_k4(s12: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """get_scale_min_k4 for all 8 groups at once: (n, 12) -> (n, 8), (n, 8)."""
    s = s12.astype(np.uint8)
    sc = np.empty((s.shape[0], 8), dtype=np.uint8)
    mn = np.empty((s.shape[0], 8), dtype=np.uint8)
    sc[:, 0:4] = s[:, 0:4] & 63
    mn[:, 0:4] = s[:, 4:8] & 63
    sc[:, 4:8] = (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:8] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return sc, mn


def gen_blocks(ggml_type: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """Row-major GGUF blocks of `ggml_type` for a [cols, rows] tensor (uint8, flat)."""
    if cols % QK:
        raise ValueError("cols must be a multiple of 256")
    n = rows * (cols // QK)
    rng = _rng(seed)
    if ggml_type in (12, 13):
        bb = BLOCK_BYTES[ggml_type]
        out = np.empty((n, bb), dtype=np.uint8)
        dm = np.empty((n, 2), dtype=np.uint16)
        dm[:, 0] = _half_scale(rng, n)
        dm[:, 1] = _half_scale(rng, n)
        out[:, 0:4] = dm.view(np.uint8).reshape(n, 4)
        sc = rng.integers(0, 64, size=(n, 8), dtype=np.uint8)
        mn = rng.integers(0, 64, size=(n, 8), dtype=np.uint8)
        out[:, 4:16] = pack_scale_min_k4(sc, mn)
        out[:, 16:] = rng.integers(0, 256, size=(n, bb - 16), dtype=np.uint8)
        return out.reshape(-1)
    if ggml_type == 14:
        out = np.empty((n, 210), dtype=np.uint8)
        out[:, 0:192] = rng.integers(0, 256, size=(n, 192), dtype=np.uint8)
        out[:, 192:208] = rng.integers(-128, 128, size=(n, 16), dtype=np.int16).astype(np.int8).view(np.uint8)
        out[:, 208:210] = _half_scale(rng, n).view(np.uint8).reshape(n, 2)
        return out.reshape(-1)
    if ggml_type == 23:
        out = np.empty((n, 136), dtype=np.uint8)
        out[:, 0:2] = _half_scale(rng, n).view(np.uint8).reshape(n, 2)
        out[:, 2:] = rng.integers(0, 256, size=(n, 134), dtype=np.uint8)
        return out.reshape(-1)
    raise ValueError(f"unsupported ggml type {ggml_type}")


def repack_q5k_soa(blocks: np.ndarray, align: int = 128) -> tuple[np.ndarray, int, int]:
    """Lossless Q5_K -> SoA planes in one buffer: META20 | QH32 | QS128.

    Same transform as repack_q5_k_sm86_block (src/quant.cpp:401-423) applied to
    every block, laid out as the converter stores it
    (tools/gguf_to_q38pack.py:240-299): each plane starts `align`-aligned.
    Returns (buffer, qh_offset, qs_offset).
    """
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, 176)
    n = b.shape[0]
    meta = np.empty((n, 20), dtype=np.uint8)
    meta[:, 0:4] = b[:, 0:4]
    sc, mn = unpack_scale_min_k4(b[:, 4:16])
    meta[:, 4:20:2] = sc
    meta[:, 5:20:2] = mn
    qh_off = (n * 20 + align - 1) // align * align
    qs_off = (qh_off + n * 32 + align - 1) // align * align
    buf = np.zeros(qs_off + n * 128, dtype=np.uint8)
    buf[: n * 20] = meta.reshape(-1)
    buf[qh_off: qh_off + n * 32] = b[:, 16:48].reshape(-1)
    buf[qs_off:] = b[:, 48:176].reshape(-1)
    return buf, qh_off, qs_off


def q5k_soa_records(blocks: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-block META20 / QH32 / QS128 arrays of Q5_K blocks (n, 176) -> (n, 20), (n, 32), (n, 128)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, 176)
    meta = np.empty((b.shape[0], 20), dtype=np.uint8)
    meta[:, 0:4] = b[:, 0:4]
    sc, mn = unpack_scale_min_k4(b[:, 4:16])
    meta[:, 4:20:2] = sc
    meta[:, 5:20:2] = mn
    return meta, b[:, 16:48], b[:, 48:176]


TILE_ROWS = 4
TILE_BYTES = TILE_ROWS * 4 * 180  # 2880


def repack_q5k_tiled(blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Lossless Q5_K -> B200 tiled execution layout (Q38PACK layout 2).

    Tiles of 4 rows x 4 super-blocks, 2880 bytes each (QS [4][4][128] | QH
    [4][4][32] | META [4][4][20]), stored quad-major.  The per-block bytes are
    those of the SoA planes (repack_q5_k_sm86_block, src/quant.cpp:401-423); a
    row count that is not a multiple of 4 is padded with all-zero rows
    (d = dmin = 0).
    """
    if cols % 1024:
        raise ValueError("the tiled layout needs cols to be a multiple of 1024")
    nb = cols // 256
    meta, qh, qs = q5k_soa_records(blocks)
    nq = (rows + TILE_ROWS - 1) // TILE_ROWS
    pad = TILE_ROWS * nq - rows

    def grid(a, width):
        a = a.reshape(rows, nb, width)
        if pad:
            a = np.concatenate([a, np.zeros((pad, nb, width), dtype=np.uint8)], axis=0)
        # (quad, row-in-quad, chunk, block-in-chunk, width) -> (quad, chunk, row, block, width)
        a = a.reshape(nq, TILE_ROWS, nb // 4, 4, width).transpose(0, 2, 1, 3, 4)
        return a.reshape(nq, nb // 4, TILE_ROWS * 4 * width)

    tiles = np.concatenate([grid(qs, 128), grid(qh, 32), grid(meta, 20)], axis=2)
    return np.ascontiguousarray(tiles).reshape(-1)


def untile_q5k(tiles: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Inverse of repack_q5k_tiled: layout-2 tiles -> row-major GGUF Q5_K blocks."""
    nb = cols // 256
    nq = (rows + TILE_ROWS - 1) // TILE_ROWS
    t = np.ascontiguousarray(tiles, dtype=np.uint8).reshape(nq, nb // 4, TILE_BYTES)

    def plane(off, width):
        a = t[:, :, off: off + TILE_ROWS * 4 * width].reshape(nq, nb // 4, TILE_ROWS, 4, width)
        return a.transpose(0, 2, 1, 3, 4).reshape(TILE_ROWS * nq, nb, width)[:rows].reshape(-1, width)

    qs, qh, meta = plane(0, 128), plane(TILE_ROWS * 4 * 128, 32), plane(TILE_ROWS * 4 * 160, 20)
    out = np.empty((qs.shape[0], 176), dtype=np.uint8)
    out[:, 0:4] = meta[:, 0:4]
    out[:, 4:16] = pack_scale_min_k4(meta[:, 4:20:2], meta[:, 5:20:2])
    out[:, 16:48] = qh
    out[:, 48:176] = qs
    return out.reshape(-1)


def gen_x(cols: int, seed: int, batch: int = 1) -> np.ndarray:
    return _rng(seed).standard_normal((batch, cols)).astype(np.float32)


def gen_f32(n: int, seed: int, scale: float = 1.0, offset: float = 0.0) -> np.ndarray:
    return (_rng(seed).standard_normal(n) * scale + offset).astype(np.float32)
