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


def _half_scale(rng: np.random.Generator, n: int, d_exp: int = -8) -> np.ndarray:
    return (np.abs(rng.standard_normal(n)) * 2.0 ** d_exp).astype(np.float16).view(np.uint16)


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


def gen_blocks(ggml_type: int, rows: int, cols: int, seed: int, d_exp: int = -8) -> np.ndarray:
    """Row-major GGUF blocks of `ggml_type` for a [cols, rows] tensor (uint8, flat).
    d (and dmin) are fp16(|N(0,1)| * 2^d_exp): -8 is the benchmark's spec; a
    smaller exponent gives weights nearer a trained model's magnitude,
    for chains of layers whose activations must stay O(1)."""
    if cols % QK:
        raise ValueError("cols must be a multiple of 256")
    n = rows * (cols // QK)
    rng = _rng(seed)
    if ggml_type in (12, 13):
        bb = BLOCK_BYTES[ggml_type]
        out = np.empty((n, bb), dtype=np.uint8)
        dm = np.empty((n, 2), dtype=np.uint16)
        dm[:, 0] = _half_scale(rng, n, d_exp)
        dm[:, 1] = _half_scale(rng, n, d_exp)
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
        out[:, 208:210] = _half_scale(rng, n, d_exp).view(np.uint8).reshape(n, 2)
        return out.reshape(-1)
    if ggml_type == 23:
        out = np.empty((n, 136), dtype=np.uint8)
        out[:, 0:2] = _half_scale(rng, n, d_exp).view(np.uint8).reshape(n, 2)
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


TILE_ROWS = 8           # layout-2 tile: 8 weight rows x 2 super-blocks
TILE_BLOCKS = 2
TILE_BYTES = {13: 2880, 12: 2368, 14: 3360, 23: 2208}  # Q5_K: QS 2048 | QH 512 | SC 256 | DM 64; Q4_K: no QH;
# Q6_K and IQ4_XS below


def tiled_bytes(ggml_type: int, rows: int, cols: int) -> int:
    """Bytes of a rows x cols matrix in layout 2."""
    return ((rows + TILE_ROWS - 1) // TILE_ROWS) * (cols // 512) * TILE_BYTES[ggml_type]


def _tile_fields(ggml_type: int, blocks: np.ndarray, rows: int, nb: int):
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(rows, nb, BLOCK_BYTES[ggml_type])
    dm = b[:, :, 0:4]
    sc, mn = unpack_scale_min_k4(b[:, :, 4:16].reshape(-1, 12))
    scm = np.concatenate([sc, mn], axis=1).reshape(rows, nb, 16)
    if ggml_type == 13:
        return dm, scm, b[:, :, 16:48], b[:, :, 48:176].reshape(rows, nb, 4, 32)
    return dm, scm, None, b[:, :, 16:144].reshape(rows, nb, 4, 32)


# Q6_K element n of a block: its low nibble sits in ql[Q6_QL[n]] >> Q6_QLSH[n],
# its top two bits in qh[Q6_QH[n]] >> Q6_QHSH[n] (src/quant.cpp's Q6_K layout).
_n = np.arange(256)
_h, _tq, _l = _n >> 7, (_n & 127) >> 5, _n & 31
Q6_QL = 64 * _h + _l + 32 * (_tq & 1)
Q6_QLSH = np.where(_tq < 2, 0, 4).astype(np.uint8)
Q6_QH = 32 * _h + _l
Q6_QHSH = (2 * _tq).astype(np.uint8)


def q6k_codes(blocks: np.ndarray) -> np.ndarray:
    """(n, 210) Q6_K blocks -> (n, 256) 6-bit codes (q, the weight is d * sc * (q - 32))."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, 210)
    lo = (b[:, Q6_QL] >> Q6_QLSH) & 15
    hi = (b[:, 128 + Q6_QH] >> Q6_QHSH) & 3
    return (lo | (hi << 4)).astype(np.uint8)


def _repack_q6_tiled(blocks: np.ndarray, rows: int, nb: int) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(rows, nb, 210)
    no, nkc = (rows + 7) // 8, nb // 2
    pad = no * 8 - rows
    q = q6k_codes(b).reshape(rows, nb, 8, 2, 4, 4)  # (j, parity, t, k)
    lo = (q[:, :, :, 0] & 15) | ((q[:, :, :, 1] & 15) << 4)  # (rows, nb, j, t, k)
    hi2 = (q >> 4).reshape(rows, nb, 2, 4, 2, 4, 4)  # (jh, jl, parity, t, k)
    hi = np.zeros((rows, nb, 2, 2, 4, 4), np.uint32)  # (jh, parity, t, k)
    for jl in range(4):
        hi |= hi2[:, :, :, jl].transpose(0, 1, 2, 3, 4, 5).astype(np.uint32) << (2 * jl)
    hi = hi.astype(np.uint8)
    sc = b[:, :, 192:208]
    d = b[:, :, 208:210]

    def padr(a):
        return np.concatenate([a, np.zeros((pad,) + a.shape[1:], dtype=a.dtype)], axis=0) if pad else a

    # LO: [s][g][t][j][k]; HI: [s][g][t][parity][jh][k]; SC [s][g][16]; D [s][g][2]
    lo_t = padr(lo).reshape(no, 8, nkc, 2, 8, 4, 4).transpose(0, 2, 3, 1, 5, 4, 6).reshape(no, nkc, 2048)
    hi_t = padr(hi.transpose(0, 1, 4, 3, 2, 5)).reshape(no, 8, nkc, 2, 4, 2, 2, 4)
    hi_t = hi_t.transpose(0, 2, 3, 1, 4, 5, 6, 7).reshape(no, nkc, 1024)
    sc_t = padr(sc).reshape(no, 8, nkc, 2, 16).transpose(0, 2, 3, 1, 4).reshape(no, nkc, 256)
    d_t = padr(d).reshape(no, 8, nkc, 2, 2).transpose(0, 2, 3, 1, 4).reshape(no, nkc, 32)
    return np.ascontiguousarray(np.concatenate([lo_t, hi_t, sc_t, d_t], axis=2)).reshape(-1)


def _untile_q6(tiles: np.ndarray, rows: int, nb: int) -> np.ndarray:
    no, nkc = (rows + 7) // 8, nb // 2
    t = np.ascontiguousarray(tiles, dtype=np.uint8).reshape(no, nkc, 3360)
    lo = t[:, :, 0:2048].reshape(no, nkc, 2, 8, 4, 8, 4).transpose(0, 3, 1, 2, 5, 4, 6)  # (o, g, kc, s, j, t, k)
    lo = lo.reshape(no * 8, nb, 8, 4, 4)[:rows]
    hi = t[:, :, 2048:3072].reshape(no, nkc, 2, 8, 4, 2, 2, 4).transpose(0, 3, 1, 2, 4, 5, 6, 7)
    hi = hi.reshape(no * 8, nb, 4, 2, 2, 4)[:rows]  # (t, parity, jh, k)
    q = np.zeros((rows, nb, 8, 2, 4, 4), np.uint8)  # (j, parity, t, k)
    for j in range(8):
        for par in range(2):
            lo4 = (lo[:, :, j] >> (4 * par)) & 15  # (rows, nb, t, k)
            hi2 = (hi[:, :, :, par, j >> 2] >> (2 * (j & 3))) & 3
            q[:, :, j, par] = lo4 | (hi2 << 4)
    q = q.reshape(rows * nb, 256)
    out = np.zeros((rows * nb, 210), np.uint8)
    np.bitwise_or.at(out, (slice(None), Q6_QL), ((q & 15) << Q6_QLSH).astype(np.uint8))
    np.bitwise_or.at(out, (slice(None), 128 + Q6_QH), ((q >> 4) << Q6_QHSH).astype(np.uint8))
    sc = t[:, :, 3072:3328].reshape(no, nkc, 2, 8, 16).transpose(0, 3, 1, 2, 4).reshape(no * 8, nb, 16)[:rows]
    d = t[:, :, 3328:3360].reshape(no, nkc, 2, 8, 2).transpose(0, 3, 1, 2, 4).reshape(no * 8, nb, 2)[:rows]
    out[:, 192:208] = sc.reshape(-1, 16)
    out[:, 208:210] = d.reshape(-1, 2)
    return out.reshape(-1)


def iq4xs_fields(blocks: np.ndarray):
    """(n, 136) IQ4_XS blocks -> d bytes (n, 2), signed group scales ls - 32 (n, 8), codes (n, 8, 32)."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, 136)
    sh = b[:, 2].astype(np.uint32) | (b[:, 3].astype(np.uint32) << 8)
    g = np.arange(8)
    ls = ((b[:, 4 + g // 2] >> (4 * (g & 1))) & 15).astype(np.int32) | (((sh[:, None] >> (2 * g)) & 3) << 4).astype(np.int32)
    qs = b[:, 8:136].reshape(-1, 8, 16)
    codes = np.concatenate([qs & 15, qs >> 4], axis=2)  # positions 0..15 low nibbles, 16..31 high
    return b[:, 0:2], (ls - 32).astype(np.int8), codes


def iq4_tile_code(c):
    """An IQ4_XS code as stored in a layout-2 tile: rotated right by one bit,
    (c & 1) << 3 | c >> 1, so the codebook entries 2i and 2i + 1 (same sign)
    share the byte_perm slot i."""
    return ((c & 1) << 3) | (c >> 1)


def iq4_code_from_tile(e):
    """Inverse of iq4_tile_code."""
    return ((e & 7) << 1) | (e >> 3)


def _repack_iq4_tiled(blocks: np.ndarray, rows: int, nb: int) -> np.ndarray:
    no, nkc = (rows + 7) // 8, nb // 2
    pad = no * 8 - rows
    d, sc, codes = iq4xs_fields(blocks)
    c = iq4_tile_code(codes.reshape(rows, nb, 4, 2, 4, 2, 4).astype(np.uint32))  # (pair, parity, t, half, k)
    w = np.zeros((rows, nb, 4, 4, 2), np.uint32)  # (pair, t, half)
    for par in range(2):
        for k in range(4):
            w |= c[:, :, :, par, :, :, k] << (16 * par + 4 * k)
    w8 = w.view(np.uint8).reshape(rows, nb, 4, 4, 8)  # (pair, t, 8 bytes)

    def padr(a):
        return np.concatenate([a, np.zeros((pad,) + a.shape[1:], dtype=a.dtype)], axis=0) if pad else a

    # QS: [s][c][g][t][pair & 1][8 B]
    qs_t = padr(w8).reshape(no, 8, nkc, 2, 2, 2, 4, 8).transpose(0, 2, 3, 4, 1, 6, 5, 7).reshape(no, nkc, 2048)
    sc_t = padr(sc.view(np.uint8).reshape(rows, nb, 8)).reshape(no, 8, nkc, 2, 8).transpose(0, 2, 3, 1, 4)
    d_t = padr(d.reshape(rows, nb, 2)).reshape(no, 8, nkc, 2, 2).transpose(0, 2, 3, 1, 4)
    return np.ascontiguousarray(np.concatenate([qs_t, sc_t.reshape(no, nkc, 128), d_t.reshape(no, nkc, 32)],
                                               axis=2)).reshape(-1)


def _untile_iq4(tiles: np.ndarray, rows: int, nb: int) -> np.ndarray:
    no, nkc = (rows + 7) // 8, nb // 2
    t = np.ascontiguousarray(tiles, dtype=np.uint8).reshape(no, nkc, 2208)
    w8 = t[:, :, 0:2048].reshape(no, nkc, 2, 2, 8, 4, 2, 8).transpose(0, 4, 1, 2, 3, 6, 5, 7)
    w = np.ascontiguousarray(w8).reshape(no * 8, nb, 4, 4, 8).view(np.uint32).reshape(no * 8, nb, 4, 4, 2)[:rows]
    codes = np.zeros((rows, nb, 4, 2, 4, 2, 4), np.uint8)  # (pair, parity, t, half, k)
    for par in range(2):
        for k in range(4):
            codes[:, :, :, par, :, :, k] = iq4_code_from_tile((w >> (16 * par + 4 * k)) & 15)
    codes = codes.reshape(rows * nb, 8, 32)
    sc = t[:, :, 2048:2176].reshape(no, nkc, 2, 8, 8).transpose(0, 3, 1, 2, 4).reshape(no * 8, nb, 8)[:rows]
    d = t[:, :, 2176:2208].reshape(no, nkc, 2, 8, 2).transpose(0, 3, 1, 2, 4).reshape(no * 8, nb, 2)[:rows]
    ls = (sc.reshape(-1, 8).view(np.int8).astype(np.int32) + 32).astype(np.uint32)
    out = np.zeros((rows * nb, 136), np.uint8)
    out[:, 0:2] = d.reshape(-1, 2)
    sh = np.zeros(rows * nb, np.uint32)
    for g in range(8):
        sh |= ((ls[:, g] >> 4) & 3) << (2 * g)
        out[:, 4 + g // 2] |= ((ls[:, g] & 15) << (4 * (g & 1))).astype(np.uint8)
    out[:, 2] = sh & 255
    out[:, 3] = sh >> 8
    out[:, 8:136] = (codes[:, :, :16] | (codes[:, :, 16:] << 4)).reshape(-1, 128)
    return out.reshape(-1)


def repack_tiled(ggml_type: int, blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Lossless GGUF Q5_K / Q4_K -> B200 fragment tiles (Q38PACK layout 2).

    A tile holds 8 rows x 2 super-blocks in the order the tensor-core GEMV's
    lanes read them (lane = 4*row + t owns positions 8t..8t+7 of every group
    pair): QS [s][c][lane][16] (pairs 2c, 2c+1: 8 bytes each), QH [lane][16]
    (Q5_K), SC [s][row][16] (6-bit scales then mins), DM [s][row][4] (d, dmin).
    A QS byte holds the even group's weight in the low nibble (Q5_K: its low 4
    bits) and the odd group's in the high nibble (Q5_K: its top 4 bits); a
    Q5_K QH byte holds, for each pair p, the even group's fifth bit at bit
    2p+1 and the odd group's lowest bit at bit 2p.  Rows pad to a multiple of
    8 with all-zero rows (d = dmin = 0).
    """
    if ggml_type not in TILE_BYTES:
        raise ValueError("layout 2 holds Q5_K, Q4_K, Q6_K and IQ4_XS")
    if cols % 512:
        raise ValueError("layout 2 needs cols to be a multiple of 512")
    nb = cols // 256
    if ggml_type == 14:
        return _repack_q6_tiled(blocks, rows, nb)
    if ggml_type == 23:
        return _repack_iq4_tiled(blocks, rows, nb)
    dm, scm, qh, qs = _tile_fields(ggml_type, blocks, rows, nb)
    no = (rows + TILE_ROWS - 1) // TILE_ROWS
    pad = no * TILE_ROWS - rows

    def padr(a):
        return np.concatenate([a, np.zeros((pad,) + a.shape[1:], dtype=np.uint8)], axis=0) if pad else a

    qs = qs.astype(np.uint8)
    if ggml_type == 13:
        p2 = (2 * np.arange(4, dtype=np.uint8)).reshape(1, 1, 4, 1)
        hb = qh.reshape(rows, nb, 1, 32)
        w_odd = (qs >> 4) | (((hb >> (p2 + 1)) & 1) << 4)
        e5 = (hb >> p2) & 1
        qs_new = (qs & 15) | ((w_odd >> 1) << 4)
        nh = (((e5 << (p2 + 1)) | ((w_odd & 1) << p2)).sum(axis=2, dtype=np.uint32)).astype(np.uint8)  # (rows, nb, 32)
    else:
        qs_new = qs
    nkc = nb // 2
    # QS: (o, g, kc, s, c, pp, t, jj) -> (o, kc, s, c, g, t, pp, jj)
    a = padr(qs_new).reshape(no, 8, nkc, 2, 2, 2, 4, 8).transpose(0, 2, 3, 4, 1, 6, 5, 7).reshape(no, nkc, 2048)
    parts = [a]
    if ggml_type == 13:
        # QH: (o, g, kc, s, t, jj) -> (o, kc, g, t, s, jj)
        h = padr(nh).reshape(no, 8, nkc, 2, 4, 8).transpose(0, 2, 1, 4, 3, 5).reshape(no, nkc, 512)
        parts.append(h)
    parts.append(padr(scm).reshape(no, 8, nkc, 2, 16).transpose(0, 2, 3, 1, 4).reshape(no, nkc, 256))
    parts.append(padr(dm).reshape(no, 8, nkc, 2, 4).transpose(0, 2, 3, 1, 4).reshape(no, nkc, 64))
    return np.ascontiguousarray(np.concatenate(parts, axis=2)).reshape(-1)


def untile(ggml_type: int, tiles: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Inverse of repack_tiled: layout-2 tiles -> row-major GGUF blocks."""
    nb = cols // 256
    if ggml_type == 14:
        return _untile_q6(tiles, rows, nb)
    if ggml_type == 23:
        return _untile_iq4(tiles, rows, nb)
    nkc = nb // 2
    no = (rows + TILE_ROWS - 1) // TILE_ROWS
    t = np.ascontiguousarray(tiles, dtype=np.uint8).reshape(no, nkc, TILE_BYTES[ggml_type])
    qs = t[:, :, 0:2048].reshape(no, nkc, 2, 2, 8, 4, 2, 8).transpose(0, 4, 1, 2, 3, 6, 5, 7)
    qs = qs.reshape(no * 8, nb, 4, 32)[:rows]
    off = 2048
    if ggml_type == 13:
        nh = t[:, :, 2048:2560].reshape(no, nkc, 8, 4, 2, 8).transpose(0, 2, 1, 4, 3, 5).reshape(no * 8, nb, 32)[:rows]
        off = 2560
    scm = t[:, :, off:off + 256].reshape(no, nkc, 2, 8, 16).transpose(0, 3, 1, 2, 4).reshape(no * 8, nb, 16)[:rows]
    dm = t[:, :, off + 256:off + 320].reshape(no, nkc, 2, 8, 4).transpose(0, 3, 1, 2, 4).reshape(no * 8, nb, 4)[:rows]
    out = np.empty((rows, nb, BLOCK_BYTES[ggml_type]), dtype=np.uint8)
    out[:, :, 0:4] = dm
    out[:, :, 4:16] = pack_scale_min_k4(scm[:, :, 0:8].reshape(-1, 8), scm[:, :, 8:16].reshape(-1, 8)).reshape(rows, nb, 12)
    if ggml_type == 13:
        p2 = (2 * np.arange(4, dtype=np.uint8)).reshape(1, 1, 4, 1)
        h = nh.reshape(rows, nb, 1, 32)
        w_odd = ((qs >> 4) << 1) | ((h >> p2) & 1)
        e5 = (h >> (p2 + 1)) & 1
        out[:, :, 48:176] = ((qs & 15) | ((w_odd & 15) << 4)).reshape(rows, nb, 128)
        qh = (((e5 << p2) | ((w_odd >> 4) << (p2 + 1))).sum(axis=2, dtype=np.uint32)).astype(np.uint8)
        out[:, :, 16:48] = qh
    else:
        out[:, :, 16:144] = qs.reshape(rows, nb, 128)
    return out.reshape(-1)


def repack_q5k_tiled(blocks: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Q5_K blocks -> layout-2 tiles (repack_tiled for Q5_K)."""
    return repack_tiled(13, blocks, rows, cols)


def untile_q5k(tiles: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Layout-2 Q5_K tiles -> GGUF blocks (untile for Q5_K)."""
    return untile(13, tiles, rows, cols)


def gen_x(cols: int, seed: int, batch: int = 1) -> np.ndarray:
    return _rng(seed).standard_normal((batch, cols)).astype(np.float32)


def gen_f32(n: int, seed: int, scale: float = 1.0, offset: float = 0.0) -> np.ndarray:
    return (_rng(seed).standard_normal(n) * scale + offset).astype(np.float32)
