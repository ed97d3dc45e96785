"""NumPy restatement of the x-fragment format (test infrastructure).

The tensor-core GEMVs read f32 activations as x-fragments: per super-block of
256 values, 1088 bytes --

* 1024 bytes of int8 limbs.  Each value is quantised to
  xi = round_half_even(v * 2^s) with s = 30 - e, where max|v| over the block
  is m * 2^e (m in [0.5, 1)), and written as four balanced base-256 digits
  (limbs, each in [-128, 127]; xi = sum_k limb_k * 256^k).  Lane
  L = 4G + t of a warp holds values 8L .. 8L+7; limb k of value 8L + j sits at
  byte (p >> 1) * 512 + (p & 1) * 8 + (4 * (2k + (G & 1)) + t) * 16 + j with
  p = G >> 1 -- the B-operand order of mma.m16n8k32 with the limbs and the
  two 32-value groups of a group pair as its eight columns.
* 64 bytes of records, one per limb k (16 bytes each): a double
  unit * 256^k / 8 (unit = 2^-s), then two floats: the sums
  (sum of xi over 32-value group) * unit of groups 2k and 2k + 1.

A block whose largest magnitude is 0 has unit 0 and zero limbs; one holding an
infinity, a NaN or a magnitude above 3e38 has unit NaN and zero limbs.
"""
from __future__ import annotations

import numpy as np

BLOCK_BYTES = 1088
META_OFF = 1024
LIMIT = 2139062143  # 0x7f7f7f7f, the largest balanced four-digit value


def _shift(amax: np.float32) -> int:
    _, e = np.frexp(np.float32(amax))
    s = 30 - int(e)
    if float(np.ldexp(np.float32(amax), s)) > LIMIT:
        s -= 1
    return s


def quantise_block(v: np.ndarray) -> tuple[np.ndarray, np.float32]:
    """(xi int64 [256], unit float32) of one super-block of float32 values."""
    v = np.asarray(v, dtype=np.float32)
    amax = np.float32(np.max(np.abs(v)))
    if not amax <= np.float32(3.0e38):  # the kernels treat these as non-finite
        return np.zeros(256, dtype=np.int64), np.float32(np.nan)
    if amax == 0:
        return np.zeros(256, dtype=np.int64), np.float32(0.0)
    s = _shift(amax)
    with np.errstate(over="ignore", under="ignore"):
        scaled = np.ldexp(v, s).astype(np.float32)  # exact power-of-two scaling
        unit = np.float32(np.ldexp(np.float32(1.0), -s))
    return np.rint(scaled).astype(np.int64), unit


def limbs_of(xi: np.ndarray) -> np.ndarray:
    """Balanced base-256 digits [n, 4] (int8) of |xi| <= 0x7f7f7f7f."""
    r = np.asarray(xi, dtype=np.int64).copy()
    out = np.zeros((r.size, 4), dtype=np.int8)
    for k in range(4):
        lk = ((r + 128) & 255) - 128
        out[:, k] = lk
        r = (r - lk) >> 8
    return out


def byte_offset(value: int, limb: int) -> int:
    lane, j = divmod(value, 8)
    G, t = divmod(lane, 4)
    p = G >> 1
    return (p >> 1) * 512 + (p & 1) * 8 + (4 * (2 * limb + (G & 1)) + t) * 16 + j


def pack(x: np.ndarray) -> np.ndarray:
    """x-fragments (uint8 [K / 256 * 1088]) of a float32 vector of K (K % 256 == 0)."""
    x = np.asarray(x, dtype=np.float32)
    nb = x.size // 256
    out = np.zeros(nb * BLOCK_BYTES, dtype=np.uint8)
    offs = np.array([[byte_offset(i, k) for k in range(4)] for i in range(256)])
    for b in range(nb):
        blk = out[b * BLOCK_BYTES:(b + 1) * BLOCK_BYTES]
        xi, unit = quantise_block(x[b * 256:(b + 1) * 256])
        blk[offs.ravel()] = limbs_of(xi).view(np.uint8).ravel()
        meta = blk[META_OFF:].view(np.uint8)
        for k in range(4):
            rec = np.zeros(16, dtype=np.uint8)
            rec[:8] = np.frombuffer(np.float64(np.float64(unit) * 256.0 ** k * 0.125).tobytes(), np.uint8)
            sums = []
            for g in (2 * k, 2 * k + 1):
                gs = float(np.sum(xi[32 * g:32 * g + 32]))
                sums.append(np.float32(gs * np.float64(unit)))
            rec[8:] = np.frombuffer(np.array(sums, dtype=np.float32).tobytes(), np.uint8)
            meta[16 * k:16 * k + 16] = rec
    return out


def unpack_values(frag: np.ndarray, nb: int) -> np.ndarray:
    """xi * unit (float64 [nb * 256]) decoded from x-fragments."""
    frag = np.asarray(frag, dtype=np.uint8)
    offs = np.array([[byte_offset(i, k) for k in range(4)] for i in range(256)])
    out = np.zeros(nb * 256, dtype=np.float64)
    for b in range(nb):
        blk = frag[b * BLOCK_BYTES:(b + 1) * BLOCK_BYTES]
        limbs = blk[offs].view(np.int8).astype(np.int64)
        xi = limbs @ (256 ** np.arange(4, dtype=np.int64))
        unit8 = blk[META_OFF:META_OFF + 8].view(np.float64)[0]  # unit / 8
        out[b * 256:(b + 1) * 256] = xi * unit8 * 8.0
    return out
