"""Layout 2 (B200 fragment tiles) on the CPU: the numpy repack is lossless,
and reading the tiles the way the tensor-core GEMV's lanes do -- the same
word offsets and the same rotate/mask decode (gemv_frag.cuh, frag_decode) --
yields exactly GGML's 5-bit (Q5_K) / 4-bit (Q4_K) weights, 6-bit scales and
mins, and d / dmin of every (row, super-block, group)."""
from __future__ import annotations

import numpy as np
import pytest

from qwen382743090_b200 import synth

M32 = 0xFFFFFFFF


def ggml_weights(ggml_type, blocks, rows, nb):
    """GGML's quantised weight q (before scales) of every (row, block, group, position)."""
    b = blocks.reshape(rows, nb, synth.BLOCK_BYTES[ggml_type])
    qs = b[:, :, 48:176] if ggml_type == 13 else b[:, :, 16:144]
    qs = qs.reshape(rows, nb, 4, 32).astype(np.uint32)
    w = np.empty((rows, nb, 8, 32), np.uint32)
    w[:, :, 0::2] = qs & 15
    w[:, :, 1::2] = qs >> 4
    if ggml_type == 13:
        qh = b[:, :, 16:48].astype(np.uint32)  # (rows, nb, 32): bit g = fifth bit of group g
        for g in range(8):
            w[:, :, g] |= ((qh >> g) & 1) << 4
    return w


def rotl(v, r):
    r %= 32
    return ((v << r) | (v >> (32 - r))) & M32 if r else v


def lane_decode(ggml_type, q, h, p):
    """frag_decode<T, p>: (even group weights, odd group weights x8 / x16) as 4 bytes each."""
    if ggml_type == 13:
        R = rotl(h, (3 - 2 * p) & 31)
        return (q & 0x0F0F0F0F) | (R & 0x10101010), (q & 0xF0F0F0F0) | (R & 0x08080808)
    return q & 0x0F0F0F0F, q & 0xF0F0F0F0


def word(t, off):
    return int(np.frombuffer(t[off:off + 4].tobytes(), np.uint32)[0])


@pytest.mark.parametrize("ggml_type", [13, 12])
@pytest.mark.parametrize("rows,cols", [(8, 512), (13, 1024), (16, 1536)])
def test_lanes_decode_ggml_weights(ggml_type, rows, cols):
    nb = cols // 256
    blocks = synth.gen_blocks(ggml_type, rows, cols, seed=rows * 100 + cols + ggml_type)
    tiles = synth.repack_tiled(ggml_type, blocks, rows, cols)
    assert tiles.nbytes == synth.tiled_bytes(ggml_type, rows, cols)
    np.testing.assert_array_equal(synth.untile(ggml_type, tiles, rows, cols), blocks)

    tb = synth.TILE_BYTES[ggml_type]
    qh_off, sc_off = (2048, 2560) if ggml_type == 13 else (None, 2048)
    dm_off = sc_off + 256
    odd_scale = 8 if ggml_type == 13 else 16
    w = ggml_weights(ggml_type, blocks, rows, nb)
    b3 = blocks.reshape(rows, nb, -1)
    sc_ref, mn_ref = synth.unpack_scale_min_k4(b3[:, :, 4:16].reshape(-1, 12))
    sc_ref, mn_ref = sc_ref.reshape(rows, nb, 8), mn_ref.reshape(rows, nb, 8)
    nkc, no = nb // 2, (rows + 7) // 8
    tiles = tiles.reshape(no, nkc, tb)
    for o in range(no):
        for kc in range(nkc):
            t = tiles[o, kc]
            for lane in range(32):
                g, tt = lane >> 2, lane & 3
                r = 8 * o + g
                h4 = [word(t, qh_off + lane * 16 + 4 * k) for k in range(4)] if qh_off else [0] * 4
                for s in range(2):
                    blk = 2 * kc + s
                    sc_bytes = t[sc_off + s * 128 + g * 16: sc_off + s * 128 + g * 16 + 16]
                    dm_bytes = t[dm_off + s * 32 + g * 4: dm_off + s * 32 + g * 4 + 4]
                    if r >= rows:  # pad rows are all zero
                        assert not sc_bytes.any() and not dm_bytes.any()
                        continue
                    np.testing.assert_array_equal(sc_bytes[:8], sc_ref[r, blk])
                    np.testing.assert_array_equal(sc_bytes[8:], mn_ref[r, blk])
                    np.testing.assert_array_equal(dm_bytes, b3[r, blk, 0:4])
                    for p in range(4):
                        base = s * 1024 + (p >> 1) * 512 + lane * 16 + (p & 1) * 8
                        for half in range(2):  # Q0: positions 8t..8t+3, Q1: 8t+4..8t+7
                            q = word(t, base + 4 * half)
                            ev, od = lane_decode(ggml_type, q, h4[2 * s + half], p)
                            pos = 8 * tt + 4 * half + np.arange(4)
                            evb = np.frombuffer(np.uint32(ev).tobytes(), np.uint8).astype(np.uint32)
                            odb = np.frombuffer(np.uint32(od).tobytes(), np.uint8).astype(np.uint32)
                            np.testing.assert_array_equal(evb, w[r, blk, 2 * p, pos])
                            np.testing.assert_array_equal(odb, odd_scale * w[r, blk, 2 * p + 1, pos])


def test_tiled_rejects_bad_shapes():
    b = synth.gen_blocks(13, 4, 768, seed=1)
    with pytest.raises(ValueError):
        synth.repack_tiled(13, b, 4, 768)
    with pytest.raises(ValueError):
        synth.repack_tiled(23, synth.gen_blocks(23, 4, 256, seed=1), 4, 256)  # one super-block: not a tile


@pytest.mark.parametrize("rows,cols", [(8, 512), (13, 1024)])
def test_q6k_lanes_decode_signed_codes(rows, cols):
    """Q6_K tiles: lane (g, t)'s A bytes for group pair j, built as the GEMV
    builds them (LO nibbles shifted into bits 2-5, the HI two-bit field into
    bits 6-7, then ^ 0x80), are 4 (q - 32) of row g's codes of groups 2j / 2j+1
    at positions 4t..4t+3; scales and d are the block's."""
    nb = cols // 256
    blocks = synth.gen_blocks(14, rows, cols, seed=rows + cols)
    tiles = synth.repack_tiled(14, blocks, rows, cols)
    assert tiles.nbytes == synth.tiled_bytes(14, rows, cols)
    np.testing.assert_array_equal(synth.untile(14, tiles, rows, cols), blocks)
    q = synth.q6k_codes(blocks).reshape(rows, nb, 256).astype(np.int32)
    b3 = blocks.reshape(rows, nb, 210)
    no, nkc = (rows + 7) // 8, nb // 2
    tiles = tiles.reshape(no, nkc, 3360)
    m32 = 0xFFFFFFFF
    for o in range(no):
        for kc in range(nkc):
            t = tiles[o, kc]
            for lane in range(32):
                g, tt = lane >> 2, lane & 3
                r = 8 * o + g
                for s in range(2):
                    blk = 2 * kc + s
                    if r >= rows:
                        continue
                    assert t[3072 + s * 128 + g * 16: 3072 + s * 128 + g * 16 + 16].tobytes() == b3[r, blk, 192:208].tobytes()
                    assert t[3328 + s * 16 + g * 2: 3328 + s * 16 + g * 2 + 2].tobytes() == b3[r, blk, 208:210].tobytes()
                    hi = [word(t, 2048 + s * 512 + lane * 16 + 4 * w) for w in range(4)]
                    for j in range(8):
                        L = word(t, s * 1024 + lane * 32 + 4 * j)
                        E, O = (hi[0], hi[2]) if j < 4 else (hi[1], hi[3])
                        sh = 6 - 2 * (j & 3)
                        ae = ((L << 2) & 0x3C3C3C3C) | ((((E << sh) & m32) & 0xC0C0C0C0) ^ 0x80808080)
                        ao = ((L >> 2) & 0x3C3C3C3C) | ((((O << sh) & m32) & 0xC0C0C0C0) ^ 0x80808080)
                        pos = 4 * tt + np.arange(4)
                        for val, grp in ((ae, 2 * j), (ao, 2 * j + 1)):
                            got = np.frombuffer(np.uint32(val).tobytes(), np.int8).astype(np.int32)
                            np.testing.assert_array_equal(got, 4 * (q[r, blk, 16 * grp + pos] - 32))


def test_xfrag_limb_bytes_from_one_add():
    """The packers take all four balanced base-256 limbs of xi at once as the
    bytes of (xi + 0x80808080) ^ 0x80808080; that equals the digit-by-digit
    form over the whole range |xi| <= 0x7f7f7f7f."""
    from xfrag_format import LIMIT, limbs_of

    rng = np.random.default_rng(5)
    xi = np.concatenate([rng.integers(-LIMIT, LIMIT + 1, 200000), [0, 1, -1, 127, 128, -128, -129, LIMIT, -LIMIT],
                         rng.integers(-300, 300, 1000)]).astype(np.int64)
    words = ((xi.astype(np.int64) + 0x80808080) & 0xFFFFFFFF) ^ 0x80808080
    fast = words.astype(np.uint32).view(np.uint8).reshape(-1, 4).view(np.int8)
    np.testing.assert_array_equal(fast, limbs_of(xi))
    # the limb sums give back sum(xi) exactly
    s = limbs_of(xi).astype(np.int64).sum(axis=0) @ (256 ** np.arange(4, dtype=np.int64))
    assert s == xi.sum()


def test_xfrag_restatement_round_trip():
    """Decoding the restated x-fragments gives x within half a unit of the
    block scale (2^-30 of the block's power-of-two ceiling)."""
    from xfrag_format import pack, unpack_values

    rng = np.random.default_rng(9)
    x = rng.standard_normal(1024).astype(np.float32)
    x[256:512] *= 1e-3
    x[512:768] = 0.0
    got = unpack_values(pack(x), 4)
    for b in range(4):
        blk = x[b * 256:(b + 1) * 256].astype(np.float64)
        amax = np.abs(blk).max()
        if amax == 0:
            assert not got[b * 256:(b + 1) * 256].any()
            continue
        ceil2 = 2.0 ** np.ceil(np.log2(amax))
        assert np.abs(got[b * 256:(b + 1) * 256] - blk).max() <= ceil2 * 2.0 ** -31


@pytest.mark.parametrize("rows,cols", [(8, 512), (13, 1024)])
def test_iq4xs_lanes_select_codes(rows, cols):
    """IQ4_XS tiles: lane (g, t)'s words for group pair p hold row g's 4-bit
    codes of groups 2p (low 16 bits) and 2p+1 (high 16 bits) at positions
    8t..8t+3 and 8t+4..8t+7, code k in bits 4k..4k+3, each stored rotated
    ((c & 1) << 3 | c >> 1); scales are ls - 32."""
    nb = cols // 256
    blocks = synth.gen_blocks(23, rows, cols, seed=rows * 3 + cols)
    tiles = synth.repack_tiled(23, blocks, rows, cols)
    assert tiles.nbytes == synth.tiled_bytes(23, rows, cols)
    np.testing.assert_array_equal(synth.untile(23, tiles, rows, cols), blocks)
    d, sc, codes = synth.iq4xs_fields(blocks)
    codes = codes.reshape(rows, nb, 8, 32)
    sc = sc.reshape(rows, nb, 8)
    no, nkc = (rows + 7) // 8, nb // 2
    tiles = tiles.reshape(no, nkc, 2208)
    for o in range(no):
        for kc in range(nkc):
            t = tiles[o, kc]
            for lane in range(32):
                g, tt = lane >> 2, lane & 3
                r = 8 * o + g
                if r >= rows:
                    continue
                for s in range(2):
                    blk = 2 * kc + s
                    got_sc = np.frombuffer(t[2048 + s * 64 + g * 8: 2048 + s * 64 + g * 8 + 8].tobytes(), np.int8)
                    np.testing.assert_array_equal(got_sc, sc[r, blk])
                    for p in range(4):
                        for half in range(2):
                            w = word(t, s * 1024 + (p >> 1) * 512 + lane * 16 + (p & 1) * 8 + half * 4)
                            pos = 8 * tt + 4 * half + np.arange(4)
                            for par in range(2):
                                got = [(w >> (16 * par + 4 * k)) & 15 for k in range(4)]
                                want = [((c & 1) << 3) | (c >> 1) for c in codes[r, blk, 2 * p + par, pos]]
                                np.testing.assert_array_equal(got, want)


def _prmt(a, b, sel):
    """PTX prmt.b32 (default mode): selector nibble k picks byte (nibble & 7)
    of b:a into result byte k, or, with its bit 3 set, that byte's sign
    replicated over the result byte."""
    src = [(a >> (8 * k)) & 255 for k in range(4)] + [(b >> (8 * k)) & 255 for k in range(4)]
    out = 0
    for k in range(4):
        n = (sel >> (4 * k)) & 15
        v = src[n & 7]
        if n & 8:
            v = 255 if v & 128 else 0
        out |= v << (8 * k)
    return out


def test_iq4xs_tile_codes_decode_to_the_codebook():
    """iq4_codes8's two byte_perm lookups and XOR, with the table words as
    gemv_frag.cuh writes them, turn every stored code iq4_tile_code(c) (in
    every nibble position and both halves of a word) into the oracle's
    codebook entry kIQ4NL[c]."""
    import re
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    src = (root / "qwen382743090_b200" / "csrc" / "gemv_frag.cuh").read_text()
    words = {}
    for name in ("kIq4L0", "kIq4L1", "kIq4H0", "kIq4H1"):
        m = re.search(rf"constexpr uint32_t {name} = iq4nl_word\(([^)]*)\);", src)
        assert m, name
        vals = [int(eval(v.strip(), {})) for v in m.group(1).split(",")]  # "~-104" etc.: int literals
        words[name] = sum((v & 255) << (8 * k) for k, v in enumerate(vals))
    oc = (root / "oracle" / "q38_oracle.c").read_text()
    m = re.search(r"kIQ4NL\[16\]\s*=\s*\{([^}]*)\}", oc)
    kv = [int(v) for v in m.group(1).split(",")]
    assert len(kv) == 16

    def codes8(q):
        f = q ^ 0x88888888
        even = _prmt(words["kIq4L0"], words["kIq4L1"], q & 0xFFFF) ^ _prmt(words["kIq4H0"], words["kIq4H1"], f & 0xFFFF)
        odd = _prmt(words["kIq4L0"], words["kIq4L1"], q >> 16) ^ _prmt(words["kIq4H0"], words["kIq4H1"], f >> 16)
        return even, odd

    rng = np.random.default_rng(7)
    cases = [np.full(8, c) for c in range(16)] + [rng.integers(0, 16, 8) for _ in range(200)]
    for cs in cases:
        q = sum(int(synth.iq4_tile_code(int(c))) << (4 * k) for k, c in enumerate(cs))
        even, odd = codes8(q)
        got = [(((w >> (8 * k)) & 255) ^ 128) - 128 for w in (even, odd) for k in range(4)]
        assert got == [kv[int(c)] for c in cs], cs
    for c in range(16):
        assert synth.iq4_code_from_tile(synth.iq4_tile_code(c)) == c
