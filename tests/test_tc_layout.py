"""The tcgen05 batched GEMM (csrc/gemm_tc.cuh) on the CPU: its descriptors and
its shared-memory layouts.

* The hand-built UMMA instruction and shared-memory descriptors equal the ones
  CUTLASS's own encoders (cute/arch/mma_sm100_desc.hpp) produce for the same
  operand types, shape and layout (compiled with nvcc, run on the host).
* A NumPy emulation of the kernel's data path -- the activation limbs at the
  byte offsets xtc_pack_kernel writes, the weight codes at the offsets
  tc_decode writes (read from the layout-2 tiles exactly as its lanes do), one
  MMA per 32-weight group read through the canonical K-major, no-swizzle UMMA
  layout ((8, n), 2) : ((16 B, SBO), LBO), and the epilogue's integer group
  scales / int64 limb join / fp64 block scale / split-K sum -- gives the FP64 oracle's GEMV
  within the GEMV tolerance, and the decoded A operand holds GGML's codes.
"""
from __future__ import annotations

import os
import shutil
import site
import subprocess
from pathlib import Path

import numpy as np
import pytest

from qwen382743090_b200 import synth
from test_tiled_layout import ggml_weights, lane_decode, word
from xfrag_format import limbs_of, quantise_block

ROOT = Path(__file__).resolve().parents[1]
TC_ROWS, META = 128, 64


def _cutlass_include():
    for sp in site.getsitepackages():
        p = Path(sp) / "flashinfer" / "data" / "cutlass" / "include"
        if (p / "cute" / "arch" / "mma_sm100_desc.hpp").exists():
            return p
    return None


DESC_SRC = r"""
#include <cstdio>
#include <cute/arch/mma_sm100_desc.hpp>
#include "gemm_tc.cuh"
int main() {
    using namespace cute;
    int bad = 0;
    auto d32 = UMMA::make_instr_desc<uint8_t, int8_t, int32_t, 128, 32, UMMA::Major::K, UMMA::Major::K>();
    auto d16 = UMMA::make_instr_desc<uint8_t, int8_t, int32_t, 128, 16, UMMA::Major::K, UMMA::Major::K>();
    bad |= uint32_t(d32) != q38::umma_idesc_u8s8(128, 32);
    bad |= uint32_t(d16) != q38::umma_idesc_u8s8(128, 16);
    const uint32_t cases[4][3] = {{0x0u, 2048u, 128u}, {0x10400u, 512u, 128u}, {0x35f30u, 256u, 128u},
                                  {0x3fff0u, 2048u, 128u}};
    for (auto& c : cases) {
        UMMA::SmemDescriptor s;
        s.desc_ = 0;
        s.start_address_ = static_cast<uint16_t>(c[0] >> 4);
        s.leading_byte_offset_ = static_cast<uint16_t>(c[1] >> 4);
        s.stride_byte_offset_ = static_cast<uint16_t>(c[2] >> 4);
        s.version_ = 1;
        s.base_offset_ = 0;
        s.lbo_mode_ = 0;
        s.layout_type_ = uint8_t(UMMA::LayoutType::SWIZZLE_NONE);
        bad |= s.desc_ != q38::umma_smem_desc(c[0], c[1], c[2]);
    }
    std::printf("idesc %08x %08x\n", uint32_t(d32), uint32_t(d16));
    return bad;
}
"""


def test_descriptors_match_cutlass(tmp_path):
    inc = _cutlass_include()
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if inc is None or not os.path.exists(nvcc):
        pytest.skip("CUTLASS headers or nvcc not available")
    src = tmp_path / "desc.cu"
    src.write_text(DESC_SRC)
    exe = tmp_path / "desc"
    res = subprocess.run([nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", f"-I{inc}",
                          f"-I{ROOT / 'qwen382743090_b200' / 'csrc'}", "-o", str(exe), str(src)],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-2000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True)
    assert run.returncode == 0, f"descriptor mismatch: {run.stdout}"
    assert "08080420 08040420" in run.stdout


# ---- the data path ---------------------------------------------------------------
def pack_xu(x: np.ndarray, slots: int) -> np.ndarray:
    """xtc_pack_kernel's output for activation rows x [nbatch][K]."""
    nbatch, K = x.shape
    nb, N = K // 256, 4 * slots
    xsb, lbob = slots * (1024 + META), (N // 8) * 128
    xu = np.zeros(nb * xsb, np.uint8)
    k = np.arange(256)
    for s in range(nb):
        base = s * xsb
        for b in range(slots):
            if b < nbatch:
                xi, unit = quantise_block(x[b, 256 * s:256 * s + 256])
            else:
                xi, unit = np.zeros(256, np.int64), np.float32(0)
            limbs = limbs_of(xi).view(np.uint8)
            for l in range(4):
                n = 4 * b + l
                xu[base + (k // 16) * lbob + (n >> 3) * 128 + (n & 7) * 16 + (k % 16)] = limbs[:, l]
            meta = base + N * 256 + b * META
            unw = np.array([np.float64(unit) * 256.0 ** l * 0.125 for l in range(4)], np.float64)
            xu[meta:meta + 32] = np.frombuffer(unw.tobytes(), np.uint8)
            gs = np.array([np.float32(float(xi[32 * g:32 * g + 32].sum()) * np.float64(unit)) for g in range(8)],
                          np.float32)
            xu[meta + 32:meta + 64] = np.frombuffer(gs.tobytes(), np.uint8)
    return xu


def decode_a(ggml_type, tiles, tb, tile_index, octs, half):
    """tc_decode of one super-block for the CTA's octets: A bytes [32768] and
    the side buffer's (scales/mins [128][16], d/dmin words [128])."""
    A = np.zeros(TC_ROWS * 256, np.uint8)
    sc = np.zeros((TC_ROWS, 16), np.uint8)
    dm = np.zeros(TC_ROWS, np.uint32)
    sc_off = 2560 if ggml_type == 13 else 2048
    for o in range(octs):
        t0 = tile_index(o) * tb
        tile = tiles[t0:t0 + tb]
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            h0 = h1 = 0
            if ggml_type == 13:
                qh = [word(tile, 2048 + lane * 16 + 4 * i) for i in range(4)]
                h0, h1 = (qh[2], qh[3]) if half else (qh[0], qh[1])
            qa = [word(tile, half * 1024 + lane * 16 + 4 * i) for i in range(4)]
            qb = [word(tile, half * 1024 + 512 + lane * 16 + 4 * i) for i in range(4)]
            base = o * 128 + g * 16 + (t & 1) * 8 + (t >> 1) * 2048
            for p, (wa, wb) in enumerate(((qa[0], qa[1]), (qa[2], qa[3]), (qb[0], qb[1]), (qb[2], qb[3]))):
                e0, o0 = lane_decode(ggml_type, wa, h0, p)
                e1, o1 = lane_decode(ggml_type, wb, h1, p)
                for grp, (lo, hi) in ((2 * p, (e0, e1)), (2 * p + 1, (o0, o1))):
                    off = base + grp * 4096
                    A[off:off + 8] = np.frombuffer(np.array([lo, hi], np.uint32).tobytes(), np.uint8)
            if t == 0:
                r = 8 * o + g
                sc[r] = tile[sc_off + half * 128 + g * 16:sc_off + half * 128 + g * 16 + 16]
                dm[r] = word(tile, sc_off + 256 + half * 32 + g * 4)
    return A, sc, dm


def umma(Abuf, a_start, Bbuf, b_start, lbo_a, lbo_b, N):
    """D [128][N] = A [128][32] (u8) x B [N][32]^T (s8), both read through the
    canonical K-major no-swizzle layout: element (row, k) at
    start + (row // 8) * SBO + (row % 8) * 16 + (k // 16) * LBO + k % 16, SBO = 128."""
    m = np.arange(TC_ROWS)[:, None]
    n = np.arange(N)[:, None]
    k = np.arange(32)[None, :]
    A = Abuf[a_start + (m // 8) * 128 + (m % 8) * 16 + (k // 16) * lbo_a + k % 16].astype(np.int64)
    B = Bbuf[b_start + (n // 8) * 128 + (n % 8) * 16 + (k // 16) * lbo_b + k % 16].view(np.int8).astype(np.int64)
    return A @ B.T


def half_bits(w):
    return np.frombuffer(np.uint16(w & 0xFFFF).tobytes(), np.float16)[0].astype(np.float32)


def emulate(ggml_type, tiles, x, rows, cols, sm_count=148):
    nbatch = x.shape[0]
    slots = 4 if nbatch <= 4 else 8
    N, xsb, lbob = 4 * slots, slots * (1024 + META), (4 * slots // 8) * 128
    tb = synth.TILE_BYTES[ggml_type]
    nb, nkc, nocts = cols // 256, cols // 512, (rows + 7) // 8
    nrb = (nocts + 15) // 16
    S = max(1, min(nkc, sm_count // nrb))
    xu = pack_xu(x, slots)
    odd_shift = 0 if ggml_type == 13 else 1
    y = np.zeros((nbatch, rows), np.float64)
    checked_a = False
    for rb in range(nrb):
        o0, octs = 16 * rb, min(16, nocts - 16 * rb)
        parts = []
        for sl in range(S):
            cb, cr = divmod(nkc, S)
            c0, nch = sl * cb + min(sl, cr), cb + (1 if sl < cr else 0)
            acc = np.zeros((TC_ROWS, slots), np.float64)
            mn = np.zeros((TC_ROWS, slots), np.float32)
            for kk in range(nch):
                kc = c0 + kk
                for half in range(2):
                    A, sc, dm = decode_a(ggml_type, tiles, tb, lambda o: (o0 + o) * nkc + kc, octs, half)
                    if not checked_a:  # the decoded codes are GGML's (odd groups x8 / x16)
                        wq = ggml_weights(ggml_type, synth_blocks_cache[0], rows, nb)
                        for G in range(8):
                            D_rows = A[G * 4096 + (np.arange(8 * octs)[:, None] // 8) * 128 +
                                       (np.arange(8 * octs)[:, None] % 8) * 16 +
                                       (np.arange(32)[None, :] // 16) * 2048 + np.arange(32)[None, :] % 16]
                            want = wq[8 * o0:8 * o0 + 8 * octs, 2 * kc + half, G] * (
                                1 if G % 2 == 0 else (8 if ggml_type == 13 else 16))
                            valid = min(8 * octs, rows - 8 * o0)
                            np.testing.assert_array_equal(D_rows[:valid], want[:valid])
                        checked_a = True
                    s = 2 * kc + half
                    sbase = s * xsb
                    D = [umma(A, G * 4096, xu, sbase + 2 * G * lbob, 2048, lbob, N) for G in range(8)]
                    d = np.array([half_bits(v) for v in dm], np.float32)
                    dmin = np.array([half_bits(v >> 16) for v in dm], np.float32)
                    for b in range(nbatch):
                        meta = sbase + N * 256 + b * META
                        unw0 = xu[meta:meta + 8].view(np.float64)[0]  # unit / 8
                        xs = xu[meta + 32:meta + 64].view(np.float32)
                        A = np.zeros(TC_ROWS, np.int64)  # sum_l A8_l 256^l, exact
                        for l in range(4):
                            Ae = sum(sc[:, G].astype(np.int64) * D[G][:, 4 * b + l] for G in (0, 2, 4, 6))
                            Ao = sum(sc[:, G].astype(np.int64) * D[G][:, 4 * b + l] for G in (1, 3, 5, 7))
                            A8 = Ae * 8 + (Ao >> odd_shift)
                            assert np.abs(A8).max() < 2 ** 31  # the kernel's int32 sums are exact
                            A += A8 * (256 ** l)
                        acc[:, b] += A.astype(np.float64) * (d.astype(np.float64) * unw0)
                        pm = sc[:, 8].astype(np.float32) * xs[0]
                        for g in range(1, 8):
                            pm = sc[:, 8 + g].astype(np.float32) * xs[g] + pm
                        mn[:, b] = dmin * pm + mn[:, b]
                        if half:
                            acc[:, b] -= mn[:, b].astype(np.float64)
                            mn[:, b] = 0
            parts.append(acc)
        tot = parts[0]
        for p in parts[1:]:
            tot = tot + p
        r0, r1 = 8 * o0, min(rows, 8 * o0 + TC_ROWS)
        y[:, r0:r1] = tot[:r1 - r0, :nbatch].T
    return y.astype(np.float32)


synth_blocks_cache = [None]


@pytest.mark.parametrize("ggml_type", [13, 12])
@pytest.mark.parametrize("rows,cols,batch,sms", [(21, 1024, 3, 148), (136, 2048, 6, 2), (8, 512, 2, 148)])
def test_tc_datapath_emulation(port, ggml_type, rows, cols, batch, sms):
    blocks = synth.gen_blocks(ggml_type, rows, cols, seed=rows + cols + batch)
    synth_blocks_cache[0] = blocks
    tiles = synth.repack_tiled(ggml_type, blocks, rows, cols)
    x = synth.gen_x(cols, seed=batch + cols, batch=batch).reshape(batch, cols)
    y = emulate(ggml_type, tiles, x, rows, cols, sm_count=sms)
    ref = port.gemv(ggml_type, blocks, x, rows, cols, threads=4)
    err = np.abs(y.astype(np.float64) - ref)
    assert not ((err > 1e-4) & (err > 1e-3 * np.abs(ref))).any(), err.max()
