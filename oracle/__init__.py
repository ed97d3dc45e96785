"""CPU parity checker for the Q38RT B200 runtime -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may
import this package.  The runtime in ``qwen382743090_b200`` never imports it
and has no CPU fallback.

Two libraries are exposed through numpy-friendly wrappers:

* ``port()``  -- ``_build/liboracle.so``, the plain-C restatement in
  ``q38_oracle.c`` (every function cites the reference file:line it follows);
* ``ref()``   -- ``_ref/libq38ref.so``, the reference's own ``src/quant.cpp``
  compiled from the reference tree by ``Makefile`` together with
  ``ref_shim.cpp``.  It exists only where the reference tree was present at
  build time (or where the built file was carried along); ``ref()`` returns
  ``None`` otherwise.

Both expose the same GEMV/dequant surface so tests can run one against the
other.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_SO = HERE / "_build" / "liboracle.so"
REF_SO = HERE / "_ref" / "libq38ref.so"

QK = 256
BLOCK_BYTES = {12: 144, 13: 176, 14: 210, 15: 292, 23: 136, 1013: 180}

_u8p = C.POINTER(C.c_uint8)
_f32p = C.POINTER(C.c_float)
_f64p = C.POINTER(C.c_double)


def reference_root() -> Path | None:
    """The reference source tree: $Q38_REFERENCE when set, else a checkout
    named `reference` beside this repository; None when neither exists."""
    env = os.environ.get("Q38_REFERENCE")
    p = Path(env) if env else HERE.parent.parent / "reference"
    return p if (p / "src" / "quant.cpp").exists() else None


def build(quiet: bool = True) -> None:
    """Run oracle/Makefile (gcc only; the reference part only if present)."""
    out = subprocess.run(["make", "-C", str(HERE)], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def _ptr(a: np.ndarray, ty):
    return a.ctypes.data_as(ty)


class _Lib:
    """Common numpy wrappers over either the port or the reference shim."""

    def __init__(self, path: Path, prefix: str):
        self.path = path
        self.lib = C.CDLL(str(path))
        self.p = prefix
        L = self.lib
        if prefix == "q38o_":
            L.q38o_fp16_to_fp32.restype = C.c_float
            L.q38o_fp16_to_fp32.argtypes = [C.c_uint16]
            L.q38o_fp32_to_fp16.restype = C.c_uint16
            L.q38o_fp32_to_fp16.argtypes = [C.c_float]
            L.q38o_dequant_block.argtypes = [C.c_int, _u8p, _f32p]
            L.q38o_dequant_q5k_soa.argtypes = [_u8p, _f32p]
            L.q38o_repack_q5k_soa.argtypes = [_u8p, _u8p]
            L.q38o_quantize_q8k.argtypes = [_f32p, C.c_size_t, _u8p]
            L.q38o_quantize_q8_1.argtypes = [_f32p, C.c_size_t, _u8p]
            L.q38o_gemv.argtypes = [C.c_int, _u8p, _f32p, C.c_size_t, C.c_size_t, C.c_size_t, _f64p, C.c_int]
            L.q38o_gemv_q8k.argtypes = [C.c_int, _u8p, _u8p, C.c_size_t, C.c_size_t, C.c_size_t, _f64p, C.c_int]
            L.q38o_gemv_q5k_soa.argtypes = [_u8p, _u8p, _u8p, _f32p, C.c_size_t, C.c_size_t, C.c_size_t, _f64p, C.c_int]
        else:
            L.q38ref_fp16_to_fp32.restype = C.c_float
            L.q38ref_fp16_to_fp32.argtypes = [C.c_uint16]
            L.q38ref_fp32_to_fp16.restype = C.c_uint16
            L.q38ref_fp32_to_fp16.argtypes = [C.c_float]
            L.q38ref_dequant.argtypes = [C.c_int, _u8p, _f32p]
            L.q38ref_repack_q5k_soa.argtypes = [_u8p, _u8p]
            L.q38ref_quantize_q8k.argtypes = [_f32p, C.c_size_t, _u8p]
            L.q38ref_quantize_q8_1.argtypes = [_f32p, C.c_size_t, _u8p]
            L.q38ref_gemv.argtypes = [C.c_int, _u8p, _f32p, C.c_size_t, C.c_size_t, C.c_size_t, _f64p, C.c_int]
            L.q38ref_gemv_q8k.argtypes = [C.c_int, _u8p, _u8p, C.c_size_t, C.c_size_t, C.c_size_t, _f64p, C.c_int]
            L.q38ref_gemv_q5k_soa.argtypes = [_u8p, _u8p, _u8p, _f32p, C.c_size_t, C.c_size_t, C.c_size_t, _f64p, C.c_int]

    # ---- scalar conversions -------------------------------------------------
    def fp16_to_fp32(self, h: int) -> float:
        return getattr(self.lib, self.p + "fp16_to_fp32")(h)

    def fp32_to_fp16(self, f: float) -> int:
        return getattr(self.lib, self.p + "fp32_to_fp16")(f)

    # ---- blocks --------------------------------------------------------------
    def dequant(self, type_id: int, blocks: np.ndarray) -> np.ndarray:
        """Dequantise a run of blocks (uint8, n*block_bytes) -> float32[n*256]."""
        bb = BLOCK_BYTES[type_id]
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
        n = blocks.size // bb
        out = np.empty(n * QK, dtype=np.float32)
        for i in range(n):
            src = blocks[i * bb:(i + 1) * bb]
            dst = out[i * QK:(i + 1) * QK]
            if self.p == "q38o_":
                if type_id == 1013:
                    self.lib.q38o_dequant_q5k_soa(_ptr(src, _u8p), _ptr(dst, _f32p))
                    rc = 0
                else:
                    rc = self.lib.q38o_dequant_block(type_id, _ptr(src, _u8p), _ptr(dst, _f32p))
            else:
                rc = self.lib.q38ref_dequant(type_id, _ptr(src, _u8p), _ptr(dst, _f32p))
            if rc != 0:
                raise ValueError(f"dequant of type {type_id} failed")
        return out

    def repack_q5k_soa_block(self, src176: np.ndarray) -> np.ndarray:
        src = np.ascontiguousarray(src176, dtype=np.uint8)
        dst = np.zeros(180, dtype=np.uint8)
        getattr(self.lib, self.p + "repack_q5k_soa")(_ptr(src, _u8p), _ptr(dst, _u8p))
        return dst

    def quantize_q8k(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        out = np.zeros(x.size // QK * 292, dtype=np.uint8)
        rc = getattr(self.lib, self.p + "quantize_q8k")(_ptr(x, _f32p), x.size, _ptr(out, _u8p))
        if rc != 0:
            raise ValueError("Q8_K quantize rejected its input")
        return out

    def quantize_q8_1(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
        out = np.zeros(x.size // 32 * 36, dtype=np.uint8)
        rc = getattr(self.lib, self.p + "quantize_q8_1")(_ptr(x, _f32p), x.size, _ptr(out, _u8p))
        if rc != 0:
            raise ValueError("Q8_1 quantize rejected its input")
        return out

    @staticmethod
    def dequant_q8_1(blocks: np.ndarray) -> np.ndarray:
        """d * q per value (dequantize_q8_1_block_cpu, src/quant.cpp:316-333)."""
        b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, 36)
        d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
        return (d * b[:, 4:].view(np.int8).astype(np.float32)).reshape(-1).astype(np.float32)

    # ---- GEMV ----------------------------------------------------------------
    def gemv(self, type_id: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int,
             threads: int = 1) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
        w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
        y = np.zeros((x.shape[0], rows), dtype=np.float64)
        rc = getattr(self.lib, self.p + "gemv")(type_id, _ptr(w, _u8p), _ptr(x, _f32p), rows, cols,
                                                x.shape[0], _ptr(y, _f64p), threads)
        if rc != 0:
            raise ValueError("gemv rejected its arguments")
        return y

    def gemv_q8k(self, type_id: int, w: np.ndarray, xq8: np.ndarray, rows: int, cols: int,
                 batch: int = 1, threads: int = 1) -> np.ndarray:
        w = np.ascontiguousarray(w, dtype=np.uint8).reshape(-1)
        xq8 = np.ascontiguousarray(xq8, dtype=np.uint8).reshape(-1)
        y = np.zeros((batch, rows), dtype=np.float64)
        rc = getattr(self.lib, self.p + "gemv_q8k")(type_id, _ptr(w, _u8p), _ptr(xq8, _u8p), rows, cols,
                                                    batch, _ptr(y, _f64p), threads)
        if rc != 0:
            raise ValueError("gemv_q8k rejected its arguments")
        return y

    def gemv_q5k_soa(self, meta: np.ndarray, qh: np.ndarray, qs: np.ndarray, x: np.ndarray,
                     rows: int, cols: int, threads: int = 1) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
        meta, qh, qs = (np.ascontiguousarray(a, dtype=np.uint8).reshape(-1) for a in (meta, qh, qs))
        y = np.zeros((x.shape[0], rows), dtype=np.float64)
        rc = getattr(self.lib, self.p + "gemv_q5k_soa")(_ptr(meta, _u8p), _ptr(qh, _u8p), _ptr(qs, _u8p),
                                                        _ptr(x, _f32p), rows, cols, x.shape[0],
                                                        _ptr(y, _f64p), threads)
        if rc != 0:
            raise ValueError("gemv_q5k_soa rejected its arguments")
        return y


class _Port(_Lib):
    """Extra entry points that only the C restatement has (layer math)."""

    def __init__(self, path: Path):
        super().__init__(path, "q38o_")
        L = self.lib
        L.q38o_rmsnorm.argtypes = [_f32p, _f32p, C.c_size_t, C.c_float, _f32p]
        L.q38o_conv4_silu_roll.argtypes = [_f32p, _f32p, _f32p, C.c_size_t, _f32p, _f32p]
        L.q38o_l2norm_heads.argtypes = [_f32p, C.c_size_t, C.c_size_t, C.c_float, _f32p]
        L.q38o_beta_gate.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_size_t, _f32p, _f32p]
        L.q38o_gdn_step.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, C.c_size_t, C.c_size_t,
                                    C.c_size_t, _f32p, _f32p]
        L.q38o_gated_rmsnorm_silu.argtypes = [_f32p, _f32p, _f32p, C.c_size_t, C.c_size_t, C.c_float, _f32p]
        L.q38o_silu_mul.argtypes = [_f32p, _f32p, C.c_size_t, _f32p]
        L.q38o_gdn_smoke_inputs.argtypes = [C.c_size_t, C.c_size_t, C.c_size_t, _f32p, _f32p, _f32p, _f32p, _f32p,
                                            _f32p]
        L.q38o_add.argtypes = [_f32p, _f32p, C.c_size_t, _f32p]
        L.q38o_rope.argtypes = [_f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, C.c_double]
        L.q38o_attn_decode.argtypes = [_f32p, C.POINTER(C.c_uint16), C.POINTER(C.c_uint16), C.c_size_t,
                                       C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, _f32p]

    @staticmethod
    def _f(a):
        return np.ascontiguousarray(a, dtype=np.float32).reshape(-1)

    def rmsnorm(self, x, w, eps=1e-6):
        x, w = self._f(x), self._f(w)
        y = np.empty_like(x)
        self.lib.q38o_rmsnorm(_ptr(x, _f32p), _ptr(w, _f32p), x.size, eps, _ptr(y, _f32p))
        return y

    def conv4_silu_roll(self, state, x, w):
        state, x, w = self._f(state), self._f(x), self._f(w)
        out = np.empty_like(x)
        st = np.empty_like(state)
        self.lib.q38o_conv4_silu_roll(_ptr(state, _f32p), _ptr(x, _f32p), _ptr(w, _f32p), x.size,
                                      _ptr(out, _f32p), _ptr(st, _f32p))
        return out, st

    def l2norm_heads(self, x, heads, dim, eps=1e-6):
        x = self._f(x)
        y = np.empty_like(x)
        self.lib.q38o_l2norm_heads(_ptr(x, _f32p), heads, dim, eps, _ptr(y, _f32p))
        return y

    def beta_gate(self, b, a, dt_bias, A):
        b, a, dt_bias, A = (self._f(v) for v in (b, a, dt_bias, A))
        beta = np.empty_like(b)
        g = np.empty_like(b)
        self.lib.q38o_beta_gate(_ptr(b, _f32p), _ptr(a, _f32p), _ptr(dt_bias, _f32p), _ptr(A, _f32p), b.size,
                                _ptr(beta, _f32p), _ptr(g, _f32p))
        return beta, g

    def gdn_step(self, q, k, v, g, beta, state, hq, hv, d):
        q, k, v, g, beta, state = (self._f(a) for a in (q, k, v, g, beta, state))
        out = np.empty(hv * d, dtype=np.float32)
        st = np.empty_like(state)
        self.lib.q38o_gdn_step(_ptr(q, _f32p), _ptr(k, _f32p), _ptr(v, _f32p), _ptr(g, _f32p),
                               _ptr(beta, _f32p), _ptr(state, _f32p), hq, hv, d, _ptr(out, _f32p),
                               _ptr(st, _f32p))
        return out, st

    def gdn_smoke_inputs(self, hq=16, hv=48, d=128):
        """q, k, v, g, beta, state of the reference's GDN decode-core smoke."""
        q, k = np.empty(hq * d, np.float32), np.empty(hq * d, np.float32)
        v, g, beta = np.empty(hv * d, np.float32), np.empty(hv, np.float32), np.empty(hv, np.float32)
        st = np.empty(hv * d * d, np.float32)
        self.lib.q38o_gdn_smoke_inputs(hq, hv, d, *(_ptr(a, _f32p) for a in (q, k, v, g, beta, st)))
        return q, k, v, g, beta, st

    def gated_rmsnorm_silu(self, o, z, w, heads, d, eps=1e-6):
        o, z, w = self._f(o), self._f(z), self._f(w)
        y = np.empty_like(o)
        self.lib.q38o_gated_rmsnorm_silu(_ptr(o, _f32p), _ptr(z, _f32p), _ptr(w, _f32p), heads, d, eps,
                                         _ptr(y, _f32p))
        return y

    def silu_mul(self, g, u):
        g, u = self._f(g), self._f(u)
        y = np.empty_like(g)
        self.lib.q38o_silu_mul(_ptr(g, _f32p), _ptr(u, _f32p), g.size, _ptr(y, _f32p))
        return y

    def add(self, a, b):
        a, b = self._f(a), self._f(b)
        y = np.empty_like(a)
        self.lib.q38o_add(_ptr(a, _f32p), _ptr(b, _f32p), a.size, _ptr(y, _f32p))
        return y

    def rope(self, x, heads, d, rope_dim, pos, theta):
        x = self._f(x).copy()
        self.lib.q38o_rope(_ptr(x, _f32p), heads, d, rope_dim, pos, theta)
        return x

    def attn_decode(self, q, kc, vc, hq, hkv, d, t, ld_t):
        q = self._f(q)
        kc = np.ascontiguousarray(kc, dtype=np.uint16).reshape(-1)
        vc = np.ascontiguousarray(vc, dtype=np.uint16).reshape(-1)
        out = np.empty(hq * d, dtype=np.float32)
        self.lib.q38o_attn_decode(_ptr(q, _f32p), kc.ctypes.data_as(C.POINTER(C.c_uint16)),
                                  vc.ctypes.data_as(C.POINTER(C.c_uint16)), hq, hkv, d, t, ld_t,
                                  _ptr(out, _f32p))
        return out


_port = None
_ref = None


def port() -> _Port:
    """The C restatement (always available once built)."""
    global _port
    if _port is None:
        if not PORT_SO.exists():
            build()
        _port = _Port(PORT_SO)
    return _port


def ref():
    """The reference's own quant.cpp, or None when it was never built here."""
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            try:
                build()  # rebuilds _ref only where the reference tree is present
            except RuntimeError:
                return None
        if not REF_SO.exists():
            return None
        _ref = _Lib(REF_SO, "q38ref_")
    return _ref
