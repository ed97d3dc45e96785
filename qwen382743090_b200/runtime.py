"""ctypes binding of the Q38RT C ABI (include/q38rt.h).

This is the host-side mirror used by tests, bench.py and the Python tools.
It loads the in-tree lib/libq38rt_b200.so and raises if it is missing: there
is no CPU or PyTorch fallback for any kernel.
"""
from __future__ import annotations

import ctypes as C
import re
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from .build import LIB, ROOT

HEADER = ROOT / "include" / "q38rt.h"

Q38_OK = 0
STATUS = {0: "OK", 1: "INVALID", 2: "CUDA", 3: "UNSUPPORTED", 4: "NOMEM", 5: "NO_DEVICE", 6: "FAULT"}


class Q38Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"q38rt {STATUS.get(code, code)}: {msg}")
        self.code = code


class q38_weight_desc(C.Structure):
    _fields_ = [
        ("ggml_type", C.c_uint32),
        ("layout", C.c_uint32),
        ("rows", C.c_uint32),
        ("cols", C.c_uint32),
        ("data", C.c_uint64),
        ("aux0", C.c_uint64),
        ("aux1", C.c_uint64),
    ]


class q38_tp_exchange_desc(C.Structure):
    _fields_ = [
        ("x_in", C.c_uint64),
        ("x_out", C.c_uint64),
        ("part", C.c_uint64),
        ("region", C.c_uint64 * 8),
        ("step", C.c_uint64),
        ("norm_w", C.c_uint64),
        ("xfrag", C.c_uint64),
        ("n", C.c_uint32),
        ("rank", C.c_uint32),
        ("size", C.c_uint32),
        ("instance", C.c_uint32),
        ("eps", C.c_float),
    ]


class q38_device_info(C.Structure):
    _fields_ = [
        ("ordinal", C.c_int),
        ("sm_major", C.c_int),
        ("sm_minor", C.c_int),
        ("sm_count", C.c_int),
        ("total_memory", C.c_size_t),
        ("l2_bytes", C.c_size_t),
        ("vmm_granularity", C.c_size_t),
        ("vmm_supported", C.c_int),
        ("driver_version", C.c_int),
        ("name", C.c_char * 128),
    ]


class q38_gdn_fused_args(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("qkv", "conv_w", "conv_in", "conv_out", "beta_raw", "alpha_raw",
                                           "dt_bias", "ssm_a", "state_in", "state_out", "z", "norm_w", "out")] + [
        ("qk_heads", C.c_uint32), ("value_heads", C.c_uint32), ("eps", C.c_float), ("scale", C.c_float)]


class q38_model_config(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_layers", "attn_every", "hidden", "ffn", "vocab", "gdn_qk_heads",
                                           "gdn_v_heads", "attn_q_heads", "attn_kv_heads", "rope_dim", "ctx")] + [
        ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("seed", C.c_uint64), ("tp_rank", C.c_uint32),
        ("tp_size", C.c_uint32), ("ffn_gate_type", C.c_uint32)]


class q38_shard_info(C.Structure):
    _fields_ = [("qk_head0", C.c_uint32), ("qk_heads", C.c_uint32), ("v_heads", C.c_uint32),
                ("v_head", C.c_uint32 * 64), ("ffn_row0", C.c_uint32), ("ffn_row1", C.c_uint32),
                ("q_head0", C.c_uint32), ("q_heads", C.c_uint32), ("kv_head0", C.c_uint32), ("kv_heads", C.c_uint32),
                ("vocab0", C.c_uint32), ("vocab1", C.c_uint32)]


class q38_model_stats(C.Structure):
    _fields_ = [("weight_bytes_per_step", C.c_uint64), ("state_bytes_per_step", C.c_uint64),
                ("arena_bytes", C.c_uint64)]


_lib = None


def header_functions() -> list[str]:
    """Names of every function declared in include/q38rt.h."""
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"\b(q38_[a-z0-9_]+)\s*\(", text)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            raise Q38Error(5, f"{LIB} is missing: build it with `python -m qwen382743090_b200.build`")
        L = C.CDLL(str(LIB))
        u64, u32, sz, vp = C.c_uint64, C.c_uint32, C.c_size_t, C.c_void_p
        L.q38_last_error.restype = C.c_char_p
        L.q38_version.restype = C.c_char_p
        L.q38_device_count.argtypes = [C.POINTER(C.c_int)]
        L.q38_device_query.argtypes = [C.c_int, C.POINTER(q38_device_info)]
        L.q38_quantize_q8_1.argtypes = [u64, u32, u64, vp]
        L.q38_iq4xs_q8_1_gemv.argtypes = [u64, u64, u64, u32, u32, vp]
        L.q38_check_conv4.argtypes = [u64, u64, u64, u64, u64, u32, vp]
        L.q38_check_l2norm.argtypes = [u64, u32, u32, C.c_float, u64, vp]
        L.q38_check_beta_gate.argtypes = [u64, u64, u64, u64, u32, u64, u64, vp]
        L.q38_check_gdn.argtypes = [u64, u64, u64, u64, u64, u64, u64, u64, u32, u32, u32, vp]
        L.q38_check_rmsnorm.argtypes = [u64, u64, u64, u32, u32, C.c_float, u64, vp]
        L.q38_check_silu_mul.argtypes = [u64, u64, u32, u64, vp]
        L.q38_scratch_bytes.argtypes = [C.c_int, C.POINTER(sz)]
        L.q38_ctx_open.argtypes = [C.c_int, C.POINTER(vp)]
        L.q38_ctx_close.argtypes = [vp]
        L.q38_alloc.argtypes = [vp, sz, C.POINTER(u64)]
        L.q38_free.argtypes = [vp, u64]
        L.q38_memcpy_h2d.argtypes = [u64, vp, sz, vp]
        L.q38_memcpy_d2h.argtypes = [vp, u64, sz, vp]
        L.q38_memcpy_d2d.argtypes = [u64, u64, sz, vp]
        L.q38_memset_d8.argtypes = [u64, C.c_uint8, sz, vp]
        L.q38_stream_synchronize.argtypes = [vp]
        L.q38_fault_status.argtypes = [C.POINTER(u32)]
        L.q38_xpack_bytes.argtypes = [u32, u32, u32]
        L.q38_xpack_bytes.restype = sz
        L.q38_xpack_f32.argtypes = [u64, u32, u32, u64, vp]
        L.q38_xpack_f32_limbs.argtypes = [u64, u32, u32, u32, u64, vp]
        L.q38_xpack_q8k.argtypes = [u64, u32, u32, u64, vp]
        L.q38_gemv_packed.argtypes = [C.POINTER(q38_weight_desc), u64, u32, u32, u64, vp]
        L.q38_q5k_sm86_soa_gemv_vec.argtypes = [u64, u64, u64, u64, u64, u32, u32, vp]
        L.q38_q5k_sm86_soa_gemv_vec_noalloc.argtypes = [u64, u64, u64, u64, u64, u32, u32, vp]
        L.q38_q5k_sm86_soa_q8k_gemv.argtypes = [u64, u64, u64, u64, u64, u32, u32, vp]
        L.q38_q5k_tiled_gemv.argtypes = [u64, u64, u64, u32, u32, vp]
        L.q38_gemv_f32.argtypes = [C.POINTER(q38_weight_desc), u64, u64, vp]
        L.q38_gemv_f32_host.argtypes = [C.POINTER(q38_weight_desc), vp, vp, vp]
        L.q38_gemv_f32_host_fed.argtypes = [C.POINTER(q38_weight_desc), vp, vp, vp]
        L.q38_check_rows.argtypes = [C.POINTER(q38_weight_desc), u32, u64, u64, u64, vp]
        L.q38_quantize_q8k.argtypes = [u64, u32, u64, vp]
        L.q38_rmsnorm_q8k.argtypes = [u64, u64, u32, C.c_float, u64, u64, vp]
        L.q38_gemv_xfrag_pair.argtypes = [C.POINTER(q38_weight_desc), C.POINTER(q38_weight_desc), u64, u64, u64, vp]
        L.q38_gemv_q8k.argtypes = [C.POINTER(q38_weight_desc), u64, u64, vp]
        L.q38_gemm_f32.argtypes = [C.POINTER(q38_weight_desc), u64, u32, u64, vp]
        L.q38_gemm_f32_tc.argtypes = [C.POINTER(q38_weight_desc), u64, u32, u64, vp]
        f32 = C.c_float
        L.q38_rmsnorm.argtypes = [u64, u64, u64, u32, u32, f32, vp]
        L.q38_conv4_silu_roll.argtypes = [u64, u64, u64, u64, u64, u32, vp]
        L.q38_qk_l2norm.argtypes = [u64, u64, u64, u32, f32, vp]
        L.q38_beta_gate.argtypes = [u64, u64, u64, u64, u64, u64, u32, vp]
        L.q38_gdn_step.argtypes = [u64] * 8 + [u32, u32, f32, vp]
        L.q38_gated_rmsnorm_silu.argtypes = [u64, u64, u64, u64, u32, f32, vp]
        L.q38_add_residual.argtypes = [u64, u64, u64, u32, vp]
        L.q38_ffn_silu_mul.argtypes = [u64, u64, u64, u32, vp]
        L.q38_gdn_fused.argtypes = [C.POINTER(q38_gdn_fused_args), vp]
        L.q38_model_create.argtypes = [C.POINTER(q38_model_config), C.POINTER(vp)]
        L.q38_repack_tiled.argtypes = [u32, u64, u32, u32, u64, vp]
        L.q38_model_create_from_pack.argtypes = [C.POINTER(q38_model_config), vp, C.POINTER(vp)]
        L.q38_model_set_comm.argtypes = [vp, vp]
        L.q38_model_shard_info.argtypes = [C.POINTER(q38_model_config), C.POINTER(q38_shard_info)]
        L.q38_comm_unique_id.argtypes = [C.POINTER(C.c_uint8)]
        L.q38_comm_init.argtypes = [C.c_int, C.c_int, C.POINTER(C.c_uint8), C.POINTER(vp)]
        L.q38_comm_destroy.argtypes = [vp]
        L.q38_comm_allreduce_f32.argtypes = [vp, u64, sz, vp]
        L.q38_tp_exchange_bytes.argtypes = [u32]
        L.q38_tp_exchange_bytes.restype = sz
        L.q38_tp_exchange.argtypes = [C.POINTER(q38_tp_exchange_desc), vp]
        L.q38_model_destroy.argtypes = [vp]
        L.q38_model_info.argtypes = [vp, C.POINTER(q38_model_stats)]
        L.q38_model_set_position.argtypes = [vp, C.c_int32, C.c_int32, u64]
        L.q38_model_get_position.argtypes = [vp, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]
        L.q38_model_reset.argtypes = [vp, C.c_int32]
        L.q38_model_set_token.argtypes = [vp, C.c_int32]
        L.q38_model_step.argtypes = [vp, vp]
        L.q38_model_layer.argtypes = [vp, u32, u64, vp]
        L.q38_model_capture.argtypes = [vp, u32, vp]
        L.q38_model_replay.argtypes = [vp, vp]
        L.q38_model_tensor.argtypes = [vp, C.c_char_p, C.POINTER(q38_weight_desc)]
        for name in ("q38_q4k_gemv_f32", "q38_q5k_gemv_f32", "q38_q6k_gemv_f32", "q38_iq4xs_gemv_f32",
                     "q38_q5k_q8k_dp4a_gemv"):
            getattr(L, name).argtypes = [u64, u64, u64, u32, u32, vp]
        L.q38_q5k_tiled_bytes.argtypes = [u32, u32]
        L.q38_q5k_tiled_bytes.restype = sz
        L.q38_tiled_bytes.argtypes = [u32, u32, u32]
        L.q38_tiled_bytes.restype = sz
        L.q38_xfrag_bytes.argtypes = [u32, u32]
        L.q38_xfrag_bytes.restype = sz
        L.q38_xfrag_f32.argtypes = [u64, u32, u32, u64, vp]
        L.q38_xfrag_q8k.argtypes = [u64, u32, u32, u64, vp]
        L.q38_gemv_xfrag.argtypes = [C.POINTER(q38_weight_desc), u64, u64, vp]
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != Q38_OK:
        raise Q38Error(rc, lib().q38_last_error().decode())


def device_count() -> int:
    n = C.c_int(0)
    rc = lib().q38_device_count(C.byref(n))
    return n.value if rc == Q38_OK else 0


def device_query(dev: int = 0) -> q38_device_info:
    info = q38_device_info()
    check(lib().q38_device_query(dev, C.byref(info)))
    return info


@dataclass
class DeviceBuffer:
    ctx: "Context"
    ptr: int
    nbytes: int

    def upload(self, a: np.ndarray, offset: int = 0, stream=None) -> None:
        a = np.ascontiguousarray(a)
        if offset + a.nbytes > self.nbytes:
            raise ValueError("upload exceeds buffer")
        check(lib().q38_memcpy_h2d(self.ptr + offset, a.ctypes.data, a.nbytes, stream))
        if stream is None:
            check(lib().q38_stream_synchronize(None))

    def download(self, dtype, count: int, offset: int = 0, stream=None) -> np.ndarray:
        out = np.empty(count, dtype=dtype)
        if offset + out.nbytes > self.nbytes:
            raise ValueError("download exceeds buffer")
        check(lib().q38_memcpy_d2h(out.ctypes.data, self.ptr + offset, out.nbytes, stream))
        check(lib().q38_stream_synchronize(stream))
        return out

    def fill(self, value: int = 0) -> None:
        check(lib().q38_memset_d8(self.ptr, value, self.nbytes, None))
        check(lib().q38_stream_synchronize(None))

    def free(self) -> None:
        if self.ptr:
            check(lib().q38_free(self.ctx.handle, self.ptr))
            self.ptr = 0


class Context:
    """One device context (q38_ctx_open); allocations are VMM-backed."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        check(lib().q38_ctx_open(device, C.byref(h)))
        self.handle = h
        self.device = device

    def alloc(self, nbytes: int) -> DeviceBuffer:
        p = C.c_uint64(0)
        check(lib().q38_alloc(self.handle, max(1, int(nbytes)), C.byref(p)))
        return DeviceBuffer(self, p.value, int(nbytes))

    def upload(self, a: np.ndarray) -> DeviceBuffer:
        a = np.ascontiguousarray(a)
        b = self.alloc(a.nbytes)
        b.upload(a)
        return b

    def close(self) -> None:
        if self.handle:
            check(lib().q38_ctx_close(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def synchronize(stream=None) -> None:
    check(lib().q38_stream_synchronize(stream))


def scratch_bytes(dev: int = 0) -> int:
    """Bytes of lazily grown device scratch the library holds on dev
    (q38_scratch_bytes)."""
    n = C.c_size_t()
    check(lib().q38_scratch_bytes(dev, C.byref(n)))
    return int(n.value)


def fault_status() -> int:
    s = C.c_uint32(0)
    check(lib().q38_fault_status(C.byref(s)))
    return s.value


def fault_clear() -> None:
    check(lib().q38_fault_clear())


def xpack_bytes(nl: int, cols: int, batch: int = 1) -> int:
    return int(lib().q38_xpack_bytes(nl, cols, batch))


def xpack_f32(x: int, cols: int, batch: int, xpack: int, stream=None) -> None:
    check(lib().q38_xpack_f32(x, cols, batch, xpack, stream))


def xpack_f32_limbs(x: int, cols: int, batch: int, nl: int, xpack: int, stream=None) -> None:
    check(lib().q38_xpack_f32_limbs(x, cols, batch, nl, xpack, stream))


def f32_limbs(cols: int) -> int:
    """Limb count the library's own f32 entry points use for an x-pack of `cols`."""
    return 3 if cols <= 6144 else 4


def xpack_q8k(xq8: int, cols: int, batch: int, xpack: int, stream=None) -> None:
    check(lib().q38_xpack_q8k(xq8, cols, batch, xpack, stream))


def weight_desc(ggml_type: int, layout: int, rows: int, cols: int, data: int, aux0: int = 0,
                aux1: int = 0) -> q38_weight_desc:
    return q38_weight_desc(ggml_type, layout, rows, cols, data, aux0, aux1)


def gemv_packed(desc: q38_weight_desc, xpack: int, nl: int, batch: int, y: int, stream=None) -> None:
    check(lib().q38_gemv_packed(C.byref(desc), xpack, nl, batch, y, stream))


def gemv_f32(desc: q38_weight_desc, x: int, y: int, stream=None) -> None:
    check(lib().q38_gemv_f32(C.byref(desc), x, y, stream))


def tp_exchange_bytes(n: int) -> int:
    return int(lib().q38_tp_exchange_bytes(n))


def tp_exchange(x_in: int, x_out: int, part: int, regions, step: int, n: int, rank: int, size: int,
                instance: int, norm_w: int = 0, xfrag: int = 0, eps: float = 1e-6, stream=None) -> None:
    """One tensor-parallel exchange (q38_tp_exchange); regions: device
    addresses of every rank's exchange region as mapped in this process."""
    d = q38_tp_exchange_desc()
    d.x_in, d.x_out, d.part, d.step, d.norm_w, d.xfrag = x_in, x_out, part, step, norm_w, xfrag
    for i, r in enumerate(regions):
        d.region[i] = r
    d.n, d.rank, d.size, d.instance, d.eps = n, rank, size, instance, eps
    check(lib().q38_tp_exchange(C.byref(d), stream))


def gemv_xfrag_pair(wa: q38_weight_desc, wb: q38_weight_desc, xfrag: int, ya: int, yb: int, stream=None) -> None:
    """ya = Wa x and yb = Wb x in one launch (layout 2, one Q5_K and one Q4_K)."""
    check(lib().q38_gemv_xfrag_pair(C.byref(wa), C.byref(wb), xfrag, ya, yb, stream))


def quantize_q8k(x: int, cols: int, out: int, stream=None) -> None:
    """f32 x [cols] -> Q8_K blocks on the device (q38_quantize_q8k)."""
    check(lib().q38_quantize_q8k(x, cols, out, stream))


def rmsnorm_q8k(x: int, w: int, n: int, eps: float, out: int, y: int = 0, stream=None) -> None:
    """Q8_K blocks of RMSNorm(x) * w (q38_rmsnorm_q8k); y optionally gets the f32 values."""
    check(lib().q38_rmsnorm_q8k(x, w, n, eps, y, out, stream))


def check_rows(desc: q38_weight_desc, nrows: int, x: int = 0, y64: int = 0, deq: int = 0, stream=None) -> None:
    """Plain device reference of the first nrows rows: FP64 dots with x and/or
    the dequantised f32 weights (q38_check_rows)."""
    check(lib().q38_check_rows(C.byref(desc), nrows, x, y64, deq, stream))


def quantize_q8_1(x: int, cols: int, out: int, stream=None) -> None:
    """f32 x -> Q8_1 blocks (q38_quantize_q8_1)."""
    check(lib().q38_quantize_q8_1(x, cols, out, stream))


def iq4xs_q8_1_gemv(w: int, xq81: int, y: int, cols: int, rows: int, stream=None) -> None:
    """y = W x for IQ4_XS blocks and Q8_1 x (q38_iq4xs_q8_1_gemv)."""
    check(lib().q38_iq4xs_q8_1_gemv(w, xq81, y, cols, rows, stream))


def check_conv4(qkv: int, w: int, state_in: int, out: int, state_out: int, channels: int, stream=None) -> None:
    check(lib().q38_check_conv4(qkv, w, state_in, out, state_out, channels, stream))


def check_l2norm(x: int, heads: int, dim: int, eps: float, y: int, stream=None) -> None:
    check(lib().q38_check_l2norm(x, heads, dim, eps, y, stream))


def check_beta_gate(b: int, a: int, dt: int, A: int, n: int, beta: int, gate: int, stream=None) -> None:
    check(lib().q38_check_beta_gate(b, a, dt, A, n, beta, gate, stream))


def check_gdn(q: int, k: int, v: int, g: int, beta: int, st_in: int, out: int, st_out: int, hq: int, hv: int,
              dim: int, stream=None) -> None:
    check(lib().q38_check_gdn(q, k, v, g, beta, st_in, out, st_out, hq, hv, dim, stream))


def check_rmsnorm(x: int, w: int, z: int, groups: int, dim: int, eps: float, y: int, stream=None) -> None:
    check(lib().q38_check_rmsnorm(x, w, z, groups, dim, eps, y, stream))


def check_silu_mul(g: int, u: int, n: int, y: int, stream=None) -> None:
    check(lib().q38_check_silu_mul(g, u, n, y, stream))


def gemv_f32_host(desc: q38_weight_desc, x_host: int, y_host: int, stream=None) -> None:
    """y = W x with x and y in page-locked host memory (addresses as ints)."""
    check(lib().q38_gemv_f32_host(C.byref(desc), x_host, y_host, stream))


def gemv_f32_host_fed(desc: q38_weight_desc, x_host: int, y_host: int, stream=None) -> None:
    """gemv_f32_host for x written by the host (not by earlier device work on the stream)."""
    check(lib().q38_gemv_f32_host_fed(C.byref(desc), x_host, y_host, stream))


def gemm_f32(desc: q38_weight_desc, x: int, batch: int, y: int, stream=None) -> None:
    """Y[b] = W X[b] for batch rows (x [batch][cols], y [batch][rows])."""
    check(lib().q38_gemm_f32(C.byref(desc), x, batch, y, stream))


def gemm_f32_tc(desc: q38_weight_desc, x: int, batch: int, y: int, stream=None) -> None:
    """Y[b] = W X[b] on tcgen05 (kind::i8, TMEM accumulators); Q5_K / Q4_K layout 2."""
    check(lib().q38_gemm_f32_tc(C.byref(desc), x, batch, y, stream))


def gemv_q8k(desc: q38_weight_desc, xq8: int, y: int, stream=None) -> None:
    check(lib().q38_gemv_q8k(C.byref(desc), xq8, y, stream))


# Drop-ins named after the reference's PTX entries (weights, x, y, cols, rows).
REFERENCE_GEMV_ENTRIES = {12: "q38_q4k_gemv_f32", 13: "q38_q5k_gemv_f32", 14: "q38_q6k_gemv_f32",
                          23: "q38_iq4xs_gemv_f32"}


def reference_gemv_f32(ggml_type: int, w: int, x: int, y: int, cols: int, rows: int, stream=None) -> None:
    check(getattr(lib(), REFERENCE_GEMV_ENTRIES[ggml_type])(w, x, y, cols, rows, stream))


def q5k_q8k_dp4a_gemv(w: int, xq8: int, y: int, cols: int, rows: int, stream=None) -> None:
    check(lib().q38_q5k_q8k_dp4a_gemv(w, xq8, y, cols, rows, stream))


def q5k_soa_gemv(meta: int, qh: int, qs: int, x: int, y: int, cols: int, rows: int, stream=None) -> None:
    check(lib().q38_q5k_sm86_soa_gemv_vec(meta, qh, qs, x, y, cols, rows, stream))


def q5k_soa_gemv_noalloc(meta: int, qh: int, qs: int, x: int, y: int, cols: int, rows: int, stream=None) -> None:
    """q5k_soa_gemv through the fixed device scratch: allocates nothing, cols <= 32768,
    and overlapping calls on one device race on the scratch."""
    check(lib().q38_q5k_sm86_soa_gemv_vec_noalloc(meta, qh, qs, x, y, cols, rows, stream))


def q5k_soa_q8k_gemv(meta: int, qh: int, qs: int, xq8: int, y: int, cols: int, rows: int, stream=None) -> None:
    check(lib().q38_q5k_sm86_soa_q8k_gemv(meta, qh, qs, xq8, y, cols, rows, stream))


def q5k_tiled_bytes(cols: int, rows: int) -> int:
    return int(lib().q38_q5k_tiled_bytes(cols, rows))


def tiled_bytes(ggml_type: int, cols: int, rows: int) -> int:
    """Bytes of a Q5_K / Q4_K / Q6_K matrix in layout 2 (0 if the shape or type does not fit)."""
    return int(lib().q38_tiled_bytes(ggml_type, cols, rows))


def repack_tiled(ggml_type: int, blocks: int, cols: int, rows: int, tiles: int, stream=None) -> None:
    """GGUF blocks on the device -> layout-2 tiles on the device (q38_repack_tiled)."""
    check(lib().q38_repack_tiled(ggml_type, blocks, cols, rows, tiles, stream))


def xfrag_bytes(cols: int, batch: int = 1) -> int:
    return int(lib().q38_xfrag_bytes(cols, batch))


def xfrag_f32(x: int, cols: int, batch: int, xfrag: int, stream=None) -> None:
    """f32 activations -> x-fragments (the activation format of layout-2 GEMVs)."""
    check(lib().q38_xfrag_f32(x, cols, batch, xfrag, stream))


def xfrag_q8k(xq8: int, cols: int, batch: int, xfrag: int, stream=None) -> None:
    check(lib().q38_xfrag_q8k(xq8, cols, batch, xfrag, stream))


def gemv_xfrag(desc: "q38_weight_desc", xfrag: int, y: int, stream=None) -> None:
    """y = W x for layout-2 weights from pre-packed x-fragments (tensor-core GEMV)."""
    check(lib().q38_gemv_xfrag(C.byref(desc), xfrag, y, stream))


def q5k_tiled_gemv(w: int, x: int, y: int, cols: int, rows: int, stream=None) -> None:
    check(lib().q38_q5k_tiled_gemv(w, x, y, cols, rows, stream))


# ---- layer ops ----------------------------------------------------------------

def rmsnorm(x: int, w: int, y: int, n: int, rows: int = 1, eps: float = 1e-6, stream=None) -> None:
    check(lib().q38_rmsnorm(x, w, y, n, rows, eps, stream))


def conv4_silu_roll(qkv: int, weight: int, state_in: int, conv_out: int, state_out: int, channels: int,
                    stream=None) -> None:
    check(lib().q38_conv4_silu_roll(qkv, weight, state_in, conv_out, state_out, channels, stream))


def qk_l2norm(conv: int, q: int, k: int, qk_heads: int, eps: float = 1e-6, stream=None) -> None:
    check(lib().q38_qk_l2norm(conv, q, k, qk_heads, eps, stream))


def beta_gate(beta_raw: int, alpha_raw: int, dt_bias: int, ssm_a: int, beta: int, gate: int, heads: int,
              stream=None) -> None:
    check(lib().q38_beta_gate(beta_raw, alpha_raw, dt_bias, ssm_a, beta, gate, heads, stream))


def gdn_step(q: int, k: int, v: int, gate: int, beta: int, state_in: int, out: int, state_out: int, qk_heads: int,
             value_heads: int, scale: float, stream=None) -> None:
    check(lib().q38_gdn_step(q, k, v, gate, beta, state_in, out, state_out, qk_heads, value_heads, scale, stream))


def gated_rmsnorm_silu(inp: int, weight: int, z: int, out: int, heads: int, eps: float = 1e-6, stream=None) -> None:
    check(lib().q38_gated_rmsnorm_silu(inp, weight, z, out, heads, eps, stream))


def add_residual(x: int, residual: int, out: int, n: int, stream=None) -> None:
    check(lib().q38_add_residual(x, residual, out, n, stream))


def ffn_silu_mul(gate: int, up: int, out: int, n: int, stream=None) -> None:
    check(lib().q38_ffn_silu_mul(gate, up, out, n, stream))


def gdn_fused(args: q38_gdn_fused_args, stream=None) -> None:
    check(lib().q38_gdn_fused(C.byref(args), stream))


# ---- decode engine ------------------------------------------------------------------

QWEN_HYBRID_64 = dict(n_layers=64, attn_every=4, hidden=5120, ffn=17408, vocab=151936, gdn_qk_heads=16,
                      gdn_v_heads=48, attn_q_heads=24, attn_kv_heads=4, rope_dim=64, ctx=4096 + 256,
                      rope_theta=1.0e7, rms_eps=1e-6, seed=1234, tp_rank=0, tp_size=1, ffn_gate_type=0)


def shard_info(**cfg) -> q38_shard_info:
    """The slice a tensor-parallel rank holds (host-side plan, no device)."""
    full = dict(QWEN_HYBRID_64)
    full.update(cfg)
    out = q38_shard_info()
    check(lib().q38_model_shard_info(C.byref(q38_model_config(**full)), C.byref(out)))
    return out


class Comm:
    """NCCL communicator over this process's current device (q38_comm_*)."""

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_uint8 * 128)()
        check(lib().q38_comm_unique_id(buf))
        return bytes(buf)

    def __init__(self, nranks: int, rank: int, uid: bytes):
        buf = (C.c_uint8 * 128).from_buffer_copy(uid)
        h = C.c_void_p()
        check(lib().q38_comm_init(nranks, rank, buf, C.byref(h)))
        self.handle = h

    def allreduce_f32(self, ptr: int, count: int, stream=None) -> None:
        check(lib().q38_comm_allreduce_f32(self.handle, ptr, count, stream))

    def close(self):
        if self.handle:
            check(lib().q38_comm_destroy(self.handle))
            self.handle = None


class Model:
    """The hybrid model on the current device (q38_model_*): seeded weights, or
    with `pack` (a path or an open q38pack.Pack) the pack's weights, this
    rank's shard of them (q38_model_create_from_pack)."""

    def __init__(self, pack=None, **cfg):
        full = dict(QWEN_HYBRID_64)
        full.update(cfg)
        self.cfg = full
        c = q38_model_config(**full)
        h = C.c_void_p()
        if pack is None:
            check(lib().q38_model_create(C.byref(c), C.byref(h)))
        else:
            from . import q38pack
            own = not isinstance(pack, q38pack.Pack)
            p = q38pack.open_pack(pack) if own else pack
            try:
                check(lib().q38_model_create_from_pack(C.byref(c), p.handle, C.byref(h)))
            finally:
                if own:
                    p.close()
        self.handle = h

    def close(self):
        if self.handle:
            check(lib().q38_model_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def set_comm(self, comm: "Comm") -> None:
        check(lib().q38_model_set_comm(self.handle, comm.handle))

    def info(self) -> q38_model_stats:
        st = q38_model_stats()
        check(lib().q38_model_info(self.handle, C.byref(st)))
        return st

    def set_position(self, token: int, pos: int, kv_seed: int = 7) -> None:
        check(lib().q38_model_set_position(self.handle, token, pos, kv_seed))

    def position(self) -> tuple[int, int]:
        t, p = C.c_int32(), C.c_int32()
        check(lib().q38_model_get_position(self.handle, C.byref(t), C.byref(p)))
        return t.value, p.value

    def reset(self, token: int) -> None:
        """A fresh sequence: zero recurrent states, position 0, next input `token`."""
        check(lib().q38_model_reset(self.handle, token))

    def set_token(self, token: int) -> None:
        """The next step's input token (position and caches kept)."""
        check(lib().q38_model_set_token(self.handle, token))

    def step(self, stream=None) -> None:
        check(lib().q38_model_step(self.handle, stream))

    def layer(self, layer: int, x: int, stream=None) -> None:
        check(lib().q38_model_layer(self.handle, layer, x, stream))

    def capture(self, steps: int, stream) -> None:
        check(lib().q38_model_capture(self.handle, steps, stream))

    def replay(self, stream) -> None:
        check(lib().q38_model_replay(self.handle, stream))

    def tensor(self, name: str) -> q38_weight_desc:
        d = q38_weight_desc()
        check(lib().q38_model_tensor(self.handle, name.encode(), C.byref(d)))
        return d

    def download(self, name: str) -> tuple[q38_weight_desc, np.ndarray]:
        """Raw bytes of a named tensor as stored (tiles for layout 2)."""
        d = self.tensor(name)
        if d.ggml_type == 0:
            n = 4 * d.cols
        elif d.layout == 2:
            n = tiled_bytes(d.ggml_type, d.cols, d.rows)
        else:
            n = d.rows * (d.cols // 256) * {12: 144, 13: 176, 14: 210, 23: 136}[d.ggml_type]
        out = np.empty(n, dtype=np.uint8)
        check(lib().q38_memcpy_d2h(out.ctypes.data, d.data, n, None))
        check(lib().q38_stream_synchronize(None))
        return d, out
