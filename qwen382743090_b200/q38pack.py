"""Q38PACK container: reader (through the library's mmap reader), writer and
the B200 converter.

The byte format is the reference's (docs/Q38PACK.md; tools/q38pack_format.py
HEADER_STRUCT / ENTRY_STRUCT_V2): a 256-byte little-endian header, 256-byte
tensor directory entries, a JSON manifest, the source GGUF metadata, then the
tensor payloads at `alignment`.  Version 3 is this library's: entries are the
v2 layout and layout 2 (B200 fragment tiles of 8 rows x 2 super-blocks for
Q5_K and Q4_K, synth.repack_tiled) is allowed.  A reference reader accepts
versions 1..2 only, so it rejects a v3 pack instead of handing a tiled tensor
to a kernel that cannot read it.

`convert_to_b200` rewrites a v1/v2 pack with every Q5_K and Q4_K matrix whose
K is a multiple of 512 in layout 2 (from GGUF blocks or from the SoA planes;
the decoded weights are unchanged), everything else copied byte for byte.
"""
from __future__ import annotations

import ctypes as C
import json
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import runtime as rt
from . import synth

MAGIC = b"Q38PACK\0"
VERSION = 3
HEADER_BYTES = 256
ENTRY_BYTES = 256
HEADER_FMT = struct.Struct("<8sIIIIIIQQQQQQQQQQ")
ENTRY_FMT = struct.Struct("<160sII4Q3QIIIIQQ")

ROLE = {"unknown": 0, "embedding": 1, "output_norm": 2, "output": 3, "attention": 4, "deltanet": 5, "ffn": 6,
        "norm": 7, "mtp": 8}
LAYOUT_NAME = {0: "GGUF_NATIVE", 1: "SM86_Q5K_SOA", 2: "B200_TILED"}
TYPE_NAME = {0: "F32", 1: "F16", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K", 15: "Q8_K", 23: "IQ4_XS"}
BLOCK_BYTES = {12: 144, 13: 176, 14: 210, 23: 136}


class q38_pack_header_info(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("version", "header_bytes", "flags", "tensor_count", "alignment")] + [
        (n, C.c_uint64) for n in ("directory_offset", "directory_bytes", "manifest_offset", "manifest_bytes",
                                  "raw_gguf_meta_offset", "raw_gguf_meta_bytes", "data_offset", "data_bytes",
                                  "source_file_size", "source_data_offset")]


class q38_tensor_record(C.Structure):
    _fields_ = [("name", C.c_char * 164), ("ndim", C.c_uint32), ("ggml_type", C.c_uint32),
                ("dims", C.c_uint64 * 4), ("data_offset", C.c_uint64), ("stored_bytes", C.c_uint64),
                ("source_offset", C.c_uint64), ("role", C.c_uint32), ("flags", C.c_uint32), ("layout", C.c_uint32),
                ("layout_flags", C.c_uint32), ("aux0_offset", C.c_uint64), ("aux1_offset", C.c_uint64)]


class q38_plan_stats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("page_bytes", "tensor_payload_bytes", "reserved_va_bytes",
                                          "page_padding_bytes", "page_count")]


def _bind():
    L = rt.lib()
    if getattr(L, "_q38pack_bound", False):
        return L
    vp, u32, u64 = C.c_void_p, C.c_uint32, C.c_uint64
    L.q38_pack_open.argtypes = [C.c_char_p, C.POINTER(vp)]
    L.q38_pack_close.argtypes = [vp]
    L.q38_pack_header.argtypes = [vp, C.POINTER(q38_pack_header_info)]
    L.q38_pack_tensor.argtypes = [vp, u32, C.POINTER(q38_tensor_record)]
    L.q38_pack_find.argtypes = [vp, C.c_char_p, C.POINTER(u32)]
    L.q38_pack_host_data.argtypes = [vp, u32, C.POINTER(vp)]
    L.q38_pack_plan.argtypes = [vp, u64, C.POINTER(q38_plan_stats), C.POINTER(u64)]
    L.q38_pack_upload.argtypes = [vp, vp, u64, C.POINTER(u64)]
    L.q38_pack_weight_desc.argtypes = [vp, u32, u64, C.POINTER(rt.q38_weight_desc)]
    L._q38pack_bound = True
    return L


class Pack:
    """An open Q38PACK file (q38_pack_open); payloads are views of the mmap."""

    def __init__(self, path):
        L = _bind()
        h = C.c_void_p()
        rt.check(L.q38_pack_open(str(path).encode(), C.byref(h)))
        self.handle = h
        self.header = q38_pack_header_info()
        rt.check(L.q38_pack_header(h, C.byref(self.header)))
        self.tensors = []
        for i in range(self.header.tensor_count):
            r = q38_tensor_record()
            rt.check(L.q38_pack_tensor(h, i, C.byref(r)))
            self.tensors.append(r)

    def close(self):
        if self.handle:
            rt.check(rt.lib().q38_pack_close(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def find(self, name: str) -> int:
        i = C.c_uint32()
        rt.check(rt.lib().q38_pack_find(self.handle, name.encode(), C.byref(i)))
        return i.value

    def data(self, index: int) -> np.ndarray:
        """The stored bytes of tensor `index` (a read-only view of the mapping)."""
        p = C.c_void_p()
        rt.check(rt.lib().q38_pack_host_data(self.handle, index, C.byref(p)))
        n = self.tensors[index].stored_bytes
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(C.c_uint8)), shape=(n,)) if n else np.zeros(0, np.uint8)

    def plan(self, page_bytes: int = 2 << 20) -> tuple[q38_plan_stats, np.ndarray]:
        st = q38_plan_stats()
        off = (C.c_uint64 * max(1, len(self.tensors)))()
        rt.check(rt.lib().q38_pack_plan(self.handle, page_bytes, C.byref(st), off))
        return st, np.array(off[: len(self.tensors)], dtype=np.uint64)

    def upload(self, ctx: rt.Context, page_bytes: int = 2 << 20) -> int:
        base = C.c_uint64()
        rt.check(rt.lib().q38_pack_upload(self.handle, ctx.handle, page_bytes, C.byref(base)))
        return base.value

    def weight_desc(self, index: int, base: int) -> rt.q38_weight_desc:
        d = rt.q38_weight_desc()
        rt.check(rt.lib().q38_pack_weight_desc(self.handle, index, base, C.byref(d)))
        return d

    def manifest(self) -> dict:
        with open(self._path_of(), "rb") as f:
            f.seek(self.header.manifest_offset)
            raw = f.read(self.header.manifest_bytes)
        return json.loads(raw) if raw else {}

    def _path_of(self):
        return self._path

    def blocks(self, index: int) -> np.ndarray:
        """Row-major GGUF blocks of a quantised tensor, whatever its layout."""
        t = self.tensors[index]
        rows, cols = int(t.dims[1]), int(t.dims[0])
        raw = self.data(index)
        if t.layout == 0:
            return raw[: rows * (cols // 256) * BLOCK_BYTES[t.ggml_type]]
        if t.layout == 1:
            n = rows * (cols // 256)
            qh = int(t.aux0_offset - t.data_offset)
            qs = int(t.aux1_offset - t.data_offset)
            meta = raw[: n * 20].reshape(n, 20)
            out = np.empty((n, 176), np.uint8)
            out[:, 0:4] = meta[:, 0:4]
            out[:, 4:16] = synth.pack_scale_min_k4(meta[:, 4:20:2], meta[:, 5:20:2])
            out[:, 16:48] = raw[qh: qh + n * 32].reshape(n, 32)
            out[:, 48:176] = raw[qs: qs + n * 128].reshape(n, 128)
            return out.reshape(-1)
        return synth.untile(t.ggml_type, raw[: synth.tiled_bytes(t.ggml_type, rows, cols)], rows, cols)


def open_pack(path) -> Pack:
    p = Pack(path)
    p._path = str(path)
    return p


@dataclass
class Tensor:
    """One tensor to write: GGUF dims (dims[0] = K), type, role, layout and the
    payload planes (one array, or META/QH/QS for layout 1)."""
    name: str
    ggml_type: int
    dims: tuple
    payload: list = field(default_factory=list)
    role: int = 0
    flags: int = 0
    layout: int = 0
    source_offset: int = 0


class LazyPlane:
    """A payload plane of known size whose bytes are produced when the pack is
    written (fn() -> uint8 array of nbytes), so a large model is written one
    tensor at a time."""

    def __init__(self, nbytes: int, fn):
        self.nbytes = int(nbytes)
        self.fn = fn


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def write_pack(path, tensors: list[Tensor], manifest: dict | None = None, raw_meta: bytes = b"",
               alignment: int = 128, version: int = VERSION, source_file_size: int = 0,
               source_data_offset: int = 0) -> None:
    """Write a Q38PACK file.  Layout-1 tensors take [META, QH, QS] planes, each
    starting on `alignment`; every other tensor takes one payload array."""
    man = json.dumps(manifest or {}, separators=(",", ":")).encode()
    n = len(tensors)
    dir_off = HEADER_BYTES
    man_off = dir_off + n * ENTRY_BYTES
    raw_off = man_off + len(man)
    data_off = _align(raw_off + len(raw_meta), alignment)
    cursor = data_off
    entries, chunks = [], []
    for t in tensors:
        cursor = _align(cursor, alignment)
        start = cursor
        offs = []
        for k, plane in enumerate(t.payload):
            if k:
                cursor = _align(cursor, alignment)
            offs.append(cursor)
            b = plane if isinstance(plane, LazyPlane) else np.ascontiguousarray(plane, dtype=np.uint8).reshape(-1)
            chunks.append((cursor, b))
            cursor += b.nbytes
        aux0 = offs[1] if t.layout == 1 else 0
        aux1 = offs[2] if t.layout == 1 else 0
        dims = list(t.dims) + [1] * (4 - len(t.dims))
        entries.append(ENTRY_FMT.pack(t.name.encode()[:160].ljust(160, b"\0"), len(t.dims), t.ggml_type, *dims,
                                      start, cursor - start, t.source_offset, t.role, t.flags, t.layout, 0, aux0,
                                      aux1))
    data_bytes = cursor - data_off
    hdr = HEADER_FMT.pack(MAGIC, version, HEADER_BYTES, 0, n, alignment, 0, dir_off, n * ENTRY_BYTES, man_off,
                          len(man), raw_off, len(raw_meta), data_off, data_bytes, source_file_size,
                          source_data_offset)
    with open(path, "wb") as f:
        f.write(hdr + bytes(HEADER_BYTES - len(hdr)))
        for e in entries:
            f.write(e + bytes(ENTRY_BYTES - len(e)))
        f.write(man)
        f.write(raw_meta)
        for off, b in chunks:
            f.seek(off)
            if isinstance(b, LazyPlane):
                arr = np.ascontiguousarray(b.fn(), dtype=np.uint8).reshape(-1)
                if arr.nbytes != b.nbytes:
                    raise ValueError(f"lazy plane produced {arr.nbytes} bytes, declared {b.nbytes}")
                b = arr
            f.write(memoryview(b))
        f.truncate(cursor)


def convert_to_b200(src, dst, alignment: int = 128) -> dict:
    """v1/v2 (or v3) pack -> v3 pack with Q5_K and Q4_K matrices in layout 2.
    Returns a summary {converted, copied, bytes_before, bytes_after}."""
    with open_pack(src) as p:
        man = p.manifest()
        with open(src, "rb") as f:
            f.seek(p.header.raw_gguf_meta_offset)
            raw_meta = f.read(p.header.raw_gguf_meta_bytes)
        out, conv = [], 0
        before = after = 0
        for i, t in enumerate(p.tensors):
            dims = tuple(int(d) for d in t.dims[: t.ndim])
            before += t.stored_bytes
            if t.ggml_type in (12, 13) and t.ndim == 2 and dims[0] % 512 == 0:
                rows, cols = dims[1], dims[0]
                tiles = synth.repack_tiled(t.ggml_type, p.blocks(i), rows, cols)
                out.append(Tensor(t.name.decode(), t.ggml_type, dims, [tiles], t.role, t.flags, 2, t.source_offset))
                conv += 1
                after += tiles.nbytes
            else:
                planes = [np.array(p.data(i))]
                if t.layout == 1:  # keep the planes, re-aligned in the new file
                    raw = planes[0]
                    qh, qs = int(t.aux0_offset - t.data_offset), int(t.aux1_offset - t.data_offset)
                    nblk = int(t.dims[1]) * (int(t.dims[0]) // 256)
                    planes = [raw[: nblk * 20], raw[qh: qh + nblk * 32], raw[qs: qs + nblk * 128]]
                out.append(Tensor(t.name.decode(), t.ggml_type, dims, planes, t.role, t.flags, t.layout,
                                  t.source_offset))
                after += sum(x.nbytes for x in planes)
        man = dict(man)
        man["q38rt_b200"] = {"layout2_tensors": conv,
                             "tile": "8 rows x 2 super-blocks (Q5_K 2880 B, Q4_K 2368 B)"}
        write_pack(dst, out, man, raw_meta, alignment, VERSION, p.header.source_file_size,
                   p.header.source_data_offset)
    return {"converted": conv, "copied": len(out) - conv, "bytes_before": before, "bytes_after": after}


def synthetic_pack(path, seed: int = 1234, hidden: int = 1024, layers: int = 1, q5k_layout: int = 1,
                   version: int = 2) -> list[str]:
    """A small seeded pack with the reference's tensor roles and types:
    Q5_K attention/deltanet projections (in `q5k_layout`), Q4_K and IQ4_XS ffn,
    Q6_K output, F32 norms.  Returns the tensor names."""
    ts = []
    rng_seed = seed
    for L in range(layers):
        for name, t, rows, role in ((f"blk.{L}.attn_qkv.weight", 13, 2 * hidden, ROLE["deltanet"]),
                                    (f"blk.{L}.attn_gate.weight", 13, hidden + 512, ROLE["deltanet"]),
                                    (f"blk.{L}.ssm_beta.weight", 12, 48, ROLE["deltanet"]),
                                    (f"blk.{L}.ffn_gate.weight", 23, 2 * hidden, ROLE["ffn"]),
                                    (f"blk.{L}.ffn_up.weight", 12, 2 * hidden, ROLE["ffn"])):
            rng_seed += 1
            blocks = synth.gen_blocks(t, rows, hidden, rng_seed)
            if t == 13 and q5k_layout == 1:
                meta, qh, qs = synth.q5k_soa_records(blocks)
                ts.append(Tensor(name, 13, (hidden, rows), [meta, qh, qs], role, 0, 1))
            elif t == 13 and q5k_layout == 2:
                ts.append(Tensor(name, 13, (hidden, rows), [synth.repack_q5k_tiled(blocks, rows, hidden)], role, 0, 2))
            else:
                ts.append(Tensor(name, t, (hidden, rows), [blocks], role))
        norm = synth.gen_f32(hidden, rng_seed, 0.1, 1.0)
        ts.append(Tensor(f"blk.{L}.attn_norm.weight", 0, (hidden,), [norm.view(np.uint8)], ROLE["norm"]))
    rng_seed += 1
    ts.append(Tensor("output.weight", 14, (hidden, 512), [synth.gen_blocks(14, 512, hidden, rng_seed)],
                     ROLE["output"]))
    write_pack(path, ts, {"synthetic": True, "seed": seed, "hidden": hidden}, b"GGUF-meta-placeholder",
               version=max(version, 3 if q5k_layout == 2 else version))
    return [t.name for t in ts]


# The recurrent decoder layer of the reference's model, as its Runtime finds it
# (src/runtime.cpp:368-460): names, GGML types, execution layouts and dims.
LAYER_TENSORS = (
    # suffix, type, dims (K, N), layout
    ("attn_norm.weight", 0, (5120,), 0),
    ("attn_qkv.weight", 13, (5120, 10240), 1),
    ("attn_gate.weight", 13, (5120, 6144), 1),
    ("ssm_beta.weight", 12, (5120, 48), 0),
    ("ssm_alpha.weight", 12, (5120, 48), 0),
    ("ssm_conv1d.weight", 0, (4, 10240), 0),
    ("ssm_dt.bias", 0, (48,), 0),
    ("ssm_a", 0, (48,), 0),
    ("ssm_norm.weight", 0, (128,), 0),
    ("ssm_out.weight", 13, (6144, 5120), 1),
    ("post_attention_norm.weight", 0, (5120,), 0),
    ("ffn_gate.weight", 23, (5120, 17408), 0),
    ("ffn_up.weight", 13, (5120, 17408), 1),
    ("ffn_down.weight", 13, (17408, 5120), 1),
)


def synthetic_layer_pack(path, seed: int = 1234, layers=(0,), d_exp: int = -17) -> list[str]:
    """A seeded v2 pack holding the recurrent layers `layers` with the
    reference's tensor names, types, layouts and shapes (hidden 5120, qkv
    10240, z 6144, 48 beta/alpha rows, conv [10240][4], 128-wide gated norm,
    FFN 17408 with an IQ4_XS gate): what q38::Runtime::run_layer0_full /
    run_recurrent_layer read.  Quantised weights use d = |N(0,1)| * 2^d_exp
    so activations stay O(1) through the layer; norms are 1 + N(0, 0.1),
    conv weights N(0, 0.3), dt_bias N(0, 0.5), A = -exp(N(0, 0.5))."""
    roles = {"attn": ROLE["deltanet"], "ssm": ROLE["deltanet"], "ffn": ROLE["ffn"], "post": ROLE["norm"]}
    ts = []
    k = seed
    for L in layers:
        for suffix, ty, dims, layout in LAYER_TENSORS:
            k += 1
            name = f"blk.{L}.{suffix}"
            role = ROLE["norm"] if "norm" in suffix else roles.get(suffix.split("_")[0], ROLE["deltanet"])
            if ty == 0:
                n = int(np.prod(dims))
                if suffix.endswith("norm.weight"):
                    v = synth.gen_f32(n, k, 0.1, 1.0)
                elif suffix == "ssm_conv1d.weight":
                    v = synth.gen_f32(n, k, 0.3)
                elif suffix == "ssm_dt.bias":
                    v = synth.gen_f32(n, k, 0.5)
                else:
                    v = (-np.exp(synth.gen_f32(n, k, 0.5))).astype(np.float32)
                ts.append(Tensor(name, 0, dims, [v.view(np.uint8)], role))
                continue
            cols, rows = dims
            blocks = synth.gen_blocks(ty, rows, cols, k, d_exp)
            if layout == 1:
                meta, qh, qs = synth.q5k_soa_records(blocks)
                ts.append(Tensor(name, 13, dims, [meta, qh, qs], role, 0, 1))
            else:
                ts.append(Tensor(name, ty, dims, [blocks], role))
    write_pack(path, ts, {"synthetic": True, "seed": seed, "layers": list(layers)}, b"GGUF-meta-placeholder",
               version=2)
    return [t.name for t in ts]


def model_tensor_names(cfg: dict) -> list[str]:
    """The pack tensors q38_model_create_from_pack reads for a model config,
    in the order export_model_pack writes them (the reference's names)."""
    names = []
    for L in range(cfg["n_layers"]):
        b = f"blk.{L}."
        names.append(b + "attn_norm.weight")
        if L % cfg["attn_every"] == cfg["attn_every"] - 1:
            names += [b + s for s in ("attn_q.weight", "attn_k.weight", "attn_v.weight", "attn_output.weight",
                                      "attn_q_norm.weight", "attn_k_norm.weight")]
        else:
            names += [b + s for s in ("attn_qkv.weight", "attn_gate.weight", "ssm_beta.weight", "ssm_alpha.weight",
                                      "ssm_out.weight", "ssm_conv1d.weight", "ssm_dt.bias", "ssm_a",
                                      "ssm_norm.weight")]
        names += [b + s for s in ("post_attention_norm.weight", "ffn_gate.weight", "ffn_up.weight",
                                  "ffn_down.weight")]
    return names + ["token_embd.weight", "output.weight", "output_norm.weight"]


def export_model_pack(model, path, q5k_layout: int = 2, q4k_layout: int = 2) -> list[str]:
    """Write the weights of a tp_size-1 model (rt.Model, seeded or loaded) as a
    Q38PACK with the reference's tensor names, types and shapes
    (model_tensor_names): the fused qkv|z and beta|alpha matrices split back
    into attn_qkv / attn_gate and ssm_beta / ssm_alpha, Q5_K matrices in
    `q5k_layout` (0 GGUF blocks, 1 the reference's SoA planes, 2 B200 tiles),
    Q4_K in `q4k_layout` (0 or 2), Q6_K and IQ4_XS as GGUF blocks.  Version 3
    when a tensor is tiled, else 2 (what the reference reads).  Loading the
    pack with q38_model_create_from_pack at any tp_size gives the model's
    weights bit for bit.  Tensors are read from the device one at a time while
    the file is written; tiles stay tiles when the layout does not change."""
    cfg = model.cfg
    if cfg.get("tp_size", 1) != 1:
        raise ValueError("export a tp_size 1 model")
    if q5k_layout not in (0, 1, 2) or q4k_layout not in (0, 2):
        raise ValueError("layouts: Q5_K 0/1/2, Q4_K 0/2")
    D, AD = 128, 256
    C = 2 * cfg["gdn_qk_heads"] * D + cfg["gdn_v_heads"] * D
    Hv = cfg["gdn_v_heads"]
    ts: list[Tensor] = []
    cache: dict = {}

    def fetch(name):
        """(desc, raw bytes as stored) of an engine tensor, the last one kept."""
        if cache.get("name") != name:
            cache.clear()
            cache["name"] = name
            cache["v"] = model.download(name)
        return cache["v"]

    def gguf_rows(name, r0, r1):
        d, raw = fetch(name)
        if d.layout == 2:
            if r0 % 8 == 0 and (r1 % 8 == 0 or r1 == d.rows):
                per_oct = synth.tiled_bytes(d.ggml_type, 8, d.cols)
                part = raw[r0 // 8 * per_oct: (r1 + 7) // 8 * per_oct]
                return synth.untile(d.ggml_type, part, r1 - r0, d.cols).reshape(r1 - r0, -1)
            return synth.untile(d.ggml_type, raw, d.rows, d.cols).reshape(d.rows, -1)[r0:r1]
        return raw.reshape(d.rows, -1)[r0:r1]

    def tiles_rows(name, r0, r1):
        d, raw = fetch(name)
        per_oct = synth.tiled_bytes(d.ggml_type, 8, d.cols)
        return raw[r0 // 8 * per_oct: (r1 + 7) // 8 * per_oct]

    def mat(pack_name, model_name, r0, r1, role):
        d = model.tensor(model_name)
        t, cols, rows = d.ggml_type, d.cols, r1 - r0
        nb = cols // 256
        lay = q5k_layout if t == 13 else q4k_layout if t == 12 else 0
        if lay == 1:
            n = rows * nb
            planes = [LazyPlane(n * w, (lambda k: lambda: synth.q5k_soa_records(
                gguf_rows(model_name, r0, r1).reshape(-1))[k])(k)) for k, w in enumerate((20, 32, 128))]
            ts.append(Tensor(pack_name, t, (cols, rows), planes, role, 0, 1))
        elif lay == 2:
            nbytes = synth.tiled_bytes(t, rows, cols)
            if d.layout == 2 and r0 % 8 == 0 and (r1 % 8 == 0 or r1 == d.rows):
                fn = lambda: tiles_rows(model_name, r0, r1)
            else:
                fn = lambda: synth.repack_tiled(t, gguf_rows(model_name, r0, r1).reshape(-1), rows, cols)
            ts.append(Tensor(pack_name, t, (cols, rows), [LazyPlane(nbytes, fn)], role, 0, 2))
        else:
            ts.append(Tensor(pack_name, t, (cols, rows),
                             [LazyPlane(rows * nb * BLOCK_BYTES[t], lambda: gguf_rows(model_name, r0, r1))], role))

    def whole(pack_name, model_name, role):
        mat(pack_name, model_name, 0, model.tensor(model_name).rows, role)

    def split(names, model_name, at, role):
        rows = model.tensor(model_name).rows
        mat(names[0], model_name, 0, at, role)
        mat(names[1], model_name, at, rows, role)

    def vec(pack_name, model_name, dims, role):
        n = int(np.prod(dims))
        ts.append(Tensor(pack_name, 0, dims, [LazyPlane(4 * n, lambda: model.download(model_name)[1])], role))

    for L in range(cfg["n_layers"]):
        b = f"blk.{L}."
        vec(b + "attn_norm.weight", b + "attn_norm", (cfg["hidden"],), ROLE["norm"])
        if L % cfg["attn_every"] == cfg["attn_every"] - 1:
            for s in ("attn_q", "attn_k", "attn_v", "attn_output"):
                whole(b + s + ".weight", b + s, ROLE["attention"])
            vec(b + "attn_q_norm.weight", b + "attn_q_norm", (AD,), ROLE["norm"])
            vec(b + "attn_k_norm.weight", b + "attn_k_norm", (AD,), ROLE["norm"])
        else:
            split((b + "attn_qkv.weight", b + "attn_gate.weight"), b + "attn_qkvz", C, ROLE["deltanet"])
            split((b + "ssm_beta.weight", b + "ssm_alpha.weight"), b + "ssm_ba", Hv, ROLE["deltanet"])
            whole(b + "ssm_out.weight", b + "ssm_out", ROLE["deltanet"])
            vec(b + "ssm_conv1d.weight", b + "ssm_conv1d", (4, C), ROLE["deltanet"])
            vec(b + "ssm_dt.bias", b + "ssm_dt", (Hv,), ROLE["deltanet"])
            vec(b + "ssm_a", b + "ssm_a", (Hv,), ROLE["deltanet"])
            vec(b + "ssm_norm.weight", b + "ssm_norm", (D,), ROLE["norm"])
        vec(b + "post_attention_norm.weight", b + "post_attention_norm", (cfg["hidden"],), ROLE["norm"])
        for s in ("ffn_gate", "ffn_up", "ffn_down"):
            whole(b + s + ".weight", b + s, ROLE["ffn"])
    whole("token_embd.weight", "token_embd", ROLE["embedding"])
    whole("output.weight", "output", ROLE["output"])
    vec("output_norm.weight", "output_norm", (cfg["hidden"],), ROLE["output_norm"])
    tiled = any(t.layout == 2 for t in ts)
    write_pack(path, ts, {"exported_from": "q38_model", "seed": cfg.get("seed"), "config": dict(cfg)},
               b"GGUF-meta-placeholder", version=3 if tiled else 2)
    return [t.name for t in ts]
