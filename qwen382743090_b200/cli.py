"""Command-line entry points with the reference's binary names and output
contract (`key: value` lines and a final `...: PASS`), over this library:

    python -m qwen382743090_b200.cli q38-plan --model M.q38pack [--page-bytes N] [--list]
    python -m qwen382743090_b200.cli q38-q5k-sm86-gemv (--model M --tensor T | --synthetic --seed S)
    python -m qwen382743090_b200.cli q38-gemv (--model M --tensor T | --synthetic --type Q4_K ...)
    python -m qwen382743090_b200.cli q38-pack-b200 SRC DST

q38-plan reproduces src/plan.cpp:64-162; the GEMV commands replace
src/q5k_sm86_gemv.cpp and the per-type q38-*-gemv mains (CMakeLists.txt:21-94):
they upload the weights, run the B200 kernel, check every row against FP64
reference rows computed plainly on the device from the GGUF blocks
(q38_check_rows: one thread per weight, the reference's dequantisation, a
fixed-order FP64 sum; a row fails only beyond 1e-4 absolute and 1e-3
relative) and time it.  The layer commands are the C++ ones in bin/.
"""
from __future__ import annotations

import argparse
import sys
import time

import numpy as np

ROLE_NAME = {0: "unknown", 1: "embedding", 2: "output_norm", 3: "output", 4: "attention", 5: "deltanet", 6: "ffn",
             7: "norm", 8: "mtp"}
TYPES = {"Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ4_XS": 23}
GIB = float(1 << 30)


def _plan(args) -> int:
    from . import q38pack

    with q38pack.open_pack(args.model) as p:
        st, off = p.plan(args.page_bytes)
        by_role, type_b, type_n, lay_b, lay_n = {}, {}, {}, {}, {}
        for t in p.tensors:
            by_role[t.role] = by_role.get(t.role, 0) + t.stored_bytes
            type_b[t.ggml_type] = type_b.get(t.ggml_type, 0) + t.stored_bytes
            type_n[t.ggml_type] = type_n.get(t.ggml_type, 0) + 1
            lay_b[t.layout] = lay_b.get(t.layout, 0) + t.stored_bytes
            lay_n[t.layout] = lay_n.get(t.layout, 0) + 1
        print("Q38 GPU placement plan")
        print(f"Q38PACK version: {p.header.version}")
        print(f"GPU page: {st.page_bytes} bytes")
        print(f"tensors: {len(p.tensors)}")
        print(f"payload: {st.tensor_payload_bytes / GIB:.3f} GiB")
        print(f"reserved VA: {st.reserved_va_bytes / GIB:.3f} GiB")
        print(f"page padding: {st.page_padding_bytes / GIB:.3f} GiB")
        print(f"pages: {st.page_count}")
        for r in sorted(by_role):
            print(f"role[{ROLE_NAME.get(r, 'unknown')}]: {by_role[r] / GIB:.3f} GiB")
        print("execution layouts:")
        for lay in sorted(lay_n):
            print(f"  layout[{lay}/{q38pack.LAYOUT_NAME.get(lay, 'UNKNOWN')}]: {lay_n[lay]} tensors, "
                  f"{lay_b[lay] / GIB:.3f} GiB")
        print("tensor types (physical stored bytes):")
        for ty in sorted(type_n):
            print(f"  type[{ty}/{q38pack.TYPE_NAME.get(ty, 'UNKNOWN')}]: {type_n[ty]} tensors, {type_b[ty] / GIB:.3f} GiB")
        if args.list:
            for t, o in zip(p.tensors, off):
                print(f"{t.name.decode()} role={ROLE_NAME.get(t.role, 'unknown')} va=0x{int(o):x} "
                      f"page_off={int(o) % st.page_bytes} bytes={t.stored_bytes} "
                      f"layout={q38pack.LAYOUT_NAME.get(t.layout, 'UNKNOWN')}")
    return 0


def _time(fn, iters: int) -> float:
    from . import runtime as rt

    for _ in range(3):
        fn()
    rt.synchronize()
    t0 = time.perf_counter()
    for _ in range(iters):
        fn()
    rt.synchronize()
    return (time.perf_counter() - t0) * 1e3 / iters


def _check_rows(y, ref) -> tuple[float, float, bool]:
    y = np.asarray(y, np.float64)
    err = np.abs(y - ref)
    rel = err / np.maximum(np.abs(ref), 1e-30)
    ok = bool(np.all((err <= 1e-4) | (err <= 1e-3 * np.abs(ref))))
    return float(err.max()), float(rel.max()), ok


def _gemv(args, q5k_sm86: bool) -> int:
    from . import q38pack, runtime as rt, synth

    ctx = rt.Context(0)
    info = rt.device_query(0)
    if args.synthetic:
        ty = 13 if q5k_sm86 else TYPES[args.type]
        rows, cols = args.rows, args.cols
        blocks = synth.gen_blocks(ty, rows, cols, args.seed)
        if ty == 13 and args.layout == "soa":
            buf = synth.repack_q5k_soa(blocks)[0]
        elif ty in (12, 13) and args.layout == "tiled":
            buf = synth.repack_tiled(ty, blocks, rows, cols)
        else:
            buf = blocks
        dev = ctx.upload(buf)
        if args.layout == "soa":
            _, qh, qs = synth.repack_q5k_soa(blocks)
            desc = rt.weight_desc(13, 1, rows, cols, dev.ptr, dev.ptr + qh, dev.ptr + qs)
        else:
            desc = rt.weight_desc(ty, 2 if args.layout == "tiled" else 0, rows, cols, dev.ptr)
        name, version = "synthetic", "-"
    else:
        p = q38pack.open_pack(args.model)
        i = p.find(args.tensor)
        t = p.tensors[i]
        ty, rows, cols = t.ggml_type, int(t.dims[1]), int(t.dims[0])
        blocks = p.blocks(i)
        base = p.upload(ctx)
        desc = p.weight_desc(i, base)
        name, version = args.tensor, p.header.version
    x = synth.gen_x(cols, args.seed + 1)[0]
    xd = ctx.upload(x)
    yd = ctx.alloc(4 * rows)
    rt.gemv_f32(desc, xd.ptr, yd.ptr)
    rt.synchronize()
    y = yd.download(np.float32, rows)
    # FP64 reference rows on the device from the GGUF blocks (any stored layout)
    bd = ctx.upload(np.ascontiguousarray(blocks))
    y64 = ctx.alloc(8 * rows)
    rt.check_rows(rt.weight_desc(ty, 0, rows, cols, bd.ptr), rows, x=xd.ptr, y64=y64.ptr)
    rt.synchronize()
    ref = y64.download(np.float64, rows)
    bd.free()
    y64.free()
    max_abs, max_rel, ok = _check_rows(y, ref)
    ms = _time(lambda: rt.gemv_f32(desc, xd.ptr, yd.ptr), args.iters)
    orig = rows * (cols // 256) * q38pack.BLOCK_BYTES[ty]
    print("Q38RT-B200 " + ("Q5_K SoA GEMV vectorized" if q5k_sm86 else f"{q38pack.TYPE_NAME[ty]} GEMV"))
    print(f"q38pack_version: {version}")
    print(f"tensor: {name}")
    print(f"shape: [{cols},{rows}]")
    print(f"layout: {q38pack.LAYOUT_NAME.get(desc.layout, desc.layout)}")
    print(f"original_{q38pack.TYPE_NAME[ty]}_bytes: {orig}")
    print(f"device: {info.name.decode()}")
    print(f"max_abs_error: {max_abs:.6e}")
    print(f"max_rel_error: {max_rel:.6e}")
    print(f"kernel_ms: {ms:.4f}")
    print(f"original_equiv_weight_bandwidth_GBps: {orig / (ms * 1e-3) / 1e9:.4f}")
    print(f"rows_checked: {rows}")
    tag = "q5_k_sm86" if q5k_sm86 else q38pack.TYPE_NAME[ty].lower()
    print(f"{tag}: {'PASS' if ok else 'FAIL'}")
    return 0 if ok else 1


def _convert(args) -> int:
    from . import q38pack

    s = q38pack.convert_to_b200(args.src, args.dst)
    for k, v in s.items():
        print(f"{k}: {v}")
    print("q38pack_b200: PASS")
    return 0


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    ap = argparse.ArgumentParser(prog="qwen382743090_b200.cli")
    sub = ap.add_subparsers(dest="cmd", required=True)
    sp = sub.add_parser("q38-plan")
    sp.add_argument("--model", required=True)
    sp.add_argument("--page-bytes", type=int, default=2 << 20)
    sp.add_argument("--list", action="store_true")
    for name in ("q38-q5k-sm86-gemv", "q38-gemv"):
        g = sub.add_parser(name)
        g.add_argument("--model")
        g.add_argument("--tensor")
        g.add_argument("--synthetic", action="store_true")
        g.add_argument("--seed", type=int, default=1234)
        g.add_argument("--rows", type=int, default=6144)
        g.add_argument("--cols", type=int, default=5120)
        g.add_argument("--type", default="Q5_K", choices=sorted(TYPES))
        g.add_argument("--layout", default="soa" if name == "q38-q5k-sm86-gemv" else "gguf",
                       choices=["gguf", "soa", "tiled"])
        g.add_argument("--iters", type=int, default=200)
    cv = sub.add_parser("q38-pack-b200")
    cv.add_argument("src")
    cv.add_argument("dst")
    args = ap.parse_args(argv)
    if args.cmd == "q38-plan":
        return _plan(args)
    if args.cmd in ("q38-q5k-sm86-gemv", "q38-gemv"):
        if not args.synthetic and not (args.model and args.tensor):
            ap.error("--model and --tensor, or --synthetic")
        return _gemv(args, args.cmd == "q38-q5k-sm86-gemv")
    return _convert(args)


if __name__ == "__main__":
    sys.exit(main())
