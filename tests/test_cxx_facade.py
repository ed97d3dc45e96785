"""The C++ host facade (include/q38/driver.hpp, lib/libq38driver_b200.so):
host code written against the reference's q38::NvidiaDriver interface
compiles and links unchanged, and on a B200 its smokes run the B200 kernels
and pass their checks (tests/cxx/facade_smoke.cpp)."""
from __future__ import annotations

import re
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from qwen382743090_b200 import build, synth

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "q38" / "driver.hpp"


def _methods() -> list[str]:
    text = HEADER.read_text()
    body = text[text.index("class NvidiaDriver"):]
    inline = set(re.findall(r"(\w+)\(\) const noexcept \{", body))
    return sorted(set(re.findall(r"\b(?:bool|void)\s+(\w+)\(", body)) - inline)


def _compile(tmp_path: Path) -> Path:
    build.build()
    exe = tmp_path / "facade_smoke"
    lib = build.LIB_DIR
    cmd = [shutil.which("g++") or "g++", "-std=c++17", "-O1", "-I", str(ROOT / "include"),
           str(ROOT / "tests" / "cxx" / "facade_smoke.cpp"), "-o", str(exe), f"-L{lib}", "-lq38driver_b200",
           "-lq38rt_b200", f"-Wl,-rpath,{lib}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return exe


def test_facade_exports_every_method():
    build.build()
    out = subprocess.run(["nm", "-DC", "--defined-only", str(build.DRIVER_LIB)], capture_output=True, text=True)
    assert out.returncode == 0
    names = _methods()
    assert "run_q5k_sm86_gemv_smoke" in names and "run_q4k_gemv_smoke" in names
    for m in names:
        assert f"q38::NvidiaDriver::{m}(" in out.stdout, m


def test_host_program_compiles_and_links(tmp_path):
    assert _compile(tmp_path).exists()


def _iq4xs_soa(blocks: np.ndarray):
    """IQ4_XS GGUF blocks -> the reference's SoA planes D [2 B] | SCALES
    [8 x int8 ls - 32] | QS [128 B] (src/quant.cpp:505-534); returns
    (buffer, scale_offset, qs_offset)."""
    b = blocks.reshape(-1, 136)
    n = b.shape[0]
    sh = b[:, 2:4].copy().view(np.uint16).reshape(n).astype(np.int32)
    sl = b[:, 4:8].astype(np.int32)
    ls = np.empty((n, 8), np.int32)
    for g in range(8):
        ls[:, g] = ((sl[:, g // 2] >> (4 * (g % 2))) & 15) | (((sh >> (2 * g)) & 3) << 4)
    scale_off, qs_off = n * 2, n * 2 + n * 8
    buf = np.zeros(qs_off + n * 128, np.uint8)
    buf[:scale_off] = b[:, 0:2].reshape(-1)
    buf[scale_off:qs_off] = (ls - 32).astype(np.int8).view(np.uint8).reshape(-1)
    buf[qs_off:] = b[:, 8:136].reshape(-1)
    return buf, scale_off, qs_off


@pytest.fixture(scope="module")
def layer_pack(tmp_path_factory):
    """A seeded pack with the reference model's recurrent layers 0 and 1
    (names, types, layouts and shapes of src/runtime.cpp:368-460)."""
    from qwen382743090_b200 import q38pack

    p = tmp_path_factory.mktemp("layer") / "layers.q38pack"
    q38pack.synthetic_layer_pack(p, layers=(0, 1))
    return p


@pytest.mark.gpu
def test_facade_smokes_on_b200(tmp_path, layer_pack):
    """Every method of the facade runs and passes its check on a B200."""
    exe = _compile(tmp_path)
    cols, rows = 5120, 64
    lines = []
    for kind, t in (("q4k", 12), ("q5k", 13), ("q6k", 14), ("iq4xs", 23)):
        p = tmp_path / f"{kind}.bin"
        synth.gen_blocks(t, rows, cols, seed=t).tofile(p)
        lines.append(f"{kind} {p} {cols} {rows}")
    buf, qh, qs = synth.repack_q5k_soa(synth.gen_blocks(13, 6144, cols, seed=1234))
    p = tmp_path / "q5k_sm86.bin"
    buf.tofile(p)
    lines.append(f"q5k_sm86 {p} {cols} 6144 {qh} {qs}")
    ibuf, so, qo = _iq4xs_soa(synth.gen_blocks(23, 512, cols, seed=23))
    p = tmp_path / "iq4xs_sm86.bin"
    ibuf.tofile(p)
    lines.append(f"iq4xs_sm86 {p} {cols} 512 {so} {qo}")
    man = tmp_path / "manifest.txt"
    man.write_text("\n".join(lines) + "\n")
    res = subprocess.run([str(exe), str(man), str(layer_pack)], capture_output=True, text=True, timeout=900)
    kv = dict(l.split(": ", 1) for l in res.stdout.splitlines() if ": " in l)
    assert res.returncode == 0 and res.stdout.strip().endswith("PASS"), res.stdout + res.stderr
    assert kv["is_target_sm"] == "1"
    for m in _methods():
        if m not in ("open", "close"):  # called around the others
            assert kv.get(f"{m}_ok") == "1", m
    for k in ("run_q4k_gemv_smoke", "run_q5k_sm86_gemv_smoke", "run_iq4xs_q8_1_gemv_smoke"):
        assert float(kv[f"{k}_gbps"]) > 0
    assert float(kv["gdn_state_gbps"]) > 0 and float(kv["layer_chain_ms"]) > 0


def _packs(tmp_path: Path) -> dict:
    from qwen382743090_b200 import q38pack

    out = {}
    for layout in (0, 1):
        p = tmp_path / f"layout{layout}.q38pack"
        q38pack.synthetic_pack(p, q5k_layout=layout, version=2)
        out[layout] = p
    return out


def test_cli_host_side_errors(tmp_path):
    """The C++ q38-q5k-sm86-gemv keeps the reference's exit codes on the host
    side: 2 without --model, 3 for an unknown tensor, 4 for a non-Q5_K one."""
    build.build()
    exe = str(build.CLI_Q5K_SM86)
    packs = _packs(tmp_path)
    assert subprocess.run([exe], capture_output=True).returncode == 2
    assert subprocess.run([exe, "--model", str(packs[1]), "--tensor", "nope"], capture_output=True).returncode == 3
    r = subprocess.run([exe, "--model", str(packs[1]), "--tensor", "blk.0.ssm_beta.weight"], capture_output=True,
                       text=True)
    assert r.returncode == 4 and "GGML_TYPE_Q5_K" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("layout", [1, 0])
def test_cli_runs_the_headline_gemv(tmp_path, layout):
    """On a B200 the command passes on a persisted SoA tensor and on GGUF
    blocks it repacks itself (decoded weights unchanged), with the
    reference's key: value lines."""
    build.build()
    p = _packs(tmp_path)[layout]
    r = subprocess.run([str(build.CLI_Q5K_SM86), "--model", str(p)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    kv = dict(l.split(": ", 1) for l in r.stdout.splitlines() if ": " in l)
    assert kv["q5_k_sm86"] == "PASS"
    assert kv["source_layout"] == ("persisted_v2" if layout == 1 else "temporary_from_native")
    if layout == 0:
        assert float(kv["repack_decode_max_abs_error"]) == 0.0
    assert float(kv["max_abs_error"]) <= 2e-3
    assert float(kv["original_equiv_weight_bandwidth_GBps"]) > 0


@pytest.mark.parametrize("layout", [0, 1, 2])
def test_cxx_plan_matches_python_cli(tmp_path, layout):
    """The C++ q38-plan (host only) prints exactly what the Python q38-plan
    prints for the same pack, tensor list included."""
    import sys

    from qwen382743090_b200 import q38pack

    build.build()
    p = tmp_path / f"plan{layout}.q38pack"
    q38pack.synthetic_pack(p, q5k_layout=layout, version=2, layers=2)
    cpp = subprocess.run([str(build.CLI_PLAN), "--model", str(p), "--list", "--page-bytes", "65536"],
                         capture_output=True, text=True)
    py = subprocess.run([sys.executable, "-m", "qwen382743090_b200.cli", "q38-plan", "--model", str(p), "--list",
                         "--page-bytes", "65536"], capture_output=True, text=True, cwd=ROOT)
    assert cpp.returncode == 0 and py.returncode == 0, cpp.stderr + py.stderr
    assert cpp.stdout == py.stdout
    assert subprocess.run([str(build.CLI_PLAN)], capture_output=True).returncode == 2


KQUANT_CMDS = {"q38-q4k-gemv": (12, None), "q38-q5k-gemv": (13, None), "q38-q6k-gemv": (14, "output.weight"),
               "q38-iq4xs-gemv": (23, None)}


def test_kquant_commands_host_side_errors(tmp_path):
    """The C++ K-quant GEMV commands keep the reference's exit codes on the
    host side: 2 without --model, 3 for an unknown tensor, 4 for a tensor of
    another type or layout."""
    build.build()
    p = _packs(tmp_path)[1]  # Q5_K persisted in the SoA layout
    for name in KQUANT_CMDS:
        exe = str(build.BIN_DIR / name)
        assert subprocess.run([exe], capture_output=True).returncode == 2
        assert subprocess.run([exe, "--model", str(p), "--tensor", "nope"], capture_output=True).returncode == 3
    r = subprocess.run([str(build.BIN_DIR / "q38-q5k-gemv"), "--model", str(p)], capture_output=True, text=True)
    assert r.returncode == 4 and "GGUF_NATIVE" in r.stderr


@pytest.mark.gpu
def test_kquant_commands_run_on_b200(tmp_path):
    """Each C++ K-quant GEMV command passes on its GGUF-native tensor of a
    synthetic pack, with the reference's key: value lines."""
    build.build()
    p = _packs(tmp_path)[0]  # every Q5_K tensor GGUF-native
    for name, (_, tensor) in KQUANT_CMDS.items():
        cmd = [str(build.BIN_DIR / name), "--model", str(p)] + (["--tensor", tensor] if tensor else [])
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, name + ": " + r.stdout + r.stderr
        kv = dict(l.split(": ", 1) for l in r.stdout.splitlines() if ": " in l)
        tag = {"q38-q4k-gemv": "q4_k_gemv", "q38-q5k-gemv": "q5_k_gemv", "q38-q6k-gemv": "q6_k_gemv",
               "q38-iq4xs-gemv": "iq4_xs_gemv"}[name]
        assert kv[tag] == "PASS"
        assert float(kv["max_abs_error"]) <= 2e-3
        assert float(kv["effective_weight_bandwidth_GBps"]) > 0


LAYER_CMDS = ("q38-layer0-projections", "q38-layer0-gate", "q38-layer0-recurrent-front",
              "q38-layer0-recurrent-attention", "q38-layer0-full")


def test_layer_commands_host_side(tmp_path):
    """Host-side contract of the layer and probe commands: 2 without the
    required arguments; q38-runtime and q38-layer-topology work without a GPU
    and name the kernel each tensor dispatches to."""
    from qwen382743090_b200 import q38pack

    build.build()
    for name in LAYER_CMDS + ("q38-recurrent-prep", "q38-q5k-q8k-gemv", "q38-q4k-smoke", "q38-recurrent-layer",
                              "q38-layer-topology", "q38-runtime"):
        assert subprocess.run([str(build.BIN_DIR / name)], capture_output=True).returncode == 2, name
    p = tmp_path / "tiled.q38pack"
    q38pack.synthetic_pack(p, q5k_layout=2, version=3, layers=2)
    r = subprocess.run([str(build.BIN_DIR / "q38-runtime"), "--model", str(p), "--no-gpu", "--list-tensors"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "blk.0.attn_qkv.weight type=13" in r.stdout and "kernel=Q5K_B200_TILED" in r.stdout
    assert "kernel=IQ4XS_PRMT" in r.stdout and "kernel=Q6K_NATIVE_VEC" in r.stdout
    r = subprocess.run([str(build.BIN_DIR / "q38-layer-topology"), "--model", str(p)], capture_output=True, text=True)
    assert r.returncode == 0 and "layer_topology: PASS" in r.stdout
    assert "layer[0]: MISSING" in r.stdout  # no ssm_conv1d / attention tensors in this small pack


@pytest.mark.gpu
def test_layer_commands_on_b200(layer_pack, tmp_path):
    """The layer, recurrent and probe commands pass on the seeded pack of the
    reference model's recurrent layers, with the reference's PASS lines."""
    from qwen382743090_b200 import q38pack

    build.build()
    tags = {"q38-layer0-projections": "layer0_projections", "q38-layer0-gate": "layer0_gate",
            "q38-layer0-recurrent-front": "layer0_recurrent_front",
            "q38-layer0-recurrent-attention": "layer0_recurrent_attention", "q38-layer0-full": "layer0_full",
            "q38-recurrent-prep": "recurrent_prep", "q38-q4k-smoke": "q4_k", "q38-q5k-smoke": "q5_k",
            "q38-iq4xs-smoke": "iq4_xs"}
    for name, tag in tags.items():
        r = subprocess.run([str(build.BIN_DIR / name), "--model", str(layer_pack)], capture_output=True, text=True,
                           timeout=600)
        assert r.returncode == 0, name + ": " + r.stdout + r.stderr
        assert f"{tag}: PASS" in r.stdout, name
    r = subprocess.run([str(build.BIN_DIR / "q38-recurrent-layer"), "--model", str(layer_pack), "--layer", "1"],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "recurrent_layer: PASS" in r.stdout, r.stdout + r.stderr
    kv = dict(l.split(": ", 1) for l in r.stdout.splitlines() if ": " in l)
    assert float(kv["layer_chain_ms"]) > 0 and float(kv["layer_output_max_abs_error"]) <= 4e-3
    for name, tag in (("q38-gpu-smoke", "smoke"), ("q38-rmsnorm-smoke", "rmsnorm"), ("q38-gdn-ar-smoke", "gdn_ar")):
        r = subprocess.run([str(build.BIN_DIR / name)], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0 and f"{tag}: PASS" in r.stdout, name + ": " + r.stdout + r.stderr
    # Q5_K x Q8_K needs GGUF-native Q5_K (exit 11 on the SoA pack, as the reference)
    r = subprocess.run([str(build.BIN_DIR / "q38-q5k-q8k-gemv"), "--model", str(layer_pack)], capture_output=True)
    assert r.returncode == 11
    p = tmp_path / "gguf.q38pack"
    q38pack.synthetic_pack(p, q5k_layout=0, version=2)
    r = subprocess.run([str(build.BIN_DIR / "q38-q5k-q8k-gemv"), "--model", str(p)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "q5_k_x_q8_k: PASS" in r.stdout, r.stdout + r.stderr
