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


@pytest.mark.gpu
def test_facade_smokes_on_b200(tmp_path):
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
    man = tmp_path / "manifest.txt"
    man.write_text("\n".join(lines) + "\n")
    res = subprocess.run([str(exe), str(man)], capture_output=True, text=True, timeout=300)
    kv = dict(l.split(": ", 1) for l in res.stdout.splitlines() if ": " in l)
    assert res.returncode == 0 and res.stdout.strip().endswith("PASS"), res.stdout + res.stderr
    assert kv["is_target_sm"] == "1"
    for kind in ("q4k", "q5k", "q6k", "iq4xs", "q5k_sm86"):
        assert kv[f"{kind}_ok"] == "1"
        assert float(kv[f"{kind}_max_abs"]) <= 2e-3
        assert float(kv[f"{kind}_gbps"]) > 0
    assert "not provided by the B200 facade" in kv["gdn_ar_smoke"]


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
