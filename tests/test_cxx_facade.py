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
