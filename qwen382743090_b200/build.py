"""Build the in-tree CUDA library lib/libq38rt_b200.so for sm_100a, and the
C++ host facade lib/libq38driver_b200.so on top of it.

    python -m qwen382743090_b200.build [--verbose]

The whole device side is one translation unit (csrc/q38rt.cu), compiled by
nvcc with the CUDA runtime linked statically; nothing is JIT-compiled and no
architecture other than sm_100a is emitted.  The facade (cxx/, the
q38::NvidiaDriver interface of include/q38/driver.hpp) is plain C++ over the
C ABI, compiled by g++ and linked against the CUDA library, and so are the
C++ commands in bin/ (q38-q5k-sm86-gemv, q38-q4k/q5k/q6k/iq4xs-gemv, q38-plan).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libq38rt_b200.so"
CXX_DIR = PKG / "cxx"
DRIVER_LIB = LIB_DIR / "libq38driver_b200.so"
BIN_DIR = PKG / "bin"
CLI_Q5K_SM86 = BIN_DIR / "q38-q5k-sm86-gemv"
CLI_PLAN = BIN_DIR / "q38-plan"
# command -> (source, extra g++ flags); the four K-quant GEMV commands share one source
CLIS = {CLI_Q5K_SM86: (CXX_DIR / "q38_q5k_sm86_gemv.cpp", []), CLI_PLAN: (CXX_DIR / "q38_plan.cpp", [])}
for _name, _type in (("q38-q4k-gemv", 12), ("q38-q5k-gemv", 13), ("q38-q6k-gemv", 14), ("q38-iq4xs-gemv", 23)):
    CLIS[BIN_DIR / _name] = (CXX_DIR / "q38_kquant_gemv.cpp", [f"-DQ38_KQUANT={_type}"])
# the layer, recurrent and probe commands share one source (q38_layer_cmds.cpp)
LAYER_CMDS = ("q38-gpu-smoke", "q38-rmsnorm-smoke", "q38-gdn-ar-smoke", "q38-recurrent-prep", "q38-q5k-q8k-gemv",
              "q38-q4k-smoke", "q38-q5k-smoke", "q38-iq4xs-smoke", "q38-layer0-projections", "q38-layer0-gate",
              "q38-layer0-recurrent-front", "q38-layer0-recurrent-attention", "q38-layer0-full",
              "q38-recurrent-layer", "q38-layer-topology", "q38-runtime")
for _i, _name in enumerate(LAYER_CMDS, 1):
    CLIS[BIN_DIR / _name] = (CXX_DIR / "q38_layer_cmds.cpp", [f"-DQ38_CMD={_i}"])

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-Wno-format-truncation",
    "-shared",
    "-ldl",
]


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.cpp")) +
                  list(CSRC.glob("*.h")) + [ROOT / "include" / "q38rt.h"])


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found: the Q38RT library needs the CUDA toolkit to build")
    return exe


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources())


DRIVER_CPP = ["nvidia_driver.cpp", "layer_smokes.cpp", "runtime.cpp"]


def driver_sources() -> list[Path]:
    return [CXX_DIR / n for n in DRIVER_CPP] + [CXX_DIR / "facade_util.hpp", ROOT / "include" / "q38" / "driver.hpp",
                                                ROOT / "include" / "q38" / "q38pack.hpp",
                                                ROOT / "include" / "q38" / "runtime.hpp", ROOT / "include" / "q38rt.h"]


def _gxx(cmd: list[str], what: str) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed ({what}):\n" + res.stdout + res.stderr)


def build_cli(force: bool = False) -> Path:
    """g++ the C++ commands (q38-q5k-sm86-gemv, the K-quant GEMVs, q38-plan) into bin/
    (they need both libraries)."""
    BIN_DIR.mkdir(parents=True, exist_ok=True)
    for exe, (src, flags) in CLIS.items():
        deps = [src, DRIVER_LIB, LIB, *(ROOT / "include" / "q38").glob("*.hpp"), ROOT / "include" / "q38rt.h"]
        if not force and exe.exists() and all(p.stat().st_mtime <= exe.stat().st_mtime for p in deps):
            continue
        tmp = exe.with_suffix(".tmp")
        _gxx([shutil.which("g++") or "g++", "-std=c++17", "-O2", "-Wall", "-Wextra", f"-I{ROOT / 'include'}", *flags,
              "-o", str(tmp), str(src),
              f"-L{LIB_DIR}", "-lq38driver_b200", "-lq38rt_b200", "-Wl,-rpath,$ORIGIN/../lib"], exe.name)
        os.replace(tmp, exe)
    return BIN_DIR


def build_driver(force: bool = False, verbose: bool = False) -> Path:
    """g++ the C++ facade into lib/libq38driver_b200.so (needs the CUDA library)."""
    if not force and DRIVER_LIB.exists() and LIB.exists():
        t = DRIVER_LIB.stat().st_mtime
        if all(p.stat().st_mtime <= t for p in driver_sources() + [LIB]):
            return DRIVER_LIB
    gxx = shutil.which("g++") or "g++"
    tmp = DRIVER_LIB.with_suffix(".so.tmp")
    cmd = [gxx, "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", f"-I{ROOT / 'include'}", "-o", str(tmp),
           *(str(CXX_DIR / n) for n in DRIVER_CPP), f"-L{LIB_DIR}", "-lq38rt_b200", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd))
    _gxx(cmd, "libq38driver_b200.so")
    os.replace(tmp, DRIVER_LIB)
    return DRIVER_LIB


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        build_driver(force, verbose)
        build_cli(force)
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *NVCC_FLAGS, "-o", str(tmp), str(CSRC / "q38rt.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        print(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    build_driver(True, verbose)
    build_cli(True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(LIB)
