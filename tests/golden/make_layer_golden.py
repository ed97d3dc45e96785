#!/usr/bin/env python3
"""Generate tests/golden/layer_golden.npz from the reference's own CPU code.

The decoder-layer ops have no standalone CPU functions in the reference: their
expected values are computed by plain C++ loops inside the GPU smoke hosts of
src/driver.cpp.  This script compiles those loops where they lie (it reads
src/driver.cpp from the reference tree, cuts three regions out by exact
anchor lines, wraps them in functions that declare the variables they use,
and builds that in a temporary directory with g++; no reference source is
written into this repository) and runs them:

* run_gdn_ar_smoke's input generator and CPU reference (src/driver.cpp:
  11198-11301), on its own shape (state_dim 128, 16 q/k heads, 48 value
  heads, as src/gdn_ar_smoke.cpp passes): the GDN step on the reference's own
  smoke inputs;
* run_qwen35_layer0_full's composition check (src/driver.cpp:8080-8242):
  conv4 + SiLU + state roll, per-head q/k L2 norm, beta/gate with its
  softplus branches, the GDN step and the gated RMSNorm * SiLU(z), on the
  seeded config-3 inputs of tests/golden/layer_inputs.py;
* its FFN check (src/driver.cpp:8365-8393): RMSNorm of the residual and
  SiLU(gate) * up, on seeded inputs.

Arrays up to a few tens of thousands of floats are stored whole; the GDN
states (786,432 floats) as a sha256 of their bytes plus 4096 sampled values.
The seeded inputs are stored as digests (the tests regenerate them and check
the digest first).  Run here, where the reference tree exists:

    python tests/golden/make_layer_golden.py
"""
from __future__ import annotations

import hashlib
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

import layer_inputs as LI  # noqa: E402
import oracle  # noqa: E402  (only to locate the reference tree)

# (enclosing function, start anchor, end anchor (excluded)) of each region:
# the first match of the start line after the function's definition
GDN_SMOKE = "bool NvidiaDriver::run_gdn_ar_smoke(\n"
LAYER0 = "bool NvidiaDriver::run_qwen35_layer0_full(\n"
REGIONS = {
    "gdn_smoke": (GDN_SMOKE, "        for (std::uint32_t h = 0; h < qk_heads; ++h) {\n            double q_ss = 0.0;\n",
                  "        const std::size_t q_bytes = q.size() * sizeof(float);\n"),
    "layer": (LAYER0, "            std::vector<float> conv_ref(kQkvRows);\n",
              "            constexpr std::size_t kTailCheckedRows = 8;\n"),
    "ffn": (LAYER0, "            std::vector<float> ffn_normed_ref(kCols);\n",
            "            constexpr std::size_t kFfnCheckedRows = 8;\n"),
}

HARNESS = r"""
#include <array>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <vector>

static std::vector<float> rd(std::FILE* f, std::size_t n) {
    std::vector<float> v(n);
    if (std::fread(v.data(), 4, n, f) != n) { std::fprintf(stderr, "short input\n"); std::exit(3); }
    return v;
}
static void wr(std::FILE* f, const std::vector<float>& v) { std::fwrite(v.data(), 4, v.size(), f); }

static void gdn_smoke(std::FILE* out) {
    const std::uint32_t state_dim = 128, qk_heads = 16, value_heads = 48;
    constexpr float kEps = 1.0e-6f;
    const std::size_t qk_values = static_cast<std::size_t>(qk_heads) * state_dim;
    const std::size_t v_values = static_cast<std::size_t>(value_heads) * state_dim;
    const std::size_t state_values = static_cast<std::size_t>(value_heads) * state_dim * state_dim;
    std::vector<float> q(qk_values), k(qk_values), v(v_values), g(value_heads), beta(value_heads);
    std::vector<float> state_in(state_values), out_ref(v_values), state_ref(state_values);
@@gdn_smoke@@
    wr(out, q); wr(out, k); wr(out, v); wr(out, g); wr(out, beta); wr(out, state_in); wr(out, out_ref); wr(out, state_ref);
}

static void layer(std::FILE* in, std::FILE* out) {
    constexpr std::uint32_t kQkvRows = 10240, kSmallRows = 48, kHeadDim = 128, kQkHeads = 16, kValueHeads = 48;
    constexpr std::uint32_t kKeyDim = kQkHeads * kHeadDim, kValueDim = kValueHeads * kHeadDim, kConvStateSteps = 3;
    constexpr std::size_t kGdnStateValues = static_cast<std::size_t>(kValueHeads) * kHeadDim * kHeadDim;
    const float rms_eps = 1.0e-6f;
    const std::vector<float> qkv_gpu = rd(in, kQkvRows), conv_state_in = rd(in, 3 * kQkvRows);
    const std::vector<float> conv_w = rd(in, 4 * kQkvRows), beta_raw_gpu = rd(in, kSmallRows);
    const std::vector<float> alpha_raw_gpu = rd(in, kSmallRows), dt_b = rd(in, kSmallRows), a_v = rd(in, kSmallRows);
    const std::vector<float> gdn_state_in = rd(in, kGdnStateValues), z_gpu = rd(in, kValueDim);
    const std::vector<float> norm_w = rd(in, kHeadDim);
    const float* conv_weight = conv_w.data();
    const float* dt_bias = dt_b.data();
    const float* ssm_a = a_v.data();
    const float* ssm_norm_weight = norm_w.data();
@@layer@@
    wr(out, conv_ref); wr(out, conv_state_ref); wr(out, q_ref); wr(out, k_ref); wr(out, beta_ref); wr(out, gate_ref);
    wr(out, gdn_out_ref); wr(out, gdn_state_ref); wr(out, gated_norm_ref);
}

static void ffn(std::FILE* in, std::FILE* out) {
    constexpr std::uint32_t kCols = 5120, kFfnDim = 17408;
    const float rms_eps = 1.0e-6f;
    const std::vector<float> residual_gpu = rd(in, kCols), pn = rd(in, kCols);
    const std::vector<float> ffn_gate_gpu = rd(in, kFfnDim), ffn_up_gpu = rd(in, kFfnDim);
    const float* post_norm_weight = pn.data();
@@ffn@@
    wr(out, ffn_normed_ref); wr(out, ffn_mul_ref);
}

int main(int argc, char** argv) {
    if (argc != 3) return 2;
    std::FILE* in = std::fopen(argv[1], "rb");
    std::FILE* out = std::fopen(argv[2], "wb");
    if (!in || !out) return 2;
    gdn_smoke(out);
    layer(in, out);
    ffn(in, out);
    std::fclose(in);
    std::fclose(out);
    return 0;
}
"""


def cut(text: str, fn: str, start: str, end: str) -> tuple[str, int, int]:
    if text.count(fn) != 1:
        raise SystemExit(f"function not found exactly once: {fn!r}")
    f = text.index(fn)
    nxt = text.find("\nbool NvidiaDriver::", f + len(fn))
    a = text.find(start, f)
    if a < 0 or (nxt >= 0 and a > nxt):
        raise SystemExit(f"anchor not found in {fn.strip()}: {start!r}")
    b = text.index(end, a)
    first = text.count("\n", 0, a) + 1
    last = text.count("\n", 0, b)
    return text[a:b], first, last


def main() -> int:
    ref = oracle.reference_root()
    if ref is None:
        raise SystemExit("reference tree not found (set Q38_REFERENCE)")
    drv = (ref / "src" / "driver.cpp").read_text()
    src = HARNESS
    lines = {}
    for name, (fn, s, e) in REGIONS.items():
        body, first, last = cut(drv, fn, s, e)
        src = src.replace(f"@@{name}@@", body)
        lines[name] = (first, last)
    li, fi = LI.layer_inputs(), LI.ffn_inputs()
    order_l = ["qkv", "conv_state_in", "conv_weight", "beta_raw", "alpha_raw", "dt_bias", "ssm_a", "gdn_state_in",
               "z", "ssm_norm_weight"]
    order_f = ["residual", "post_norm_weight", "ffn_gate", "ffn_up"]
    with tempfile.TemporaryDirectory() as td:
        td = Path(td)
        (td / "h.cpp").write_text(src)
        subprocess.run(["g++", "-std=c++20", "-O2", "-ffp-contract=off", "-o", str(td / "h"), str(td / "h.cpp")],
                       check=True)
        with open(td / "in.bin", "wb") as f:
            for k in order_l:
                f.write(li[k].tobytes())
            for k in order_f:
                f.write(fi[k].tobytes())
        subprocess.run([str(td / "h"), str(td / "in.bin"), str(td / "out.bin")], check=True)
        raw = np.fromfile(td / "out.bin", np.float32)
    H, Hq, D, C, S = LI.VALUE_HEADS, LI.QK_HEADS, LI.HEAD_DIM, LI.QKV_ROWS, LI.VALUE_HEADS * 128 * 128
    sizes = [("smoke_q", Hq * D), ("smoke_k", Hq * D), ("smoke_v", H * D), ("smoke_g", H), ("smoke_beta", H),
             ("smoke_state_in", S), ("smoke_out", H * D), ("smoke_state_out", S),
             ("conv_out", C), ("conv_state_out", 3 * C), ("q", LI.KEY_DIM), ("k", LI.KEY_DIM), ("beta", H),
             ("gate", H), ("gdn_out", LI.VALUE_DIM), ("gdn_state_out", S), ("gated", LI.VALUE_DIM),
             ("ffn_normed", LI.HIDDEN), ("ffn_mul", LI.FFN_DIM)]
    assert raw.size == sum(n for _, n in sizes), (raw.size, sum(n for _, n in sizes))
    arr, off = {}, 0
    for name, n in sizes:
        arr[name] = raw[off: off + n]
        off += n
    idx = LI.sample_index(S)
    out = {}
    for name, a in arr.items():
        if a.size == S or name == "conv_state_out":
            out[name + "_sha256"] = np.array(LI.digest(a))
            if a.size == S:
                out[name + "_sample"] = a[idx]
        else:
            out[name] = a
    out["state_sample_index"] = idx
    for k, v in {**li, **fi}.items():
        out["input_" + k + "_sha256"] = np.array(LI.digest(v))
    out["reference_driver_cpp_sha256"] = np.array(hashlib.sha256(drv.encode()).hexdigest())
    for name, (a, b) in lines.items():
        out[f"lines_{name}"] = np.array([a, b], np.int64)
    np.savez_compressed(HERE / "layer_golden.npz", **out)
    print("wrote", HERE / "layer_golden.npz", {k: tuple(v) for k, v in lines.items()})
    return 0


if __name__ == "__main__":
    sys.exit(main())
