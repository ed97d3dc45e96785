"""The decoder-layer restatements in oracle/q38_oracle.c against the
reference's own CPU code.

tests/golden/layer_golden.npz holds what the reference's C++ check loops
(run_gdn_ar_smoke, src/driver.cpp:11198-11301; run_qwen35_layer0_full,
src/driver.cpp:8080-8242 and 8365-8393) computed when compiled and run by
tests/golden/make_layer_golden.py.  Every oracle output must equal them bit
for bit: whole arrays where the fixture stores them, the sha256 of the
float32 bytes for the GDN states.  No GPU needed.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import layer_inputs as LI  # noqa: E402


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(GOLDEN / "layer_golden.npz"))


def same(a, b, what):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    assert a.shape == b.shape, what
    bad = np.flatnonzero(a.view(np.uint32) != b.view(np.uint32))
    assert bad.size == 0, f"{what}: {bad.size} values differ, first at {bad[0]}: {a[bad[0]]!r} vs {b[bad[0]]!r}"


def test_seeded_inputs_are_the_fixture_inputs(gold):
    for k, v in {**LI.layer_inputs(), **LI.ffn_inputs()}.items():
        assert LI.digest(v) == str(gold["input_" + k + "_sha256"]), k


def test_gdn_step_on_the_reference_smoke_inputs(port, gold):
    q, k, v, g, beta, st = port.gdn_smoke_inputs()
    for name, a in (("q", q), ("k", k), ("v", v), ("g", g), ("beta", beta)):
        same(a, gold["smoke_" + name], "smoke input " + name)
    assert LI.digest(st) == str(gold["smoke_state_in_sha256"])
    out, st_out = port.gdn_step(q, k, v, g, beta, st, 16, 48, 128)
    same(out, gold["smoke_out"], "GDN output")
    same(st_out[gold["state_sample_index"]], gold["smoke_state_out_sample"], "GDN state sample")
    assert LI.digest(st_out) == str(gold["smoke_state_out_sha256"])


def test_layer_chain_matches_the_reference_check(port, gold):
    x = LI.layer_inputs()
    C, K = LI.QKV_ROWS, LI.KEY_DIM
    conv, conv_st = port.conv4_silu_roll(x["conv_state_in"], x["qkv"], x["conv_weight"])
    same(conv, gold["conv_out"], "conv4 + SiLU")
    assert LI.digest(conv_st) == str(gold["conv_state_out_sha256"])
    q = port.l2norm_heads(conv[:K], LI.QK_HEADS, LI.HEAD_DIM)
    k = port.l2norm_heads(conv[K:2 * K], LI.QK_HEADS, LI.HEAD_DIM)
    same(q, gold["q"], "q L2 norm")
    same(k, gold["k"], "k L2 norm")
    beta, gate = port.beta_gate(x["beta_raw"], x["alpha_raw"], x["dt_bias"], x["ssm_a"])
    same(beta, gold["beta"], "beta")
    same(gate, gold["gate"], "gate")
    o, st = port.gdn_step(q, k, conv[2 * K:C], gate, beta, x["gdn_state_in"], LI.QK_HEADS, LI.VALUE_HEADS,
                          LI.HEAD_DIM)
    same(o, gold["gdn_out"], "GDN output")
    assert LI.digest(st) == str(gold["gdn_state_out_sha256"])
    y = port.gated_rmsnorm_silu(o, x["z"], x["ssm_norm_weight"], LI.VALUE_HEADS, LI.HEAD_DIM)
    same(y, gold["gated"], "gated RMSNorm * SiLU(z)")


def test_ffn_pointwise_matches_the_reference_check(port, gold):
    f = LI.ffn_inputs()
    same(port.rmsnorm(f["residual"], f["post_norm_weight"]), gold["ffn_normed"], "RMSNorm")
    same(port.silu_mul(f["ffn_gate"], f["ffn_up"]), gold["ffn_mul"], "SiLU(gate) * up")
