"""The decoder-layer kernels against values computed by the reference's own CPU
code (tests/golden/layer_golden.npz, made by tests/golden/make_layer_golden.py
from src/driver.cpp:8080-8242, 8365-8393 and 11198-11301).

Each device op runs on the fixture's inputs: the seeded config-3 / FFN inputs
(regenerated and checked against the fixture's digests) and the reference's
own GDN smoke inputs (restated by the oracle, whose bit-exactness to the
reference's generator tests/test_layer_golden.py pins).  Tolerances are those
of the layer-op tests: 2e-6 of the vector's max magnitude for the pointwise
ops, 1e-5 for one GDN step and 1e-4 for what follows the recurrent state
(the gated norm of the device's own GDN output, the fused recurrent core).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

from qwen382743090_b200 import runtime as rt

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import layer_inputs as LI  # noqa: E402

pytestmark = pytest.mark.gpu
HQ, HV, D, C, K = LI.QK_HEADS, LI.VALUE_HEADS, LI.HEAD_DIM, LI.QKV_ROWS, LI.KEY_DIM


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(GOLDEN / "layer_golden.npz"))


def close(got, ref, tol, what):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    err = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
    assert err <= tol, f"{what}: max error {err:.3g} of max |ref| (tol {tol})"


def test_gdn_step_on_the_reference_smoke_inputs(ctx, port, gold):
    q, k, v, g, beta, st = port.gdn_smoke_inputs()
    assert LI.digest(st) == str(gold["smoke_state_in_sha256"])
    bufs = [ctx.upload(a) for a in (q, k, v, g, beta, st)]
    od = ctx.alloc(4 * HV * D)
    qd, kd, vd, gd, bd, sd = bufs
    rt.gdn_step(qd.ptr, kd.ptr, vd.ptr, gd.ptr, bd.ptr, sd.ptr, od.ptr, sd.ptr, HQ, HV, 1.0 / np.sqrt(D))
    close(od.download(np.float32, HV * D), gold["smoke_out"], 1e-5, "GDN output")
    st_out = sd.download(np.float32, HV * D * D)
    close(st_out[gold["state_sample_index"]], gold["smoke_state_out_sample"], 1e-5, "GDN state sample")
    assert rt.fault_status() == 0
    for b in (*bufs, od):
        b.free()


def test_layer_ops_on_the_reference_check_inputs(ctx, gold):
    x = LI.layer_inputs()
    for k, v in x.items():
        assert LI.digest(v) == str(gold["input_" + k + "_sha256"]), k
    qkv, w = ctx.upload(x["qkv"]), ctx.upload(x["conv_weight"])
    sin, sout, conv = ctx.upload(x["conv_state_in"]), ctx.alloc(4 * 3 * C), ctx.alloc(4 * C)
    rt.conv4_silu_roll(qkv.ptr, w.ptr, sin.ptr, conv.ptr, sout.ptr, C)
    close(conv.download(np.float32, C), gold["conv_out"], 2e-6, "conv4 + SiLU")
    assert LI.digest(sout.download(np.float32, 3 * C)) == str(gold["conv_state_out_sha256"])
    qd, kd = ctx.alloc(4 * K), ctx.alloc(4 * K)
    rt.qk_l2norm(conv.ptr, qd.ptr, kd.ptr, HQ, 1e-6)
    close(qd.download(np.float32, K), gold["q"], 2e-6, "q L2 norm")
    close(kd.download(np.float32, K), gold["k"], 2e-6, "k L2 norm")
    br, ar, dt, A = (ctx.upload(x[n]) for n in ("beta_raw", "alpha_raw", "dt_bias", "ssm_a"))
    beta, gate = ctx.alloc(4 * HV), ctx.alloc(4 * HV)
    rt.beta_gate(br.ptr, ar.ptr, dt.ptr, A.ptr, beta.ptr, gate.ptr, HV)
    close(beta.download(np.float32, HV), gold["beta"], 1e-6, "beta")
    close(gate.download(np.float32, HV), gold["gate"], 1e-6, "gate")
    # the GDN step on the device's own q, k, v, gate and beta
    st, od = ctx.upload(x["gdn_state_in"]), ctx.alloc(4 * HV * D)
    rt.gdn_step(qd.ptr, kd.ptr, conv.ptr + 4 * 2 * K, gate.ptr, beta.ptr, st.ptr, od.ptr, st.ptr, HQ, HV,
                1.0 / np.sqrt(D))
    close(od.download(np.float32, HV * D), gold["gdn_out"], 1e-5, "GDN output")
    close(st.download(np.float32, HV * D * D)[gold["state_sample_index"]], gold["gdn_state_out_sample"], 1e-5,
          "GDN state sample")
    zd, nw, yd = ctx.upload(x["z"]), ctx.upload(x["ssm_norm_weight"]), ctx.alloc(4 * HV * D)
    rt.gated_rmsnorm_silu(od.ptr, nw.ptr, zd.ptr, yd.ptr, HV, 1e-6)
    close(yd.download(np.float32, HV * D), gold["gated"], 1e-4, "gated RMSNorm * SiLU(z) after the GDN step")
    assert rt.fault_status() == 0
    for b in (qkv, w, sin, sout, conv, qd, kd, br, ar, dt, A, beta, gate, st, od, zd, nw, yd):
        b.free()


def test_fused_recurrent_core_on_the_reference_check_inputs(ctx, gold):
    x = LI.layer_inputs()
    dev = {n: ctx.upload(x[n]) for n in ("qkv", "conv_weight", "conv_state_in", "beta_raw", "alpha_raw", "dt_bias",
                                         "ssm_a", "gdn_state_in", "z", "ssm_norm_weight")}
    cout, yd = ctx.alloc(4 * 3 * C), ctx.alloc(4 * HV * D)
    args = rt.q38_gdn_fused_args(dev["qkv"].ptr, dev["conv_weight"].ptr, dev["conv_state_in"].ptr, cout.ptr,
                                 dev["beta_raw"].ptr, dev["alpha_raw"].ptr, dev["dt_bias"].ptr, dev["ssm_a"].ptr,
                                 dev["gdn_state_in"].ptr, dev["gdn_state_in"].ptr, dev["z"].ptr,
                                 dev["ssm_norm_weight"].ptr, yd.ptr, HQ, HV, 1e-6, 1.0 / np.sqrt(D))
    rt.gdn_fused(args)
    close(yd.download(np.float32, HV * D), gold["gated"], 1e-4, "fused core output")
    assert LI.digest(cout.download(np.float32, 3 * C)) == str(gold["conv_state_out_sha256"])
    st = dev["gdn_state_in"].download(np.float32, HV * D * D)
    close(st[gold["state_sample_index"]], gold["gdn_state_out_sample"], 1e-4, "fused core state sample")
    assert rt.fault_status() == 0
    for b in (*dev.values(), cout, yd):
        b.free()


def test_ffn_pointwise_on_the_reference_check_inputs(ctx, gold):
    f = LI.ffn_inputs()
    r, w, y = ctx.upload(f["residual"]), ctx.upload(f["post_norm_weight"]), ctx.alloc(4 * LI.HIDDEN)
    rt.rmsnorm(r.ptr, w.ptr, y.ptr, LI.HIDDEN, 1, 1e-6)
    close(y.download(np.float32, LI.HIDDEN), gold["ffn_normed"], 2e-6, "RMSNorm")
    g, u, m = ctx.upload(f["ffn_gate"]), ctx.upload(f["ffn_up"]), ctx.alloc(4 * LI.FFN_DIM)
    rt.ffn_silu_mul(g.ptr, u.ptr, m.ptr, LI.FFN_DIM)
    close(m.download(np.float32, LI.FFN_DIM), gold["ffn_mul"], 2e-6, "SiLU(gate) * up")
    for b in (r, w, y, g, u, m):
        b.free()


def ulp_close(got, ref, what, ulps=2):
    """Elementwise within a couple of float ulps: only the device's double
    exp / log1p / sqrt differ from the host's."""
    got, ref = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    tol = ulps * np.spacing(np.abs(ref)) + 1e-30
    bad = np.abs(got.astype(np.float64) - ref.astype(np.float64)) > tol
    assert not bad.any(), f"{what}: {bad.sum()} values beyond {ulps} ulp"


def test_device_check_entries_reproduce_the_reference_loops(ctx, port, gold):
    """The plain FP64 device checks (q38_check_*) that the C++ facade's layer
    smokes compare against, on the fixture's inputs."""
    x, f = LI.layer_inputs(), LI.ffn_inputs()
    d = {n: ctx.upload(a) for n, a in {**x, **f}.items()}
    conv, sout = ctx.alloc(4 * C), ctx.alloc(4 * 3 * C)
    rt.check_conv4(d["qkv"].ptr, d["conv_weight"].ptr, d["conv_state_in"].ptr, conv.ptr, sout.ptr, C)
    ulp_close(conv.download(np.float32, C), gold["conv_out"], "conv4")
    assert LI.digest(sout.download(np.float32, 3 * C)) == str(gold["conv_state_out_sha256"])
    qd, kd = ctx.alloc(4 * K), ctx.alloc(4 * K)
    rt.check_l2norm(conv.ptr, HQ, D, 1e-6, qd.ptr)
    rt.check_l2norm(conv.ptr + 4 * K, HQ, D, 1e-6, kd.ptr)
    ulp_close(qd.download(np.float32, K), gold["q"], "q norm")
    ulp_close(kd.download(np.float32, K), gold["k"], "k norm")
    beta, gate = ctx.alloc(4 * HV), ctx.alloc(4 * HV)
    rt.check_beta_gate(d["beta_raw"].ptr, d["alpha_raw"].ptr, d["dt_bias"].ptr, d["ssm_a"].ptr, HV, beta.ptr, gate.ptr)
    ulp_close(beta.download(np.float32, HV), gold["beta"], "beta")
    ulp_close(gate.download(np.float32, HV), gold["gate"], "gate")
    od, so = ctx.alloc(4 * HV * D), ctx.alloc(4 * HV * D * D)
    rt.check_gdn(qd.ptr, kd.ptr, conv.ptr + 8 * K, gate.ptr, beta.ptr, d["gdn_state_in"].ptr, od.ptr, so.ptr, HQ, HV, D)
    ulp_close(od.download(np.float32, HV * D), gold["gdn_out"], "GDN out", ulps=4)
    ulp_close(so.download(np.float32, HV * D * D)[gold["state_sample_index"]], gold["gdn_state_out_sample"],
              "GDN state", ulps=4)
    yd = ctx.alloc(4 * HV * D)
    rt.check_rmsnorm(od.ptr, d["ssm_norm_weight"].ptr, d["z"].ptr, HV, D, 1e-6, yd.ptr)
    ulp_close(yd.download(np.float32, HV * D), gold["gated"], "gated norm", ulps=8)
    fn, fm = ctx.alloc(4 * LI.HIDDEN), ctx.alloc(4 * LI.FFN_DIM)
    rt.check_rmsnorm(d["residual"].ptr, d["post_norm_weight"].ptr, 0, 1, LI.HIDDEN, 1e-6, fn.ptr)
    ulp_close(fn.download(np.float32, LI.HIDDEN), gold["ffn_normed"], "RMSNorm")
    rt.check_silu_mul(d["ffn_gate"].ptr, d["ffn_up"].ptr, LI.FFN_DIM, fm.ptr)
    ulp_close(fm.download(np.float32, LI.FFN_DIM), gold["ffn_mul"], "SiLU * up")
    # the GDN check on the reference's own smoke inputs
    q, k, v, g, b, st = port.gdn_smoke_inputs()
    s = [ctx.upload(a) for a in (q, k, v, g, b, st)]
    o2, st2 = ctx.alloc(4 * HV * D), ctx.alloc(4 * HV * D * D)
    rt.check_gdn(*(a.ptr for a in s), o2.ptr, st2.ptr, HQ, HV, D)
    ulp_close(o2.download(np.float32, HV * D), gold["smoke_out"], "smoke GDN out", ulps=4)
    ulp_close(st2.download(np.float32, HV * D * D)[gold["state_sample_index"]], gold["smoke_state_out_sample"],
              "smoke GDN state", ulps=4)
    for bf in (*d.values(), conv, sout, qd, kd, beta, gate, od, so, yd, fn, fm, *s, o2, st2):
        bf.free()
