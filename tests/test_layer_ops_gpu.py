"""GPU parity of the decoder-layer ops against the FP64 oracle, through the C ABI.

Shapes are the reference's (config 3): hidden 5120, qkv 10240 channels
(q 2048 | k 2048 | v 6144), 16 q/k heads and 48 value heads of 128, state
[48][128][128].  Inputs follow the synthetic spec: beta_raw ~ N(0,1),
g = ln(decay) with decay = exp(-softplus(N(0,1)) * 0.1), state N(0, 0.02).
Tolerance: 2e-5 relative to the vector's max magnitude for the pointwise
ops (fp32 arithmetic against FP64), 1e-4 for the recurrent state chain.
"""
from __future__ import annotations

import numpy as np
import pytest

from qwen382743090_b200 import runtime as rt
from qwen382743090_b200 import synth

pytestmark = pytest.mark.gpu

HQ, HV, D = 16, 48, 128
C = 2 * HQ * D + HV * D  # 10240


def close(got, ref, tol, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = max(np.abs(ref).max(), 1e-30)
    err = np.abs(got - ref).max() / scale
    assert err <= tol, f"{what}: max error {err:.3g} of max |ref| (tol {tol})"


def test_rmsnorm(ctx, port):
    for n in (5120, 17408, 1000):
        x = synth.gen_f32(n, seed=n)
        w = synth.gen_f32(n, seed=n + 1, scale=0.1, offset=1.0)
        xd, wd, yd = ctx.upload(x), ctx.upload(w), ctx.alloc(4 * n)
        rt.rmsnorm(xd.ptr, wd.ptr, yd.ptr, n, 1, 1e-6)
        close(yd.download(np.float32, n), port.rmsnorm(x, w, 1e-6), 2e-6, f"rmsnorm {n}")
        for b in (xd, wd, yd):
            b.free()


def test_conv4_silu_roll_in_place_and_separate(ctx, port):
    qkv = synth.gen_f32(C, seed=1)
    st = synth.gen_f32(3 * C, seed=2)
    w = synth.gen_f32(4 * C, seed=3, scale=0.5)
    out_ref, st_ref = port.conv4_silu_roll(st, qkv, w)
    qd, wd, sd, od = ctx.upload(qkv), ctx.upload(w), ctx.upload(st), ctx.alloc(4 * C)
    s2 = ctx.alloc(4 * 3 * C)
    rt.conv4_silu_roll(qd.ptr, wd.ptr, sd.ptr, od.ptr, s2.ptr, C)
    close(od.download(np.float32, C), out_ref, 2e-6, "conv out")
    np.testing.assert_array_equal(s2.download(np.float32, 3 * C), st_ref)
    rt.conv4_silu_roll(qd.ptr, wd.ptr, sd.ptr, od.ptr, sd.ptr, C)  # in place
    np.testing.assert_array_equal(sd.download(np.float32, 3 * C), st_ref)
    for b in (qd, wd, sd, od, s2):
        b.free()


def test_qk_l2norm_and_beta_gate(ctx, port):
    conv = synth.gen_f32(C, seed=4)
    cd, qd, kd = ctx.upload(conv), ctx.alloc(4 * HQ * D), ctx.alloc(4 * HQ * D)
    rt.qk_l2norm(cd.ptr, qd.ptr, kd.ptr, HQ, 1e-6)
    close(qd.download(np.float32, HQ * D), port.l2norm_heads(conv[: HQ * D], HQ, D, 1e-6), 2e-6, "q norm")
    close(kd.download(np.float32, HQ * D), port.l2norm_heads(conv[HQ * D: 2 * HQ * D], HQ, D, 1e-6), 2e-6, "k norm")
    b = synth.gen_f32(HV, seed=5)
    a = synth.gen_f32(HV, seed=6, scale=10.0)  # reaches both softplus branches
    a[:3] = [25.0, -25.0, 20.5]
    dt = synth.gen_f32(HV, seed=7)
    A = -np.abs(synth.gen_f32(HV, seed=8))
    bd, ad, dd, Ad = (ctx.upload(v) for v in (b, a, dt, A))
    beta_d, g_d = ctx.alloc(4 * HV), ctx.alloc(4 * HV)
    rt.beta_gate(bd.ptr, ad.ptr, dd.ptr, Ad.ptr, beta_d.ptr, g_d.ptr, HV)
    beta_ref, g_ref = port.beta_gate(b, a, dt, A)
    close(beta_d.download(np.float32, HV), beta_ref, 1e-6, "beta")
    close(g_d.download(np.float32, HV), g_ref, 1e-6, "gate")
    for buf in (cd, qd, kd, bd, ad, dd, Ad, beta_d, g_d):
        buf.free()


def gdn_inputs(seed):
    rng = np.random.default_rng(seed)
    q = port_norm(rng.standard_normal(HQ * D).astype(np.float32))
    k = port_norm(rng.standard_normal(HQ * D).astype(np.float32))
    v = rng.standard_normal(HV * D).astype(np.float32)
    sp = np.log1p(np.exp(rng.standard_normal(HV)))
    g = np.log(np.exp(-sp * 0.1)).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-rng.standard_normal(HV)))).astype(np.float32)
    state = (rng.standard_normal(HV * D * D) * 0.02).astype(np.float32)
    return q, k, v, g, beta, state


def port_norm(x):
    x = x.reshape(-1, D)
    return (x / np.sqrt((x.astype(np.float64) ** 2).sum(1, keepdims=True) + 1e-6)).astype(np.float32).reshape(-1)


def test_gdn_step_matches_oracle_in_place(ctx, port):
    q, k, v, g, beta, state = gdn_inputs(11)
    out_ref, st_ref = port.gdn_step(q, k, v, g, beta, state, HQ, HV, D)
    bufs = [ctx.upload(a) for a in (q, k, v, g, beta, state)]
    od = ctx.alloc(4 * HV * D)
    qd, kd, vd, gd, bd, sd = bufs
    rt.gdn_step(qd.ptr, kd.ptr, vd.ptr, gd.ptr, bd.ptr, sd.ptr, od.ptr, sd.ptr, HQ, HV, 1.0 / np.sqrt(D))
    close(od.download(np.float32, HV * D), out_ref, 1e-5, "gdn out")
    close(sd.download(np.float32, HV * D * D), st_ref, 1e-5, "gdn state")
    for b in (*bufs, od):
        b.free()


def test_gated_rmsnorm_silu_add_silu_mul(ctx, port):
    o = synth.gen_f32(HV * D, seed=21)
    z = synth.gen_f32(HV * D, seed=22)
    w = synth.gen_f32(D, seed=23, scale=0.1, offset=1.0)
    od, zd, wd, yd = ctx.upload(o), ctx.upload(z), ctx.upload(w), ctx.alloc(4 * HV * D)
    rt.gated_rmsnorm_silu(od.ptr, wd.ptr, zd.ptr, yd.ptr, HV, 1e-6)
    close(yd.download(np.float32, HV * D), port.gated_rmsnorm_silu(o, z, w, HV, D, 1e-6), 2e-6, "gated norm")
    n = 17408
    g = synth.gen_f32(n, seed=24, scale=3.0)
    u = synth.gen_f32(n, seed=25)
    gd, ud, yd2 = ctx.upload(g), ctx.upload(u), ctx.alloc(4 * n)
    rt.ffn_silu_mul(gd.ptr, ud.ptr, yd2.ptr, n)
    close(yd2.download(np.float32, n), port.silu_mul(g, u), 2e-6, "silu_mul")
    rt.add_residual(gd.ptr, ud.ptr, yd2.ptr, n)
    close(yd2.download(np.float32, n), port.add(g, u), 1e-7, "add")
    for b in (od, zd, wd, yd, gd, ud, yd2):
        b.free()


def test_gdn_fused_equals_op_chain_and_oracle(ctx, port):
    """The fused recurrent core against the FP64 chain conv -> norms -> gates
    -> GDN -> gated norm, over two consecutive tokens (state carried)."""
    rng = np.random.default_rng(31)
    conv_w = (rng.standard_normal(4 * C) * 0.5).astype(np.float32)
    conv_st = rng.standard_normal(3 * C).astype(np.float32)
    dt = rng.standard_normal(HV).astype(np.float32)
    A = -np.exp(rng.standard_normal(HV)).astype(np.float32)
    norm_w = (1.0 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    state = (rng.standard_normal(HV * D * D) * 0.02).astype(np.float32)
    dev = {n: ctx.upload(a) for n, a in dict(conv_w=conv_w, dt=dt, A=A, norm_w=norm_w, state=state).items()}
    cin, cout = ctx.upload(conv_st), ctx.alloc(4 * 3 * C)
    yd = ctx.alloc(4 * HV * D)
    ref_conv, ref_state = conv_st, state
    for tok in range(2):
        qkv = rng.standard_normal(C).astype(np.float32)
        braw = rng.standard_normal(HV).astype(np.float32)
        araw = rng.standard_normal(HV).astype(np.float32)
        z = rng.standard_normal(HV * D).astype(np.float32)
        tok_dev = [ctx.upload(a) for a in (qkv, braw, araw, z)]
        args = rt.q38_gdn_fused_args(tok_dev[0].ptr, dev["conv_w"].ptr, cin.ptr, cout.ptr, tok_dev[1].ptr,
                                     tok_dev[2].ptr, dev["dt"].ptr, dev["A"].ptr, dev["state"].ptr,
                                     dev["state"].ptr, tok_dev[3].ptr, dev["norm_w"].ptr, yd.ptr, HQ, HV, 1e-6,
                                     1.0 / np.sqrt(D))
        rt.gdn_fused(args)
        # FP64 reference chain
        conv, ref_conv = port.conv4_silu_roll(ref_conv, qkv, conv_w)
        qn = port.l2norm_heads(conv[: HQ * D], HQ, D, 1e-6)
        kn = port.l2norm_heads(conv[HQ * D: 2 * HQ * D], HQ, D, 1e-6)
        beta, g = port.beta_gate(braw, araw, dt, A)
        o, ref_state = port.gdn_step(qn, kn, conv[2 * HQ * D:], g, beta, ref_state, HQ, HV, D)
        y_ref = port.gated_rmsnorm_silu(o, z, norm_w, HV, D, 1e-6)
        close(yd.download(np.float32, HV * D), y_ref, 1e-4, f"fused out token {tok}")
        np.testing.assert_array_equal(cout.download(np.float32, 3 * C), ref_conv)
        close(dev["state"].download(np.float32, HV * D * D), ref_state, 1e-4, f"fused state token {tok}")
        cin, cout = cout, cin  # ping-pong the conv state
        for b in tok_dev:
            b.free()
    with pytest.raises(rt.Q38Error):
        bad = rt.q38_gdn_fused_args(*([8 * 1024] * 13), HQ, HV, 1e-6, 0.1)
        rt.gdn_fused(bad)  # conv_in == conv_out is rejected before any launch
    for b in (*dev.values(), cin, cout, yd):
        b.free()
