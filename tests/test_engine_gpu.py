"""The decode engine against an FP64 oracle chain at the full layer dimensions.

A 4-layer model (3 Gated DeltaNet layers, then one GQA attention layer) with
hidden 5120, FFN 17408 and the real head geometry; vocab and context are cut
down so the FP64 chain runs in seconds.  The oracle rebuilds every layer from
the engine's own weights, read back from the device: GEMVs are FP64 dots of
the dequantised GGUF blocks (layout-2 tensors are un-tiled on the host first),
the pointwise ops are the restatements of the reference's composition check.
Tolerance (config 4): layer outputs within 2e-3 of max |ref|.
"""
from __future__ import annotations

import numpy as np
import pytest

from qwen382743090_b200 import runtime as rt
from qwen382743090_b200 import synth

pytestmark = pytest.mark.gpu

HQ, HV, D = 16, 48, 128
AQ, AK, AD = 24, 4, 256
H, F = 5120, 17408
C = 2 * HQ * D + HV * D
SMALL = dict(n_layers=4, attn_every=4, vocab=4096, ctx=512, seed=99)
EPS = 1e-6
LAYER_TOL = 2e-3


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)


class Chain:
    """FP64 oracle chain over a model's downloaded weights."""

    def __init__(self, model, port):
        self.m, self.port = model, port

    def f32(self, name):
        return self.m.download(name)[1].view(np.float32).copy()

    def gemv(self, name, x):
        d, raw = self.m.download(name)
        blocks = raw if d.layout == 0 else synth.untile(d.ggml_type, raw, d.rows, d.cols)
        return self.port.gemv(d.ggml_type, blocks, np.asarray(x, np.float32), d.rows, d.cols, threads=16)[0]

    def ffn(self, L, x1):
        p = self.port
        h2 = p.rmsnorm(x1, self.f32(f"blk.{L}.post_attention_norm"), EPS)
        g = self.gemv(f"blk.{L}.ffn_gate", h2).astype(np.float32)
        u = self.gemv(f"blk.{L}.ffn_up", h2).astype(np.float32)
        mm = p.silu_mul(g, u)
        return (x1.astype(np.float64) + self.gemv(f"blk.{L}.ffn_down", mm)).astype(np.float32)

    def recurrent(self, L, x, conv_in, state):
        p = self.port
        h = p.rmsnorm(x, self.f32(f"blk.{L}.attn_norm"), EPS)
        qkvz = self.gemv(f"blk.{L}.attn_qkvz", h).astype(np.float32)
        ba = self.gemv(f"blk.{L}.ssm_ba", h).astype(np.float32)
        conv, conv_out = p.conv4_silu_roll(conv_in, qkvz[:C], self.f32(f"blk.{L}.ssm_conv1d"))
        qn = p.l2norm_heads(conv[: HQ * D], HQ, D, EPS)
        kn = p.l2norm_heads(conv[HQ * D: 2 * HQ * D], HQ, D, EPS)
        beta, g = p.beta_gate(ba[:HV], ba[HV:], self.f32(f"blk.{L}.ssm_dt"), self.f32(f"blk.{L}.ssm_a"))
        o, state_out = p.gdn_step(qn, kn, conv[2 * HQ * D:], g, beta, state, HQ, HV, D)
        y = p.gated_rmsnorm_silu(o, qkvz[C:], self.f32(f"blk.{L}.ssm_norm"), HV, D, EPS)
        x1 = (x.astype(np.float64) + self.gemv(f"blk.{L}.ssm_out", y)).astype(np.float32)
        return self.ffn(L, x1), conv_out, state_out

    def attention(self, L, x, kc, vc, pos, ctx, rope_dim=64, theta=1.0e7):
        p = self.port
        h = p.rmsnorm(x, self.f32(f"blk.{L}.attn_norm"), EPS)
        qg = self.gemv(f"blk.{L}.attn_q", h).astype(np.float32).reshape(AQ, 2 * AD)
        k = self.gemv(f"blk.{L}.attn_k", h).astype(np.float32).reshape(AK, AD)
        v = self.gemv(f"blk.{L}.attn_v", h).astype(np.float32).reshape(AK, AD)
        qnw, knw = self.f32(f"blk.{L}.attn_q_norm"), self.f32(f"blk.{L}.attn_k_norm")
        q = np.stack([p.rmsnorm(qg[i, :AD], qnw, EPS) for i in range(AQ)]).reshape(-1)
        kn = np.stack([p.rmsnorm(k[i], knw, EPS) for i in range(AK)]).reshape(-1)
        q = p.rope(q, AQ, AD, rope_dim, pos, theta)
        kn = p.rope(kn, AK, AD, rope_dim, pos, theta)
        kc = kc.reshape(AK, ctx, AD).copy()
        vc = vc.reshape(AK, ctx, AD).copy()
        kc[:, pos] = kn.reshape(AK, AD).astype(np.float16).view(np.uint16)
        vc[:, pos] = v.astype(np.float16).view(np.uint16)
        o = p.attn_decode(q, kc, vc, AQ, AK, AD, pos + 1, ctx).reshape(AQ, AD).astype(np.float64)
        gate = qg[:, AD:].astype(np.float64)
        o = (o / (1.0 + np.exp(-gate))).astype(np.float32).reshape(-1)
        x1 = (x.astype(np.float64) + self.gemv(f"blk.{L}.attn_output", o)).astype(np.float32)
        return self.ffn(L, x1), kc, vc


@pytest.fixture(scope="module")
def model(ctx):
    m = rt.Model(**SMALL)
    yield m
    m.close()


def test_recurrent_layer_matches_oracle(model, ctx, port):
    model.set_position(token=5, pos=36, kv_seed=3)  # even position: conv state 0 is the input
    ch = Chain(model, port)
    conv_in = ch.f32("blk.0.conv_state0")
    state = ch.f32("blk.0.ssm_state")
    x = synth.gen_f32(H, seed=1)
    xd = ctx.upload(x)
    model.layer(0, xd.ptr)
    got = xd.download(np.float32, H)
    ref, conv_ref, state_ref = ch.recurrent(0, x, conv_in, state)
    assert rel_err(got, ref) <= LAYER_TOL, rel_err(got, ref)
    conv_got = ch.f32("blk.0.conv_state1")
    np.testing.assert_array_equal(conv_got[: 2 * C], conv_ref[: 2 * C])  # rolled columns move exactly
    assert rel_err(conv_got[2 * C:], conv_ref[2 * C:]) <= 1e-5  # the new column is the qkv GEMV output
    assert rel_err(ch.f32("blk.0.ssm_state"), state_ref) <= 1e-4
    assert rt.fault_status() == 0
    xd.free()


def test_attention_layer_matches_oracle(model, ctx, port):
    pos = 300
    model.set_position(token=9, pos=pos, kv_seed=11)
    ch = Chain(model, port)
    kc = model.download("blk.3.k_cache")[1].view(np.uint16)
    vc = model.download("blk.3.v_cache")[1].view(np.uint16)
    x = synth.gen_f32(H, seed=2)
    xd = ctx.upload(x)
    model.layer(3, xd.ptr)
    got = xd.download(np.float32, H)
    ref, kc_ref, vc_ref = ch.attention(3, x, kc, vc, pos, SMALL["ctx"])
    assert rel_err(got, ref) <= LAYER_TOL, rel_err(got, ref)
    kc_got = model.download("blk.3.k_cache")[1].view(np.float16).reshape(AK, -1, AD)
    assert rel_err(kc_got[:, pos], kc_ref.view(np.float16)[:, pos]) <= 2e-3
    vc_got = model.download("blk.3.v_cache")[1].view(np.float16).reshape(AK, -1, AD)
    assert rel_err(vc_got[:, pos], vc_ref.view(np.float16)[:, pos]) <= 2e-3  # fp16 of the v GEMV output
    xd.free()


def test_attention_long_context_multi_chunk(ctx, port):
    """A context long enough that every split CTA streams its tokens in more
    than one shared-memory chunk (online softmax across chunks)."""
    long_ctx, pos = 10240, 9000
    m = rt.Model(**dict(SMALL, ctx=long_ctx))
    try:
        m.set_position(token=5, pos=pos, kv_seed=13)
        ch = Chain(m, port)
        kc = m.download("blk.3.k_cache")[1].view(np.uint16)
        vc = m.download("blk.3.v_cache")[1].view(np.uint16)
        x = synth.gen_f32(H, seed=4)
        xd = ctx.upload(x)
        m.layer(3, xd.ptr)
        got = xd.download(np.float32, H)
        ref, _, _ = ch.attention(3, x, kc, vc, pos, long_ctx)
        assert rel_err(got, ref) <= LAYER_TOL, rel_err(got, ref)
        assert rt.fault_status() == 0
        xd.free()
    finally:
        m.close()


def test_decode_step_matches_oracle_chain(model, port):
    """embed -> 3 GDN layers -> attention layer -> norm -> lm_head -> argmax."""
    pos, token = 128, 1234
    model.set_position(token=token, pos=pos, kv_seed=5)
    ch = Chain(model, port)
    convs = [ch.f32(f"blk.{L}.conv_state0") for L in range(3)]
    states = [ch.f32(f"blk.{L}.ssm_state") for L in range(3)]
    kc = model.download("blk.3.k_cache")[1].view(np.uint16)
    vc = model.download("blk.3.v_cache")[1].view(np.uint16)
    model.step()
    tok, new_pos = model.position()
    logits = ch.f32("logits")
    d, emb = model.download("token_embd")
    nb = H // 256
    x = port.dequant(14, emb.reshape(-1, nb * 210)[token])
    for L in range(3):
        x, _, _ = ch.recurrent(L, x, convs[L], states[L])
    x, _, _ = ch.attention(3, x, kc, vc, pos, SMALL["ctx"])
    h = port.rmsnorm(x, ch.f32("output_norm"), EPS)
    ref = ch.gemv("output", h)
    assert new_pos == pos + 1
    assert rel_err(logits, ref) <= LAYER_TOL, rel_err(logits, ref)
    assert tok == int(np.argmax(logits))
    top2 = np.sort(ref)[-2:]
    if top2[1] - top2[0] > 4 * LAYER_TOL * np.abs(ref).max():
        assert tok == int(np.argmax(ref))


def test_graph_replay_equals_eager_steps(ctx):
    torch = pytest.importorskip("torch")
    a = rt.Model(**SMALL)
    b = rt.Model(**SMALL)
    try:
        for m in (a, b):
            m.set_position(token=17, pos=40, kv_seed=9)
        toks_a = []
        for _ in range(4):
            a.step()
            toks_a.append(a.position())
        s = torch.cuda.Stream()
        b.capture(2, s.cuda_stream)
        toks_b = []
        for _ in range(2):
            b.replay(s.cuda_stream)
            s.synchronize()
            toks_b.append(b.position())
        assert toks_b == [toks_a[1], toks_a[3]]
        la = a.download("logits")[1]
        lb = b.download("logits")[1]
        np.testing.assert_array_equal(la, lb)
        assert rt.fault_status() == 0
    finally:
        a.close()
        b.close()


def test_iq4xs_ffn_gate_layer_matches_oracle(ctx, port):
    """The reference model's ffn_gate is IQ4_XS (src/layer_topology.cpp:87):
    with ffn_gate_type 23 the gate is an IQ4_XS tile matrix paired with ffn_up
    in one launch over the post-attention norm's x-fragments."""
    with rt.Model(**dict(SMALL, n_layers=1), ffn_gate_type=23) as m:
        assert m.tensor("blk.0.ffn_gate").ggml_type == 23 and m.tensor("blk.0.ffn_gate").layout == 2
        m.set_position(token=5, pos=36, kv_seed=3)
        ch = Chain(m, port)
        conv_in = ch.f32("blk.0.conv_state0")
        state = ch.f32("blk.0.ssm_state")
        x = synth.gen_f32(H, seed=8)
        xd = ctx.upload(x)
        m.layer(0, xd.ptr)
        got = xd.download(np.float32, H)
        ref, _, _ = ch.recurrent(0, x, conv_in, state)
        assert rel_err(got, ref) <= LAYER_TOL, rel_err(got, ref)
        assert rt.fault_status() == 0
        xd.free()
