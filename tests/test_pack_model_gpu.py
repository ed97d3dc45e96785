"""Decode from a Q38PACK (q38_model_create_from_pack): a seeded model's weights
written as a pack with the reference's tensor names -- Q5_K as GGUF blocks, as
the reference's SoA planes or as B200 tiles -- and loaded back give the same
tensors byte for byte and the same greedy tokens and logits bit for bit; a
pack that does not match the config is refused with the tensor's name."""
from __future__ import annotations

import numpy as np
import pytest

from qwen382743090_b200 import q38pack
from qwen382743090_b200 import runtime as rt

pytestmark = pytest.mark.gpu

# 3 recurrent layers and one attention layer at small widths (every
# dimension rule of the engine holds: hidden and ffn multiples of 1024,
# 8 value heads over 4 q/k heads, 12 query heads over 4 KV heads)
TINY = dict(n_layers=4, attn_every=4, hidden=1024, ffn=2048, vocab=4096, gdn_qk_heads=4, gdn_v_heads=8,
            attn_q_heads=12, attn_kv_heads=4, rope_dim=64, ctx=256, seed=7)
STEPS = 8


def engine_names(cfg):
    out = ["token_embd", "output", "output_norm"]
    for L in range(cfg["n_layers"]):
        b = f"blk.{L}."
        out += [b + s for s in ("attn_norm", "post_attention_norm", "ffn_gate", "ffn_up", "ffn_down")]
        if L % cfg["attn_every"] == cfg["attn_every"] - 1:
            out += [b + s for s in ("attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm", "attn_k_norm")]
        else:
            out += [b + s for s in ("attn_qkvz", "ssm_ba", "ssm_out", "ssm_conv1d", "ssm_dt", "ssm_a", "ssm_norm",
                                    "conv_state0", "ssm_state")]
    return out


def decode(m, steps=STEPS):
    m.set_position(token=11, pos=20, kv_seed=5)
    toks, logits = [], []
    for _ in range(steps):
        m.step()
        toks.append(m.position()[0])
        logits.append(m.download("logits")[1].copy())
    return toks, logits


@pytest.fixture(scope="module")
def seeded(ctx):
    """Seeded models, their tensors as created (decoding updates the states)
    and their greedy decode."""
    out = {}
    for gate in (0, 23):
        m = rt.Model(**TINY, ffn_gate_type=gate)
        first = {n: m.download(n) for n in engine_names(TINY)}
        out[gate] = (m, first, decode(m))
    yield out
    for m, _, _ in out.values():
        m.close()


@pytest.mark.parametrize("gate", [0, 23])
@pytest.mark.parametrize("q5k_layout,q4k_layout", [(2, 2), (1, 0), (0, 0)])
def test_pack_roundtrip_bit_exact(seeded, tmp_path, gate, q5k_layout, q4k_layout):
    src, first, (toks, logits) = seeded[gate]
    path = tmp_path / "model.q38pack"
    names = q38pack.export_model_pack(src, path, q5k_layout=q5k_layout, q4k_layout=q4k_layout)
    assert names == q38pack.model_tensor_names(src.cfg)
    with q38pack.open_pack(path) as p:
        layouts = {t.name.decode(): t.layout for t in p.tensors}
        assert layouts["blk.0.attn_qkv.weight"] == q5k_layout
        assert p.header.version == (3 if 2 in (q5k_layout, q4k_layout) else 2)
    with rt.Model(pack=path, **TINY, ffn_gate_type=gate) as m:
        for n in engine_names(TINY):
            d0, a = first[n]
            d1, b = m.download(n)
            assert (d0.ggml_type, d0.layout, d0.rows, d0.cols) == (d1.ggml_type, d1.layout, d1.rows, d1.cols), n
            np.testing.assert_array_equal(a, b, err_msg=n)
        t2, l2 = decode(m)
    assert t2 == toks
    for a, b in zip(logits, l2):
        np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    assert rt.fault_status() == 0


def test_pack_refused_when_shapes_differ(seeded, tmp_path):
    src = seeded[0][0]
    path = tmp_path / "model.q38pack"
    q38pack.export_model_pack(src, path)
    with pytest.raises(rt.Q38Error, match="attn_norm.weight"):
        rt.Model(pack=path, **dict(TINY, hidden=2048))
    with pytest.raises(rt.Q38Error, match="ffn_gate.weight"):
        rt.Model(pack=path, **TINY, ffn_gate_type=23)  # the pack's gate is Q4_K
    with pytest.raises(rt.Q38Error, match="no tensor 'blk.4"):
        rt.Model(pack=path, **dict(TINY, n_layers=8))
