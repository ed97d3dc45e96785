"""Host side of decode-from-pack, on the CPU: export_model_pack writes the
reference's tensor names, shapes, types and layouts from a model's tensors
(here a stand-in that serves seeded GGUF blocks in the engine's storage), and
the pack reader gives back exactly those blocks whatever the layout."""
from __future__ import annotations

import numpy as np
import pytest

from qwen382743090_b200 import q38pack, synth
from qwen382743090_b200 import runtime as rt

CFG = dict(n_layers=4, attn_every=4, hidden=1024, ffn=2048, vocab=1024, gdn_qk_heads=4, gdn_v_heads=8,
           attn_q_heads=12, attn_kv_heads=4, tp_size=1, seed=3)
H, F, V = 1024, 2048, 1024
D, AD, HQ, HV, AQ, AK = 128, 256, 4, 8, 12, 4
C = 2 * HQ * D + HV * D


class FakeModel:
    """Serves tensors as q38_model_tensor / Model.download would: layout-2
    tiles for Q5_K / Q4_K, GGUF blocks for Q6_K / IQ4_XS, f32 vectors."""

    def __init__(self, gate_type=12):
        self.cfg = dict(CFG)
        self.gate_type = gate_type
        self.blocks = {}

    def shape(self, n):
        f = n.split(".")[-1]
        table = {"attn_qkvz": (13, C + HV * D, H), "ssm_ba": (12, 2 * HV, H), "ssm_out": (13, H, HV * D),
                 "ffn_gate": (self.gate_type, F, H), "ffn_up": (13, F, H), "ffn_down": (13, H, F),
                 "attn_q": (13, 2 * AQ * AD, H), "attn_k": (13, AK * AD, H), "attn_v": (14, AK * AD, H),
                 "attn_output": (13, H, AQ * AD), "token_embd": (14, V, H), "output": (14, V, H)}
        vecs = {"attn_norm": H, "post_attention_norm": H, "ssm_conv1d": 4 * C, "ssm_dt": HV, "ssm_a": HV,
                "ssm_norm": D, "attn_q_norm": AD, "attn_k_norm": AD, "output_norm": H}
        return table.get(f), vecs.get(f)

    def tensor(self, n):
        mat, vec = self.shape(n)
        if vec:
            return rt.q38_weight_desc(0, 0, 1, vec, 0, 0, 0)
        t, rows, cols = mat
        return rt.q38_weight_desc(t, 2 if t in (12, 13) else 0, rows, cols, 0, 0, 0)

    def download(self, n):
        mat, vec = self.shape(n)
        seed = sum(map(ord, n))
        if vec:
            d = rt.q38_weight_desc(0, 0, 1, vec, 0, 0, 0)
            return d, synth.gen_f32(vec, seed).view(np.uint8)
        t, rows, cols = mat
        b = synth.gen_blocks(t, rows, cols, seed)
        self.blocks[n] = b.reshape(rows, -1)
        if t in (12, 13):
            return rt.q38_weight_desc(t, 2, rows, cols, 0, 0, 0), synth.repack_tiled(t, b, rows, cols)
        return rt.q38_weight_desc(t, 0, rows, cols, 0, 0, 0), b


@pytest.mark.parametrize("q5k_layout,q4k_layout,gate", [(2, 2, 12), (1, 0, 23), (0, 0, 12)])
def test_export_names_shapes_layouts_and_blocks(tmp_path, q5k_layout, q4k_layout, gate):
    m = FakeModel(gate)
    path = tmp_path / "m.q38pack"
    names = q38pack.export_model_pack(m, path, q5k_layout=q5k_layout, q4k_layout=q4k_layout)
    assert names == q38pack.model_tensor_names(CFG)
    with q38pack.open_pack(path) as p:
        assert p.header.version == (3 if 2 in (q5k_layout, q4k_layout) else 2)
        rec = {t.name.decode(): (i, t) for i, t in enumerate(p.tensors)}

        def blocks(name):
            return p.blocks(rec[name][0]).reshape(int(rec[name][1].dims[1]), -1)

        i, t = rec["blk.0.attn_qkv.weight"]
        assert (t.ggml_type, t.dims[0], t.dims[1], t.layout) == (13, H, C, q5k_layout)
        np.testing.assert_array_equal(blocks("blk.0.attn_qkv.weight"), m.blocks["blk.0.attn_qkvz"][:C])
        np.testing.assert_array_equal(blocks("blk.0.attn_gate.weight"), m.blocks["blk.0.attn_qkvz"][C:])
        assert rec["blk.0.ssm_beta.weight"][1].layout == q4k_layout
        np.testing.assert_array_equal(blocks("blk.0.ssm_beta.weight"), m.blocks["blk.0.ssm_ba"][:HV])
        np.testing.assert_array_equal(blocks("blk.0.ssm_alpha.weight"), m.blocks["blk.0.ssm_ba"][HV:])
        g = rec["blk.1.ffn_gate.weight"][1]
        assert (g.ggml_type, g.layout) == (gate, q4k_layout if gate == 12 else 0)
        np.testing.assert_array_equal(blocks("blk.1.ffn_gate.weight"), m.blocks["blk.1.ffn_gate"])
        np.testing.assert_array_equal(blocks("blk.2.ffn_down.weight"), m.blocks["blk.2.ffn_down"])
        np.testing.assert_array_equal(blocks("blk.3.attn_output.weight"), m.blocks["blk.3.attn_output"])
        assert rec["blk.3.attn_v.weight"][1].layout == 0
        np.testing.assert_array_equal(blocks("output.weight"), m.blocks["output"])
        conv = rec["blk.0.ssm_conv1d.weight"][1]
        assert (conv.ggml_type, conv.ndim, conv.dims[0], conv.dims[1]) == (0, 2, 4, C)
        np.testing.assert_array_equal(p.data(rec["blk.0.ssm_conv1d.weight"][0]).view(np.float32),
                                      synth.gen_f32(4 * C, sum(map(ord, "blk.0.ssm_conv1d"))))
        assert "blk.3.attn_qkv.weight" not in rec and "blk.0.attn_q.weight" not in rec


def test_export_refuses_a_shard():
    m = FakeModel()
    m.cfg["tp_size"] = 2
    with pytest.raises(ValueError):
        q38pack.export_model_pack(m, "/nonexistent/x.q38pack")
