"""Q38PACK container: the library's mmap reader against files written here,
the reference's own Python reader (when its sources are present), the
placement plan arithmetic of PlacementPlan::build (src/placement.cpp:23-60),
the v1/v2 -> v3 converter and the q38-plan CLI.  No GPU needed.
"""
from __future__ import annotations

import io
import sys
from contextlib import redirect_stdout
from pathlib import Path

import numpy as np
import pytest

from qwen382743090_b200 import cli, q38pack, runtime as rt, synth

import oracle  # noqa: E402  (locates the reference tree; test infrastructure)

_REF_ROOT = oracle.reference_root()
REF_TOOLS = (_REF_ROOT / "tools") if _REF_ROOT else Path("reference-tree-absent")


@pytest.fixture
def pack2(tmp_path):
    path = tmp_path / "m.q38pack"
    names = q38pack.synthetic_pack(path, seed=9, hidden=1024, layers=2, q5k_layout=1, version=2)
    return path, names


def test_reader_round_trip(pack2):
    path, names = pack2
    with q38pack.open_pack(path) as p:
        assert p.header.version == 2 and p.header.tensor_count == len(names)
        assert [t.name.decode() for t in p.tensors] == names
        for i, t in enumerate(p.tensors):
            assert t.data_offset % 128 == 0 and t.data_offset >= p.header.data_offset
            if t.layout == 1:
                assert t.data_offset <= t.aux0_offset <= t.aux1_offset < t.data_offset + t.stored_bytes
        i = p.find("blk.1.attn_qkv.weight")
        blocks = synth.gen_blocks(13, 2048, 1024, 9 + 6)  # the generator's seed sequence
        assert np.array_equal(p.blocks(i), blocks)
        with pytest.raises(rt.Q38Error):
            p.find("missing.weight")


def test_plan_matches_placement_rule(pack2):
    path, _ = pack2
    with q38pack.open_pack(path) as p:
        st, off = p.plan(2 << 20)
        cursor, payload = 0, 0
        for t, o in zip(p.tensors, off):
            cursor = (cursor + 255) // 256 * 256
            assert int(o) == cursor
            cursor += t.stored_bytes
            payload += t.stored_bytes
        assert st.tensor_payload_bytes == payload
        assert st.reserved_va_bytes == (cursor + (2 << 20) - 1) // (2 << 20) * (2 << 20)
        assert st.page_count == st.reserved_va_bytes // (2 << 20)
        with pytest.raises(rt.Q38Error):
            p.plan(3 << 20)


def test_converter_keeps_weights_and_bumps_version(pack2, tmp_path):
    path, names = pack2
    dst = tmp_path / "m3.q38pack"
    s = q38pack.convert_to_b200(path, dst)
    with q38pack.open_pack(path) as a:
        n2 = sum(1 for t in a.tensors if t.ggml_type in (12, 13) and t.ndim == 2 and int(t.dims[0]) % 512 == 0)
    assert n2 > 0 and s["converted"] == n2 and s["copied"] == len(names) - n2
    with q38pack.open_pack(path) as a, q38pack.open_pack(dst) as b:
        assert b.header.version == 3
        for i, t in enumerate(b.tensors):
            j = a.find(t.name.decode())
            if t.ggml_type in (12, 13, 14, 23):
                assert np.array_equal(b.blocks(i), a.blocks(j))
            else:
                assert np.array_equal(b.data(i), a.data(j))
            assert t.layout == (2 if t.ggml_type in (12, 13) else a.tensors[j].layout)


def test_corrupt_files_are_rejected(tmp_path, pack2):
    path, _ = pack2
    raw = bytearray(path.read_bytes())
    bad = tmp_path / "bad.q38pack"
    raw2 = bytearray(raw)
    raw2[0] = ord("X")
    bad.write_bytes(bytes(raw2))
    with pytest.raises(rt.Q38Error):
        q38pack.open_pack(bad)
    raw3 = bytearray(raw)
    raw3[8] = 9  # version 9
    bad.write_bytes(bytes(raw3))
    with pytest.raises(rt.Q38Error):
        q38pack.open_pack(bad)
    bad.write_bytes(bytes(raw[: 256 + 100]))  # truncated directory
    with pytest.raises(rt.Q38Error):
        q38pack.open_pack(bad)


@pytest.mark.skipif(not REF_TOOLS.exists(), reason="reference sources not present")
def test_reference_reader_reads_v2_and_rejects_v3(pack2, tmp_path):
    sys.path.insert(0, str(REF_TOOLS))
    try:
        import q38pack_format as ref
    finally:
        sys.path.pop(0)
    path, names = pack2
    with ref.PackReader(path) as r:
        assert r.header.version == 2
        assert [t.name for t in r.tensors] == names
        with q38pack.open_pack(path) as p:
            for a, b in zip(r.tensors, p.tensors):
                assert (a.ggml_type, a.data_offset, a.stored_bytes, a.layout, a.aux0_offset, a.aux1_offset) == (
                    b.ggml_type, b.data_offset, b.stored_bytes, b.layout, b.aux0_offset, b.aux1_offset)
    dst = tmp_path / "m3.q38pack"
    q38pack.convert_to_b200(path, dst)
    with pytest.raises(ValueError):
        ref.PackReader(dst).open()


def test_plan_cli_output(pack2):
    path, names = pack2
    buf = io.StringIO()
    with redirect_stdout(buf):
        assert cli.main(["q38-plan", "--model", str(path), "--list"]) == 0
    out = buf.getvalue().splitlines()
    assert out[0] == "Q38 GPU placement plan"
    assert "Q38PACK version: 2" in out and f"tensors: {len(names)}" in out
    assert any(line.startswith("  layout[1/SM86_Q5K_SOA]: 4 tensors") for line in out)
    assert sum(1 for line in out if " va=0x" in line) == len(names)
