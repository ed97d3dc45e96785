"""The OpenAI-compatible surface on the GPU: a request's greedy tokens are the
engine's own (prompt fed one step per token from a reset sequence), repeat
requests are independent, and a model loaded from a Q38PACK serves the same
tokens as the seeded model it was written from."""
from __future__ import annotations

import json
import threading
from urllib import request

import pytest

from qwen382743090_b200 import q38pack
from qwen382743090_b200 import runtime as rt
from qwen382743090_b200 import server as srv

pytestmark = pytest.mark.gpu

TINY = dict(n_layers=4, attn_every=4, hidden=1024, ffn=2048, vocab=4096, gdn_qk_heads=4, gdn_v_heads=8,
            attn_q_heads=12, attn_kv_heads=4, rope_dim=64, ctx=256, seed=21)
PROMPT = [7, 1234, 99, 4000, 256, 3]


def direct(m, prompt, n):
    m.reset(prompt[0])
    for t in prompt[1:]:
        m.step()
        m.set_token(t)
    out = []
    for _ in range(n):
        m.step()
        out.append(m.position()[0])
    return out


def post(url, payload):
    req = request.Request(url + "/v1/chat/completions", data=json.dumps(payload).encode(), method="POST",
                          headers={"Content-Type": "application/json"})
    with request.urlopen(req, timeout=120) as r:
        return json.loads(r.read())


def serve(model):
    s = srv.make_server(srv.State(None, "tiny", None, None, srv.Generator(model)), "127.0.0.1", 0, verbose=False)
    threading.Thread(target=s.serve_forever, daemon=True).start()
    return s, f"http://127.0.0.1:{s.server_address[1]}"


def test_served_tokens_are_the_engines(ctx, tmp_path):
    with rt.Model(**TINY) as m:
        ref = direct(m, PROMPT, 10)
        s, url = serve(m)
        try:
            a = post(url, {"prompt_token_ids": PROMPT, "max_tokens": 10})["choices"][0]["token_ids"]
            b = post(url, {"prompt_token_ids": PROMPT, "max_tokens": 10})["choices"][0]["token_ids"]
        finally:
            s.shutdown()
            s.server_close()
        assert a == ref and b == ref
        path = tmp_path / "tiny.q38pack"
        q38pack.export_model_pack(m, path)
    with rt.Model(pack=path, **TINY) as m2:
        s, url = serve(m2)
        try:
            c = post(url, {"prompt_token_ids": PROMPT, "max_tokens": 10})["choices"][0]["token_ids"]
        finally:
            s.shutdown()
            s.server_close()
    assert c == ref
    assert rt.fault_status() == 0
