"""The OpenAI-compatible surface (qwen382743090_b200/server.py) on the CPU:
the reference's endpoints and error shapes (server/q38_openai.py:38-161), the
prompt fed one decode step per token then greedy steps, SSE streaming, stop
ids, limits, and the upstream proxy -- against a stand-in model whose next
token is a known function of (input token, position)."""
from __future__ import annotations

import json
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from urllib import error, request

import pytest

from qwen382743090_b200 import server as srv

VOCAB, CTX = 4096, 64


class ToyModel:
    """step(): consumes the input token at the position, outputs (7 t + 3 pos) % V."""

    def __init__(self):
        self.cfg = {"vocab": VOCAB, "ctx": CTX}
        self.tok, self.pos, self.log = 0, 0, []

    def reset(self, token):
        self.tok, self.pos = token, 0
        self.log.append(("reset", token))

    def set_token(self, token):
        self.tok = token

    def step(self, stream=None):
        self.log.append(("step", self.tok, self.pos))
        self.tok = (7 * self.tok + 3 * self.pos) % VOCAB
        self.pos += 1

    def position(self):
        return self.tok, self.pos


def expected(prompt, n, stop=()):
    pos, out = len(prompt) - 1, []
    tok = (7 * prompt[-1] + 3 * pos) % VOCAB
    pos += 1
    for _ in range(n):
        out.append(tok)
        if tok in stop:
            break
        tok = (7 * tok + 3 * pos) % VOCAB
        pos += 1
    return out


@pytest.fixture()
def served():
    model = ToyModel()
    state = srv.State(None, "toy", None, None, srv.Generator(model), 3, "qwen35-hybrid")
    server = srv.make_server(state, "127.0.0.1", 0, verbose=False)
    th = threading.Thread(target=server.serve_forever, daemon=True)
    th.start()
    yield f"http://127.0.0.1:{server.server_address[1]}", model
    server.shutdown()
    server.server_close()


def call(url, path, payload=None, raw=None):
    data = raw if raw is not None else (json.dumps(payload).encode() if payload is not None else None)
    req = request.Request(url + path, data=data, method="POST" if data is not None else "GET",
                          headers={"Content-Type": "application/json"})
    try:
        with request.urlopen(req, timeout=30) as r:
            return r.status, r.read().decode()
    except error.HTTPError as e:
        return e.code, e.read().decode()


def test_health_models_and_errors(served):
    url, _ = served
    code, body = call(url, "/health")
    h = json.loads(body)
    assert code == 200 and h["native_decode_ready"] is True and h["model"] == "toy" and h["tensor_count"] == 3
    code, body = call(url, "/v1/models")
    assert code == 200 and json.loads(body)["data"][0]["id"] == "toy"
    code, body = call(url, "/nope")
    assert code == 404 and json.loads(body)["error"]["code"] == "not_found"
    code, body = call(url, "/v1/chat/completions", raw=b"{not json")
    assert code == 400 and json.loads(body)["error"]["code"] == "invalid_json"
    code, body = call(url, "/v1/chat/completions", {"prompt_token_ids": [1, VOCAB]})
    assert code == 400
    code, body = call(url, "/v1/chat/completions", {"prompt_token_ids": list(range(60)), "max_tokens": 10})
    assert code == 400 and "context" in json.loads(body)["error"]["message"]


def test_prompt_ids_prefill_then_greedy(served):
    url, model = served
    prompt = [5, 900, 17, 4000]
    code, body = call(url, "/v1/chat/completions", {"prompt_token_ids": prompt, "max_tokens": 6})
    r = json.loads(body)
    assert code == 200
    ch = r["choices"][0]
    assert ch["token_ids"] == expected(prompt, 6) and ch["finish_reason"] == "length"
    assert r["usage"] == {"prompt_tokens": 4, "completion_tokens": 6, "total_tokens": 10}
    # one reset, then the prompt's tokens as the inputs of the first steps
    assert model.log[0] == ("reset", 5)
    assert [e[1] for e in model.log[1:5]] == prompt and [e[2] for e in model.log[1:5]] == [0, 1, 2, 3]


def test_messages_as_bytes_and_stop(served):
    url, _ = served
    msgs = [{"role": "user", "content": "héllo"}]
    ids = srv.messages_to_ids(msgs)
    assert bytes(ids).decode() == "user: héllo\nassistant: "
    full = expected(ids, 8)
    stop = full[2]
    code, body = call(url, "/v1/chat/completions", {"messages": msgs, "max_tokens": 8, "stop_token_ids": [stop]})
    ch = json.loads(body)["choices"][0]
    assert ch["token_ids"] == full[:3] and ch["finish_reason"] == "stop"
    assert ch["message"]["content"] == srv.ids_to_text(full[:3])
    assert srv.ids_to_text([104, 105, 300]) == "hi<|300|>"


def test_streaming_matches_non_streaming(served):
    url, _ = served
    prompt = [11, 22, 33]
    code, body = call(url, "/v1/chat/completions", {"prompt_token_ids": prompt, "max_tokens": 5, "stream": True})
    assert code == 200
    events = [line[6:] for line in body.split("\n") if line.startswith("data: ")]
    assert events[-1] == "[DONE]"
    chunks = [json.loads(e) for e in events[:-1]]
    assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
    ids = [t for c in chunks for t in c.get("token_ids", [])]
    assert ids == expected(prompt, 5)
    assert chunks[-1]["choices"][0]["finish_reason"] == "length"


def test_no_model_is_503_and_proxy_forwards():
    class Up(BaseHTTPRequestHandler):
        def do_POST(self):
            body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
            raw = json.dumps({"upstream_model": body.get("model")}).encode()
            self.send_response(200)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(raw)))
            self.end_headers()
            self.wfile.write(raw)

        def log_message(self, *a):
            pass

    up = ThreadingHTTPServer(("127.0.0.1", 0), Up)
    threading.Thread(target=up.serve_forever, daemon=True).start()
    servers = []
    try:
        for base in (None, f"http://127.0.0.1:{up.server_address[1]}"):
            st = srv.State(None, "m", base, "upstream-name", None)
            s = srv.make_server(st, "127.0.0.1", 0, verbose=False)
            threading.Thread(target=s.serve_forever, daemon=True).start()
            servers.append(s)
        u0 = f"http://127.0.0.1:{servers[0].server_address[1]}"
        code, body = call(u0, "/v1/chat/completions", {"messages": [{"role": "user", "content": "x"}]})
        assert code == 503 and json.loads(body)["error"]["code"] == "native_decode_not_ready"
        u1 = f"http://127.0.0.1:{servers[1].server_address[1]}"
        code, body = call(u1, "/v1/chat/completions", {"messages": [{"role": "user", "content": "x"}]})
        assert code == 200 and json.loads(body) == {"upstream_model": "upstream-name"}
    finally:
        for s in servers + [up]:
            s.shutdown()
            s.server_close()
