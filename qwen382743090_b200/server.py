"""OpenAI-compatible HTTP surface over the native decode.

The reference's server (server/q38_openai.py:38-161) answers GET /health and
GET /v1/models, and POST /v1/chat/completions with 503 until its native decode
exists, or proxies to an upstream OpenAI-compatible server
(--reference-base-url).  This one keeps those endpoints, error shapes and
flags and wires POST /v1/chat/completions to the library's batch-1 greedy
decode (q38_model_*): the prompt is fed one decode step per token
(q38_model_reset, q38_model_set_token), then up to max_tokens greedy steps,
as one JSON response or as server-sent events with stream=true.

Neither project has a tokenizer.  A request may give its prompt as token ids
(`prompt_token_ids`, the vLLM field); otherwise the chat messages are turned
into byte-level ids (the UTF-8 bytes of "role: content" lines, then
"assistant: ").  Replies carry the generated ids (`token_ids`) and a byte-level
rendering as the message content (ids >= 256 as <|id|>).  With the synthetic
weights the text means nothing; the surface is what is exercised.

    python -m qwen382743090_b200.server --model model.q38pack --port 8000
    python -m qwen382743090_b200.server --seeded --config '{"n_layers": 4}'
"""
from __future__ import annotations

import argparse
import json
import sys
import threading
import time
import uuid
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path
from typing import Any, Iterator
from urllib import error, request


def send_json(handler: BaseHTTPRequestHandler, status: int, payload: dict[str, Any]) -> None:
    raw = json.dumps(payload, ensure_ascii=False, separators=(",", ":")).encode("utf-8")
    handler.send_response(status)
    handler.send_header("Content-Type", "application/json; charset=utf-8")
    handler.send_header("Content-Length", str(len(raw)))
    handler.end_headers()
    handler.wfile.write(raw)


def openai_error(message: str, code: str, err_type: str = "server_error") -> dict[str, Any]:
    return {"error": {"message": message, "type": err_type, "param": None, "code": code}}


# ---- byte-level token ids (no tokenizer exists for the model) ----------------------
def messages_to_ids(messages: list[dict[str, Any]]) -> list[int]:
    lines = []
    for m in messages:
        content = m.get("content", "")
        if isinstance(content, list):  # content parts: keep the text ones
            content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
        lines.append(f"{m.get('role', 'user')}: {content}")
    return list(("\n".join(lines) + "\nassistant: ").encode("utf-8"))


def ids_to_text(ids: list[int]) -> str:
    out, run = [], bytearray()
    for t in ids:
        if 0 <= t < 256:
            run.append(t)
            continue
        if run:
            out.append(run.decode("utf-8", errors="replace"))
            run = bytearray()
        out.append(f"<|{t}|>")
    if run:
        out.append(run.decode("utf-8", errors="replace"))
    return "".join(out)


class Generator:
    """Greedy batch-1 generation on one model, one sequence at a time."""

    def __init__(self, model):
        self.model = model
        self.vocab = int(model.cfg["vocab"])
        self.ctx = int(model.cfg["ctx"])
        self.lock = threading.Lock()

    def check(self, prompt: list[int], max_tokens: int) -> str | None:
        if not prompt:
            return "the prompt is empty"
        if any(not isinstance(t, int) or t < 0 or t >= self.vocab for t in prompt):
            return f"prompt token ids must be integers in [0, {self.vocab})"
        if len(prompt) + max_tokens > self.ctx:
            return f"prompt ({len(prompt)}) + max_tokens ({max_tokens}) exceeds the context ({self.ctx})"
        return None

    def generate(self, prompt: list[int], max_tokens: int, stop_ids: set[int]) -> Iterator[int]:
        with self.lock:
            m = self.model
            m.reset(prompt[0])
            for t in prompt[1:]:  # prefill: one decode step per prompt token
                m.step()
                m.set_token(t)
            for _ in range(max_tokens):
                m.step()
                tok = int(m.position()[0])
                yield tok
                if tok in stop_ids:
                    return


class State:
    def __init__(self, model_path: Path | None, model_id: str, reference_base_url: str | None,
                 reference_model: str | None, generator: Generator | None, tensor_count: int = 0,
                 architecture: str | None = None):
        self.model_path = model_path
        self.model_id = model_id
        self.reference_base_url = reference_base_url.rstrip("/") if reference_base_url else None
        self.reference_model = reference_model
        self.generator = generator
        self.tensor_count = tensor_count
        self.architecture = architecture

    @property
    def native_ready(self) -> bool:
        return self.generator is not None


class Handler(BaseHTTPRequestHandler):
    server_version = "q38rt-b200/0.1"

    @property
    def state(self) -> State:
        return self.server.state  # type: ignore[attr-defined]

    def log_message(self, fmt: str, *args: Any) -> None:
        if getattr(self.server, "verbose", True):
            sys.stderr.write("%s - - [%s] %s\n" % (self.address_string(), self.log_date_time_string(), fmt % args))

    def do_GET(self) -> None:
        if self.path == "/health":
            send_json(self, 200, {
                "status": "ok",
                "native_decode_ready": self.state.native_ready,
                "reference_backend": bool(self.state.reference_base_url),
                "model": self.state.model_id,
                "architecture": self.state.architecture,
                "tensor_count": self.state.tensor_count,
            })
            return
        if self.path == "/v1/models":
            send_json(self, 200, {"object": "list", "data": [{
                "id": self.state.model_id, "object": "model", "created": int(time.time()), "owned_by": "q38rt"}]})
            return
        send_json(self, 404, openai_error("Not found", "not_found", "invalid_request_error"))

    def do_POST(self) -> None:
        if self.path != "/v1/chat/completions":
            send_json(self, 404, openai_error("Not found", "not_found", "invalid_request_error"))
            return
        try:
            length = int(self.headers.get("Content-Length", "0"))
            payload = json.loads(self.rfile.read(length).decode("utf-8"))
            if not isinstance(payload, dict):
                raise ValueError("the body is not a JSON object")
        except Exception as exc:
            send_json(self, 400, openai_error(f"Invalid JSON request: {exc}", "invalid_json", "invalid_request_error"))
            return
        if self.state.generator is not None:
            self.native(payload)
            return
        if self.state.reference_base_url:
            self.proxy_reference(payload)
            return
        send_json(self, 503, openai_error("No model is loaded and no reference backend is configured.",
                                          "native_decode_not_ready"))

    # ---- native greedy decode --------------------------------------------------------
    def native(self, payload: dict[str, Any]) -> None:
        gen = self.state.generator
        try:
            if "prompt_token_ids" in payload:
                prompt = list(payload["prompt_token_ids"])
            else:
                msgs = payload.get("messages")
                if not isinstance(msgs, list) or not msgs:
                    raise ValueError("messages must be a non-empty list")
                prompt = messages_to_ids(msgs)
            max_tokens = int(payload.get("max_tokens", payload.get("max_completion_tokens", 16)))
            if max_tokens < 1:
                raise ValueError("max_tokens must be at least 1")
            stop_ids = {int(t) for t in payload.get("stop_token_ids", [])}
        except Exception as exc:
            send_json(self, 400, openai_error(f"Invalid request: {exc}", "invalid_request", "invalid_request_error"))
            return
        why = gen.check(prompt, max_tokens)
        if why:
            send_json(self, 400, openai_error(why, "invalid_request", "invalid_request_error"))
            return
        rid = "chatcmpl-" + uuid.uuid4().hex[:24]
        created = int(time.time())
        model_id = self.state.model_id
        if payload.get("stream"):
            self.send_response(200)
            self.send_header("Content-Type", "text/event-stream")
            self.send_header("Cache-Control", "no-cache")
            self.send_header("Connection", "close")
            self.end_headers()

            def event(delta: dict[str, Any], finish: str | None, extra: dict[str, Any] | None = None) -> None:
                chunk = {"id": rid, "object": "chat.completion.chunk", "created": created, "model": model_id,
                         "choices": [{"index": 0, "delta": delta, "finish_reason": finish}]}
                if extra:
                    chunk.update(extra)
                self.wfile.write(b"data: " + json.dumps(chunk, ensure_ascii=False).encode("utf-8") + b"\n\n")
                self.wfile.flush()

            event({"role": "assistant", "content": ""}, None)
            ids: list[int] = []
            for tok in gen.generate(prompt, max_tokens, stop_ids):
                ids.append(tok)
                event({"content": ids_to_text([tok])}, None, {"token_ids": [tok]})
            event({}, "stop" if ids and ids[-1] in stop_ids else "length")
            self.wfile.write(b"data: [DONE]\n\n")
            self.wfile.flush()
            return
        ids = list(gen.generate(prompt, max_tokens, stop_ids))
        finish = "stop" if ids and ids[-1] in stop_ids else "length"
        send_json(self, 200, {
            "id": rid, "object": "chat.completion", "created": created, "model": model_id,
            "choices": [{"index": 0, "message": {"role": "assistant", "content": ids_to_text(ids)},
                         "finish_reason": finish, "token_ids": ids}],
            "usage": {"prompt_tokens": len(prompt), "completion_tokens": len(ids),
                      "total_tokens": len(prompt) + len(ids)},
        })

    # ---- upstream proxy (the reference's --reference-base-url) ---------------------------
    def proxy_reference(self, payload: dict[str, Any]) -> None:
        forwarded = dict(payload)
        if self.state.reference_model:
            forwarded["model"] = self.state.reference_model
        url = self.state.reference_base_url + "/v1/chat/completions"
        req = request.Request(url, data=json.dumps(forwarded, ensure_ascii=False).encode("utf-8"), method="POST",
                              headers={"Content-Type": "application/json"})
        auth = self.headers.get("Authorization")
        if auth:
            req.add_header("Authorization", auth)
        try:
            upstream = request.urlopen(req, timeout=600)
        except error.HTTPError as exc:
            body = exc.read()
            self.send_response(exc.code)
            self.send_header("Content-Type", exc.headers.get("Content-Type", "application/json"))
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)
            return
        except Exception as exc:
            send_json(self, 502, openai_error(f"Reference backend failed: {exc}", "reference_backend_error"))
            return
        content_type = upstream.headers.get("Content-Type", "application/json")
        if not payload.get("stream"):
            body = upstream.read()
            self.send_response(upstream.status)
            self.send_header("Content-Type", content_type)
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)
            return
        self.send_response(upstream.status)
        self.send_header("Content-Type", content_type)
        self.send_header("Cache-Control", "no-cache")
        self.send_header("Connection", "close")
        self.end_headers()
        while True:
            chunk = upstream.read(8192)
            if not chunk:
                break
            self.wfile.write(chunk)
            self.wfile.flush()


def make_server(state: State, host: str = "127.0.0.1", port: int = 8000, verbose: bool = True) -> ThreadingHTTPServer:
    server = ThreadingHTTPServer((host, port), Handler)
    server.state = state  # type: ignore[attr-defined]
    server.verbose = verbose  # type: ignore[attr-defined]
    return server


def load_model(model_path: Path | None, seeded: bool, overrides: dict[str, Any]):
    """The model to serve and its pack facts: the pack's weights with the
    config its manifest records (a pack written by export_model_pack) or the
    real model's dimensions, the IQ4_XS ffn_gate detected from the pack; or
    the seeded synthetic model."""
    from . import q38pack
    from . import runtime as rt

    cfg: dict[str, Any] = {}
    tensor_count, arch = 0, None
    if model_path is not None and not seeded:
        with q38pack.open_pack(model_path) as p:
            tensor_count = int(p.header.tensor_count)
            man = p.manifest()
            arch = (man.get("model") or {}).get("architecture")
            known = set(rt.QWEN_HYBRID_64)
            cfg.update({k: v for k, v in (man.get("config") or {}).items() if k in known})
            names = {t.name.decode(): t for t in p.tensors}
            gate = names.get("blk.0.ffn_gate.weight")
            if gate is not None and gate.ggml_type == 23:
                cfg["ffn_gate_type"] = 23
    cfg.update(overrides)
    cfg["tp_rank"], cfg["tp_size"] = 0, 1
    model = rt.Model(pack=None if seeded else model_path, **cfg)
    return model, tensor_count, arch or "qwen35-hybrid"


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="Q38RT-B200 OpenAI-compatible server")
    ap.add_argument("--model", type=Path, help="Q38PACK model")
    ap.add_argument("--seeded", action="store_true", help="serve the seeded synthetic model instead of a pack")
    ap.add_argument("--config", default="{}", help="JSON overrides of the model config (n_layers, ctx, ...)")
    ap.add_argument("--model-id", default="qwen3.8-27b-q38")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--reference-base-url", help="OpenAI-compatible upstream used when no model is loaded")
    ap.add_argument("--reference-model", help="model name sent to the reference backend")
    args = ap.parse_args(argv)
    if args.model is None and not args.seeded and not args.reference_base_url:
        ap.error("give --model, --seeded or --reference-base-url")
    gen, count, arch = None, 0, None
    if args.model is not None or args.seeded:
        model, count, arch = load_model(args.model, args.seeded, json.loads(args.config))
        gen = Generator(model)
    state = State(args.model, args.model_id, args.reference_base_url, args.reference_model, gen, count, arch)
    server = make_server(state, args.host, args.port)
    print(f"q38rt serving http://{args.host}:{args.port} model={args.model_id}")
    print(f"native_decode_ready={state.native_ready} reference_backend={bool(state.reference_base_url)}")
    try:
        server.serve_forever()
    except KeyboardInterrupt:
        pass
    finally:
        server.server_close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
