"""OpenAI-compatible HTTP front end over OffloadEngine's token loop (mlx-qwen38/server.py: the
request handling of do_GET / do_POST, server.py:491-620, and the single generation worker,
server.py:202-254).

Kept: GET /v1/models, /health, /api/status (the engine's decode cache totals); POST
/v1/completions and /v1/chat/completions with max_tokens / max_completion_tokens,
temperature, top_p, seed, stop strings and `stream` (server-sent events, optional usage
chunk); 400 for malformed requests, 404 for unknown paths; every generation on one worker
thread, one request at a time. Left out (not on the MoE path): the Responses API, tool calls,
thinking splits, the prompt cache, the web UI and the chat template of a real tokenizer (a chat
prompt here is "role: content" lines and "assistant: ", encoded by the engine's tokenizer).

    python -m moe_offload_b200.server --port 8000 --vocab 248320 [--budget-pct 20]
"""
from __future__ import annotations

import argparse
import json
import queue
import threading
import time
import uuid
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Any, Iterator

MAX_BODY_BYTES = 16 << 20


class GenerationWorker:
    """Runs engine.generate_stream on one thread (the engine's CUDA state belongs to it) and
    hands tokens to the requesting thread through a queue; a client that goes away cancels."""

    def __init__(self, engine):
        self.engine = engine
        self.jobs: queue.Queue = queue.Queue()
        self.busy = threading.Lock()
        self.thread = threading.Thread(target=self._loop, name="moe-gen-worker", daemon=True)
        self.thread.start()

    def _loop(self) -> None:
        while True:
            args, kwargs, out_q, cancel = self.jobs.get()
            with self.busy:
                gen = None
                try:
                    gen = self.engine.generate_stream(*args, **kwargs)
                    for tok in gen:
                        if cancel.is_set():
                            break
                        out_q.put(("tok", tok))
                except BaseException as exc:  # noqa: BLE001
                    out_q.put(("err", exc))
                finally:
                    if gen is not None:
                        try:
                            gen.close()
                        except Exception:  # noqa: BLE001
                            pass
                    out_q.put(("done", dict(getattr(self.engine, "_last_timings", {}) or {})))

    def stream(self, *args, timings: dict | None = None, **kwargs) -> Iterator[int]:
        """Yields token ids; once the generation has ended, `timings` (when given) holds that
        generation's prefill / decode timings."""
        out_q: queue.Queue = queue.Queue()
        cancel = threading.Event()
        self.jobs.put((args, kwargs, out_q, cancel))
        finished = False
        try:
            while True:
                kind, val = out_q.get()
                if kind == "tok":
                    yield val
                elif kind == "err":
                    raise val
                else:
                    if timings is not None:
                        timings.update(val)
                    finished = True
                    return
        finally:
            if not finished:
                cancel.set()
                while True:
                    kind, val = out_q.get()
                    if kind == "done":
                        if timings is not None:
                            timings.update(val)
                        break


def _requested_max(req: dict, default: int) -> int:
    for key in ("max_tokens", "max_completion_tokens"):
        v = req.get(key)
        if v is not None:
            if isinstance(v, bool) or not isinstance(v, int) or v < 1:
                raise ValueError(f"'{key}' must be a positive integer")
            return v
    return default


def _stop_strings(raw) -> list[str]:
    if raw is None:
        return []
    if isinstance(raw, str):
        return [raw] if raw else []
    if isinstance(raw, list) and all(isinstance(s, str) for s in raw):
        return [s for s in raw if s]
    raise ValueError("'stop' must be a string or a list of strings")


def chat_prompt(messages) -> str:
    if not isinstance(messages, list) or not messages:
        raise ValueError("'messages' must be a non-empty list")
    lines = []
    for m in messages:
        if not isinstance(m, dict) or not isinstance(m.get("role"), str):
            raise ValueError("every message needs a string 'role'")
        content = m.get("content", "")
        if isinstance(content, list):      # content parts: keep the text ones
            content = "".join(p.get("text", "") for p in content if isinstance(p, dict))
        if not isinstance(content, str):
            raise ValueError("message 'content' must be a string or a list of text parts")
        lines.append(f"{m['role']}: {content}\n")
    return "".join(lines) + "assistant: "


class Handler(BaseHTTPRequestHandler):
    server_version = "moe-offload-b200"
    protocol_version = "HTTP/1.1"

    def log_message(self, fmt, *args) -> None:       # quiet by default
        if getattr(self.server, "verbose", False):
            super().log_message(fmt, *args)

    # ------------------------------------------------------------------ replies
    def _send_json(self, code: int, obj: Any) -> None:
        body = json.dumps(obj).encode()
        self.send_response(code)
        self.send_header("Content-Type", "application/json")
        self.send_header("Content-Length", str(len(body)))
        self.end_headers()
        self.wfile.write(body)

    def _send_error_json(self, code: int, msg: str, kind: str) -> None:
        self._send_json(code, {"error": {"message": msg, "type": kind, "code": code}})

    def _sse(self, obj: Any) -> None:
        data = obj if isinstance(obj, str) else json.dumps(obj)
        chunk = f"data: {data}\n\n".encode()
        self.wfile.write(f"{len(chunk):x}\r\n".encode() + chunk + b"\r\n")
        self.wfile.flush()

    # ------------------------------------------------------------------ GET
    def do_GET(self) -> None:  # noqa: N802
        path = self.path.split("?", 1)[0]
        srv = self.server
        if path in ("/health", "/healthz"):
            self._send_json(200, {"status": "ok", "model": srv.model_id, "busy": srv.worker.busy.locked()})
        elif path == "/v1/models":
            self._send_json(200, {"object": "list", "data": [{"id": srv.model_id, "object": "model",
                                                              "created": srv.created_ts, "owned_by": "local"}]})
        elif path == "/api/status":
            try:
                lru, pref, dem, req, dem_b, pref_b = srv.engine._snapshot_decode_totals()
                cache = {"decode_requests": req, "lru_hits": lru, "prefetch_hits": pref, "demand_misses": dem,
                         "hit_rate": round((lru + pref) / req, 4) if req else None,
                         "demand_read_bytes": dem_b, "prefetch_read_bytes": pref_b}
            except Exception as exc:  # noqa: BLE001
                cache = {"error": type(exc).__name__}
            self._send_json(200, {"status": "ok", "model": srv.model_id, "busy": srv.worker.busy.locked(),
                                  "expert_cache_since_start": cache, "last_request": srv.last_request})
        else:
            self._send_error_json(404, f"Unknown endpoint: {path}", "not_found_error")

    # ------------------------------------------------------------------ POST
    def do_POST(self) -> None:  # noqa: N802
        path = self.path.split("?", 1)[0]
        if path not in ("/v1/completions", "/v1/chat/completions"):
            self._send_error_json(404, f"Unknown endpoint: {path}", "not_found_error")
            return
        srv = self.server
        try:
            n = int(self.headers.get("Content-Length", "0"))
            if n > MAX_BODY_BYTES:
                self.close_connection = True          # the unread body must not reach the next request
                self._send_error_json(413, f"request body over {MAX_BODY_BYTES} bytes", "invalid_request_error")
                return
            req = json.loads(self.rfile.read(n) or b"{}")
            if not isinstance(req, dict):
                raise ValueError("the request body must be a JSON object")
            is_chat = path == "/v1/chat/completions"
            if is_chat:
                prompt = chat_prompt(req.get("messages"))
            else:
                prompt = req.get("prompt")
                if not isinstance(prompt, str) or not prompt:
                    raise ValueError("'prompt' must be a non-empty string")
            prompt_ids = srv.engine.tokenizer.encode(prompt)
            if not prompt_ids:
                raise ValueError("Encoded prompt produced 0 tokens")
            max_tokens = _requested_max(req, srv.default_max_tokens)
            temperature = float(req.get("temperature", 0.0) or 0.0)
            top_p = float(1.0 if req.get("top_p") is None else req.get("top_p"))
            if not 0.0 < top_p <= 1.0:
                raise ValueError("'top_p' must be in (0, 1]")
            seed = req.get("seed")
            seed = int(seed) if seed is not None else int(time.time_ns() & 0xFFFFFFFF)
            stops = _stop_strings(req.get("stop"))
            stream = bool(req.get("stream", False))
            opts = req.get("stream_options") or {}
            include_usage = bool(isinstance(opts, dict) and opts.get("include_usage", False))
        except Exception as exc:  # noqa: BLE001
            self._send_error_json(400, str(exc), "invalid_request_error")
            return
        try:
            self._generate(is_chat, prompt_ids, max_tokens, temperature, top_p, seed, stops, stream, include_usage)
        except Exception as exc:  # noqa: BLE001
            try:
                self._send_error_json(500, str(exc), "server_error")
            except Exception:  # noqa: BLE001
                pass

    def _generate(self, is_chat, prompt_ids, max_tokens, temperature, top_p, seed, stops, stream,
                  include_usage) -> None:
        srv = self.server
        tok = srv.engine.tokenizer
        rid = ("chatcmpl-" if is_chat else "cmpl-") + uuid.uuid4().hex[:24]
        created = int(time.time())
        obj = "chat.completion" if is_chat else "text_completion"
        ids: list[int] = []
        text, sent, finish = "", 0, "length"
        t0 = time.perf_counter()
        timings: dict = {}
        gen = srv.worker.stream(prompt_ids, max_tokens, temperature=temperature, top_p=top_p, seed=seed,
                                timings=timings)
        if stream:
            self.send_response(200)
            self.send_header("Content-Type", "text/event-stream")
            self.send_header("Cache-Control", "no-cache")
            self.send_header("Transfer-Encoding", "chunked")
            self.end_headers()
            if is_chat:
                self._sse(self._chunk(rid, created, is_chat, {"role": "assistant", "content": ""}, None))
        try:
            for t in gen:
                ids.append(t)
                text = tok.decode(ids)
                hit = min((text.find(s) for s in stops if s in text), default=-1)
                if hit >= 0:
                    text, finish = text[:hit], "stop"
                if stream and len(text) > sent and "�" not in text[sent:]:
                    self._sse(self._chunk(rid, created, is_chat, text[sent:], None))
                    sent = len(text)
                if hit >= 0:
                    break
        finally:
            gen.close()
        if finish == "length" and timings.get("stopped_by_token"):
            finish = "stop"
        usage = {"prompt_tokens": len(prompt_ids), "completion_tokens": len(ids),
                 "total_tokens": len(prompt_ids) + len(ids)}
        srv.last_request = {"id": rid, "prompt_tokens": len(prompt_ids), "completion_tokens": len(ids),
                            "seconds": round(time.perf_counter() - t0, 4), "timings": timings}
        if stream:
            if len(text) > sent:
                self._sse(self._chunk(rid, created, is_chat, text[sent:], None))
            self._sse(self._chunk(rid, created, is_chat, "" if not is_chat else {}, finish))
            if include_usage:
                self._sse({"id": rid, "object": obj + ".chunk", "created": created, "model": srv.model_id,
                           "choices": [], "usage": usage})
            self._sse("[DONE]")
            self.wfile.write(b"0\r\n\r\n")
            self.wfile.flush()
            return
        choice = ({"index": 0, "message": {"role": "assistant", "content": text}, "finish_reason": finish}
                  if is_chat else {"index": 0, "text": text, "finish_reason": finish})
        self._send_json(200, {"id": rid, "object": obj, "created": created, "model": srv.model_id,
                              "choices": [choice], "usage": usage})

    def _chunk(self, rid, created, is_chat, delta, finish) -> dict:
        srv = self.server
        if is_chat:
            d = delta if isinstance(delta, dict) else {"content": delta}
            choice = {"index": 0, "delta": d, "finish_reason": finish}
            return {"id": rid, "object": "chat.completion.chunk", "created": created, "model": srv.model_id,
                    "choices": [choice]}
        return {"id": rid, "object": "text_completion", "created": created, "model": srv.model_id,
                "choices": [{"index": 0, "text": delta, "finish_reason": finish}]}


def make_server(engine, host: str = "127.0.0.1", port: int = 8000, model_id: str = "moe-offload-b200",
                default_max_tokens: int = 256) -> ThreadingHTTPServer:
    """An HTTP server bound to (host, port) over `engine` (anything with `tokenizer` and
    `generate_stream(prompt_ids, max_tokens, temperature=, top_p=, seed=)`); call
    serve_forever() on it."""
    srv = ThreadingHTTPServer((host, port), Handler)
    srv.engine = engine
    srv.worker = GenerationWorker(engine)
    srv.model_id = model_id
    srv.created_ts = int(time.time())
    srv.default_max_tokens = default_max_tokens
    srv.last_request = None
    srv.verbose = False
    return srv


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--model", default=None, help="model directory in the reference's shard layout (else synthetic)")
    ap.add_argument("--vocab", type=int, default=248_320)
    ap.add_argument("--budget-pct", type=float, default=20.0)
    ap.add_argument("--max-tokens", type=int, default=256)
    args = ap.parse_args()
    from .engine import OffloadEngine
    eng = OffloadEngine(model_path=args.model, budget_pct=args.budget_pct, vocab_size=args.vocab)
    srv = make_server(eng, args.host, args.port, default_max_tokens=args.max_tokens)
    print(f"serving on http://{args.host}:{args.port}", flush=True)
    try:
        srv.serve_forever()
    finally:
        eng.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
