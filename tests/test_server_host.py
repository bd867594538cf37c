"""The HTTP front end (server.py) on CPU with a stand-in engine: request validation, the
OpenAI response shapes of /v1/completions and /v1/chat/completions, server-sent-event
streaming, stop strings, the stop-token finish reason, /v1/models, /health, /api/status and
404s (the reference's do_GET / do_POST, mlx-qwen38/server.py:491-620)."""
import http.client
import json
import threading

import pytest


class FakeEngine:
    """Emits the bytes of `reply` as token ids, then the eos id (a stop token)."""

    def __init__(self, reply: str = "Hello, world! Bye."):
        from moe_offload_b200.tokens import ByteTokenizer
        self.tokenizer = ByteTokenizer(300)
        self.reply = reply
        self.calls = []
        self._last_timings = {}

    def generate_stream(self, prompt_ids, max_tokens, temperature=0.0, top_p=1.0, stop_ids=None, seed=0):
        self.calls.append(dict(prompt_ids=list(prompt_ids), max_tokens=max_tokens, temperature=temperature,
                               top_p=top_p, seed=seed))
        self._last_timings = {"prefill_s": 0.0, "decode_s": 0.0, "decode_tok_per_s": 0.0, "stopped_by_token": False}
        ids = self.tokenizer.encode(self.reply) + [self.tokenizer.eos_token_id]
        n = 0
        for t in ids:
            if t == self.tokenizer.eos_token_id:
                self._last_timings["stopped_by_token"] = True
                return
            if n >= max_tokens:
                return
            n += 1
            yield t

    def _snapshot_decode_totals(self):
        return (8, 1, 1, 10, 1000, 200)


@pytest.fixture()
def server():
    from moe_offload_b200.server import make_server
    eng = FakeEngine()
    srv = make_server(eng, "127.0.0.1", 0, model_id="test-model", default_max_tokens=64)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    yield srv, eng
    srv.shutdown()
    srv.server_close()


def _req(srv, method, path, body=None):
    c = http.client.HTTPConnection("127.0.0.1", srv.server_address[1], timeout=10)
    c.request(method, path, body=None if body is None else json.dumps(body),
              headers={"Content-Type": "application/json"})
    r = c.getresponse()
    data = r.read()
    c.close()
    return r.status, r.getheader("Content-Type"), data


def test_get_routes(server):
    srv, _ = server
    st, _, data = _req(srv, "GET", "/v1/models")
    assert st == 200 and json.loads(data)["data"][0]["id"] == "test-model"
    st, _, data = _req(srv, "GET", "/health")
    assert st == 200 and json.loads(data)["status"] == "ok"
    st, _, data = _req(srv, "GET", "/api/status")
    assert st == 200 and json.loads(data)["expert_cache_since_start"]["hit_rate"] == 0.9
    st, _, data = _req(srv, "GET", "/nope")
    assert st == 404 and json.loads(data)["error"]["type"] == "not_found_error"


def test_completion_and_chat(server):
    srv, eng = server
    st, _, data = _req(srv, "POST", "/v1/completions", {"prompt": "Hi", "max_tokens": 5, "temperature": 0.5,
                                                        "top_p": 0.9, "seed": 3})
    out = json.loads(data)
    assert st == 200 and out["object"] == "text_completion"
    assert out["choices"][0]["text"] == "Hello" and out["choices"][0]["finish_reason"] == "length"
    assert out["usage"] == {"prompt_tokens": 2, "completion_tokens": 5, "total_tokens": 7}
    assert eng.calls[-1] == dict(prompt_ids=[72, 105], max_tokens=5, temperature=0.5, top_p=0.9, seed=3)
    st, _, data = _req(srv, "POST", "/v1/chat/completions",
                       {"messages": [{"role": "user", "content": "yo"}], "stop": ["!"]})
    out = json.loads(data)
    assert st == 200 and out["object"] == "chat.completion"
    assert out["choices"][0]["message"] == {"role": "assistant", "content": "Hello, world"}
    assert out["choices"][0]["finish_reason"] == "stop"
    assert eng.tokenizer.decode(eng.calls[-1]["prompt_ids"]) == "user: yo\nassistant: "
    # the stop token ends the reply with finish_reason "stop"
    st, _, data = _req(srv, "POST", "/v1/completions", {"prompt": "x"})
    out = json.loads(data)
    assert out["choices"][0]["text"] == "Hello, world! Bye." and out["choices"][0]["finish_reason"] == "stop"
    assert srv.last_request["completion_tokens"] == len("Hello, world! Bye.")


def test_streaming(server):
    srv, _ = server
    st, ctype, data = _req(srv, "POST", "/v1/chat/completions",
                           {"messages": [{"role": "user", "content": "yo"}], "stream": True, "max_tokens": 7,
                            "stream_options": {"include_usage": True}})
    assert st == 200 and ctype == "text/event-stream"
    events = [ln[len("data: "):] for ln in data.decode().split("\n") if ln.startswith("data: ")]
    assert events[-1] == "[DONE]"
    chunks = [json.loads(e) for e in events[:-1]]
    assert chunks[0]["choices"][0]["delta"] == {"role": "assistant", "content": ""}
    text = "".join(c["choices"][0]["delta"].get("content", "") for c in chunks if c["choices"])
    assert text == "Hello, "
    assert [c["choices"][0]["finish_reason"] for c in chunks if c["choices"]][-1] == "length"
    assert chunks[-1]["usage"]["completion_tokens"] == 7


@pytest.mark.parametrize("path,body,msg", [
    ("/v1/completions", {"prompt": ""}, "prompt"),
    ("/v1/completions", {"prompt": "a", "max_tokens": 0}, "max_tokens"),
    ("/v1/completions", {"prompt": "a", "top_p": 0}, "top_p"),
    ("/v1/completions", {"prompt": "a", "stop": 5}, "stop"),
    ("/v1/chat/completions", {"messages": []}, "messages"),
    ("/v1/chat/completions", {"messages": [{"content": "x"}]}, "role"),
])
def test_bad_requests(server, path, body, msg):
    srv, _ = server
    st, _, data = _req(srv, "POST", path, body)
    out = json.loads(data)
    assert st == 400 and out["error"]["type"] == "invalid_request_error" and msg in out["error"]["message"]


def test_oversized_body_refused(server):
    srv, _ = server
    from moe_offload_b200.server import MAX_BODY_BYTES
    c = http.client.HTTPConnection("127.0.0.1", srv.server_address[1], timeout=10)
    c.putrequest("POST", "/v1/completions")
    c.putheader("Content-Type", "application/json")
    c.putheader("Content-Length", str(MAX_BODY_BYTES + 1))
    c.endheaders()
    r = c.getresponse()
    assert r.status == 413
    c.close()
