"""HTTP/SSE front end, serve loop and metrics against the scripted mock backend (no GPU)."""

import http.client
import json
import socket
import time

import pytest

from zstep_b200 import _master as M
from tests.test_tokenizer import build_hf_tokenizer


@pytest.fixture(scope="module")
def tok(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("srvtok"))
    build_hf_tokenizer(d)
    t = M.Tokenizer()
    t.load_dir(d)
    return t


def engine_cfg(**kw):
    c = M.EngineConfig()
    c.max_seqs, c.max_step_tokens, c.max_prefill_chunk = 4, 256, 64
    c.page_size, c.num_pages, c.max_model_len = 16, 256, 1024
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def request(port, method, path, body=None, headers=None, timeout=30):
    conn = http.client.HTTPConnection("127.0.0.1", port, timeout=timeout)
    data = json.dumps(body) if body is not None else None
    h = {"Content-Type": "application/json"}
    h.update(headers or {})
    conn.request(method, path, body=data, headers=h)
    r = conn.getresponse()
    raw = r.read()
    conn.close()
    return r.status, dict(r.getheaders()), raw


def chat(port, **kw):
    body = {"model": "m", "messages": [{"role": "user", "content": "hello there"}], "max_tokens": 8}
    body.update(kw.pop("body", {}))
    return request(port, "POST", "/v1/chat/completions", body, **kw)


def sse_events(raw: bytes):
    out = []
    for block in raw.decode().split("\n\n"):
        if block.startswith("data: "):
            payload = block[6:]
            out.append(payload if payload == "[DONE]" else json.loads(payload))
    return out


# Mock output tokens are drawn from a run of ids whose bytes are printable ASCII (the
# tokenizer trained by build_hf_tokenizer puts the byte alphabet first).
LOW, HIGH = 3, 96


def expected_tokens(tok, n, low=LOW, high=HIGH):
    """The mock backend's greedy continuation of the rendered prompt."""
    ids = tok.encode(M.render_chat([("user", "hello there", "")]))
    out, last, pos = [], ids[-1], len(ids) - 1
    for _ in range(n):
        nxt = M.mock_next_token(last, pos, low, high)
        out.append(nxt)
        last, pos = nxt, pos + 1
    return out


@pytest.fixture
def server(tok):
    s = M.serve_mock(tok, engine_cfg(), admin_port=0, mock_low=LOW, mock_high=HIGH)
    yield s
    s.stop()


def test_probes_and_models(server):
    p = server.port()
    assert request(p, "GET", "/livez")[0] == 200
    assert request(p, "GET", "/health")[0] == 200
    st, _, raw = request(p, "GET", "/ready")
    assert st == 200 and json.loads(raw)["status"] == "ready"
    st, _, raw = request(p, "GET", "/v1/models")
    data = json.loads(raw)["data"]
    assert st == 200 and data[0]["id"] == "zstep-mock" and data[0]["owned_by"] == "zstep"
    assert request(p, "GET", "/nope")[0] == 404


def test_chat_non_stream(server, tok):
    st, hdr, raw = chat(server.port(), headers={"x-request-id": "req-42"})
    assert st == 200, raw
    body = json.loads(raw)
    assert body["id"] == "req-42" and hdr.get("x-request-id") == "req-42"
    assert body["object"] == "chat.completion"
    exp = expected_tokens(tok, 8)
    assert body["choices"][0]["message"]["content"] == tok.decode(exp).decode("utf-8", "replace")
    assert body["choices"][0]["finish_reason"] == "length"
    u = body["usage"]
    assert u["completion_tokens"] == 8 and u["total_tokens"] == u["prompt_tokens"] + 8


def test_chat_stream_sse(server, tok):
    st, hdr, raw = chat(server.port(), body={"stream": True, "stream_options": {"include_usage": True},
                                             "logprobs": True, "top_logprobs": 2})
    assert st == 200 and hdr["Content-Type"].startswith("text/event-stream")
    ev = sse_events(raw)
    assert ev[-1] == "[DONE]"
    assert ev[0]["choices"][0]["delta"]["role"] == "assistant"
    text = "".join(e["choices"][0]["delta"].get("content", "") for e in ev[:-1] if isinstance(e, dict) and e["choices"])
    assert text == tok.decode(expected_tokens(tok, 8)).decode("utf-8", "replace")
    finals = [e for e in ev[:-1] if e["choices"] and e["choices"][0]["finish_reason"]]
    assert finals[-1]["choices"][0]["finish_reason"] == "length"
    usage = [e for e in ev[:-1] if e.get("usage")]
    assert usage and usage[-1]["usage"]["completion_tokens"] == 8 and usage[-1]["choices"] == []
    lps = [c for e in ev[:-1] if e["choices"] and e["choices"][0].get("logprobs")
           for c in e["choices"][0]["logprobs"]["content"]]
    assert len(lps) == 8 and all(len(c["top_logprobs"]) == 2 for c in lps)


@pytest.mark.parametrize("extra,msg", [
    ({"n": 2}, "n=2"), ({"tools": [{}]}, "tool calling"), ({"response_format": {"type": "json_object"}}, "response_format"),
    ({"foo": 1}, "unsupported parameter"), ({"top_logprobs": 2}, "top_logprobs"), ({"temperature": 3.0}, "temperature"),
    ({"max_tokens": 0}, "max_tokens"), ({"stop": ["a", "b", "c", "d", "e"]}, "stop"),
    ({"stream_options": {"x": 1}}, "stream_options"), ({"messages": []}, "messages"),
    ({"messages": [{"role": "tool", "content": "x"}]}, "role"), ({"max_tokens": 5000}, "max_model_len")])
def test_rejects_invalid(server, extra, msg):
    st, _, raw = chat(server.port(), body=extra)
    assert st == 400, raw
    err = json.loads(raw)["error"]
    assert msg in err["message"] and err["type"] == "invalid_request_error"


def test_stop_string_ends_request(server, tok):
    full = tok.decode(expected_tokens(tok, 8)).decode("utf-8", "replace")
    # A stop string of well-formed characters (the raw token bytes may not be UTF-8).
    stop = full[3:5]
    st, _, raw = chat(server.port(), body={"stop": stop})
    body = json.loads(raw)
    assert st == 200 and body["choices"][0]["finish_reason"] == "stop"
    assert body["choices"][0]["message"]["content"] == full[:full.index(stop)]


def test_auth_and_ops_routes(tok):
    s = M.serve_mock(tok, engine_cfg(), api_key="sekret", admin_port=0)
    try:
        p = s.port()
        assert chat(p)[0] == 401
        assert chat(p, headers={"Authorization": "Bearer wrong"})[0] == 401
        assert chat(p, headers={"Authorization": "Bearer sekret"})[0] == 200
        assert request(p, "GET", "/metrics")[0] == 401
        st, _, raw = request(p, "GET", "/metrics", headers={"Authorization": "Bearer sekret"})
        assert st == 200 and b"zstep:num_requests_running" in raw
        # The admin port only serves probes, metrics and admin routes.
        assert request(s.admin_port(), "POST", "/v1/chat/completions", {})[0] == 404
        assert request(s.admin_port(), "GET", "/health")[0] == 200
    finally:
        s.stop()


def test_metrics_and_drain(server):
    p = server.port()
    assert chat(p)[0] == 200
    st, hdr, raw = request(p, "GET", "/metrics")
    text = raw.decode()
    assert st == 200 and hdr["Content-Type"].startswith("text/plain")
    # The reference's metric names (dashboards keep working), plus this engine's own.
    for name in ("zstep:kv_cache_usage_perc", "zstep:time_to_first_token_seconds_bucket",
                 "zstep:time_per_output_token_seconds_count", "zstep:request_outcomes_total", "zstep:generation_tokens_total",
                 "zstep:num_requests_running", "zstep:num_requests_waiting", "zstep:num_preemptions_total",
                 "zstep:triton_recompilations_total"):
        assert name in text, name
    assert 'outcome="length"} 1' in text
    st, _, raw = request(p, "POST", "/admin/drain")
    assert st == 200 and json.loads(raw)["status"] == "draining"
    assert request(p, "GET", "/ready")[0] == 503
    assert request(p, "GET", "/health")[0] == 200  # still scraped while draining
    assert chat(p)[0] == 503


def test_client_disconnect_cancels_and_frees_kv(tok):
    s = M.serve_mock(tok, engine_cfg(), step_delay_us=20000)
    try:
        free0 = s.free_pages()
        sock = socket.create_connection(("127.0.0.1", s.port()))
        body = json.dumps({"messages": [{"role": "user", "content": "hello there"}], "max_tokens": 500,
                           "stream": True}).encode()
        sock.sendall(b"POST /v1/chat/completions HTTP/1.1\r\nHost: x\r\nContent-Type: application/json\r\n"
                     b"Content-Length: " + str(len(body)).encode() + b"\r\n\r\n" + body)
        sock.recv(4096)  # headers + first chunk: the request is running
        sock.close()
        for _ in range(200):
            if s.idle() and s.free_pages() == free0:
                break
            time.sleep(0.05)
        assert s.idle() and s.free_pages() == free0 and s.free_slots() == 4
        assert 'outcome="cancelled"} 1' in s.metrics_text()
    finally:
        s.stop()


def test_overload_returns_429(tok):
    s = M.serve_mock(tok, engine_cfg(), max_waiting=1, step_delay_us=50000)
    try:
        import threading

        codes = []

        def one():
            codes.append(chat(s.port(), body={"max_tokens": 20})[0])

        th = [threading.Thread(target=one) for _ in range(12)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        assert 429 in codes and 200 in codes
    finally:
        s.stop()


@pytest.mark.parametrize("stream", [True, False])
def test_backend_fault_fails_requests_and_reports_faulted(tok, stream):
    """Fault injection (the mock backend fails every step after its third, as a dead worker
    or a kernel error would): the request in flight ends with an error, the engine state
    turns to faulted, probes and new requests answer 503, and the failed request's slot
    and pages are released."""
    s = M.serve_mock(tok, engine_cfg(), admin_port=0, mock_low=LOW, mock_high=HIGH, fail_after=3)
    try:
        free0 = s.free_pages()
        status, _, raw = chat(s.port(), body={"max_tokens": 64, "stream": stream})
        if stream:
            assert status == 200  # headers went out before the fault
            events = sse_events(raw)
            errors = [e for e in events if isinstance(e, dict) and ("error" in e or any(
                c.get("finish_reason") == "error" for c in e.get("choices", [])))]
            assert errors, events
        else:
            assert status >= 500, raw
        assert s.state() == "faulted"
        assert request(s.port(), "GET", "/health")[0] == 503
        assert request(s.port(), "GET", "/ready")[0] == 503
        assert request(s.port(), "GET", "/livez")[0] == 200  # the process itself is alive
        assert chat(s.port())[0] == 503
        assert s.free_slots() == 4 and s.free_pages() == free0
        import re

        assert re.search(r"^zstep:engine_state(\{[^}]*\})? 3$", s.metrics_text(), re.M)
    finally:
        s.stop()
