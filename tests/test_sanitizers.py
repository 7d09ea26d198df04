"""The C++ control plane under sanitizers (CPU only): the master built with AddressSanitizer
+ UndefinedBehaviorSanitizer drives the mock backend through generation, prefix caching,
n-gram speculation and benchmark tiers; the ThreadSanitizer build serves HTTP requests
(streamed and not, plus metrics) while its engine thread runs, then drains on SIGTERM.
Any sanitizer report fails the test.  Skipped where no compiler with the sanitizer
runtimes exists."""

import http.client
import json
import os
import signal
import threading
import subprocess

import pytest

from tests.test_tokenizer import build_hf_tokenizer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN_DIR = os.path.join(ROOT, "zstep_b200", "bin")
REPORTS = ("AddressSanitizer", "LeakSanitizer", "runtime error:", "ThreadSanitizer")


def _build(target: str) -> str:
    path = os.path.join(BIN_DIR, f"zstep_{target}")
    r = subprocess.run(["make", "-C", os.path.join(ROOT, "csrc", "master"), target], capture_output=True, text=True,
                       timeout=900)
    if r.returncode != 0 or not os.path.exists(path):
        pytest.skip(f"no {target} build here: {r.stderr[-300:]}")
    return path


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("san_model"))
    build_hf_tokenizer(d)
    return d


def _clean(stderr: str) -> None:
    hits = [line for line in stderr.splitlines() if any(k in line for k in REPORTS)]
    assert not hits, "\n".join(hits[:20])


@pytest.mark.timeout(1200)
def test_engine_workloads_under_asan_ubsan(model_dir):
    b = _build("asan")
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1", UBSAN_OPTIONS="print_stacktrace=1")
    runs = [
        ["run", "--mock", "--model-dir", model_dir, "--prompt-ids", "5,6,7,8", "--max-tokens", "8"],
        ["run", "--mock", "--model-dir", model_dir, "--enable-prefix-caching", "--speculative-method", "ngram",
         "--bench-tiers", "t:4:8:32:16:64:2"],
        ["run", "--mock", "--model-dir", model_dir, "--max-seqs", "2", "--num-kv-pages", "24", "--enable-prefix-caching",
         "--bench-tiers", "small:3:6:40:12"],
    ]
    for args in runs:
        r = subprocess.run([b, *args], capture_output=True, text=True, timeout=600, env=env)
        assert r.returncode == 0, (args, r.stderr[-3000:])
        _clean(r.stderr)


@pytest.mark.timeout(1200)
def test_serve_loop_under_tsan(model_dir):
    b = _build("tsan")
    env = dict(os.environ, ZSTEP_API_KEY="", TSAN_OPTIONS="halt_on_error=0")
    p = subprocess.Popen([b, "serve", "--mock", "--model-dir", model_dir, "--port", "0", "--drain-timeout-secs", "10"],
                         stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, env=env)
    errors = []
    try:
        port = json.loads(p.stdout.readline())["port"]

        def client(i: int) -> None:
            try:
                conn = http.client.HTTPConnection("127.0.0.1", port, timeout=120)
                body = {"messages": [{"role": "user", "content": f"hello {i}"}], "max_tokens": 6, "stream": i % 2 == 0}
                conn.request("POST", "/v1/chat/completions", body=json.dumps(body),
                             headers={"Content-Type": "application/json"})
                r = conn.getresponse()
                r.read()
                if r.status != 200:
                    errors.append((i, r.status))
                conn.request("GET", "/metrics")
                conn.getresponse().read()
            except Exception as e:  # noqa: BLE001
                errors.append((i, repr(e)))

        # Simultaneous client connections: the connection threads tokenize, submit and
        # stream at the same time as the acceptor and the engine thread.  (This run found
        # the tokenizer's BPE memo being filled by several connection threads at once.)
        threads = [threading.Thread(target=client, args=(i,)) for i in range(6)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(timeout=300)
        assert not any(t.is_alive() for t in threads), "a client did not finish"
        assert not errors, errors
        p.send_signal(signal.SIGTERM)
        assert p.wait(timeout=120) == 0
    finally:
        if p.poll() is None:
            p.kill()
            p.wait()
    _clean(p.stderr.read())
