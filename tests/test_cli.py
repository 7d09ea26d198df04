"""The native `zstep` binary: `zstep run` (generation, greedy parity gate, bench tiers) and
`zstep serve` (HTTP server lifecycle with SIGTERM drain), on the scripted mock backend."""

import http.client
import json
import os
import signal
import subprocess

import pytest

from zstep_b200 import _master as M
from tests.test_tokenizer import build_hf_tokenizer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "zstep_b200", "bin", "zstep")


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    if not os.path.exists(BIN):
        subprocess.run(["make", "-C", os.path.join(ROOT, "csrc", "master")], check=True, capture_output=True)
    d = str(tmp_path_factory.mktemp("model"))
    build_hf_tokenizer(d)
    return d


def run(*args, timeout=120):
    return subprocess.run([BIN, *args], capture_output=True, text=True, timeout=timeout)


def mock_chain(prompt, n, high):
    out, last, pos = [], prompt[-1], len(prompt) - 1
    for _ in range(n):
        last = M.mock_next_token(last, pos, 0, high)
        out.append(last)
        pos += 1
    return out


def vocab_high(model_dir):
    t = M.Tokenizer()
    t.load_dir(model_dir)
    return min(t.vocab_size(), 256)


def test_run_prompt_ids(model_dir):
    r = run("run", "--mock", "--model-dir", model_dir, "--prompt-ids", "5,6,7", "--max-tokens", "6")
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout)
    assert out["tokens"] == mock_chain([5, 6, 7], 6, vocab_high(model_dir))


def test_verify_greedy_gate(model_dir, tmp_path):
    high = vocab_high(model_dir)
    prompts = [[1, 2, 3, 4], [9, 8, 7]]
    good = {"prompts": prompts, "expected": [mock_chain(p, 5, high) for p in prompts]}
    path = tmp_path / "v.json"
    path.write_text(json.dumps(good))
    r = run("run", "--mock", "--model-dir", model_dir, "--verify-greedy-json", str(path))
    assert r.returncode == 0, r.stdout + r.stderr
    assert json.loads(r.stdout)["mismatches"] == 0
    bad = dict(good, expected=[good["expected"][0], [0, 0, 0]])
    path.write_text(json.dumps(bad))
    r = run("run", "--mock", "--model-dir", model_dir, "--verify-greedy-json", str(path))
    assert r.returncode == 1 and json.loads(r.stdout)["mismatches"] == 1


def test_bench_tiers_report(model_dir):
    r = run("run", "--mock", "--model-dir", model_dir, "--bench-tiers", "small:2:4:16:8,tiny:1:2:8:4",
            "--bench-repeats", "2", "--max-seqs", "4", "--max-step-tokens", "256")
    assert r.returncode == 0, r.stderr
    rep = json.loads(r.stdout)
    assert [t["label"] for t in rep["tiers"]] == ["small", "tiny"]
    assert all(len(t["runs"]) == 2 and t["output_tok_s_mean"] > 0 for t in rep["tiers"])
    assert rep["tiers"][0]["runs"][0]["num_prompts"] == 4
    assert "git_sha" in rep["provenance"]


def test_bench_tiers_shared_prefix(model_dir):
    r = run("run", "--mock", "--model-dir", model_dir, "--bench-tiers", "apc:2:6:8:4:48:2", "--max-seqs", "4",
            "--max-step-tokens", "256", "--apc-node-pages", "1")
    assert r.returncode == 0, r.stderr
    run0 = json.loads(r.stdout)["tiers"][0]["runs"][0]
    assert run0["shared_prefix_len"] == 48 and run0["num_prefixes"] == 2 and run0["output_tok_s"] > 0
    assert run("run", "--mock", "--model-dir", model_dir, "--bench-tiers", "x:1:1:8:4:0:2").returncode == 2


def test_strict_flags(model_dir):
    r = run("serve", "--mock", "--model-dir", model_dir, "--bogus", "1")
    assert r.returncode == 2 and "unknown flag --bogus" in r.stderr
    r = run("serve", "--mock", "--model-dir", model_dir, "--max-seqs", "abc")
    assert r.returncode == 2
    r = run("run", "--mock", "--model-dir", model_dir, "--speculative-method", "magic", "--prompt-ids", "1")
    assert r.returncode == 2 and "speculative-method" in r.stderr
    assert run("frobnicate").returncode == 2


def test_serve_lifecycle_and_sigterm(model_dir):
    env = dict(os.environ, ZSTEP_API_KEY="")
    p = subprocess.Popen([BIN, "serve", "--mock", "--model-dir", model_dir, "--port", "0", "--served-model-name", "m1",
                          "--drain-timeout-secs", "5"], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                         env=env)
    try:
        ready = json.loads(p.stdout.readline())
        port = ready["port"]
        conn = http.client.HTTPConnection("127.0.0.1", port, timeout=30)
        conn.request("POST", "/v1/chat/completions",
                     body=json.dumps({"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4}),
                     headers={"Content-Type": "application/json"})
        r = conn.getresponse()
        body = json.loads(r.read())
        assert r.status == 200 and body["model"] == "m1" and body["usage"]["completion_tokens"] == 4
        p.send_signal(signal.SIGTERM)
        assert p.wait(timeout=30) == 0
    finally:
        if p.poll() is None:
            p.kill()
            p.wait()


def test_micro_steps_control_plane_benchmark():
    """`zstep run --micro-steps` drives synthetic plans through the shared-memory coordinator
    to two CPU workers running the micro-step model (tensor-parallel sum over gloo)."""
    import sys

    r = run("run", "--micro-steps", "12", "--token-counts", "4,16", "--device", "cpu", "--world-size", "2",
            "--max-seqs", "32", "--max-step-tokens", "64", "--micro-hidden", "256", "--micro-features", "256",
            "--micro-experts", "64", "--micro-topk", "4", "--python", sys.executable, "--worker-root", ROOT,
            timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    rep = json.loads(r.stdout.strip().splitlines()[-1])
    tiers = rep["micro_steps"]
    assert [t["token_count"] for t in tiers] == [4, 16]
    assert all(t["steps"] == 12 and t["steps_per_s"] > 0 and t["p99_step_us"] >= t["p50_step_us"] for t in tiers)
