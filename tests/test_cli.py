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
    r = run("serve", "--mock", "--model-dir", model_dir, "--max-seqs", "600", "--max-step-tokens", "8192")
    assert r.returncode == 2 and "max-seqs" in r.stderr
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
        tp = "00-0af7651916cd43dd8448eb211c80319c-b7ad6b7169203331-01"
        conn.request("POST", "/v1/chat/completions",
                     body=json.dumps({"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4,
                                      "user": "u-17"}),
                     headers={"Content-Type": "application/json", "x-request-id": "rq-1", "traceparent": tp})
        r = conn.getresponse()
        body = json.loads(r.read())
        assert r.status == 200 and body["model"] == "m1" and body["usage"]["completion_tokens"] == 4
        p.send_signal(signal.SIGTERM)
        assert p.wait(timeout=30) == 0
        log = p.stderr.read()
        line = next(x for x in log.splitlines() if x.startswith("zstep_serve request_id=rq-1 "))
        assert f"traceparent={tp}" in line and "max_tokens=4" in line and "user=u-17" in line, line
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


def test_reference_serve_flags(model_dir):
    """Every flag of the reference's `zstep serve` usage is accepted: calibration, KV dtype,
    GDN node size, loading-area alias, starvation cap, mixed-step budget, prompt lookup and
    the (ignored) host all-reduce grid flags; invalid values are rejected."""
    ok = run("run", "--mock", "--model-dir", model_dir, "--prompt-ids", "5,6,7", "--max-tokens", "4",
             "--gpu-memory-utilization", "0.5", "--kv-cache-dtype", "bf16", "--apc-gdn-node-tokens", "64",
             "--kv-loading-area-ratio", "0.2", "--prefill-starvation-cap-ms", "1000", "--max-mixed-step-tokens",
             "512", "--no-dynamic-prefill-budget", "--prompt-lookup-max", "4", "--prompt-lookup-min", "2",
             "--allreduce-blocks", "8", "--allreduce-threads", "256")
    assert ok.returncode == 0, ok.stderr
    assert json.loads(ok.stdout)["tokens"] == mock_chain([5, 6, 7], 4, vocab_high(model_dir))
    assert "allreduce-blocks accepted and ignored" in ok.stderr
    bad = [("--kv-cache-dtype", "fp8", "kv-cache-dtype"), ("--gpu-memory-utilization", "1.5", "gpu-memory"),
           ("--apc-gdn-node-tokens", "96", "apc-gdn-node-tokens"), ("--prompt-lookup-min", "7", "prompt-lookup"),
           ("--max-mixed-step-tokens", "-1", "max-mixed-step-tokens")]
    for flag, value, word in bad:
        r = run("run", "--mock", "--model-dir", model_dir, "--prompt-ids", "1", flag, value)
        assert r.returncode == 2 and word in r.stderr, (flag, value, r.stderr[-500:])


def test_multi_case_greedy_parity(model_dir, tmp_path):
    """The reference's parity-gate input: named cases run alone, batched and chunked; a report
    per case and pass, and the gates (--require-exact-greedy, --require-exact-cases, per-case
    require_exact)."""
    high = vocab_high(model_dir)
    prompts = {"short": [1, 2, 3, 4], "long": list(range(10, 60))}
    cases = [{"name": n, "prompt_token_ids": p, "max_tokens": 5, "expected_greedy_token_ids": mock_chain(p, 5, high)}
             for n, p in prompts.items()]
    ref = tmp_path / "ref.json"
    ref.write_text(json.dumps({"vllm_version": "x", "cases": cases}))
    out = tmp_path / "parity.json"
    metrics = tmp_path / "metrics.json"
    r = run("run", "--mock", "--model-dir", model_dir, "--verify-greedy-json", str(ref), "--max-prefill-chunk", "16",
            "--verify-output-json", str(out), "--metrics-output", str(metrics), "--require-exact-greedy", "true")
    assert r.returncode == 0, r.stdout + r.stderr
    rep = json.loads(out.read_text())
    assert rep == json.loads(metrics.read_text()) == json.loads(r.stdout)
    assert rep["all_matched"] and rep["batched_vs_single_exact_match"] and rep["chunked_vs_unchunked_exact_match"]
    assert [c["name"] for c in rep["cases"]] == ["short", "long"] and rep["gate"] == "ok"
    assert rep["cases"][1]["chunked_generated_token_ids"] == cases[1]["expected_greedy_token_ids"]
    # One wrong expected token: reported; fails only under a gate.
    cases[0]["expected_greedy_token_ids"][2] += 1
    ref.write_text(json.dumps({"cases": cases}))
    base = ("run", "--mock", "--model-dir", model_dir, "--verify-greedy-json", str(ref))
    r = run(*base)
    assert r.returncode == 0 and not json.loads(r.stdout)["all_matched"]
    assert json.loads(r.stdout)["cases"][0]["single_match"]["first_mismatch_token_index"] == 2
    assert run(*base, "--require-exact-greedy", "true").returncode == 1
    assert run(*base, "--require-exact-cases", "long").returncode == 0
    assert run(*base, "--require-exact-cases", "short").returncode == 1
    assert run(*base, "--require-exact-cases", "nope").returncode == 1
    cases[0]["require_exact"] = True
    ref.write_text(json.dumps({"cases": cases}))
    assert run(*base).returncode == 1
    cases[0]["max_tokens"] = 4  # expected length must equal max_tokens
    ref.write_text(json.dumps({"cases": cases}))
    assert run(*base).returncode == 2


def test_reference_run_spellings(model_dir):
    """`zstep --model-dir ...` without a subcommand, the reference's flag names for the same
    options, and ';'-separated bench tiers."""
    r = run("--mock", "--model-dir", model_dir, "--prompt-ids", "5,6,7", "--max-new-tokens", "3")
    assert r.returncode == 0, r.stderr
    assert json.loads(r.stdout)["tokens"] == mock_chain([5, 6, 7], 3, vocab_high(model_dir))
    r = run("--mock", "--model-dir", model_dir, "--bench-tiers", "a:1:2:8:4;b:2:2:8:4", "--repeats", "2",
            "--max-seqs", "4", "--max-step-tokens", "256", "--max-pages-per-seq", "64", "--max-decoder-rows", "256",
            "--heartbeat-timeout-ms", "4000")
    assert r.returncode == 0, r.stderr
    rep = json.loads(r.stdout)
    assert [t["label"] for t in rep["tiers"]] == ["a", "b"] and all(len(t["runs"]) == 2 for t in rep["tiers"])
    r = run("--mock", "--model-dir", model_dir, "--prompt-ids", "1", "--max-step-tokens", "256",
            "--max-decoder-rows", "8")
    assert r.returncode == 2 and "max-decoder-rows" in r.stderr


def test_tokenizer_mode_values(model_dir):
    base = ("run", "--mock", "--model-dir", model_dir, "--prompt", "hi", "--max-tokens", "2")
    for mode in ("auto", "chatml", "deepseek", "deepseek_v41"):
        r = run(*base, "--tokenizer-mode", mode)
        assert r.returncode == 0, (mode, r.stderr)
    r = run(*base, "--tokenizer-mode", "llama")
    assert r.returncode == 2 and "tokenizer-mode" in r.stderr


def test_micro_steps_are_the_default_mode():
    """Without a model or a mode, `zstep run` (and `zstep --steps N`, the reference's
    spelling) is the control-plane micro-step benchmark."""
    import sys

    small = ["--token-counts", "4", "--device", "cpu", "--world-size", "1", "--max-seqs", "8", "--max-step-tokens",
             "16", "--micro-hidden", "256", "--micro-features", "256", "--micro-experts", "64", "--micro-topk", "4",
             "--python", sys.executable, "--worker-root", ROOT]
    r = run("run", *small, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    assert json.loads(r.stdout.strip().splitlines()[-1])["micro_steps"][0]["steps"] == 200
    r = run("--steps", "7", *small, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    assert json.loads(r.stdout.strip().splitlines()[-1])["micro_steps"][0]["steps"] == 7
