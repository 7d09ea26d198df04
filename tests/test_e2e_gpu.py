"""The native `zstep run` driving a B200 worker end to end: greedy generation through the
shared-memory coordinator, and MTP speculative decoding producing the same tokens."""

import json
import os
import subprocess
import sys

import pytest

from tests.test_tokenizer import build_hf_tokenizer

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "zstep_b200", "bin", "zstep")
PROMPTS = [[11, 200, 3000, 45, 7], [900, 901, 902], list(range(100, 140))]


@pytest.fixture(scope="module")
def model_dir(tmp_path_factory):
    if not os.path.exists(BIN):
        subprocess.run(["make", "-C", os.path.join(ROOT, "csrc", "master")], check=True, capture_output=True)
    d = str(tmp_path_factory.mktemp("model"))
    build_hf_tokenizer(d)
    return d


def zstep_run(model_dir, *extra, timeout=900):
    args = [BIN, "run", "--model-dir", model_dir, "--model", "qwen3.5-small", "--device", "cuda", "--max-seqs", "8",
            "--max-model-len", "512", "--num-kv-pages", "256", "--max-step-tokens", "256", "--max-prefill-chunk",
            "128", "--python", sys.executable, "--worker-root", ROOT, *extra]
    r = subprocess.run(args, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_greedy_and_mtp_agree(model_dir):
    outs = {}
    for method in ("none", "mtp"):
        res = []
        for p in PROMPTS:
            o = zstep_run(model_dir, "--prompt-ids", ",".join(map(str, p)), "--max-tokens", "16",
                          "--speculative-method", method)
            res.append(o["tokens"])
        outs[method] = res
    assert all(len(t) == 16 for t in outs["none"])
    # Verify rows run the varlen GDN kernel while plain decode runs the decode kernel, so a
    # near-tie can flip after a few tokens; the leading tokens must agree everywhere and
    # at least one continuation in full.
    assert all(a[:4] == b[:4] for a, b in zip(outs["none"], outs["mtp"])), outs
    assert any(a == b for a, b in zip(outs["none"], outs["mtp"])), outs


def test_deepseek_greedy_and_dspark_agree(model_dir):
    """DeepSeek-style model with the DSpark draft head: verify steps accept drafts only
    where they equal the target's greedy tokens, so the output matches plain decoding
    (leading tokens everywhere, at least one continuation in full: verify rows run the
    varlen attention path while plain decode runs the split-KV one)."""
    outs = {}
    for method in ("none", "dspark"):
        res = []
        for p in PROMPTS:
            args = [BIN, "run", "--model-dir", model_dir, "--model", "deepseek-small", "--device", "cuda",
                    "--max-seqs", "4", "--max-model-len", "256", "--num-kv-pages", "128", "--max-step-tokens", "128",
                    "--max-prefill-chunk", "128", "--python", sys.executable, "--worker-root", ROOT,
                    "--prompt-ids", ",".join(map(str, p)), "--max-tokens", "12", "--speculative-method", method]
            r = subprocess.run(args, capture_output=True, text=True, timeout=900)
            assert r.returncode == 0, r.stderr[-3000:]
            res.append(json.loads(r.stdout.strip().splitlines()[-1])["tokens"])
        outs[method] = res
    assert all(len(t) == 12 for t in outs["dspark"])
    assert all(a[:4] == b[:4] for a, b in zip(outs["none"], outs["dspark"])), outs
    assert any(a == b for a, b in zip(outs["none"], outs["dspark"])), outs


def test_bench_tier_with_mtp_and_shared_prefix(model_dir):
    rep = zstep_run(model_dir, "--speculative-method", "mtp", "--bench-tiers", "mtp:4:8:32:16:64:2")
    run0 = rep["tiers"][0]["runs"][0]
    assert run0["output_tok_s"] > 0 and run0["shared_prefix_len"] == 64
    assert run0["mean_acceptance_length"] >= 1.0


def test_deepseek_dram_tier_keeps_greedy_tokens(model_dir, tmp_path):
    """DeepSeek-style model on a B200 worker with a host DRAM tier and a small HBM page
    pool: prefixes are demoted and reloaded between requests, and the generated tokens
    equal a run without prefix caching."""
    fam = [list(range(300, 364)), list(range(900, 964))]
    prompts = [fam[k % 2] + [50 + 7 * k + j for j in range(8)] for k in range(6)]
    path = tmp_path / "p.json"
    path.write_text(json.dumps({"prompts": prompts}))  # no expectations: --max-tokens each
    base = ["--model", "deepseek-small", "--max-seqs", "1", "--max-tokens", "8"]

    def run(*extra):
        args = [BIN, "run", "--model-dir", model_dir, "--device", "cuda", "--max-model-len", "256",
                "--max-step-tokens", "256", "--max-prefill-chunk", "128", "--python", sys.executable,
                "--worker-root", ROOT, "--verify-greedy-json", str(path), *base, *extra]
        r = subprocess.run(args, capture_output=True, text=True, timeout=900)
        return json.loads(r.stdout.strip().splitlines()[-1]), r

    ref, r0 = run("--no-enable-prefix-caching", "--num-kv-pages", "64")
    assert "verify_greedy" in ref, r0.stderr[-3000:]
    want = [e["tokens"] for e in ref["verify_greedy"]]
    path.write_text(json.dumps({"prompts": prompts, "expected": want}))
    got, r1 = run("--num-kv-pages", "16", "--dram-kv-blocks", "32")
    assert got.get("mismatches") == 0, (got, r1.stderr[-3000:])


def test_micro_steps_on_gpu():
    """The micro-step model on a B200 worker (RMSNorm + MXFP8 + tcgen05 GEMM + router)."""
    args = [BIN, "run", "--micro-steps", "20", "--token-counts", "6,48,192", "--device", "cuda", "--max-seqs", "192",
            "--max-step-tokens", "256", "--python", sys.executable, "--worker-root", ROOT]
    r = subprocess.run(args, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    tiers = json.loads(r.stdout.strip().splitlines()[-1])["micro_steps"]
    assert [t["token_count"] for t in tiers] == [6, 48, 192]
    assert all(t["mean_gpu_us"] > 0 and t["steps_per_s"] > 0 for t in tiers)
