"""Host-side pieces of the expert-parallel all-to-all and the DSpark head that need no GPU:
the symmetric block layout, the receive capacity bound, the DSpark weight shapes and
auxiliary-layer choice, and the `dspark` speculative method through the CLI."""

import os
import subprocess

import pytest

from zstep_b200.config import DeepSeekConfig, deepseek_small_gpu
from zstep_b200.models.deepseek_weights import DeepSeekRandomWeights, shape_of
from zstep_b200.ops import mx
from zstep_b200.parallel.ep import default_recv_cap, ep_layout

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "zstep_b200", "bin", "zstep")


@pytest.mark.parametrize("world,experts,hidden,topk,tokens", [(1, 64, 1024, 4, 256), (8, 256, 4096, 8, 4096),
                                                              (2, 32, 512, 2, 7)])
def test_ep_layout_is_aligned_and_covers_every_region(world, experts, hidden, topk, tokens):
    cap = default_recv_cap(world, experts, topk, tokens)
    assert cap % 128 == 0
    # Worst case: every pair of every rank on one rank, each local segment 128-row aligned.
    assert cap >= world * tokens * topk + (experts // world) * 127
    off = ep_layout(world, experts, hidden, topk, tokens, cap)
    order = ["flags", "counts", "q", "sf", "meta", "comb", "nbytes"]
    sizes = {"flags": 64 * 4, "counts": world * experts * 8, "q": cap * hidden,
             "sf": mx.atoms_bytes(cap, hidden), "meta": cap * 8, "comb": tokens * topk * hidden * 2}
    for a, b in zip(order, order[1:]):
        assert off[a] % 256 == 0 and off[b] >= off[a] + sizes[a], (a, b, off)


def test_dspark_weights_and_aux_layers():
    cfg = deepseek_small_gpu(num_layers=5, vocab=1024, experts=8)
    assert cfg.dspark_aux() == (1, 2, 4)
    assert DeepSeekConfig(num_hidden_layers=1).dspark_aux() == (0,)
    assert DeepSeekConfig(num_hidden_layers=48, dspark_aux_layers=(3, 7)).dspark_aux() == (3, 7)
    H, r = cfg.hidden_size, cfg.dspark_markov_rank
    assert shape_of(cfg, "dspark.fc") == (H, 3 * H)
    assert shape_of(cfg, "dspark.markov_w1") == (cfg.vocab_size, r)
    assert shape_of(cfg, "layers.dspark.mla.kv_a") == shape_of(cfg, "layers.0.mla.kv_a")
    w = DeepSeekRandomWeights(cfg, seed=3)
    a, b = w.get("dspark.markov_w2"), w.get("dspark.markov_w2")
    assert a.shape == (cfg.vocab_size, r) and bool((a == b).all())  # deterministic per name
    n = w.get("dspark.final_norm").float()
    assert abs(float(n.mean()) - 1.0) < 0.05  # norm scales start near one


def test_cli_accepts_dspark_and_rejects_unknown_methods(tmp_path):
    if not os.path.exists(BIN):
        subprocess.run(["make", "-C", os.path.join(ROOT, "csrc", "master")], check=True, capture_output=True)
    from tests.test_tokenizer import build_hf_tokenizer

    build_hf_tokenizer(str(tmp_path))
    ok = subprocess.run([BIN, "run", "--mock", "--model-dir", str(tmp_path), "--speculative-method", "dspark",
                         "--prompt-ids", "5,6,7", "--max-tokens", "4"], capture_output=True, text=True, timeout=120)
    assert ok.returncode == 0, ok.stderr
    bad = subprocess.run([BIN, "run", "--mock", "--model-dir", str(tmp_path), "--speculative-method", "eagle",
                          "--prompt-ids", "5", "--max-tokens", "1"], capture_output=True, text=True, timeout=120)
    assert bad.returncode == 2 and "dspark" in bad.stderr
