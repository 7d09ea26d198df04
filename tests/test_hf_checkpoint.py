"""HF-safetensors checkpoints (CPU): a checkpoint exported from random-init weights in the
HF layout loads back tensor-for-tensor through the readers the runners use, the config
round-trips through config.json, and the fp32 reference forward is bit-identical with
the loaded weights."""

import dataclasses

import torch

from zstep_b200.config import DeepSeekConfig, Qwen35Config, deepseek_tiny, qwen35_tiny
from zstep_b200.models import deepseek_weights, weights
from zstep_b200.models.deepseek_ref import DeepSeekReference
from zstep_b200.models.deepseek_weights import DeepSeekRandomWeights
from zstep_b200.models.hf_checkpoint import DeepSeekSafetensorsWeights, export_deepseek, export_qwen35
from zstep_b200.models.qwen35_ref import Qwen35Reference
from zstep_b200.models.weights import RandomWeights, SafetensorsWeights
from zstep_b200.runtime import runners


def _qwen_names(cfg):
    names = ["embed", "final_norm", "lm_head"]
    for i in range(cfg.num_hidden_layers):
        names += weights.layer_names(cfg, i)
    names += ["mtp." + n for n in ("pre_fc_norm_embedding", "pre_fc_norm_hidden", "fc", "norm")]
    names += weights.layer_names(cfg, 0, prefix="mtp.layer.")
    return names


def test_qwen35_checkpoint_round_trip(tmp_path):
    cfg = qwen35_tiny()
    src = RandomWeights(cfg, seed=7)
    d = export_qwen35(cfg, src, tmp_path / "qwen")
    loaded_cfg = Qwen35Config.from_hf(str(d))
    for f in dataclasses.fields(cfg):
        if f.name != "name":
            assert getattr(loaded_cfg, f.name) == getattr(cfg, f.name), f.name
    # The runner's own selection: a directory means an HF config + safetensors reader.
    assert isinstance(runners._weights(runners._resolve_config(str(d)), str(d), 0), SafetensorsWeights)
    ck = SafetensorsWeights(cfg, d)
    for n in _qwen_names(cfg):
        a, b = src.get(n), ck.get(n)
        assert a.shape == b.shape and torch.equal(a.to(b.dtype), b), n
    r1, r2 = Qwen35Reference(cfg, src), Qwen35Reference(cfg, ck)
    s1, s2 = r1.new_state(), r2.new_state()
    for t in (5, 77, 1000, 3, 42):
        assert torch.equal(r1.step(s1, t), r2.step(s2, t))


def test_deepseek_checkpoint_round_trip(tmp_path):
    cfg = deepseek_tiny()
    src = DeepSeekRandomWeights(cfg, seed=9)
    d = export_deepseek(cfg, src, tmp_path / "ds", with_dspark=True)
    assert DeepSeekConfig.is_hf_config(str(d))
    loaded_cfg = DeepSeekConfig.from_hf(str(d))
    for f in dataclasses.fields(cfg):
        if f.name != "name":
            assert getattr(loaded_cfg, f.name) == getattr(cfg, f.name), f.name
    ck = runners._weights(runners._resolve_config(str(d)), str(d), 0)
    assert isinstance(ck, DeepSeekSafetensorsWeights)
    names = ["embed", "final_norm", "lm_head", "hc_head.fn", "hc_head.base", "hc_head.scale",
             "dspark.fc", "dspark.final_norm", "dspark.markov_w1", "dspark.markov_w2"]
    for i in range(cfg.num_hidden_layers):
        names += deepseek_weights.layer_names(cfg, i)
    names += ["layers.dspark." + n.split(".", 2)[-1] for n in deepseek_weights.layer_names(cfg, 0)
              if not n.split(".", 2)[-1].startswith(("moe.", "mlp."))]
    for n in names:
        a, b = src.get(n), ck.get(n)
        assert a.shape == b.shape and torch.equal(a.to(b.dtype), b), n
    moe_layer = next(i for i in range(cfg.num_hidden_layers) if not cfg.is_dense(i))
    for e in (0, cfg.n_routed_experts - 1):
        for leaf in ("moe.gate", "moe.up", "moe.down"):
            n = f"layers.{moe_layer}.{leaf}"
            assert torch.equal(src.get_expert(n, e), ck.get_expert(n, e)), (n, e)
    r1, r2 = DeepSeekReference(cfg, src), DeepSeekReference(cfg, ck)
    s1, s2 = r1.new_state(), r2.new_state()
    for t in (5, 77, 300, 3):
        assert torch.equal(r1.step(s1, t), r2.step(s2, t))
