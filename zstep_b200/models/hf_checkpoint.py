"""HF-safetensors checkpoints for both model families: export and DeepSeek-style loading.

``SafetensorsWeights`` (models/weights.py) reads Qwen3.5-MoE checkpoints; this module adds
the writer that produces the same layout from any canonical weight source, and the
reader/writer pair for the DeepSeek-style MLA + DSA + mHC family.  Readers expose the
canonical ``get(name, device)`` interface (plus ``get_expert`` for routed experts), so the
GPU runners and the fp32 references load a checkpoint exactly like random-init weights.

DeepSeek-style tensor names follow the DeepSeek-V3 HF layout for the parts that exist
there, the V3.2 names for the lightning indexer, and flat ``hc_*`` names for the mHC
mixing parameters (per layer ``hc_attn_fn/base/scale`` and ``hc_ffn_*``, globally
``hc_head_*``)::

    model.embed_tokens.weight, model.norm.weight, lm_head.weight
    model.layers.{i}.input_layernorm.weight          attn_norm
    model.layers.{i}.post_attention_layernorm.weight ffn_norm
    model.layers.{i}.self_attn.{q_a_proj, q_a_layernorm, q_b_proj, kv_a_proj_with_mqa,
                                kv_a_layernorm, kv_b_proj, o_proj}.weight
    model.layers.{i}.self_attn.indexer.{wq_b, wk, k_norm, weights_proj}.weight
    model.layers.{i}.mlp.{gate_proj, up_proj, down_proj}.weight           (dense layers)
    model.layers.{i}.mlp.gate.weight, mlp.gate.e_score_correction_bias     (router)
    model.layers.{i}.mlp.experts.{e}.{gate_proj, up_proj, down_proj}.weight
    model.layers.{i}.mlp.shared_experts.{gate_proj, up_proj, down_proj}.weight
    model.layers.{i}.hc_{attn,ffn}_{fn,base,scale}, model.hc_head_{fn,base,scale}
    dspark.*  (the DSpark draft head, canonical names under a ``dspark.`` prefix)

``config.json`` carries the DeepSeek-V3 keys plus this model's (``index_*``, ``hc_*``);
``DeepSeekConfig.from_hf`` reads exactly the keys it knows.

Reference parity: the reference loads Qwen3.5 checkpoints itself
(worker/zstep_worker/models/qwen35_moe.py:852-1019) and hands DeepSeek checkpoints to
vLLM (worker/zstep_worker/models/deepseek_v41.py:408).
"""

from __future__ import annotations

import dataclasses
import json
from pathlib import Path

import torch

from ..config import DeepSeekConfig, Qwen35Config
from . import deepseek_weights


# ----------------------------------------------------------------------------- Qwen3.5
def qwen35_hf_config(cfg: Qwen35Config) -> dict:
    return {
        "model_type": "qwen3_5_moe", "_name_or_path": cfg.name, "vocab_size": cfg.vocab_size,
        "hidden_size": cfg.hidden_size, "num_hidden_layers": cfg.num_hidden_layers,
        "layer_types": list(cfg.layer_types), "rms_norm_eps": cfg.rms_norm_eps,
        "num_attention_heads": cfg.num_attention_heads, "num_key_value_heads": cfg.num_key_value_heads,
        "head_dim": cfg.head_dim, "rope_parameters": {"rope_theta": cfg.rope_theta,
                                                      "partial_rotary_factor": cfg.partial_rotary_factor},
        "linear_num_key_heads": cfg.linear_num_key_heads, "linear_key_head_dim": cfg.linear_key_head_dim,
        "linear_num_value_heads": cfg.linear_num_value_heads, "linear_value_head_dim": cfg.linear_value_head_dim,
        "linear_conv_kernel_dim": cfg.linear_conv_kernel_dim, "num_experts": cfg.num_experts,
        "num_experts_per_tok": cfg.num_experts_per_tok, "moe_intermediate_size": cfg.moe_intermediate_size,
        "shared_expert_intermediate_size": cfg.shared_expert_intermediate_size,
        "norm_topk_prob": cfg.norm_topk_prob, "mtp_num_hidden_layers": cfg.mtp_num_hidden_layers,
    }


def _qwen35_layer_tensors(cfg: Qwen35Config, src, canon_prefix: str, hf_prefix: str, gdn: bool) -> dict:
    """HF tensors of one decoder layer (inverse of SafetensorsWeights._layer)."""
    g = lambda n: src.get(canon_prefix + n, "cpu")  # noqa: E731
    lp = hf_prefix
    out = {lp + "input_layernorm.weight": g("input_norm"), lp + "post_attention_layernorm.weight": g("post_norm")}
    if gdn:
        w = g("gdn.in_proj")
        qkv = cfg.conv_dim
        hv, dv = cfg.linear_num_value_heads, cfg.linear_value_head_dim
        out[lp + "linear_attn.in_proj_qkv.weight"] = w[:qkv]
        out[lp + "linear_attn.in_proj_z.weight"] = w[qkv:qkv + hv * dv]
        out[lp + "linear_attn.in_proj_b.weight"] = w[qkv + hv * dv:qkv + hv * dv + hv]
        out[lp + "linear_attn.in_proj_a.weight"] = w[qkv + hv * dv + hv:]
        out[lp + "linear_attn.conv1d.weight"] = g("gdn.conv_w").reshape(cfg.conv_dim, 1, -1)
        out[lp + "linear_attn.A_log"] = g("gdn.a_log")
        out[lp + "linear_attn.dt_bias"] = g("gdn.dt_bias")
        out[lp + "linear_attn.norm.weight"] = g("gdn.norm")
        out[lp + "linear_attn.out_proj.weight"] = g("gdn.out_proj")
    else:
        w = g("attn.qkv")
        hq2 = cfg.num_attention_heads * 2 * cfg.head_dim
        kvd = cfg.num_key_value_heads * cfg.head_dim
        out[lp + "self_attn.q_proj.weight"] = w[:hq2]
        out[lp + "self_attn.k_proj.weight"] = w[hq2:hq2 + kvd]
        out[lp + "self_attn.v_proj.weight"] = w[hq2 + kvd:]
        for leaf in ("q_norm", "k_norm", "o_proj"):
            out[lp + f"self_attn.{leaf}.weight"] = g("attn." + leaf)
    out[lp + "mlp.gate.weight"] = g("moe.router")
    out[lp + "mlp.shared_expert_gate.weight"] = g("moe.shared_gate")
    out[lp + "mlp.experts.gate_up_proj"] = torch.cat([g("moe.gate"), g("moe.up")], 1)
    out[lp + "mlp.experts.down_proj"] = g("moe.down")
    for leaf in ("gate", "up", "down"):
        out[lp + f"mlp.shared_expert.{leaf}_proj.weight"] = g("moe.shared." + leaf)
    return out


def export_qwen35(cfg: Qwen35Config, src, out_dir: str | Path) -> Path:
    """Write ``config.json`` + ``model.safetensors`` in the HF Qwen3.5-MoE layout from any
    canonical weight source (random init, another checkpoint)."""
    from safetensors.torch import save_file

    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    t = {"model.embed_tokens.weight": src.get("embed", "cpu"), "model.norm.weight": src.get("final_norm", "cpu"),
         "lm_head.weight": src.get("lm_head", "cpu")}
    for i in range(cfg.num_hidden_layers):
        t.update(_qwen35_layer_tensors(cfg, src, f"layers.{i}.", f"model.layers.{i}.",
                                       cfg.layer_types[i] == "linear_attention"))
    if cfg.mtp_num_hidden_layers > 0:
        for leaf in ("pre_fc_norm_embedding", "pre_fc_norm_hidden", "fc", "norm"):
            t[f"mtp.{leaf}.weight"] = src.get("mtp." + leaf, "cpu")
        t.update(_qwen35_layer_tensors(cfg, src, "mtp.layer.", "mtp.layers.0.", False))
    save_file({k: v.contiguous() for k, v in t.items()}, str(out / "model.safetensors"))
    (out / "config.json").write_text(json.dumps(qwen35_hf_config(cfg), indent=1))
    return out


# ----------------------------------------------------------------------------- DeepSeek
_DS_LAYER = {
    "attn_norm": "input_layernorm.weight", "ffn_norm": "post_attention_layernorm.weight",
    "mla.q_a": "self_attn.q_a_proj.weight", "mla.q_a_norm": "self_attn.q_a_layernorm.weight",
    "mla.q_b": "self_attn.q_b_proj.weight", "mla.kv_a": "self_attn.kv_a_proj_with_mqa.weight",
    "mla.kv_a_norm": "self_attn.kv_a_layernorm.weight", "mla.kv_b": "self_attn.kv_b_proj.weight",
    "mla.o_proj": "self_attn.o_proj.weight",
    "idx.wq": "self_attn.indexer.wq_b.weight", "idx.wk": "self_attn.indexer.wk.weight",
    "idx.k_norm": "self_attn.indexer.k_norm.weight", "idx.w": "self_attn.indexer.weights_proj.weight",
    "mlp.gate": "mlp.gate_proj.weight", "mlp.up": "mlp.up_proj.weight", "mlp.down": "mlp.down_proj.weight",
    "moe.router": "mlp.gate.weight", "moe.bias": "mlp.gate.e_score_correction_bias",
    "moe.shared.gate": "mlp.shared_experts.gate_proj.weight", "moe.shared.up": "mlp.shared_experts.up_proj.weight",
    "moe.shared.down": "mlp.shared_experts.down_proj.weight",
    "hc_attn.fn": "hc_attn_fn", "hc_attn.base": "hc_attn_base", "hc_attn.scale": "hc_attn_scale",
    "hc_ffn.fn": "hc_ffn_fn", "hc_ffn.base": "hc_ffn_base", "hc_ffn.scale": "hc_ffn_scale",
}
_DS_GLOBAL = {"embed": "model.embed_tokens.weight", "final_norm": "model.norm.weight", "lm_head": "lm_head.weight",
              "hc_head.fn": "model.hc_head_fn", "hc_head.base": "model.hc_head_base",
              "hc_head.scale": "model.hc_head_scale"}
_DS_EXPERT = {"moe.gate": "gate_proj", "moe.up": "up_proj", "moe.down": "down_proj"}


def _ds_hf_name(name: str) -> str:
    if name in _DS_GLOBAL:
        return _DS_GLOBAL[name]
    if name.startswith("dspark.") or name.startswith("layers.dspark."):
        return name if name.startswith("dspark.") else "dspark.layer." + name[len("layers.dspark."):]
    _, i, leaf = name.split(".", 2)
    return f"model.layers.{i}.{_DS_LAYER[leaf]}"


class DeepSeekSafetensorsWeights:
    """DeepSeek-style checkpoint reader (``model.safetensors.index.json`` or one
    ``model.safetensors``) with the canonical interface of DeepSeekRandomWeights."""

    def __init__(self, cfg: DeepSeekConfig, model_dir: str | Path):
        from safetensors import safe_open

        self.cfg = cfg
        self.dir = Path(model_dir)
        idx = self.dir / "model.safetensors.index.json"
        if idx.exists():
            self.map = json.loads(idx.read_text())["weight_map"]
        else:
            with safe_open(str(self.dir / "model.safetensors"), "pt") as h:
                self.map = {k: "model.safetensors" for k in h.keys()}
        self._handles: dict[str, object] = {}

    def _raw(self, key: str) -> torch.Tensor:
        from safetensors import safe_open

        if key not in self.map:
            raise KeyError(f"{key} not in checkpoint {self.dir}")
        fn = self.map[key]
        if fn not in self._handles:
            self._handles[fn] = safe_open(str(self.dir / fn), "pt")
        return self._handles[fn].get_tensor(key)

    def get_expert(self, name: str, e: int, device="cpu") -> torch.Tensor:
        _, i, leaf = name.split(".", 2)
        return self._raw(f"model.layers.{i}.mlp.experts.{e}.{_DS_EXPERT[leaf]}.weight").to(device)

    def get(self, name: str, device="cpu") -> torch.Tensor:
        if name.endswith(tuple(_DS_EXPERT)) and not name.endswith(("shared.gate", "shared.up", "shared.down")):
            return torch.stack([self.get_expert(name, e, device) for e in range(self.cfg.n_routed_experts)])
        t = self._raw(_ds_hf_name(name))
        if name.endswith("moe.bias") or ".hc_" in name or name.startswith("hc_"):
            t = t.float()
        return t.to(device)


def deepseek_hf_config(cfg: DeepSeekConfig) -> dict:
    raw = {f.name: getattr(cfg, f.name) for f in dataclasses.fields(cfg)}
    raw["dspark_aux_layers"] = list(cfg.dspark_aux_layers)
    raw["model_type"] = "deepseek_mla_dsa_mhc"
    raw["_name_or_path"] = cfg.name
    return raw


def export_deepseek(cfg: DeepSeekConfig, src, out_dir: str | Path, with_dspark: bool = False) -> Path:
    """Write a DeepSeek-style checkpoint (names above) from any canonical weight source."""
    from safetensors.torch import save_file

    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    t = {hf: src.get(c, "cpu") for c, hf in _DS_GLOBAL.items()}
    for i in range(cfg.num_hidden_layers):
        for name in deepseek_weights.layer_names(cfg, i):
            leaf = name.split(".", 2)[-1]
            if leaf in _DS_EXPERT:
                for e in range(cfg.n_routed_experts):
                    t[f"model.layers.{i}.mlp.experts.{e}.{_DS_EXPERT[leaf]}.weight"] = src.get_expert(name, e, "cpu")
            else:
                t[_ds_hf_name(name)] = src.get(name, "cpu")
    if with_dspark:
        for leaf in ("dspark.fc", "dspark.final_norm", "dspark.markov_w1", "dspark.markov_w2"):
            t[leaf] = src.get(leaf, "cpu")
        for name in deepseek_weights.layer_names(cfg, 0):
            dn = "layers.dspark." + name.split(".", 2)[-1]
            if dn.split(".", 2)[-1].startswith(("moe.", "mlp.")):
                continue
            t[_ds_hf_name(dn)] = src.get(dn, "cpu")
    save_file({k: v.contiguous() for k, v in t.items()}, str(out / "model.safetensors"))
    (out / "config.json").write_text(json.dumps(deepseek_hf_config(cfg), indent=1))
    return out


__all__ = ["export_qwen35", "qwen35_hf_config", "export_deepseek", "deepseek_hf_config",
           "DeepSeekSafetensorsWeights"]
