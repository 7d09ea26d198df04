"""Weight sources for the Qwen3.5 hybrid: deterministic random init or HF safetensors.

Both expose ``get(name, device) -> Tensor`` over one *canonical* naming scheme, so
the GPU runner (which packs each tensor to MXFP8 as it arrives and drops the
original) and the fp32 reference model read identical values.

Canonical names (per layer prefix ``layers.{i}.``):
  input_norm, post_norm                         [H]          zero-centered ((1 + w) scale)
  gdn.in_proj   [conv_dim + Hv*dv + 2*Hv, H]    rows = [q | k | v | z | b | a]
  gdn.conv_w    [conv_dim, 4]; gdn.a_log, gdn.dt_bias [Hv] (fp32); gdn.norm [dv] (plain scale)
  gdn.out_proj  [H, Hv*dv]
  attn.qkv      [(2*Hq + 2*Hkv)*D, H]           rows = [per q head (q | gate) | k heads | v heads]
  attn.q_norm, attn.k_norm [D]; attn.o_proj [H, Hq*D]
  moe.router [E, H]; moe.shared_gate [1, H]
  moe.gate, moe.up [E, I, H]; moe.down [E, H, I]
  moe.shared.gate, moe.shared.up [Is, H]; moe.shared.down [H, Is]
Globals: embed [V, H], final_norm [H], lm_head [V, H].
MTP head (prefix ``mtp.``): pre_fc_norm_embedding, pre_fc_norm_hidden [H], fc [H, 2H],
norm [H], and ``mtp.layer.*`` with the full-attention layer names above.

HF mapping follows the Qwen3.5 checkpoint names the reference loads
(worker/zstep_worker/models/qwen35_moe.py:852-1019): ``linear_attn.in_proj_qkv/z/b/a``,
``mlp.experts.gate_up_proj`` ([E, 2I, H], gate rows first), ``mlp.experts.down_proj``.
"""

from __future__ import annotations

import json
import math
import zlib
from pathlib import Path

import torch

from ..config import Qwen35Config


def layer_names(cfg: Qwen35Config, i: int, prefix: str | None = None) -> list[str]:
    p = prefix if prefix is not None else f"layers.{i}."
    names = [p + "input_norm", p + "post_norm"]
    if prefix is None and cfg.layer_types[i] == "linear_attention":
        names += [p + n for n in ("gdn.in_proj", "gdn.conv_w", "gdn.a_log", "gdn.dt_bias", "gdn.norm",
                                  "gdn.out_proj")]
    else:
        names += [p + n for n in ("attn.qkv", "attn.q_norm", "attn.k_norm", "attn.o_proj")]
    names += [p + n for n in ("moe.router", "moe.shared_gate", "moe.gate", "moe.up", "moe.down",
                              "moe.shared.gate", "moe.shared.up", "moe.shared.down")]
    return names


def shape_of(cfg: Qwen35Config, name: str) -> tuple[int, ...]:
    H, E, I, Is = cfg.hidden_size, cfg.num_experts, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
    Hv, dv = cfg.linear_num_value_heads, cfg.linear_value_head_dim
    Hq, D = cfg.num_attention_heads, cfg.head_dim
    leaf = name.split(".", 2)[-1] if name.startswith("layers.") else name
    if name.startswith("mtp.layer."):
        leaf = name[len("mtp.layer."):]
    table = {
        "input_norm": (H,), "post_norm": (H,),
        "gdn.in_proj": (cfg.gdn_proj_dim, H), "gdn.conv_w": (cfg.conv_dim, cfg.linear_conv_kernel_dim),
        "gdn.a_log": (Hv,), "gdn.dt_bias": (Hv,), "gdn.norm": (dv,), "gdn.out_proj": (H, Hv * dv),
        "attn.qkv": (cfg.attn_qkv_dim, H), "attn.q_norm": (D,), "attn.k_norm": (D,),
        "attn.o_proj": (H, Hq * D),
        "moe.router": (E, H), "moe.shared_gate": (1, H),
        "moe.gate": (E, I, H), "moe.up": (E, I, H), "moe.down": (E, H, I),
        "moe.shared.gate": (Is, H), "moe.shared.up": (Is, H), "moe.shared.down": (H, Is),
        "embed": (cfg.vocab_size, H), "final_norm": (H,), "lm_head": (cfg.vocab_size, H),
        "mtp.pre_fc_norm_embedding": (H,), "mtp.pre_fc_norm_hidden": (H,), "mtp.fc": (H, 2 * H),
        "mtp.norm": (H,),
    }
    return table[leaf]


class RandomWeights:
    """Deterministic random init: every tensor is seeded from (seed, crc32(name)), so
    any subset can be generated in any order on any device of the same type."""

    def __init__(self, cfg: Qwen35Config, seed: int = 0, dtype: torch.dtype = torch.bfloat16):
        self.cfg = cfg
        self.seed = seed
        self.dtype = dtype

    def _gen(self, name: str, device) -> torch.Generator:
        g = torch.Generator(device=device)
        g.manual_seed((self.seed * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFF_FFFF_FFFF)
        return g

    def get(self, name: str, device="cpu") -> torch.Tensor:
        shape = shape_of(self.cfg, name)
        g = self._gen(name, device)
        leaf = name.rsplit(".", 1)[-1]
        std = self.cfg.initializer_range
        if name.endswith("gdn.a_log"):
            return torch.log(torch.empty(shape, device=device).uniform_(1.0, 16.0, generator=g))
        if name.endswith("gdn.dt_bias"):
            u = torch.empty(shape, device=device).uniform_(0.0, 1.0, generator=g)
            dt = torch.exp(u * (math.log(0.1) - math.log(1e-3)) + math.log(1e-3)).clamp_min(1e-4)
            return dt + torch.log(-torch.expm1(-dt))
        if name.endswith("gdn.conv_w"):
            return torch.empty(shape, device=device).uniform_(-0.5, 0.5, generator=g).to(self.dtype)
        if name.endswith("gdn.norm"):
            return torch.ones(shape, device=device, dtype=self.dtype)
        if leaf.endswith("norm") or leaf in ("input_norm", "post_norm", "final_norm", "q_norm", "k_norm") \
                or "pre_fc_norm" in name:
            # Zero-centered norms: small perturbation around the identity scale.
            return (torch.randn(shape, device=device, generator=g) * 0.02).to(self.dtype)
        if name == "embed":
            return (torch.randn(shape, device=device, generator=g) * 1.0).to(self.dtype)
        return (torch.randn(shape, device=device, generator=g, dtype=torch.float32) * std).to(self.dtype)


class SafetensorsWeights:
    """HF Qwen3.5 checkpoint reader (``model.safetensors.index.json`` or single file)."""

    def __init__(self, cfg: Qwen35Config, model_dir: str | Path):
        from safetensors import safe_open  # noqa: F401  (import check)

        self.cfg = cfg
        self.dir = Path(model_dir)
        idx = self.dir / "model.safetensors.index.json"
        if idx.exists():
            self.map = json.loads(idx.read_text())["weight_map"]
        else:
            from safetensors import safe_open as so

            f = self.dir / "model.safetensors"
            with so(str(f), "pt") as h:
                self.map = {k: "model.safetensors" for k in h.keys()}
        self.prefix = "model.language_model." if "model.language_model.norm.weight" in self.map else "model."
        self._handles: dict[str, object] = {}

    def _raw(self, key: str) -> torch.Tensor:
        from safetensors import safe_open

        fn = self.map[key]
        if fn not in self._handles:
            self._handles[fn] = safe_open(str(self.dir / fn), "pt")
        return self._handles[fn].get_tensor(key)

    def get(self, name: str, device="cpu") -> torch.Tensor:
        p = self.prefix
        if name == "embed":
            t = self._raw(p + "embed_tokens.weight")
        elif name == "final_norm":
            t = self._raw(p + "norm.weight")
        elif name == "lm_head":
            t = self._raw("lm_head.weight")
        elif name.startswith("mtp."):
            t = self._mtp(name)
        else:
            _, i, leaf = name.split(".", 2)
            t = self._layer(f"{p}layers.{i}.", leaf)
        return t.to(device)

    def _mtp(self, name: str) -> torch.Tensor:
        leaf = name[len("mtp."):]
        simple = {"pre_fc_norm_embedding": "mtp.pre_fc_norm_embedding.weight",
                  "pre_fc_norm_hidden": "mtp.pre_fc_norm_hidden.weight", "fc": "mtp.fc.weight",
                  "norm": "mtp.norm.weight"}
        if leaf in simple:
            return self._raw(simple[leaf])
        return self._layer("mtp.layers.0.", leaf[len("layer."):])

    def _layer(self, lp: str, leaf: str) -> torch.Tensor:
        r = self._raw
        if leaf == "input_norm":
            return r(lp + "input_layernorm.weight")
        if leaf == "post_norm":
            return r(lp + "post_attention_layernorm.weight")
        if leaf == "gdn.in_proj":
            return torch.cat([r(lp + "linear_attn.in_proj_qkv.weight"), r(lp + "linear_attn.in_proj_z.weight"),
                              r(lp + "linear_attn.in_proj_b.weight"), r(lp + "linear_attn.in_proj_a.weight")], 0)
        if leaf == "gdn.conv_w":
            return r(lp + "linear_attn.conv1d.weight").reshape(self.cfg.conv_dim, -1)
        if leaf == "gdn.a_log":
            return r(lp + "linear_attn.A_log").float()
        if leaf == "gdn.dt_bias":
            return r(lp + "linear_attn.dt_bias").float()
        if leaf == "gdn.norm":
            return r(lp + "linear_attn.norm.weight")
        if leaf == "gdn.out_proj":
            return r(lp + "linear_attn.out_proj.weight")
        if leaf == "attn.qkv":
            return torch.cat([r(lp + "self_attn.q_proj.weight"), r(lp + "self_attn.k_proj.weight"),
                              r(lp + "self_attn.v_proj.weight")], 0)
        if leaf in ("attn.q_norm", "attn.k_norm", "attn.o_proj"):
            return r(lp + "self_attn." + leaf.split(".")[1] + ".weight")
        if leaf == "moe.router":
            return r(lp + "mlp.gate.weight")
        if leaf == "moe.shared_gate":
            return r(lp + "mlp.shared_expert_gate.weight")
        I = self.cfg.moe_intermediate_size
        if leaf == "moe.gate":
            return r(lp + "mlp.experts.gate_up_proj")[:, :I]
        if leaf == "moe.up":
            return r(lp + "mlp.experts.gate_up_proj")[:, I:]
        if leaf == "moe.down":
            return r(lp + "mlp.experts.down_proj")
        if leaf.startswith("moe.shared."):
            return r(lp + "mlp.shared_expert." + leaf.split(".")[2] + "_proj.weight")
        raise KeyError(leaf)
