"""Weight source for the DeepSeek-style MLA + DSA + mHC MoE model: deterministic random
init over one canonical naming scheme (the GPU runner and the fp32 reference read the same
values through ``get(name, device)``).

Canonical names (per layer prefix ``layers.{i}.``):
  attn_norm, ffn_norm [H]                         plain RMSNorm scales (y = x * w)
  hc_attn.fn, hc_ffn.fn [2n + n*n, n*H] fp32      mHC mixing projections (n = hc_mult)
  hc_attn.base, hc_ffn.base [2n + n*n] fp32; hc_attn.scale, hc_ffn.scale [3] fp32
  mla.q_a [q_lora, H]; mla.q_a_norm [q_lora]; mla.q_b [heads*(nope+rope), q_lora]
  mla.kv_a [kv_lora+rope, H]; mla.kv_a_norm [kv_lora]; mla.kv_b [heads*(nope+v), kv_lora]
  mla.o_proj [H, heads*v]
  idx.wq [ih*id, q_lora]; idx.wk [id, H]; idx.k_norm [id]; idx.w [ih, H]
  dense layers: mlp.gate, mlp.up [F, H]; mlp.down [H, F]
  MoE layers: moe.router [E, H]; moe.bias [E] fp32; moe.gate, moe.up [E, I, H];
              moe.down [E, H, I]; moe.shared.gate, moe.shared.up [Is, H]; moe.shared.down [H, Is]
Globals: embed [V, H]; hc_head.fn [n, n*H], hc_head.base [n], hc_head.scale [1] (fp32);
final_norm [H]; lm_head [V, H].
DSpark draft head: dspark.fc [H, a*H] (a = number of auxiliary target layers);
layers.dspark.* (one dense MLA layer, names as above); dspark.final_norm [H];
dspark.markov_w1, dspark.markov_w2 [V, r] (r = dspark_markov_rank).

mHC initialisation: the mixing projections start small (scale 0.01) around a base that
gives pre = post-gate = sigmoid(0) and a residual matrix close to the identity (diagonal
logit 4), so the untrained network behaves like a plain residual stack.
"""

from __future__ import annotations

import zlib

import torch

from ..config import DeepSeekConfig


def shape_of(cfg: DeepSeekConfig, name: str) -> tuple[int, ...]:
    H, n = cfg.hidden_size, cfg.hc_mult
    nh, ql, kl = cfg.num_attention_heads, cfg.q_lora_rank, cfg.kv_lora_rank
    E, I = cfg.n_routed_experts, cfg.moe_intermediate_size
    Is = cfg.moe_intermediate_size * cfg.n_shared_experts
    leaf = name.split(".", 2)[-1] if name.startswith("layers.") else name
    table = {
        "attn_norm": (H,), "ffn_norm": (H,),
        "hc_attn.fn": (cfg.hc_mix_dim, n * H), "hc_ffn.fn": (cfg.hc_mix_dim, n * H),
        "hc_attn.base": (cfg.hc_mix_dim,), "hc_ffn.base": (cfg.hc_mix_dim,),
        "hc_attn.scale": (3,), "hc_ffn.scale": (3,),
        "mla.q_a": (ql, H), "mla.q_a_norm": (ql,), "mla.q_b": (nh * cfg.qk_head_dim, ql),
        "mla.kv_a": (kl + cfg.qk_rope_head_dim, H), "mla.kv_a_norm": (kl,),
        "mla.kv_b": (nh * (cfg.qk_nope_head_dim + cfg.v_head_dim), kl), "mla.o_proj": (H, nh * cfg.v_head_dim),
        "idx.wq": (cfg.index_n_heads * cfg.index_head_dim, ql), "idx.wk": (cfg.index_head_dim, H),
        "idx.k_norm": (cfg.index_head_dim,), "idx.w": (cfg.index_n_heads, H),
        "mlp.gate": (cfg.intermediate_size, H), "mlp.up": (cfg.intermediate_size, H),
        "mlp.down": (H, cfg.intermediate_size),
        "moe.router": (E, H), "moe.bias": (E,), "moe.gate": (E, I, H), "moe.up": (E, I, H), "moe.down": (E, H, I),
        "moe.shared.gate": (Is, H), "moe.shared.up": (Is, H), "moe.shared.down": (H, Is),
        "embed": (cfg.vocab_size, H), "final_norm": (H,), "lm_head": (cfg.vocab_size, H),
        "hc_head.fn": (n, n * H), "hc_head.base": (n,), "hc_head.scale": (1,),
        "dspark.fc": (H, len(cfg.dspark_aux()) * H), "dspark.final_norm": (H,),
        "dspark.markov_w1": (cfg.vocab_size, cfg.dspark_markov_rank),
        "dspark.markov_w2": (cfg.vocab_size, cfg.dspark_markov_rank),
    }
    return table[leaf]


def layer_names(cfg: DeepSeekConfig, i: int) -> list[str]:
    p = f"layers.{i}."
    names = ["attn_norm", "ffn_norm", "hc_attn.fn", "hc_attn.base", "hc_attn.scale", "hc_ffn.fn", "hc_ffn.base",
             "hc_ffn.scale", "mla.q_a", "mla.q_a_norm", "mla.q_b", "mla.kv_a", "mla.kv_a_norm", "mla.kv_b",
             "mla.o_proj", "idx.wq", "idx.wk", "idx.k_norm", "idx.w"]
    if cfg.is_dense(i):
        names += ["mlp.gate", "mlp.up", "mlp.down"]
    else:
        names += ["moe.router", "moe.bias", "moe.gate", "moe.up", "moe.down", "moe.shared.gate", "moe.shared.up",
                  "moe.shared.down"]
    return [p + n for n in names]


class DeepSeekRandomWeights:
    """Every tensor is seeded from (seed, crc32(name)), so any subset can be generated in
    any order.  ``get_expert(name, e, device)`` generates one expert's slice of a routed
    expert tensor without materialising all of them (the full model's experts are
    ~300 G parameters)."""

    def __init__(self, cfg: DeepSeekConfig, seed: int = 0, dtype: torch.dtype = torch.bfloat16):
        self.cfg = cfg
        self.seed = seed
        self.dtype = dtype

    def _gen(self, name: str, device) -> torch.Generator:
        g = torch.Generator(device=device)
        g.manual_seed((self.seed * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFF_FFFF_FFFF)
        return g

    def get_expert(self, name: str, e: int, device="cpu") -> torch.Tensor:
        shape = shape_of(self.cfg, name)[1:]
        g = self._gen(f"{name}#{e}", device)
        return (torch.randn(shape, device=device, generator=g) * self.cfg.initializer_range).to(self.dtype)

    def get(self, name: str, device="cpu") -> torch.Tensor:
        cfg = self.cfg
        if name.endswith(("moe.gate", "moe.up", "moe.down")):
            E = cfg.n_routed_experts
            return torch.stack([self.get_expert(name, e, device) for e in range(E)])
        shape = shape_of(cfg, name)
        g = self._gen(name, device)
        leaf = name.split(".", 2)[-1] if name.startswith("layers.") else name
        n = cfg.hc_mult
        if leaf.endswith(".fn"):
            return torch.randn(shape, device=device, generator=g) * cfg.initializer_range
        if leaf.endswith(".scale"):
            return torch.full(shape, 0.01, device=device)
        if leaf.endswith(".base"):
            b = torch.randn(shape, device=device, generator=g) * 0.1
            if leaf.startswith("hc_head"):
                return b
            res = b[2 * n:].view(n, n)
            res += 4.0 * torch.eye(n, device=device)
            return b
        if leaf == "moe.bias":
            return torch.randn(shape, device=device, generator=g) * 0.01
        if leaf.endswith("norm"):
            return (1.0 + torch.randn(shape, device=device, generator=g) * 0.02).to(self.dtype)
        if name == "embed":
            return torch.randn(shape, device=device, generator=g).to(self.dtype)
        return (torch.randn(shape, device=device, generator=g, dtype=torch.float32)
                * cfg.initializer_range).to(self.dtype)
