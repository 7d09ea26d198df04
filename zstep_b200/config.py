"""Model configurations.

``Qwen35Config`` describes the Qwen3.5-MoE hybrid (GatedDeltaNet + gated GQA + MoE)
backbone; ``from_hf`` reads a HuggingFace ``config.json`` (``text_config`` nesting and
``rope_parameters`` handled as in the reference's config loader,
worker/zstep_worker/models/qwen35_moe.py:82-150), without the reference's fixed
TP=8 shape check -- any head counts divisible by the tensor-parallel degree work.
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field
from pathlib import Path


@dataclass(frozen=True)
class Qwen35Config:
    vocab_size: int = 248320
    hidden_size: int = 2048
    num_hidden_layers: int = 40
    layer_types: tuple[str, ...] = field(default_factory=tuple)
    rms_norm_eps: float = 1e-6
    num_attention_heads: int = 16
    num_key_value_heads: int = 2
    head_dim: int = 256
    rope_theta: float = 1.0e7
    partial_rotary_factor: float = 0.25
    linear_num_key_heads: int = 16
    linear_key_head_dim: int = 128
    linear_num_value_heads: int = 32
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    num_experts: int = 256
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 512
    shared_expert_intermediate_size: int = 512
    norm_topk_prob: bool = True
    initializer_range: float = 0.02
    # MTP draft head (one full-attention MoE layer) -- 0 disables.
    mtp_num_hidden_layers: int = 1
    name: str = "qwen3.5-35b-a3b"

    def __post_init__(self):
        if not self.layer_types:
            object.__setattr__(self, "layer_types", tuple(
                "full_attention" if (i + 1) % 4 == 0 else "linear_attention"
                for i in range(self.num_hidden_layers)))
        assert len(self.layer_types) == self.num_hidden_layers

    # ---------------------------------------------------------------- derived sizes
    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def gdn_layers(self) -> list[int]:
        return [i for i, t in enumerate(self.layer_types) if t == "linear_attention"]

    @property
    def attn_layers(self) -> list[int]:
        return [i for i, t in enumerate(self.layer_types) if t == "full_attention"]

    @property
    def conv_dim(self) -> int:
        return (2 * self.linear_num_key_heads * self.linear_key_head_dim
                + self.linear_num_value_heads * self.linear_value_head_dim)

    @property
    def gdn_proj_dim(self) -> int:
        """Width of the fused GDN input projection [q | k | v | z | b | a]."""
        return self.conv_dim + self.linear_num_value_heads * (self.linear_value_head_dim + 2)

    @property
    def attn_qkv_dim(self) -> int:
        """Width of the fused attention projection [per-head (q | gate) | k | v]."""
        return (2 * self.num_attention_heads + 2 * self.num_key_value_heads) * self.head_dim

    def params(self) -> int:
        h, e, i = self.hidden_size, self.num_experts, self.moe_intermediate_size
        per_moe = e * 3 * h * i + 3 * h * self.shared_expert_intermediate_size + h * (e + 1)
        gdn = h * self.gdn_proj_dim + self.linear_num_value_heads * self.linear_value_head_dim * h
        attn = h * self.attn_qkv_dim + self.num_attention_heads * self.head_dim * h
        n = len(self.gdn_layers) * (gdn + per_moe) + len(self.attn_layers) * (attn + per_moe)
        return n + 2 * self.vocab_size * h

    def to_dict(self) -> dict:
        d = asdict(self)
        d["layer_types"] = list(self.layer_types)
        return d

    # ---------------------------------------------------------------- constructors
    @classmethod
    def from_hf(cls, path: str | Path) -> "Qwen35Config":
        p = Path(path)
        raw = json.loads((p / "config.json" if p.is_dir() else p).read_text(encoding="utf-8"))
        tc = raw.get("text_config", raw)
        rope = tc.get("rope_parameters") or {}
        theta = rope.get("rope_theta", tc.get("rope_theta", 1.0e7))
        prf = rope.get("partial_rotary_factor", tc.get("partial_rotary_factor", 0.25))
        return cls(
            vocab_size=int(tc["vocab_size"]),
            hidden_size=int(tc["hidden_size"]),
            num_hidden_layers=int(tc["num_hidden_layers"]),
            layer_types=tuple(tc.get("layer_types") or ()),
            rms_norm_eps=float(tc.get("rms_norm_eps", 1e-6)),
            num_attention_heads=int(tc["num_attention_heads"]),
            num_key_value_heads=int(tc["num_key_value_heads"]),
            head_dim=int(tc.get("head_dim", 256)),
            rope_theta=float(theta),
            partial_rotary_factor=float(prf),
            linear_num_key_heads=int(tc["linear_num_key_heads"]),
            linear_key_head_dim=int(tc["linear_key_head_dim"]),
            linear_num_value_heads=int(tc["linear_num_value_heads"]),
            linear_value_head_dim=int(tc["linear_value_head_dim"]),
            linear_conv_kernel_dim=int(tc.get("linear_conv_kernel_dim", 4)),
            num_experts=int(tc["num_experts"]),
            num_experts_per_tok=int(tc["num_experts_per_tok"]),
            moe_intermediate_size=int(tc["moe_intermediate_size"]),
            shared_expert_intermediate_size=int(tc["shared_expert_intermediate_size"]),
            norm_topk_prob=bool(tc.get("norm_topk_prob", True)),
            mtp_num_hidden_layers=int(tc.get("mtp_num_hidden_layers", 0)),
            name=str(raw.get("_name_or_path", tc.get("model_type", "qwen3_5_moe"))),
        )


def qwen35_35b_a3b() -> Qwen35Config:
    """The Qwen3.5-35B-A3B shape (random-init benchmark config)."""
    return Qwen35Config()


def qwen35_tiny() -> Qwen35Config:
    """CPU plumbing model: 4 layers (3 GDN + 1 GQA), hidden 256, 8 experts top-2 + shared."""
    return Qwen35Config(
        vocab_size=4096, hidden_size=256, num_hidden_layers=4,
        layer_types=("linear_attention", "linear_attention", "linear_attention", "full_attention"),
        num_attention_heads=4, num_key_value_heads=2, head_dim=64,
        linear_num_key_heads=4, linear_key_head_dim=32, linear_num_value_heads=8,
        linear_value_head_dim=32, num_experts=8, num_experts_per_tok=2,
        moe_intermediate_size=128, shared_expert_intermediate_size=128,
        mtp_num_hidden_layers=1, name="qwen3.5-tiny")


def qwen35_small_gpu(num_layers: int = 4, vocab: int = 8192, experts: int = 32) -> Qwen35Config:
    """A reduced-depth config with the full per-layer shapes the sm_100a kernels serve
    (hidden 2048, GDN 128-dim heads, GQA 256-dim heads) for fast GPU tests."""
    types = tuple("full_attention" if (i + 1) % 4 == 0 else "linear_attention" for i in range(num_layers))
    return Qwen35Config(vocab_size=vocab, num_hidden_layers=num_layers, layer_types=types,
                        num_experts=experts, name=f"qwen3.5-small-{num_layers}l")


PRESETS = {
    "qwen3.5-35b-a3b": qwen35_35b_a3b,
    "qwen3.5-tiny": qwen35_tiny,
    "qwen3.5-small": qwen35_small_gpu,
}


@dataclass(frozen=True)
class DeepSeekConfig:
    """DeepSeek-style MoE with multi-head latent attention (MLA), the DSA lightning indexer
    (sparse attention over the top-k keys per query) and manifold-constrained hyper-
    connections (mHC: ``hc_mult`` residual streams mixed by per-token sigmoid pre/post
    weights and a Sinkhorn-normalised doubly-stochastic residual matrix).

    The reference serves this family through vLLM (worker/zstep_worker/models/
    deepseek_v41.py:408, DeepSeekV41StepRunner); the model math here is written from the
    architecture's definition: MLA with absorbed k/v up-projections, a ReLU-weighted
    multi-head index score, sigmoid grouped routing with a score-correction bias."""

    vocab_size: int = 129280
    hidden_size: int = 4096
    num_hidden_layers: int = 48
    first_k_dense_replace: int = 1
    intermediate_size: int = 12288          # dense FFN layers
    rms_norm_eps: float = 1e-6
    num_attention_heads: int = 64
    q_lora_rank: int = 1024
    kv_lora_rank: int = 512
    qk_nope_head_dim: int = 128
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    rope_theta: float = 10000.0
    index_n_heads: int = 64
    index_head_dim: int = 128
    index_topk: int = 2048
    n_routed_experts: int = 256
    num_experts_per_tok: int = 8
    n_group: int = 8
    topk_group: int = 4
    routed_scaling_factor: float = 2.5
    # Router scores: "sigmoid" (DeepSeek-V3) or "sqrtsoftplus" (sqrt(softplus(logit)));
    # either way the top-k runs on score + correction bias within the kept groups and the
    # weights are the unbiased scores, renormalised and scaled.
    scoring_func: str = "sigmoid"
    moe_intermediate_size: int = 2048
    n_shared_experts: int = 1
    hc_mult: int = 4
    hc_sinkhorn_iters: int = 20
    hc_eps: float = 1e-6
    expert_format: str = "mxfp4"            # routed and shared experts; everything else MXFP8
    initializer_range: float = 0.02
    name: str = "deepseek-mla-dsa-mhc"
    # DSpark draft head: target layers whose FFN-site inputs feed it (empty: 1, L/2, L-1),
    # the rank of its Markov (previous-token) logit correction, and the filler token of
    # the draft block's non-anchor rows (-1: vocab_size - 1).
    dspark_aux_layers: tuple = ()
    dspark_markov_rank: int = 256
    dspark_noise_token: int = -1

    def dspark_aux(self) -> tuple:
        if self.dspark_aux_layers:
            return tuple(self.dspark_aux_layers)
        L = self.num_hidden_layers
        return tuple(sorted({min(1, L - 1), L // 2, L - 1}))

    @property
    def qk_head_dim(self) -> int:
        return self.qk_nope_head_dim + self.qk_rope_head_dim

    @property
    def kv_cache_dim(self) -> int:
        """Latent cache row: normalised c_kv [kv_lora_rank] then roped k_pe [qk_rope_head_dim]."""
        return self.kv_lora_rank + self.qk_rope_head_dim

    @property
    def hc_mix_dim(self) -> int:
        """Per-token mixing logits of one mHC site: pre [n], post [n], residual [n*n]."""
        n = self.hc_mult
        return 2 * n + n * n

    def is_dense(self, layer: int) -> bool:
        return layer < self.first_k_dense_replace

    def params(self) -> int:
        h = self.hidden_size
        nh = self.num_attention_heads
        attn = (h * self.q_lora_rank + self.q_lora_rank * nh * self.qk_head_dim + h * self.kv_cache_dim
                + self.kv_lora_rank * nh * (self.qk_nope_head_dim + self.v_head_dim) + nh * self.v_head_dim * h
                + self.q_lora_rank * self.index_n_heads * self.index_head_dim + h * self.index_head_dim
                + h * self.index_n_heads)
        moe = (self.n_routed_experts + self.n_shared_experts) * 3 * h * self.moe_intermediate_size \
            + h * self.n_routed_experts
        dense = 3 * h * self.intermediate_size
        nd = self.first_k_dense_replace
        return self.num_hidden_layers * attn + nd * dense + (self.num_hidden_layers - nd) * moe \
            + 2 * self.vocab_size * h

    def to_dict(self) -> dict:
        return asdict(self)

    @staticmethod
    def is_hf_config(path: str | Path) -> bool:
        p = Path(path)
        f = p / "config.json" if p.is_dir() else p
        if not f.is_file():
            return False
        return "kv_lora_rank" in json.loads(f.read_text(encoding="utf-8"))

    @classmethod
    def from_hf(cls, path: str | Path) -> "DeepSeekConfig":
        """DeepSeek-V3-style ``config.json`` keys; mHC / index fields where present."""
        p = Path(path)
        raw = json.loads((p / "config.json" if p.is_dir() else p).read_text(encoding="utf-8"))
        known = {f for f in cls.__dataclass_fields__}
        kw = {k: v for k, v in raw.items() if k in known}
        if "dspark_aux_layers" in kw:
            kw["dspark_aux_layers"] = tuple(kw["dspark_aux_layers"])
        if "scoring_func" in kw:
            kw["scoring_func"] = str(kw["scoring_func"]).replace("_", "")
            if kw["scoring_func"] not in ("sigmoid", "sqrtsoftplus"):
                raise ValueError(f"unsupported router scoring_func {raw['scoring_func']!r}")
        kw["name"] = str(raw.get("_name_or_path", raw.get("model_type", "deepseek")))
        return cls(**kw)


def deepseek_full() -> DeepSeekConfig:
    """The DeepSeek-style benchmark shape (48 layers, MLA 64 heads, DSA top-2048, mHC x4,
    256 experts top-8 in MXFP4)."""
    return DeepSeekConfig()


def deepseek_tiny() -> DeepSeekConfig:
    """CPU-sized DeepSeek-style model for the reference and plumbing tests."""
    return DeepSeekConfig(vocab_size=512, hidden_size=128, num_hidden_layers=3, first_k_dense_replace=1,
                          intermediate_size=256, num_attention_heads=4, q_lora_rank=64, kv_lora_rank=64,
                          qk_nope_head_dim=32, qk_rope_head_dim=16, v_head_dim=32, index_n_heads=4,
                          index_head_dim=32, index_topk=8, n_routed_experts=16, num_experts_per_tok=4, n_group=4,
                          topk_group=2, moe_intermediate_size=64, name="deepseek-tiny")


def deepseek_small_gpu(num_layers: int = 3, vocab: int = 8192, experts: int = 32, topk: int = 64) -> DeepSeekConfig:
    """Reduced depth/width with the full per-head shapes the sm_100a kernels serve
    (kv_lora 512, rope 64, nope/v 128, index heads 128-dim) for fast GPU tests."""
    return DeepSeekConfig(vocab_size=vocab, hidden_size=1024, num_hidden_layers=num_layers, intermediate_size=2048,
                          num_attention_heads=16, q_lora_rank=512, index_n_heads=16, index_topk=topk,
                          n_routed_experts=experts, n_group=4, topk_group=2, moe_intermediate_size=512,
                          name=f"deepseek-small-{num_layers}l")


PRESETS.update({
    "deepseek-mla-dsa-mhc": deepseek_full,
    "deepseek-tiny": deepseek_tiny,
    "deepseek-small": deepseek_small_gpu,
})
