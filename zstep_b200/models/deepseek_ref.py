"""fp32 PyTorch reference of the DeepSeek-style MLA + DSA + mHC MoE model (token at a
time, explicit per-sequence state).

It is the oracle of the GPU runner's tests.  With ``quant=True`` it applies the GPU
kernels' quantization points: dense weights MXFP8, routed experts MXFP4 (both
dequantized), every GEMM input activation fake-quantized to MXFP8, and bf16 rounding
wherever the kernels store bf16.  ``tp_rank``/``tp_size`` shard attention heads, the
dense FFN and the vocabulary, and place experts by expert parallelism (expert e on rank
e // (E / tp)); ``allreduce`` sums a rank's partial sublayer output.

Per layer (n = hc_mult residual streams X [n, H], fp32):
  for each sublayer (attention, then FFN):
    m       = (fn @ vec(X)) * rsqrt(mean(vec(X)^2) + eps)          [2n + n^2]
    pre     = sigmoid(scale0 * m[:n] + base[:n])
    post    = 2 * sigmoid(scale1 * m[n:2n] + base[n:2n])
    res     = sinkhorn(scale2 * m[2n:] + base[2n:])  (row softmax, then `iters` rounds of
              column- and row-normalisation)
    y       = sublayer(rmsnorm(pre @ X))
    X       = res @ X + post[:, None] * y
  final: h = sigmoid(scale * (fn_head @ vec(X)) * rsqrt(...) + base_head) @ X, then
  final RMSNorm and lm_head.

MLA (absorbed): c_kv = rmsnorm(kv_a[:kv_lora]), k_pe = rope(kv_a[kv_lora:]) are cached;
q_lat[h] = W_UK[h]^T q_nope[h]; score = (q_lat . c_kv + q_pe . k_pe) / sqrt(nope + rope);
o[h] = W_UV[h] (softmax(score) @ c_kv).  RoPE rotates halves (dims i and i + rope/2).
DSA indexer: iq = wq @ rmsnorm(q_a); ik = rope(rmsnorm(wk @ x)) cached;
I[s] = sum_h w_h relu(iq_h . ik_s) / sqrt(index_dim) with w = (W_w @ x) / sqrt(index_heads);
attention reads the top-k positions by I (ties: lower position first), or every
position while the context is at most k.

DSpark draft head (``load_dspark``): a context entry per target row at its position,
c = MLA projections of rmsnorm(fc @ [FFN inputs of the auxiliary layers]) into the draft
layer's own caches; a draft block of k rows [newest token, filler...] through that layer
(every row attends to the contexts and the whole block), plain residual, final norm;
draft i = argmax(lm_head . h_i + w2 . w1[previous token])
(worker/zstep_worker/models/deepseek_v41_dspark.py:123,233,387,471).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from ..config import DeepSeekConfig
from ..ops import mx
from ..ops import reference as R


@dataclass
class DsState:
    ckv: list = field(default_factory=list)   # per layer [T, kv_lora + rope] (c_kv | k_pe)
    ik: list = field(default_factory=list)    # per layer [T, index_dim]
    pos: int = 0
    dckv: torch.Tensor | None = None          # DSpark draft layer's own caches, indexed by
    dik: torch.Tensor | None = None           # position (rows never written read as zeros)


def sinkhorn(logits: torch.Tensor, iters: int) -> torch.Tensor:
    p = torch.softmax(logits, dim=-1)
    for _ in range(iters):
        p = p / p.sum(dim=0, keepdim=True)
        p = p / p.sum(dim=1, keepdim=True)
    return p


def rope_halves(x: torch.Tensor, pos: int, theta: float) -> torch.Tensor:
    d = x.shape[-1]
    cos, sin = R.rope_cos_sin(pos, d, theta)
    cos, sin = cos.to(x.device), sin.to(x.device)
    lo, hi = x[..., : d // 2], x[..., d // 2:]
    return torch.cat([lo * cos - hi * sin, hi * cos + lo * sin], dim=-1)


class DeepSeekReference:
    def __init__(self, cfg: DeepSeekConfig, src, *, device="cpu", quant: bool = False, tp_rank: int = 0,
                 tp_size: int = 1, allreduce=None):
        self.cfg = c = cfg
        self.dev = torch.device(device)
        self.quant = quant
        self.r, self.tp = tp_rank, tp_size
        self.allreduce = allreduce
        self.hl = c.num_attention_heads // tp_size
        self.e_local = c.n_routed_experts // tp_size
        g = lambda n: src.get(n, self.dev).float()  # noqa: E731
        self.embed = g("embed")
        V = c.vocab_size // tp_size
        self.lm_head = self._w(g("lm_head")[tp_rank * V:(tp_rank + 1) * V])
        self.final_norm = g("final_norm")
        self.hc_head = (g("hc_head.fn"), g("hc_head.base"), g("hc_head.scale"))
        self.layers = []
        for i in range(c.num_hidden_layers):
            p = f"layers.{i}."
            L = {"attn_norm": g(p + "attn_norm"), "ffn_norm": g(p + "ffn_norm"),
                 "hc_attn": (g(p + "hc_attn.fn"), g(p + "hc_attn.base"), g(p + "hc_attn.scale")),
                 "hc_ffn": (g(p + "hc_ffn.fn"), g(p + "hc_ffn.base"), g(p + "hc_ffn.scale"))}
            L.update(self._mla(g, p))
            if c.is_dense(i):
                F_ = c.intermediate_size // tp_size
                sl = slice(tp_rank * F_, (tp_rank + 1) * F_)
                L.update(dense=True, gate=self._w(g(p + "mlp.gate")[sl]), up=self._w(g(p + "mlp.up")[sl]),
                         down=self._w(g(p + "mlp.down")[:, sl]))
            else:
                L.update(self._moe(src, g, p))
            self.layers.append(L)

    # ------------------------------------------------------------------ weights
    def _w(self, w: torch.Tensor) -> torch.Tensor:
        return mx.fake_quant(w.reshape(-1, w.shape[-1])).reshape(w.shape) if self.quant else w

    def _w4(self, w: torch.Tensor) -> torch.Tensor:
        if not self.quant:
            return w
        if self.cfg.expert_format == "mxfp4":
            return mx.fake_quant_fp4(w.reshape(-1, w.shape[-1])).reshape(w.shape)
        return self._w(w)

    def _mla(self, g, p):
        c, hl, r = self.cfg, self.hl, self.r
        qk, nope, vd, kl = c.qk_head_dim, c.qk_nope_head_dim, c.v_head_dim, c.kv_lora_rank
        q_b = g(p + "mla.q_b")[r * hl * qk:(r + 1) * hl * qk]
        kv_b = g(p + "mla.kv_b").reshape(c.num_attention_heads, nope + vd, kl)[r * hl:(r + 1) * hl]
        bf = R.bfr if self.quant else (lambda t: t)
        return {"q_a": self._w(g(p + "mla.q_a")), "q_a_norm": g(p + "mla.q_a_norm"), "q_b": self._w(q_b),
                "kv_a": self._w(g(p + "mla.kv_a")), "kv_a_norm": g(p + "mla.kv_a_norm"),
                # The absorbed up-projections run on bf16 weights (no MXFP8 round trip).
                "w_uk": bf(kv_b[:, :nope]), "w_uv": bf(kv_b[:, nope:]),
                "o_proj": self._w(g(p + "mla.o_proj")[:, r * hl * vd:(r + 1) * hl * vd]),
                "idx_wq": self._w(g(p + "idx.wq")), "idx_wk": self._w(g(p + "idx.wk")),
                "idx_k_norm": g(p + "idx.k_norm"), "idx_w": self._w(g(p + "idx.w"))}

    def _moe(self, src, g, p):
        c, r = self.cfg, self.r
        eb = r * self.e_local
        experts = []
        for e in range(eb, eb + self.e_local):
            experts.append(tuple(self._w4(src.get_expert(p + "moe." + n, e, self.dev).float())
                                 for n in ("gate", "up", "down")))
        # The shared expert is one more MXFP4 expert that every rank computes in full; its
        # down-projection rows are masked to this rank's output slice so the sum over ranks
        # counts it once.
        sd = self._w4(g(p + "moe.shared.down"))
        if self.tp > 1:
            H = c.hidden_size
            mask = torch.zeros(H, 1, device=sd.device)
            mask[r * H // self.tp:(r + 1) * H // self.tp] = 1
            sd = sd * mask
        return {"dense": False, "router": self._w(g(p + "moe.router")), "bias": g(p + "moe.bias"),
                "experts": experts, "sgate": self._w4(g(p + "moe.shared.gate")),
                "sup": self._w4(g(p + "moe.shared.up")), "sdown": sd}

    # ------------------------------------------------------------------ helpers
    def new_state(self) -> DsState:
        c = self.cfg
        s = DsState()
        for _ in range(c.num_hidden_layers):
            s.ckv.append(torch.zeros(0, c.kv_cache_dim, device=self.dev))
            s.ik.append(torch.zeros(0, c.index_head_dim, device=self.dev))
        return s

    def clone_state(self, s: DsState) -> DsState:
        cl = lambda t: None if t is None else t.clone()  # noqa: E731
        return DsState(ckv=[t.clone() for t in s.ckv], ik=[t.clone() for t in s.ik], pos=s.pos, dckv=cl(s.dckv),
                       dik=cl(s.dik))

    def _q(self, x: torch.Tensor) -> torch.Tensor:
        if not self.quant:
            return x
        k = x.shape[-1]
        return mx.fake_quant(x.reshape(-1, k)).reshape(x.shape) if k % 32 == 0 else x

    def _bf(self, x):
        return R.bfr(x) if self.quant else x

    def _reduce(self, x):
        return self.allreduce(x) if self.tp > 1 else x

    def _mix(self, X, hc):
        c = self.cfg
        n = c.hc_mult
        fn, base, scale = hc
        xf = X.reshape(-1)
        rs = torch.rsqrt(xf.pow(2).mean() + c.rms_norm_eps)
        m = (fn @ xf) * rs
        pre = torch.sigmoid(scale[0] * m[:n] + base[:n])
        post = 2.0 * torch.sigmoid(scale[1] * m[n:2 * n] + base[n:2 * n])
        res = sinkhorn((scale[2] * m[2 * n:] + base[2 * n:]).view(n, n), c.hc_sinkhorn_iters)
        return pre, post, res

    # ------------------------------------------------------------------ forward
    def step(self, s: DsState, token: int) -> torch.Tensor:
        """Advance one token; returns this rank's logits shard [V/tp] (fp32)."""
        c = self.cfg
        eps = c.rms_norm_eps
        n = c.hc_mult
        X = self._bf(self.embed[token]).unsqueeze(0).repeat(n, 1)
        aux_layers = c.dspark_aux()
        self.last_aux = []  # FFN-site inputs of the DSpark auxiliary layers (its context source)
        for li, L in enumerate(self.layers):
            for site in ("attn", "ffn"):
                pre, post, res = self._mix(X, L["hc_" + site])
                h = pre @ X
                xq = self._q(R.rmsnorm(h, L[site + "_norm"], eps, 0.0))
                if site == "attn":
                    y = self._attention(s, li, L, xq)
                else:
                    if li in aux_layers:
                        self.last_aux.append(xq)
                    y = self._ffn(L, xq)
                y = self._bf(self._reduce(y))
                X = res @ X + post[:, None] * y
        fn, base, scale = self.hc_head
        xf = X.reshape(-1)
        rs = torch.rsqrt(xf.pow(2).mean() + eps)
        h = torch.sigmoid(scale[0] * (fn @ xf) * rs + base) @ X
        s.pos += 1
        self.last_normed = self._q(R.rmsnorm(h, self.final_norm, eps, 0.0))  # lm_head input (for tests)
        return self.lm_head @ self.last_normed

    def _attention(self, s: DsState, li: int, L, xq):
        q, entry, ik = self._mla_project(L, xq, s.pos)
        s.ckv[li] = torch.cat([s.ckv[li], entry[None]])
        s.ik[li] = torch.cat([s.ik[li], ik[None]])
        return self._mla_attend(L, q, s.ckv[li], s.ik[li])

    def _mla_project(self, L, xq, pos: int):
        """Query side (q_lat, q_pe, index query, index weights) and the cache entries
        (c_kv | k_pe, index key) of one row at `pos`."""
        c = self.cfg
        eps, hl = c.rms_norm_eps, self.hl
        nope, rope, kl = c.qk_nope_head_dim, c.qk_rope_head_dim, c.kv_lora_rank
        bf = self._bf
        qa = bf(L["q_a"] @ xq)
        kva = bf(L["kv_a"] @ xq)
        ik_raw = bf(L["idx_wk"] @ xq)
        iw = bf(L["idx_w"] @ xq) * (c.index_n_heads ** -0.5)
        qa_n = self._q(R.rmsnorm(qa, L["q_a_norm"], eps, 0.0))
        q = bf(L["q_b"] @ qa_n).view(hl, c.qk_head_dim)
        iq = bf(L["idx_wq"] @ qa_n).view(c.index_n_heads, c.index_head_dim)
        ckv = bf(R.rmsnorm(kva[:kl], L["kv_a_norm"], eps, 0.0))
        kpe = bf(rope_halves(kva[kl:], pos, c.rope_theta))
        ik = bf(R.rmsnorm(ik_raw, L["idx_k_norm"], eps, 0.0))
        ik = bf(torch.cat([ik[:c.index_head_dim - rope], rope_halves(ik[c.index_head_dim - rope:], pos, c.rope_theta)]))
        iq = bf(torch.cat([iq[:, :c.index_head_dim - rope],
                           rope_halves(iq[:, c.index_head_dim - rope:], pos, c.rope_theta)], dim=1))
        q_pe = bf(rope_halves(q[:, nope:], pos, c.rope_theta))
        q_lat = bf(torch.einsum("hd,hdc->hc", q[:, :nope], L["w_uk"]))
        return (q_lat, q_pe, iq, iw), torch.cat([ckv, kpe]), ik

    def _mla_attend(self, L, q, keys: torch.Tensor, ikeys: torch.Tensor):
        """Absorbed MLA over the cached rows `keys` [T, kv_lora + rope]: the top-k rows by
        the indexer score when T exceeds index_topk (ties: lower position first), else all."""
        c = self.cfg
        kl = c.kv_lora_rank
        q_lat, q_pe, iq, iw = q
        T = keys.shape[0]
        if T > c.index_topk:
            score = (torch.relu(ikeys @ iq.T) * (c.index_head_dim ** -0.5)) @ iw   # [T]
            sel = torch.sort(score, descending=True, stable=True).indices[:c.index_topk]
        else:
            sel = torch.arange(T, device=self.dev)
        kv = keys[sel]
        scores = (q_lat @ kv[:, :kl].T + q_pe @ kv[:, kl:].T) * (c.qk_head_dim ** -0.5)
        p = torch.softmax(scores, dim=-1)
        o_lat = self._bf(p @ kv[:, :kl])
        o = self._bf(torch.einsum("hc,hvc->hv", o_lat, L["w_uv"])).reshape(-1)
        return L["o_proj"] @ self._q(o)

    # ------------------------------------------------------------------ DSpark draft head
    def load_dspark(self, src) -> None:
        """The draft head: fc over the auxiliary layers' FFN inputs, one dense MLA layer with
        its own caches, a final norm, and the low-rank Markov correction [V, r] x 2 (vocab
        rows of w2 sharded like lm_head)."""
        c, r = self.cfg, self.r
        g = lambda n: src.get(n, self.dev).float()  # noqa: E731
        p = "layers.dspark."
        L = {"attn_norm": g(p + "attn_norm"), "ffn_norm": g(p + "ffn_norm"), "dense": True}
        L.update(self._mla(g, p))
        F_ = c.intermediate_size // self.tp
        sl = slice(r * F_, (r + 1) * F_)
        L.update(gate=self._w(g(p + "mlp.gate")[sl]), up=self._w(g(p + "mlp.up")[sl]),
                 down=self._w(g(p + "mlp.down")[:, sl]))
        V = c.vocab_size // self.tp
        self.dspark = {"layer": L, "fc": self._w(g("dspark.fc")), "final_norm": g("dspark.final_norm"),
                       "w1": self._bf(g("dspark.markov_w1")), "w2": self._w(g("dspark.markov_w2")[r * V:(r + 1) * V])}

    def _put(self, cache: torch.Tensor | None, pos: int, row: torch.Tensor) -> torch.Tensor:
        if cache is None:
            cache = torch.zeros(0, row.shape[0], device=self.dev)
        if cache.shape[0] <= pos:
            cache = torch.cat([cache, torch.zeros(pos + 1 - cache.shape[0], row.shape[0], device=self.dev)])
        cache[pos] = row
        return cache

    def dspark_context(self, s: DsState, aux: list, pos: int) -> None:
        """Context entry at `pos` from the auxiliary FFN inputs of the target row there
        (``last_aux`` after its step): fc, the draft layer's attention norm, its MLA
        projections into the draft caches."""
        D, eps = self.dspark, self.cfg.rms_norm_eps
        L = D["layer"]
        h = self._bf(D["fc"] @ torch.cat(aux))
        _, entry, ik = self._mla_project(L, self._q(R.rmsnorm(h, L["attn_norm"], eps, 0.0)), pos)
        s.dckv, s.dik = self._put(s.dckv, pos, entry), self._put(s.dik, pos, ik)

    def dspark_draft(self, s: DsState, anchor: int, pos: int, k: int, full_logits=lambda x: x) -> list[int]:
        """`k` greedy drafts after `anchor` (the newest token, at `pos`): a block of rows
        [anchor, noise * (k-1)] at pos..pos+k-1 through the draft layer, every row attending
        to the contexts and the whole block; draft i is the argmax of
        lm_head . h_i + w2 . w1[previous token].  `full_logits` gathers vocab shards."""
        c, D = self.cfg, self.dspark
        L, eps = D["layer"], c.rms_norm_eps
        noise = c.vocab_size - 1 if c.dspark_noise_token < 0 else c.dspark_noise_token
        hs, qs = [], []
        for i, t in enumerate([anchor] + [noise] * (k - 1)):
            h = self._bf(self.embed[t])
            q, entry, ik = self._mla_project(L, self._q(R.rmsnorm(h, L["attn_norm"], eps, 0.0)), pos + i)
            s.dckv, s.dik = self._put(s.dckv, pos + i, entry), self._put(s.dik, pos + i, ik)
            hs.append(h)
            qs.append(q)
        keys, ikeys = s.dckv[:pos + k], s.dik[:pos + k]
        drafts, prev = [], anchor
        for i in range(k):
            h = self._bf(hs[i] + self._reduce(self._mla_attend(L, qs[i], keys, ikeys)))
            h = self._bf(h + self._reduce(self._ffn(L, self._q(R.rmsnorm(h, L["ffn_norm"], eps, 0.0)))))
            xf = self._q(R.rmsnorm(h, D["final_norm"], eps, 0.0))
            lg = self.lm_head @ xf + D["w2"] @ self._q(D["w1"][prev])
            prev = int(torch.argmax(full_logits(lg)))
            drafts.append(prev)
        return drafts

    def _ffn(self, L, xq):
        c = self.cfg
        if L["dense"]:
            h = F.silu(L["gate"] @ xq) * (L["up"] @ xq)
            return L["down"] @ self._q(h)
        logits = L["router"] @ xq
        ids, w = R.route(logits[None], top_k=c.num_experts_per_tok, scoring=c.scoring_func, bias=L["bias"],
                         n_group=c.n_group, topk_group=c.topk_group, routed_scale=c.routed_scaling_factor)
        out = torch.zeros(c.hidden_size, device=xq.device)
        eb = self.r * self.e_local
        for e, wt in zip(ids[0].tolist(), w[0].tolist()):
            if eb <= e < eb + self.e_local:
                wg, wu, wd = L["experts"][e - eb]
                h = F.silu(wg @ xq) * (wu @ xq)
                # Expert rows are stored bf16, then weighted in fp32 by the combine.
                out = out + self._bf(wd @ self._q(h)) * wt
        h = F.silu(L["sgate"] @ xq) * (L["sup"] @ xq)
        return out + self._bf(L["sdown"] @ self._q(h))
