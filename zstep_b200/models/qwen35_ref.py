"""fp32 PyTorch reference of the Qwen3.5 hybrid model (token-at-a-time, explicit state).

Used three ways:
  * the oracle of the GPU model tests (same weights; with ``quant=True`` it applies the
    same MXFP8 quantization points as the sm_100a kernels: weights dequantized from
    MXFP8, every GEMM input activation fake-quantized, bf16 rounding where the kernels
    store bf16);
  * the CPU plumbing model of the control-plane tests (``quant=False``, any head sizes);
  * a tensor-parallel shard (``tp_rank``/``tp_size`` with an ``allreduce`` callback) so
    CPU worker ranks can run the sharded math over the master's transport.

Math follows the reference runner's decode forward
(worker/zstep_worker/models/qwen35_moe.py:1021-1168) and ops (kernels_sm120/qwen35_ops.py).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from ..config import Qwen35Config
from ..ops import mx
from ..ops import reference as R


@dataclass
class SeqState:
    gdn: list = field(default_factory=list)    # per GDN layer: (window [conv_dim,3], state [Hv,dv,dk])
    keys: list = field(default_factory=list)   # per attn layer: [T, Hkv, D]
    values: list = field(default_factory=list)
    pos: int = 0
    hidden = None                              # residual stream after the last layer (pre final norm)
    mtp_keys = None                            # MTP layer KV, indexed by position: [T, Hkv, D]
    mtp_values = None


class Qwen35Reference:
    def __init__(self, cfg: Qwen35Config, src, *, device="cpu", quant: bool = False, tp_rank: int = 0,
                 tp_size: int = 1, allreduce=None):
        self.cfg = cfg
        self.dev = torch.device(device)
        self.quant = quant
        self.r, self.tp = tp_rank, tp_size
        self.allreduce = allreduce
        c = cfg
        self.hk, self.hv = c.linear_num_key_heads // tp_size, c.linear_num_value_heads // tp_size
        self.dk, self.dv = c.linear_key_head_dim, c.linear_value_head_dim
        self.hq = c.num_attention_heads // tp_size
        self.hkv = max(1, c.num_key_value_heads // tp_size)
        self.D = c.head_dim
        self.E = c.num_experts
        self.e_local = self.E // tp_size
        g = lambda n: src.get(n, self.dev).float()  # noqa: E731
        self.embed = g("embed")
        self.final_norm = g("final_norm")
        V = c.vocab_size // tp_size
        self.vocab_local = V
        self.lm_head = self._w(g("lm_head")[tp_rank * V:(tp_rank + 1) * V])
        self.layers = []
        for i in range(c.num_hidden_layers):
            p = f"layers.{i}."
            L = {"type": c.layer_types[i], "input_norm": g(p + "input_norm"), "post_norm": g(p + "post_norm")}
            if L["type"] == "linear_attention":
                hk, hv, dk, dv = c.linear_num_key_heads, c.linear_num_value_heads, self.dk, self.dv
                w = self._shard(g(p + "gdn.in_proj"), [hk * dk, hk * dk, hv * dv, hv * dv, hv, hv])
                L["in_proj"] = self._w(w)
                L["conv_w"] = self._shard(g(p + "gdn.conv_w"), [hk * dk, hk * dk, hv * dv])
                L["a_log"] = g(p + "gdn.a_log")[tp_rank * self.hv:(tp_rank + 1) * self.hv]
                L["dt_bias"] = g(p + "gdn.dt_bias")[tp_rank * self.hv:(tp_rank + 1) * self.hv]
                L["gnorm"] = g(p + "gdn.norm")
                L["out_proj"] = self._w(g(p + "gdn.out_proj")[:, tp_rank * self.hv * dv:(tp_rank + 1) * self.hv * dv])
            else:
                L.update(self._attn(g, p))
            L.update(self._moe(g, p))
            self.layers.append(L)
        self.mtp = None
        if c.mtp_num_hidden_layers > 0:
            try:
                p = "mtp.layer."
                M = {"fc": self._w(g("mtp.fc")), "norm_e": g("mtp.pre_fc_norm_embedding"),
                     "norm_h": g("mtp.pre_fc_norm_hidden"), "norm": g("mtp.norm"),
                     "input_norm": g(p + "input_norm"), "post_norm": g(p + "post_norm")}
                M.update(self._attn(g, p))
                M.update(self._moe(g, p))
                self.mtp = M
            except KeyError:
                self.mtp = None

    # ------------------------------------------------------------------ weights
    def _w(self, w: torch.Tensor) -> torch.Tensor:
        return mx.fake_quant(w.reshape(-1, w.shape[-1])).reshape(w.shape) if self.quant else w

    def _shard(self, t, parts):
        out, o = [], 0
        for p in parts:
            n = p // self.tp
            out.append(t[o:o + p][self.r * n:(self.r + 1) * n])
            o += p
        return torch.cat(out, 0)

    def _attn(self, g, p):
        c, r = self.cfg, self.r
        Hq, Hkv, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        w = g(p + "attn.qkv")
        q = w[:Hq * 2 * D][r * self.hq * 2 * D:(r + 1) * self.hq * 2 * D]
        kvh = (r * Hkv) // self.tp if self.tp > Hkv else r * self.hkv
        k = w[Hq * 2 * D:Hq * 2 * D + Hkv * D][kvh * D:(kvh + self.hkv) * D]
        v = w[Hq * 2 * D + Hkv * D:][kvh * D:(kvh + self.hkv) * D]
        return {"qkv": self._w(torch.cat([q, k, v], 0)), "q_norm": g(p + "attn.q_norm"),
                "k_norm": g(p + "attn.k_norm"),
                "o_proj": self._w(g(p + "attn.o_proj")[:, r * self.hq * D:(r + 1) * self.hq * D])}

    def _moe(self, g, p):
        eb, ee = self.r * self.e_local, (self.r + 1) * self.e_local
        H = self.cfg.hidden_size
        sd = g(p + "moe.shared.down")
        if self.tp > 1:
            n = H // self.tp
            mask = torch.zeros(H, 1, device=sd.device)
            mask[self.r * n:(self.r + 1) * n] = 1
            sd = sd * mask
        return {"router": self._w(torch.cat([g(p + "moe.router"), g(p + "moe.shared_gate")], 0)),
                "gate": self._w(g(p + "moe.gate")[eb:ee]), "up": self._w(g(p + "moe.up")[eb:ee]),
                "down": self._w(g(p + "moe.down")[eb:ee]),
                "sgate": self._w(g(p + "moe.shared.gate")), "sup": self._w(g(p + "moe.shared.up")),
                "sdown": self._w(sd)}

    # ------------------------------------------------------------------ state
    def new_state(self) -> SeqState:
        s = SeqState()
        conv_dim = 2 * self.hk * self.dk + self.hv * self.dv
        for t in self.cfg.layer_types:
            if t == "linear_attention":
                s.gdn.append((torch.zeros(conv_dim, 3, device=self.dev),
                              torch.zeros(self.hv, self.dv, self.dk, device=self.dev)))
            else:
                s.keys.append(torch.zeros(0, self.hkv, self.D, device=self.dev))
                s.values.append(torch.zeros(0, self.hkv, self.D, device=self.dev))
        return s

    def clone_state(self, s: SeqState) -> SeqState:
        n = SeqState(gdn=[(a.clone(), b.clone()) for a, b in s.gdn], keys=[k.clone() for k in s.keys],
                     values=[v.clone() for v in s.values], pos=s.pos)
        n.hidden = None if s.hidden is None else s.hidden.clone()
        n.mtp_keys = None if s.mtp_keys is None else s.mtp_keys.clone()
        n.mtp_values = None if s.mtp_values is None else s.mtp_values.clone()
        return n

    # ------------------------------------------------------------------ forward
    def _q(self, x: torch.Tensor) -> torch.Tensor:
        """Activation entering a GEMM (MXFP8 round trip when quant)."""
        if not self.quant:
            return x
        k = x.shape[-1]
        return mx.fake_quant(x.reshape(-1, k)).reshape(x.shape) if k % 32 == 0 else x

    def _bf(self, x):
        return R.bfr(x) if self.quant else x

    def _reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp > 1:
            return self.allreduce(x)
        return x

    def step(self, s: SeqState, token: int) -> torch.Tensor:
        """Advance one token; returns this rank's logits shard [V/tp] (fp32)."""
        c = self.cfg
        eps = c.rms_norm_eps
        pos = s.pos
        res = R.bfr(self.embed[token]) if self.quant else self.embed[token].clone()
        normed = R.rmsnorm(res, self.layers[0]["input_norm"], eps)
        gi = ai = 0
        for li, L in enumerate(self.layers):
            xq = self._q(normed)
            if L["type"] == "linear_attention":
                proj = self._bf(L["in_proj"] @ xq)
                win, st = s.gdn[gi]
                if pos == 0:
                    win, st = torch.zeros_like(win), torch.zeros_like(st)
                y, win, st = self._gdn(proj, win, st, L)
                s.gdn[gi] = (win, st)
                gi += 1
                delta = self._bf(L["out_proj"] @ self._q(y))
            else:
                qkv = self._bf(L["qkv"] @ xq)
                q, gate, k, v = self._prologue(qkv, pos, L)
                s.keys[ai] = torch.cat([s.keys[ai], k[None]], 0)
                s.values[ai] = torch.cat([s.values[ai], v[None]], 0)
                out = self._attention(q, gate, s.keys[ai], s.values[ai])
                ai += 1
                delta = self._bf(L["o_proj"] @ self._q(out))
            res, normed = self._add_norm(res, self._reduce(delta), L["post_norm"], eps)
            moe = self._moe_fwd(self._q(normed), L)
            nw = self.layers[li + 1]["input_norm"] if li + 1 < len(self.layers) else self.final_norm
            res, normed = self._add_norm(res, self._reduce(moe), nw, eps)
        s.pos += 1
        s.hidden = res
        return self.lm_head @ self._q(normed)

    def mtp_step(self, s: SeqState, token: int, hidden: torch.Tensor, pos: int):
        """One multi-token-prediction step: the next token's embedding and the hidden state
        at `pos` (target's or the previous MTP step's) -> (draft logits shard, MTP hidden).
        The MTP attention layer keeps its own KV at `pos` (entries past `pos` are dropped)."""
        c, M = self.cfg, self.mtp
        eps = c.rms_norm_eps
        emb = R.bfr(self.embed[token]) if self.quant else self.embed[token]
        fc_in = torch.cat([self._bf(R.rmsnorm(emb, M["norm_e"], eps)), self._bf(R.rmsnorm(hidden, M["norm_h"], eps))])
        res = self._bf(M["fc"] @ self._q(fc_in))
        normed = R.rmsnorm(res, M["input_norm"], eps)
        qkv = self._bf(M["qkv"] @ self._q(normed))
        q, gate, k, v = self._prologue(qkv, pos, M)
        if s.mtp_keys is None:
            s.mtp_keys = torch.zeros(0, self.hkv, self.D, device=self.dev)
            s.mtp_values = torch.zeros(0, self.hkv, self.D, device=self.dev)
        keys, values = s.mtp_keys[:pos], s.mtp_values[:pos]
        if keys.shape[0] < pos:  # positions never filled (e.g. chunk boundaries) read as zeros
            pad = torch.zeros(pos - keys.shape[0], self.hkv, self.D, device=self.dev)
            keys, values = torch.cat([keys, pad]), torch.cat([values, pad])
        s.mtp_keys = torch.cat([keys, k[None]], 0)
        s.mtp_values = torch.cat([values, v[None]], 0)
        out = self._attention(q, gate, s.mtp_keys, s.mtp_values)
        delta = self._bf(M["o_proj"] @ self._q(out))
        res, normed = self._add_norm(res, self._reduce(delta), M["post_norm"], eps)
        moe = self._moe_fwd(self._q(normed), M)
        res, normed = self._add_norm(res, self._reduce(moe), M["norm"], eps)
        return self.lm_head @ self._q(normed), res

    def _add_norm(self, res, delta, w, eps):
        r = res + delta
        if self.quant:
            r = R.bfr(r)
        return r, R.rmsnorm(r, w, eps)

    def _gdn(self, proj, win, st, L):
        return R.gdn_token(proj, win, st, hk=self.hk, hv=self.hv, conv_w=L["conv_w"], a_log=L["a_log"],
                           dt_bias=L["dt_bias"], norm_w=L["gnorm"], eps=self.cfg.rms_norm_eps, dk=self.dk, dv=self.dv)

    def _prologue(self, qkv, pos, L):
        c = self.cfg
        return R.attn_prologue_row(qkv, pos, hq=self.hq, hkv=self.hkv, q_norm_w=L["q_norm"], k_norm_w=L["k_norm"],
                                   eps=c.rms_norm_eps, rotary_dim=c.rotary_dim, theta=c.rope_theta, d=self.D)

    def _attention(self, q, gate, keys, values):
        return R.gated_attention(q, gate, keys, values, 1.0 / math.sqrt(self.D))

    def _moe_fwd(self, xq, L):
        c = self.cfg
        logits = L["router"] @ xq
        ids, w = R.route(logits[None, :self.E], top_k=c.num_experts_per_tok, norm_topk=c.norm_topk_prob)
        out = torch.zeros(c.hidden_size, device=xq.device)
        terms = []
        eb = self.r * self.e_local
        for e, wt in zip(ids[0].tolist(), w[0].tolist()):
            if not (eb <= e < eb + self.e_local):
                continue
            terms.append((L["gate"][e - eb], L["up"][e - eb], L["down"][e - eb], wt))
        terms.append((L["sgate"], L["sup"], L["sdown"], torch.sigmoid(logits[self.E]).item()))
        for wg, wu, wd, wt in terms:
            h = F.silu(wg @ xq) * (wu @ xq)
            # Expert output rounded to bf16, then weighted (the GPU combine gathers the
            # bf16 expert rows and applies the routing weight in fp32).
            out = out + self._bf(wd @ self._q(h)) * wt
        return out
