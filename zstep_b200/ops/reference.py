"""PyTorch fp32 reference implementations of every fused op the sm_100a kernels run.

Layouts and rounding points mirror the kernels exactly (bf16 where the kernel stores
bf16), so GPU numerics tests can compare a kernel against these functions and the
CPU plumbing model can run the same math without a GPU.

Reference parity (math): worker/zstep_worker/kernels_sm120/qwen35_ops.py -- zero-centered
RMSNorm (:88-178), attention prologue (:187-277), paged GQA with sigmoid gate
(:325-560), causal conv1d + gated delta rule + gated RMSNorm (:659-935), router
softmax/top-k/shared gate (:1165-1222); the sigmoid grouped router follows the
DeepSeek-V3 scheme (kernels_sm120/moe_router.py:31-110).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def bfr(x: torch.Tensor) -> torch.Tensor:
    """Round to bf16 and back to fp32."""
    return x.to(torch.bfloat16).float()


# ------------------------------------------------------------------------------ norms
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, w_offset: float = 1.0) -> torch.Tensor:
    """``x * rsqrt(mean(x^2) + eps) * (w + w_offset)`` in fp32 (zero-centered when w_offset=1)."""
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return xf * rstd * (w.float() + w_offset)


def add_rmsnorm(residual: torch.Tensor, delta: torch.Tensor | None, w: torch.Tensor, eps: float,
                w_offset: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (new residual rounded to bf16 as fp32, normed fp32)."""
    r = residual.float()
    if delta is not None:
        r = r + delta.float()
    r = bfr(r)
    return r, rmsnorm(r, w, eps, w_offset)


# ------------------------------------------------------------------------------ GDN
def gdn_conv_step(x: torch.Tensor, window: torch.Tensor, conv_w: torch.Tensor):
    """One causal-conv step.  x [C], window [C, 3] (previous inputs), conv_w [C, 4].
    Returns (silu(conv) rounded to bf16, new window)."""
    acc = (window * conv_w[:, :3].float()).sum(-1) + conv_w[:, 3].float() * x
    y = bfr(F.silu(acc))
    new_window = torch.cat([window[:, 1:], x[:, None]], dim=1)
    return y, new_window


def gdn_token(proj_row: torch.Tensor, window: torch.Tensor, state: torch.Tensor, *, hk: int,
              hv: int, conv_w: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor,
              norm_w: torch.Tensor, eps: float, dk: int = 128, dv: int = 128):
    """GatedDeltaNet for one token.

    proj_row: fp32 [2*hk*dk + 2*hv*dv + 2*hv] = [q | k | v | z | b | a] (bf16 values)
    window:   fp32 [conv_dim, 3]; state: fp32 [hv, dv, dk] (updated copy returned)
    Returns (y fp32 [hv*dv] (bf16-rounded gated output), new window, new state).
    """
    conv_dim = 2 * hk * dk + hv * dv
    x = proj_row[:conv_dim]
    y, window = gdn_conv_step(x, window, conv_w)
    q = y[: hk * dk].reshape(hk, dk)
    k = y[hk * dk: 2 * hk * dk].reshape(hk, dk)
    v = y[2 * hk * dk:].reshape(hv, dv)
    zoff = conv_dim
    z = proj_row[zoff: zoff + hv * dv].reshape(hv, dv)
    b = proj_row[zoff + hv * dv: zoff + hv * dv + hv]
    a = proj_row[zoff + hv * dv + hv: zoff + hv * dv + 2 * hv]
    q = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) / math.sqrt(dk)
    k = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    ratio = hv // hk
    beta = torch.sigmoid(b)
    sp = a + dt_bias.float()
    softplus = torch.where(sp > 20.0, sp, torch.log1p(torch.exp(sp)))
    g = torch.exp(-torch.exp(a_log.float()) * softplus)
    new_state = state.clone()
    out = torch.empty(hv, dv, device=state.device)
    for h in range(hv):
        kh = h // ratio
        s = new_state[h] * g[h]
        kv = s @ k[kh]
        delta = (v[h] - kv) * beta[h]
        s = s + delta[:, None] * k[kh][None, :]
        new_state[h] = s
        out[h] = s @ q[kh]
    rstd = torch.rsqrt((out * out).mean(-1, keepdim=True) + eps)
    nrm = bfr(out * rstd) * norm_w.float()
    yout = bfr(nrm * F.silu(z))
    return yout.reshape(-1), window, new_state


# ------------------------------------------------------------------------------ attention
def rope_cos_sin(pos: int, rotary_dim: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    half = rotary_dim // 2
    i = torch.arange(half, dtype=torch.float32)
    inv_freq = theta ** (-2.0 * i / rotary_dim)
    ang = pos * inv_freq.double()
    return bfr(torch.cos(ang).float()), bfr(torch.sin(ang).float())


def attn_prologue_row(qkv_row: torch.Tensor, pos: int, *, hq: int, hkv: int, q_norm_w, k_norm_w,
                      eps: float, rotary_dim: int, theta: float, d: int = 256):
    """Returns (q [hq, d], gate [hq, d], k [hkv, d], v [hkv, d]) fp32 with bf16 rounding."""
    cos, sin = rope_cos_sin(pos, rotary_dim, theta)
    cos, sin = cos.to(qkv_row.device), sin.to(qkv_row.device)
    half = rotary_dim // 2

    def norm_rope(x, w):
        y = bfr(rmsnorm(x, w, eps, 1.0))
        lo, hi = y[..., :half].clone(), y[..., half:2 * half].clone()
        y[..., :half] = bfr(lo * cos - hi * sin)
        y[..., half:2 * half] = bfr(hi * cos + lo * sin)
        return y

    qg = qkv_row[: hq * 2 * d].reshape(hq, 2, d)
    q = norm_rope(qg[:, 0].float(), q_norm_w)
    gate = qg[:, 1].float()
    kk = qkv_row[hq * 2 * d: hq * 2 * d + hkv * d].reshape(hkv, d).float()
    vv = qkv_row[hq * 2 * d + hkv * d: hq * 2 * d + 2 * hkv * d].reshape(hkv, d).float()
    return q, gate, norm_rope(kk, k_norm_w), vv


def gated_attention(q: torch.Tensor, gate: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
                    sm_scale: float) -> torch.Tensor:
    """q, gate [hq, d]; keys/values [T, hkv, d].  Returns bf16-rounded [hq*d]."""
    hq, d = q.shape
    hkv = keys.shape[1]
    grp = hq // hkv
    out = torch.empty(hq, d, device=q.device)
    for h in range(hq):
        kvh = h // grp
        s = (keys[:, kvh] @ q[h]) * sm_scale
        p = torch.softmax(s, dim=0)
        out[h] = p @ values[:, kvh]
    return bfr(bfr(out) * torch.sigmoid(gate)).reshape(-1)


# ------------------------------------------------------------------------------ MoE routing
def route(logits: torch.Tensor, *, top_k: int, scoring: str = "softmax", norm_topk: bool = True,
          bias: torch.Tensor | None = None, n_group: int = 1, topk_group: int = 1,
          routed_scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """logits [rows, E] fp32 -> (ids [rows, k] int64, weights [rows, k] fp32).

    Ties resolve to the smallest expert id (a stable descending sort)."""
    if scoring == "softmax":
        score = torch.softmax(logits.float(), dim=-1)
        choice = score.clone()
    else:
        if scoring == "sqrtsoftplus":
            x = logits.float()
            score = torch.sqrt(torch.where(x > 20.0, x, torch.log1p(torch.exp(x))))
        elif scoring == "sigmoid":
            score = torch.sigmoid(logits.float())
        else:
            raise ValueError(f"unknown router scoring {scoring!r}")
        choice = score + (bias.float() if bias is not None else 0.0)
        if n_group > 1:
            rows, e = choice.shape
            g = choice.reshape(rows, n_group, e // n_group)
            top2 = g.topk(2, dim=-1).values.sum(-1)
            # stable: lower group index wins ties
            order = torch.sort(top2, dim=-1, descending=True, stable=True).indices[:, :topk_group]
            mask = torch.zeros(rows, n_group, dtype=torch.bool, device=choice.device)
            mask.scatter_(1, order, True)
            choice = torch.where(mask.repeat_interleave(e // n_group, dim=1), choice,
                                 torch.full_like(choice, float("-inf")))
    idx = torch.sort(choice, dim=-1, descending=True, stable=True).indices[:, :top_k]
    w = torch.gather(score, 1, idx)
    if norm_topk:
        w = w / w.sum(-1, keepdim=True).clamp_min(1e-20)
    return idx, w * routed_scale
