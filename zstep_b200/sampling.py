"""Token selection shared by every runner.

* greedy: global argmax with the smallest id on ties (``torch.argmax`` returns the first
  maximum), matching the fused lm_head argmax kernels;
* stochastic: temperature, top-k and top-p (nucleus) filtering, penalties, and a
  uniform draw from a SplitMix64 stream seeded per (request seed, generated index), so
  every tensor-parallel rank draws the same token without communication;
* speculative verify: greedy prefix acceptance of draft tokens.

Reference parity: worker/zstep_worker/sampler.py (splitmix64_uniform_f32 :47,
SlotPenaltyState :62, sample_tp8_logits :127) and spec_decode.py (verify_greedy :41).
"""

from __future__ import annotations

import torch

_MASK64 = (1 << 64) - 1


def splitmix64(state: int) -> tuple[int, int]:
    state = (state + 0x9E3779B97F4A7C15) & _MASK64
    z = state
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK64
    return state, z ^ (z >> 31)


def uniform01(seed: int) -> float:
    """Deterministic uniform in [0, 1) from a 64-bit seed (24-bit mantissa)."""
    _, z = splitmix64(seed & _MASK64)
    return (z >> 40) / float(1 << 24)


def apply_penalties(logits: torch.Tensor, history: list[int], presence: float, frequency: float,
                    repetition: float) -> torch.Tensor:
    if not history or (presence == 0 and frequency == 0 and repetition == 1.0):
        return logits
    ids = torch.tensor(history, dtype=torch.long, device=logits.device)
    counts = torch.bincount(ids, minlength=logits.numel()).to(logits.dtype)
    seen = counts > 0
    out = logits.clone()
    if repetition != 1.0:
        out = torch.where(seen, torch.where(out > 0, out / repetition, out * repetition), out)
    out = out - frequency * counts - presence * seen.to(out.dtype)
    return out


def sample_logits(logits: torch.Tensor, sp, history: list[int] | None = None) -> int:
    """``sp`` is a SamplingParams record (temperature, top_p, top_k, presence, frequency,
    repetition, seed, logprobs)."""
    logits = logits.float().reshape(-1)
    temperature = float(sp["temperature"]) if hasattr(sp, "dtype") or isinstance(sp, dict) else float(sp[0])
    if history:  # penalties shape greedy and stochastic choices alike
        logits = apply_penalties(logits, history, float(sp["presence"]), float(sp["frequency"]),
                                 float(sp["repetition"]))
    if temperature <= 0.0:
        return int(torch.argmax(logits))
    top_p = float(sp["top_p"])
    top_k = int(sp["top_k"])
    seed = int(sp["seed"])
    logits = logits / temperature
    vals, idx = torch.sort(logits, descending=True, stable=True)
    if top_k > 0:
        vals, idx = vals[:top_k], idx[:top_k]
    probs = torch.softmax(vals, dim=0)
    if top_p < 1.0:
        cdf = torch.cumsum(probs, dim=0)
        keep = int(torch.searchsorted(cdf, torch.tensor(top_p, dtype=cdf.dtype))) + 1
        probs, idx = probs[:keep], idx[:keep]
        probs = probs / probs.sum()
    u = uniform01(seed)
    cdf = torch.cumsum(probs, dim=0)
    j = int(torch.searchsorted(cdf, torch.tensor(u, dtype=cdf.dtype), right=True))
    return int(idx[min(j, idx.numel() - 1)])


def verify_greedy(drafts: list[int], targets: list[int]) -> list[int]:
    """targets[j] = the model's token after verify row j (row 0 = last accepted token).
    Accept drafts while they match; append the model's token at the first mismatch (or
    the bonus token after the last draft)."""
    out = []
    for j, d in enumerate(drafts):
        if targets[j] != d:
            out.append(targets[j])
            return out
        out.append(d)
    out.append(targets[len(drafts)])
    return out


def gumbel_noise(seed: int, pos: int, ids: torch.Tensor) -> torch.Tensor:
    """Gumbel(0, 1) noise of the GPU sampler for token ids `ids` at (seed, position):
    one SplitMix64 step of seed ^ pos*C1 ^ id*C2, 24-bit uniform in (0, 1)."""
    m = _MASK64
    z = [(((seed ^ ((pos & 0xFFFFFFFF) * 0x9E3779B97F4A7C15) ^ ((int(i) & 0xFFFFFFFF) * 0xD1B54A32D192ED03)) & m)
          + 0x9E3779B97F4A7C15) & m for i in ids.tolist()]
    out = []
    for v in z:
        v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & m
        v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & m
        v ^= v >> 31
        out.append(((v >> 40) + 0.5) / float(1 << 24))
    u = torch.tensor(out, dtype=torch.float32)
    return -torch.log(-torch.log(u))


def gumbel_sample(logits: torch.Tensor, temperature: float, seed: int, pos: int) -> int:
    """Reference of the fused lm_head sampler: argmax of logits / T + Gumbel noise
    (distributed as softmax(logits / T)); greedy when T <= 0."""
    if temperature <= 0:
        return int(torch.argmax(logits))
    ids = torch.arange(logits.numel())
    return int(torch.argmax(logits.float().cpu() / temperature + gumbel_noise(seed, pos, ids)))
