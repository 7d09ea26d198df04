"""Host-side token selection (zstep_b200/sampling.py): greedy ties, temperature / top-k /
top-p draws that every rank reproduces from the seed alone, penalties, greedy speculative
acceptance and the Gumbel reference of the fused lm_head sampler.  CPU only."""

import math

import numpy as np
import torch

from zstep_b200.runtime import wire
from zstep_b200.sampling import (apply_penalties, gumbel_sample, sample_logits, splitmix64, uniform01,
                                 verify_greedy)


def sp(temperature=0.0, top_p=1.0, top_k=0, seed=0, presence=0.0, frequency=0.0, repetition=1.0):
    rec = np.zeros(1, dtype=wire.SAMPLING_DTYPE)[0]
    rec["temperature"], rec["top_p"], rec["top_k"], rec["seed"] = temperature, top_p, top_k, seed
    rec["presence"], rec["frequency"], rec["repetition"] = presence, frequency, repetition
    return rec


def test_splitmix64_reference_vector():
    # First outputs of SplitMix64 from state 0 (the published reference sequence).
    s, a = splitmix64(0)
    _, b = splitmix64(s)
    assert (a, b) == (0xE220A8397B1DCDAF, 0x6E789E6AA1B965F4)
    assert 0.0 <= uniform01(12345) < 1.0 and uniform01(12345) == uniform01(12345)


def test_greedy_takes_the_smallest_id_on_ties():
    logits = torch.tensor([0.5, 2.0, -1.0, 2.0, 2.0])
    assert sample_logits(logits, sp()) == 1


def test_top_k_one_and_tiny_top_p_are_greedy():
    g = torch.Generator().manual_seed(0)
    for seed in range(20):
        logits = torch.randn(300, generator=g)
        best = int(torch.argmax(logits))
        assert sample_logits(logits, sp(temperature=1.0, top_k=1, seed=seed)) == best
        assert sample_logits(logits, sp(temperature=1.0, top_p=1e-6, seed=seed)) == best


def test_sampling_is_a_function_of_the_seed():
    logits = torch.randn(500, generator=torch.Generator().manual_seed(1))
    picks = [sample_logits(logits, sp(temperature=0.8, top_p=0.9, top_k=50, seed=s)) for s in range(40)]
    again = [sample_logits(logits.clone(), sp(temperature=0.8, top_p=0.9, top_k=50, seed=s)) for s in range(40)]
    assert picks == again and len(set(picks)) > 1


def test_draws_follow_the_tempered_distribution():
    logits = torch.tensor([1.0, 0.0, -1.0, 0.5])
    T = 0.7
    p = torch.softmax(logits / T, 0).tolist()
    n = 4000
    counts = [0] * 4
    for s in range(n):
        counts[sample_logits(logits, sp(temperature=T, seed=s * 7919 + 3))] += 1
    for c, q in zip(counts, p):
        assert abs(c / n - q) < 4 * math.sqrt(q * (1 - q) / n) + 0.005, (counts, p)


def test_top_p_keeps_the_smallest_nucleus():
    logits = torch.log(torch.tensor([0.5, 0.3, 0.15, 0.05]))
    seen = {sample_logits(logits, sp(temperature=1.0, top_p=0.75, seed=s)) for s in range(300)}
    assert seen == {0, 1}  # 0.5 < 0.75 <= 0.8: the first two tokens


def test_penalties():
    logits = torch.tensor([2.0, -2.0, 1.0, 0.0])
    out = apply_penalties(logits, [0, 1, 1], presence=0.5, frequency=0.25, repetition=2.0)
    # repetition divides positive / multiplies negative seen logits, then frequency x count
    # and presence are subtracted from every seen token.
    assert torch.allclose(out, torch.tensor([2.0 / 2 - 0.25 - 0.5, -2.0 * 2 - 0.5 - 0.5, 1.0, 0.0]))
    # Penalties shape greedy choices too.
    assert sample_logits(torch.tensor([1.0, 0.9]), sp(presence=0.5), history=[0]) == 1


def test_verify_greedy():
    assert verify_greedy([5, 6, 7], [5, 6, 7, 8]) == [5, 6, 7, 8]   # all accepted + bonus
    assert verify_greedy([5, 6, 7], [5, 9, 7, 8]) == [5, 9]         # stop at the first mismatch
    assert verify_greedy([5, 6, 7], [4, 6, 7, 8]) == [4]
    assert verify_greedy([], [3]) == [3]


def test_gumbel_sampler_reference():
    logits = torch.tensor([0.3, 1.2, -0.4])
    assert gumbel_sample(logits, 0.0, seed=1, pos=0) == 1
    T, n = 1.3, 3000
    p = torch.softmax(logits / T, 0).tolist()
    counts = [0] * 3
    for pos in range(n):
        counts[gumbel_sample(logits, T, seed=99, pos=pos)] += 1
    for c, q in zip(counts, p):
        assert abs(c / n - q) < 4 * math.sqrt(q * (1 - q) / n) + 0.005, (counts, p)


def test_full_distribution_head_is_used_only_when_needed():
    """Greedy and plain temperature rows stay in the lm_head GEMM (argmax / Gumbel
    epilogue); top-k, top-p, penalties or logprobs route the step to the sampling head."""
    from zstep_b200.models.sampling_head import needs_full

    def recs(**kw):
        r = np.zeros(2, dtype=wire.SAMPLING_DTYPE)
        r["top_p"], r["repetition"], r["logprobs"] = 1.0, 1.0, -1
        for k, v in kw.items():
            r[k][1] = v
        return r

    assert not needs_full(recs(), 2)
    assert not needs_full(recs(temperature=0.7), 2)
    assert not needs_full(recs(top_k=5), 2)  # greedy: top-k changes nothing
    assert needs_full(recs(temperature=0.7, top_k=5), 2)
    assert needs_full(recs(temperature=0.7, top_p=0.9), 2)
    assert needs_full(recs(presence=0.5), 2) and needs_full(recs(frequency=0.5), 2)
    assert needs_full(recs(repetition=1.1), 2) and needs_full(recs(logprobs=0), 2)
    assert not needs_full(recs(logprobs=0), 1)  # only the first n rows count
