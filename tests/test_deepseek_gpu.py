"""DeepSeek-style model on B200 kernels (mHC, MLA, DSA indexer top-k, sigmoid grouped MoE
with MXFP8 or MXFP4 experts) against the fp32 reference with the same quantization
points, on a reduced config that keeps the per-head kernel shapes.  Prompts are longer
than the index top-k so the sparse path runs."""

import pytest
import torch

from zstep_b200.config import deepseek_small_gpu
from zstep_b200.models.deepseek import DeepSeekRunner
from zstep_b200.models.deepseek_ref import DeepSeekReference
from zstep_b200.models.deepseek_weights import DeepSeekRandomWeights
from zstep_b200.ops import mx

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=["mxfp8", "mxfp4"])
def setup(request):
    cfg = deepseek_small_gpu(num_layers=3, vocab=8192, experts=32, topk=48)
    cfg = cfg.__class__(**{**cfg.to_dict(), "expert_format": request.param})
    src = DeepSeekRandomWeights(cfg, seed=13)
    runner = DeepSeekRunner(cfg, weights=src, max_seqs=8, max_prefill_tokens=256, num_pages=64, max_model_len=256)
    ref = DeepSeekReference(cfg, src, device="cuda", quant=True)
    return cfg, runner, ref


def _check_rows(runner, ref_logits, ref_normed, out):
    """The runner's lm_head input matches the reference's (cosine), its max logit matches,
    and each picked token is the reference's argmax or within a near-tie of it."""
    H = runner.cfg.hidden_size
    b = runner.buf
    n = len(out)
    hn = mx.dequantize(b["xq"][:n], mx.codes_from_atoms(b["xsf"], n, H))
    vals = b["out_vals"][:n].cpu()
    for s in range(n):
        cos = torch.nn.functional.cosine_similarity(hn[s].float(), ref_normed[s].float(), dim=0).item()
        assert cos > 0.998, (s, cos)
        lg = ref_logits[s]
        torch.testing.assert_close(vals[s], lg.max().cpu(), rtol=3e-2, atol=3e-2)
        assert lg[out[s]] >= lg.max() - 0.05, (s, out[s], int(lg.argmax()))


def test_prefill_then_decode_matches_reference(setup):
    cfg, runner, ref = setup
    g = torch.Generator().manual_seed(3)
    lens = [9, 60, 30]
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]
    for s in range(len(lens)):
        runner.set_pages(s, list(range(1 + 8 * s, 1 + 8 * (s + 1))))
    ids, pos, slots, starts = [], [], [], [0]
    for s, p in enumerate(prompts):
        ids += p
        pos += list(range(len(p)))
        slots += [s] * len(p)
        starts.append(starts[-1] + len(p))
    runner.stage(ids, pos, slots, seq_start=starts)
    first = runner.prefill_forward(len(ids), len(lens)).cpu().tolist()
    assert runner.check_error() == 0
    # lm_head rows of the prefill are gathered into xq_last: compare the max logits there.
    states = [ref.new_state() for _ in lens]
    ref_l, ref_next = [], []
    for s, p in enumerate(prompts):
        for t in p:
            lg = ref.step(states[s], t)
        ref_l.append(lg)
        ref_next.append(int(lg.argmax()))
    vals = runner.buf["out_vals"][:3].cpu()
    for s in range(3):
        torch.testing.assert_close(vals[s], ref_l[s].max().cpu(), rtol=3e-2, atol=3e-2)
        assert ref_l[s][first[s]] >= ref_l[s].max() - 0.05, (s, first, ref_next)
    toks = ref_next
    for step in range(6):
        p_now = [len(p) + step for p in prompts]
        runner.stage(toks, p_now, list(range(3)))
        out = runner.decode_step(3).cpu().tolist()
        assert runner.check_error() == 0
        logits, normed = [], []
        for s in range(3):
            logits.append(ref.step(states[s], toks[s]))
            normed.append(ref.last_normed)
        _check_rows(runner, logits, normed, out)
        toks = [int(lg.argmax()) for lg in logits]
