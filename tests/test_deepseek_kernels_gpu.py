"""DeepSeek-style kernels against PyTorch fp32 references: the tensor-core DSA indexer
scores + deterministic top-k, and the split-KV latent attention + W_UV up-projection."""

import os

import pytest
import torch

from zstep_b200.ops import _ext
from zstep_b200.ops import mx

pytestmark = pytest.mark.gpu


def _paged(n_seqs, max_len, page, dim, gen, scale=1.0):
    pages_per = (max_len + page - 1) // page
    cache = (torch.randn(1 + n_seqs * pages_per, page, dim, generator=gen) * scale).to(torch.bfloat16)
    # Non-contiguous page order per sequence.
    perm = torch.randperm(n_seqs * pages_per, generator=gen) + 1
    table = perm.view(n_seqs, pages_per).to(torch.int32)
    return cache, table


def _rows(cache, table, slot, n, page):
    idx = torch.arange(n)
    return cache[table[slot, idx // page].long(), idx % page].float()


@pytest.mark.parametrize("ih", [16, 64])
def test_dsa_index_scores_and_topk(ih):
    C = _ext.load()
    g = torch.Generator().manual_seed(1)
    page, topk, max_len = 16, 96, 700
    ctx = [5, 96, 97, 300, 700, 513]
    n = len(ctx)
    cache, table = _paged(n, max_len, page, 128, g)
    iq = (torch.randn(n, ih, 128, generator=g)).to(torch.bfloat16)
    iw = torch.randn(n, ih, generator=g)
    dev = "cuda"
    scores = torch.zeros(n, max_len, device=dev)
    sel = torch.full((n, topk), -1, dtype=torch.int32, device=dev)
    n_sel = torch.zeros(n, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    C.dsa_index(iq.to(dev), iw.to(dev), cache.to(dev), table.to(dev), page, torch.arange(n, dtype=torch.int32, device=dev),
                torch.tensor(ctx, dtype=torch.int32, device=dev), n, ih, topk, max_len, scores, sel, n_sel, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for t in range(n):
        c = ctx[t]
        if c <= topk:
            assert int(n_sel[t]) == c and sel[t, :c].cpu().tolist() == list(range(c))
            continue
        k = _rows(cache, table, t, c, page)
        ref = (torch.relu(k @ iq[t].float().T) * 128 ** -0.5) @ iw[t]
        got = scores[t, :c].cpu()
        torch.testing.assert_close(got, ref, rtol=1e-3, atol=1e-3)
        # Top-k of the kernel's own scores, ties to the lower position, ascending order.
        order = torch.sort(got, descending=True, stable=True).indices[:topk]
        assert int(n_sel[t]) == topk
        assert sel[t].cpu().tolist() == sorted(order.tolist())


def test_dsa_topk_ties_prefer_lower_positions():
    C = _ext.load()
    dev = "cuda"
    topk, ctx = 8, 40
    # Scores come from the indexer; force exact ties by giving every key the same vector.
    g = torch.Generator().manual_seed(2)
    cache = torch.zeros(4, 16, 128).to(torch.bfloat16)
    cache[1:] = torch.randn(1, 1, 128, generator=g).to(torch.bfloat16)
    table = torch.tensor([[1, 2, 3]], dtype=torch.int32)
    iq = torch.ones(1, 16, 128).to(torch.bfloat16)
    iw = torch.ones(1, 16)
    scores = torch.zeros(1, 48, device=dev)
    sel = torch.zeros(1, topk, dtype=torch.int32, device=dev)
    n_sel = torch.zeros(1, dtype=torch.int32, device=dev)
    C.dsa_index(iq.to(dev), iw.to(dev), cache.to(dev), table.to(dev), 16, torch.zeros(1, dtype=torch.int32, device=dev),
                torch.tensor([ctx], dtype=torch.int32, device=dev), 1, 16, topk, 48, scores, sel, n_sel)
    assert sel[0].cpu().tolist() == list(range(topk))


# The tensor-core latent attention (impl 2) has not run on a GPU yet: its case runs only
# when ZSTEP_TEST_MLA_TC=1 asks for it.
@pytest.mark.parametrize("impl", [1, pytest.param(2, marks=pytest.mark.skipif(
    os.environ.get("ZSTEP_TEST_MLA_TC") != "1", reason="tensor-core MLA not yet validated; ZSTEP_TEST_MLA_TC=1"))])
def test_mla_attention_and_up_projection(impl):
    C = _ext.load()
    g = torch.Generator().manual_seed(3)
    dev = "cuda"
    page, hl, kl, rope, vd = 16, 8, 512, 64, 128
    ctx = [1, 37, 200, 64]
    n = len(ctx)
    max_len = 256
    cache, table = _paged(n, max_len, page, kl + rope, g, scale=0.5)
    q_lat = (torch.randn(n, hl, kl, generator=g) * 0.1).to(torch.bfloat16)
    q_pe = (torch.randn(n, hl, rope, generator=g) * 0.1).to(torch.bfloat16)
    w_uv_t = (torch.randn(hl, kl, vd, generator=g) * 0.05).to(torch.bfloat16)
    # Selected positions: everything for short contexts, a strided subset for the long one.
    sel = torch.zeros(n, 128, dtype=torch.int32)
    n_sel = torch.zeros(n, dtype=torch.int32)
    picks = []
    for t, c in enumerate(ctx):
        p = list(range(c)) if c <= 128 else list(range(0, c, 2))[:128]
        picks.append(p)
        sel[t, :len(p)] = torch.tensor(p, dtype=torch.int32)
        n_sel[t] = len(p)
    scale = 192 ** -0.5
    for splits in (1, 4):
        part = torch.zeros(n * hl * splits * (kl + 4), device=dev)
        q = torch.zeros(128, hl * vd, dtype=torch.uint8, device=dev)
        sf = torch.zeros(mx.atoms_bytes(128, hl * vd), dtype=torch.uint8, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        C.mla_attn(q_lat.to(dev), q_pe.to(dev), cache.to(dev), table.to(dev), page,
                   torch.arange(n, dtype=torch.int32, device=dev), sel.to(dev), n_sel.to(dev), n, hl, splits, scale, part,
                   impl=impl, err=err)
        C.mla_up(part, n, hl, splits, w_uv_t.to(dev), q, sf)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        got = mx.dequantize(q[:n].cpu(), mx.codes_from_atoms(sf.cpu(), n, hl * vd))
        for t in range(n):
            kv = _rows(cache, table, t, ctx[t], page)[picks[t]]
            s = (q_lat[t].float() @ kv[:, :kl].T + q_pe[t].float() @ kv[:, kl:].T) * scale
            o_lat = torch.softmax(s, -1) @ kv[:, :kl]
            o = torch.einsum("hc,hcv->hv", o_lat.bfloat16().float(), w_uv_t.float()).reshape(-1)
            ref = mx.fake_quant(o.bfloat16().float()[None])[0]
            torch.testing.assert_close(got[t], ref, rtol=0.07, atol=2e-3)
