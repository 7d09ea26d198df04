"""Numerics of every sm_100a kernel against a PyTorch fp32 reference of the same op."""

import math

import pytest
import torch
import torch.nn.functional as F

from zstep_b200.ops import mx
from zstep_b200.ops.kv_layout import swizzle_pages, unswizzle_pages
from zstep_b200.ops import reference as ref

pytestmark = pytest.mark.gpu

EPI_BF16, EPI_F32, EPI_SILU, EPI_SCATTER, EPI_ARGMAX = 0, 1, 2, 3, 4


@pytest.fixture(scope="module")
def C():
    from zstep_b200.ops import _ext

    return _ext.load()


def gemm(C, *args, block_n=128, k_splits=1, split_stride=0, a_tiled=0):
    C.gemm_mxf8(*args, block_n, k_splits, split_stride, a_tiled)


def route(C, logits, *args, splits=1, split_stride=0, chunk_rows=128):
    C.moe_route(logits, *args, logits.shape[-1], splits, split_stride, chunk_rows)


def _pad_rows(n: int) -> int:
    return (n + 127) // 128 * 128


def _quant_weights(w: torch.Tensor):
    """w [G, N, K] fp32 -> (q [G*Npad, K] u8, atoms, dequant [G, Npad, K])."""
    g, n, k = w.shape
    npad = _pad_rows(n)
    wp = torch.zeros(g, npad, k)
    wp[:, :n] = w
    q, code = mx.quantize(wp.reshape(g * npad, k))
    deq = mx.dequantize(q, code).reshape(g, npad, k)
    return q.cuda(), mx.atoms_from_codes(code).cuda(), deq, npad


def _quant_act(x: torch.Tensor, rows_pad: int):
    rows, k = x.shape
    xp = torch.zeros(rows_pad, k)
    xp[:rows] = x
    q, code = mx.quantize(xp)
    return q.cuda(), mx.atoms_from_codes(code).cuda(), mx.dequantize(q, code)[:rows]


@pytest.mark.parametrize("m,n,k", [(200, 300, 512), (1, 128, 128), (256, 1024, 2048), (37, 129, 384)])
def test_gemm_dense_f32(C, m, n, k):
    torch.manual_seed(m + n + k)
    w = torch.randn(1, n, k) * 0.05
    x = torch.randn(m, k)
    wq, wsf, wd, npad = _quant_weights(w)
    xq, xsf, xd = _quant_act(x, _pad_rows(m))
    out = torch.zeros(m, n, device="cuda", dtype=torch.float32)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gemm(C,wq, wsf, xq, xsf, k, npad, n, 1, m, None, None, None, EPI_F32, out, n,
                None, None, None, err, 0)
    torch.cuda.synchronize()
    assert err.item() == 0
    expect = xd @ wd[0, :n].T
    torch.testing.assert_close(out.cpu(), expect, rtol=1e-4, atol=1e-3)


def test_gemm_dense_bf16(C):
    torch.manual_seed(1)
    m, n, k = 130, 640, 1024
    w = torch.randn(1, n, k) * 0.05
    x = torch.randn(m, k)
    wq, wsf, wd, npad = _quant_weights(w)
    xq, xsf, xd = _quant_act(x, _pad_rows(m))
    out = torch.zeros(m, n, device="cuda", dtype=torch.bfloat16)
    gemm(C,wq, wsf, xq, xsf, k, npad, n, 1, m, None, None, None, EPI_BF16, out, n,
                None, None, None, None, 0)
    torch.cuda.synchronize()
    expect = (xd @ wd[0, :n].T).to(torch.bfloat16)
    torch.testing.assert_close(out.cpu(), expect, rtol=1e-2, atol=1e-2)


def _grouped_setup(counts, k, n, seed=0):
    torch.manual_seed(seed)
    g = len(counts)
    w = torch.randn(g, n, k) * 0.05
    wq, wsf, wd, npad = _quant_weights(w)
    offsets, chunk_prefix, o, c = [], [0], 0, 0
    for cnt in counts:
        offsets.append(o)
        o += _pad_rows(cnt) if cnt else 0
        c += (cnt + 127) // 128
        chunk_prefix.append(c)
    rows = max(o, 128)
    x = torch.randn(rows, k)
    xq, xsf, xd = _quant_act(x, rows)
    dev = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")  # noqa: E731
    return dict(w=w, wq=wq, wsf=wsf, wd=wd, npad=npad, x=x, xq=xq, xsf=xsf, xd=xd, rows=rows,
                offsets=offsets, cnt=dev(counts), off=dev(offsets), pre=dev(chunk_prefix))


def test_gemm_grouped_f32(C):
    counts = [0, 7, 130, 16, 1, 300]
    k, n = 256, 256
    s = _grouped_setup(counts, k, n)
    out = torch.full((s["rows"], n), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gemm(C,s["wq"], s["wsf"], s["xq"], s["xsf"], k, s["npad"], n, len(counts), 0,
                s["cnt"], s["off"], s["pre"], EPI_F32, out, n, None, None, None, err, 0)
    torch.cuda.synchronize()
    assert err.item() == 0
    out = out.cpu()
    for gi, cnt in enumerate(counts):
        if cnt == 0:
            continue
        o = s["offsets"][gi]
        expect = s["xd"][o:o + cnt] @ s["wd"][gi, :n].T
        torch.testing.assert_close(out[o:o + cnt], expect, rtol=1e-4, atol=1e-3)


def test_gemm_grouped_bn32(C):
    """32-token chunks: chunks start 0/32/64/96 rows into a scale atom."""
    counts = [0, 3, 33, 64, 100, 17, 130]
    k, n = 384, 256
    s = _grouped_setup(counts, k, n, seed=4)
    pre, c = [0], 0
    for cnt in counts:
        c += (cnt + 31) // 32
        pre.append(c)
    out = torch.full((s["rows"], n), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    gemm(C, s["wq"], s["wsf"], s["xq"], s["xsf"], k, s["npad"], n, len(counts), 0, s["cnt"], s["off"],
         torch.tensor(pre, dtype=torch.int32, device="cuda"), EPI_F32, out, n, None, None, None, err, 0,
         block_n=32)
    torch.cuda.synchronize()
    assert err.item() == 0
    out = out.cpu()
    for gi, cnt in enumerate(counts):
        if cnt == 0:
            continue
        o = s["offsets"][gi]
        expect = s["xd"][o:o + cnt] @ s["wd"][gi, :n].T
        torch.testing.assert_close(out[o:o + cnt], expect, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("m,splits,bn", [(256, 4, 128), (20, 8, 32), (130, 3, 32)])
def test_gemm_split_k(C, m, splits, bn):
    torch.manual_seed(9)
    n, k = 384, 2048
    w = torch.randn(1, n, k) * 0.05
    x = torch.randn(m, k)
    wq, wsf, wd, npad = _quant_weights(w)
    xq, xsf, xd = _quant_act(x, _pad_rows(m))
    out = torch.zeros(splits, m, n, device="cuda")
    gemm(C, wq, wsf, xq, xsf, k, npad, n, 1, m, None, None, None, EPI_F32, out, n, None, None, None, None, 0,
         block_n=bn, k_splits=splits, split_stride=m * n)
    torch.cuda.synchronize()
    expect = xd @ wd[0, :n].T
    torch.testing.assert_close(out.sum(0).cpu(), expect, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("grouped", [False, True])
def test_gemm_tiled_weights(C, grouped):
    """Pre-tiled weight layout (contiguous 16 KiB blocks) gives identical results."""
    counts = [5, 40, 0, 129]
    k, n = 512, 384
    s = _grouped_setup(counts if grouped else [200], k, n, seed=12)
    g = len(counts) if grouped else 1
    wq_t = mx.tile_weight(s["wq"].cpu()).cuda()
    out = torch.full((s["rows"], n), float("nan"), device="cuda")
    if grouped:
        gemm(C, wq_t, s["wsf"], s["xq"], s["xsf"], k, s["npad"], n, g, 0, s["cnt"], s["off"], s["pre"], EPI_F32,
             out, n, None, None, None, None, 0, a_tiled=1)
    else:
        gemm(C, wq_t, s["wsf"], s["xq"], s["xsf"], k, s["npad"], n, 1, 200, None, None, None, EPI_F32, out, n,
             None, None, None, None, 0, a_tiled=1)
    torch.cuda.synchronize()
    out = out.cpu()
    for gi, cnt in enumerate(counts if grouped else [200]):
        if cnt == 0:
            continue
        o = s["offsets"][gi]
        torch.testing.assert_close(out[o:o + cnt], s["xd"][o:o + cnt] @ s["wd"][gi, :n].T, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("bn", [32, 128])
@pytest.mark.parametrize("grouped", [False, True])
def test_gemm_fp4_weights(C, grouped, bn):
    """MXFP4 weights stay packed in memory and are widened to e4m3 in shared memory by the
    converter warps: results equal an fp32 GEMM on the dequantized MXFP4 weights."""
    counts = [5, 40, 0, 129, 33]
    k, n = 512, 384
    s = _grouped_setup(counts if grouped else [200], k, n, seed=21)
    g = len(counts) if grouped else 1
    w = s["w"]
    npad = s["npad"]
    wp = torch.zeros(g, npad, k)
    wp[:, :n] = w
    packed, code = mx.quantize_fp4(wp.reshape(g * npad, k))
    wd = mx.dequantize_fp4(packed, code).reshape(g, npad, k)
    wq4 = mx.tile_weight_fp4(packed).cuda()
    wsf = mx.atoms_from_codes(code).cuda()
    out = torch.full((s["rows"], n), float("nan"), device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    if grouped:
        pre, c = [0], 0
        for cnt in counts:
            c += (cnt + bn - 1) // bn
            pre.append(c)
        C.gemm_mxf8(wq4, wsf, s["xq"], s["xsf"], k, npad, n, g, 0, s["cnt"], s["off"],
                    torch.tensor(pre, dtype=torch.int32, device="cuda"), EPI_F32, out, n, None, None, None, err, 0,
                    bn, 1, 0, 1, a_fp4=1)
    else:
        C.gemm_mxf8(wq4, wsf, s["xq"], s["xsf"], k, npad, n, 1, 200, None, None, None, EPI_F32, out, n, None,
                    None, None, err, 0, bn, 1, 0, 1, a_fp4=1)
    torch.cuda.synchronize()
    assert err.item() == 0
    out = out.cpu()
    for gi, cnt in enumerate(counts if grouped else [200]):
        if cnt == 0:
            continue
        o = s["offsets"][gi]
        torch.testing.assert_close(out[o:o + cnt], s["xd"][o:o + cnt] @ wd[gi, :n].T, rtol=1e-4, atol=1e-3)


def test_gemm_silu_quant(C):
    counts = [5, 0, 140]
    k, inter = 256, 256  # 4 tiles of (64 gate + 64 up)
    torch.manual_seed(3)
    g = len(counts)
    wg = torch.randn(g, inter, k) * 0.05
    wu = torch.randn(g, inter, k) * 0.05
    # Interleave per 128-row tile: [gate 64m..64m+63 ; up 64m..64m+63]
    packed = torch.stack([wg.reshape(g, inter // 64, 64, k), wu.reshape(g, inter // 64, 64, k)], dim=2)
    packed = packed.reshape(g, 2 * inter, k)
    s = _grouped_setup(counts, k, 2 * inter)
    wq, wsf, wd, npad = _quant_weights(packed)
    act = torch.zeros(s["rows"], inter, dtype=torch.uint8, device="cuda")
    act_sf = torch.zeros(mx.atoms_bytes(s["rows"], inter), dtype=torch.uint8, device="cuda")
    gemm(C,wq, wsf, s["xq"], s["xsf"], k, npad, 2 * inter, g, 0, s["cnt"], s["off"], s["pre"],
                EPI_SILU, act, inter, act_sf, None, None, None, 0)
    torch.cuda.synchronize()
    codes = mx.codes_from_atoms(act_sf.cpu(), s["rows"], inter)
    got = mx.dequantize(act.cpu(), codes)
    for gi, cnt in enumerate(counts):
        if cnt == 0:
            continue
        o = s["offsets"][gi]
        full = s["xd"][o:o + cnt] @ wd[gi].T  # [cnt, 2*inter] in packed order
        full = full.reshape(cnt, inter // 64, 2, 64)
        h = (F.silu(full[:, :, 0]) * full[:, :, 1]).reshape(cnt, inter)
        expect = mx.fake_quant(h)
        tol = h.abs().amax(-1, keepdim=True) / 8
        assert ((got[o:o + cnt] - expect).abs() <= tol + 1e-6).all()
        torch.testing.assert_close(got[o:o + cnt], h, rtol=0.07, atol=0.02 * h.abs().max().item())


def test_gemm_argmax_gumbel_sampling(C):
    """Sampling rows take argmax(logit / T + Gumbel(seed, pos, id)): matches the host
    reference on the kernel's own logits, and the sample frequencies follow softmax(l / T)."""
    from zstep_b200.sampling import gumbel_noise

    torch.manual_seed(5)
    m, vocab, k = 64, 1000, 256
    w = torch.randn(1, vocab, k) * 0.05
    x = torch.randn(m, k)
    wq, wsf, wd, npad = _quant_weights(w)
    xq, xsf, xd = _quant_act(x, _pad_rows(m))
    tiles = npad // 128
    logits = torch.zeros(m, vocab, device="cuda")
    gemm(C, wq, wsf, xq, xsf, k, npad, vocab, 1, m, None, None, None, EPI_F32, logits, vocab, None, None, None, None, 0)
    temp = torch.tensor([0.0 if r % 4 == 0 else 0.7 for r in range(m)], device="cuda")
    seed = torch.arange(m, dtype=torch.int64, device="cuda") * 7919 + 11
    pos = torch.arange(m, dtype=torch.int32, device="cuda") + 100
    keys = torch.zeros(m, tiles, dtype=torch.int64, device="cuda")
    C.gemm_mxf8(wq, wsf, xq, xsf, k, npad, vocab, 1, m, None, None, None, EPI_ARGMAX, keys, tiles, None, None, None,
                None, 0, 128, 1, 0, 0, 1, None, None, temp, seed, pos, 5000)
    ids = torch.zeros(m, dtype=torch.int32, device="cuda")
    C.argmax_reduce(keys, m, tiles, ids, None, None)
    torch.cuda.synchronize()
    lg = logits.cpu()
    agree = 0
    for r in range(m):
        t = float(temp[r])
        if t == 0:
            exp = int(lg[r].argmax())
        else:
            exp = int(torch.argmax(lg[r] / t + gumbel_noise(int(seed[r]), int(pos[r]), torch.arange(vocab) + 5000)))
        agree += int(exp == int(ids[r]))
    assert agree >= m - 1, agree
    # Distribution: one 4-way row repeated at many positions.
    m2, v2 = 2048, 128
    w2 = torch.zeros(1, v2, k)
    w2[0, :4, 0] = torch.tensor([1.0, 0.5, 0.0, -0.5])
    x2 = torch.zeros(m2, k)
    x2[:, 0] = 1.0
    wq2, wsf2, wd2, npad2 = _quant_weights(w2)
    xq2, xsf2, xd2 = _quant_act(x2, _pad_rows(m2))
    l2 = (xd2[0] @ wd2[0, :v2].T)[:4]
    keys2 = torch.zeros(m2, 1, dtype=torch.int64, device="cuda")
    C.gemm_mxf8(wq2, wsf2, xq2, xsf2, k, npad2, 4, 1, m2, None, None, None, EPI_ARGMAX, keys2, 1, None, None, None,
                None, 0, 128, 1, 0, 0, 1, None, None, torch.full((m2,), 0.5, device="cuda"),
                torch.full((m2,), 1234, dtype=torch.int64, device="cuda"),
                torch.arange(m2, dtype=torch.int32, device="cuda"), 0)
    ids2 = torch.zeros(m2, dtype=torch.int32, device="cuda")
    C.argmax_reduce(keys2, m2, 1, ids2, None, None)
    freq = torch.bincount(ids2.cpu().long(), minlength=4)[:4].float() / m2
    torch.testing.assert_close(freq, torch.softmax(l2 / 0.5, 0), atol=0.04, rtol=0)


def _split_ws():
    return torch.zeros(8 << 20, device="cuda"), torch.zeros(16384, dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("epi,S,bn", [(EPI_BF16, 4, 128), (EPI_F32, 8, 128), (EPI_BF16, 2, 32), (EPI_ARGMAX, 4, 128)])
def test_gemm_fix_splits_dense(C, epi, S, bn):
    # tiles * S must fit one wave: 640 features = 5 tiles x (2 or 1) token chunks.
    """In-kernel split-K (last CTA reduces) matches the unsplit kernel and the fp32
    reference, is deterministic across calls, and leaves the tile counters at zero."""
    torch.manual_seed(21)
    m = 200 if bn == 128 else 30
    n, k = 640, 1024
    w = torch.randn(1, n, k) * 0.05
    x = torch.randn(m, k)
    wq, wsf, wd, npad = _quant_weights(w)
    xq, xsf, xd = _quant_act(x, _pad_rows(m))
    ws, sem = _split_ws()
    if epi == EPI_ARGMAX:
        ldo = npad // 128
        mk = lambda: torch.zeros(m, ldo, dtype=torch.int64, device="cuda")  # noqa: E731
    else:
        ldo = n
        dt = torch.bfloat16 if epi == EPI_BF16 else torch.float32
        mk = lambda: torch.zeros(m, n, device="cuda", dtype=dt)  # noqa: E731
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    args = (wq, wsf, xq, xsf, k, npad, n, 1, m, None, None, None, epi)
    ref_out = mk()
    C.gemm_mxf8(*args, ref_out, ldo, None, None, None, err, 0, bn, 1, 0, 0)
    outs = []
    for _ in range(2):
        o = mk()
        C.gemm_mxf8(*args, o, ldo, None, None, None, err, 0, bn, 1, 0, 0, S, ws, sem)
        outs.append(o)
    torch.cuda.synchronize()
    assert err.item() == 0
    assert int(sem.abs().sum()) == 0
    assert torch.equal(outs[0], outs[1])
    if epi == EPI_ARGMAX:
        assert torch.equal(outs[0] & 0xFFFFFFFF, ref_out & 0xFFFFFFFF)
    else:
        torch.testing.assert_close(outs[0].float(), ref_out.float(), rtol=2e-3, atol=2e-3)
        expect = xd @ wd[0, :n].T
        torch.testing.assert_close(outs[0].cpu().float(), expect, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("S,bn", [(2, 128), (4, 32)])
def test_gemm_fix_splits_grouped(C, S, bn):
    counts = [0, 7, 130, 16, 1, 45]
    k, n = 512, 256
    s = _grouped_setup(counts, k, n, seed=8)
    pre, c = [0], 0
    for cnt in counts:
        c += (cnt + bn - 1) // bn
        pre.append(c)
    pre = torch.tensor(pre, dtype=torch.int32, device="cuda")
    ws, sem = _split_ws()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.full((s["rows"], n), float("nan"), device="cuda")
    C.gemm_mxf8(s["wq"], s["wsf"], s["xq"], s["xsf"], k, s["npad"], n, len(counts), 0, s["cnt"], s["off"], pre,
                EPI_F32, out, n, None, None, None, err, 0, bn, 1, 0, 0, S, ws, sem)
    torch.cuda.synchronize()
    assert err.item() == 0 and int(sem.abs().sum()) == 0
    out = out.cpu()
    for gi, cnt in enumerate(counts):
        if cnt == 0:
            continue
        o = s["offsets"][gi]
        expect = s["xd"][o:o + cnt] @ s["wd"][gi, :n].T
        torch.testing.assert_close(out[o:o + cnt], expect, rtol=1e-4, atol=1e-3)


def test_gemm_scatter_scaled(C):
    counts = [3, 9]
    k, n = 128, 256
    s = _grouped_setup(counts, k, n, seed=5)
    rows = s["rows"]
    row_dst = torch.full((rows,), -1, dtype=torch.int32)
    row_scale = torch.zeros(rows)
    perm = torch.randperm(12)
    i = 0
    for gi, cnt in enumerate(counts):
        for r in range(cnt):
            row_dst[s["offsets"][gi] + r] = perm[i]
            row_scale[s["offsets"][gi] + r] = 0.5 + i
            i += 1
    out = torch.zeros(12, n, dtype=torch.bfloat16, device="cuda")
    gemm(C,s["wq"], s["wsf"], s["xq"], s["xsf"], k, s["npad"], n, 2, 0, s["cnt"], s["off"],
                s["pre"], EPI_SCATTER, out, n, None, row_dst.cuda(), row_scale.cuda(), None, 0)
    torch.cuda.synchronize()
    out = out.cpu().float()
    for gi, cnt in enumerate(counts):
        for r in range(cnt):
            src = s["offsets"][gi] + r
            expect = (s["xd"][src] @ s["wd"][gi, :n].T) * row_scale[src]
            torch.testing.assert_close(out[row_dst[src]], expect, rtol=1e-2, atol=1e-2)


def test_gemm_argmax_ties(C):
    torch.manual_seed(7)
    m, vocab, k = 37, 1000, 256
    w = torch.randn(1, vocab, k) * 0.05
    w[0, 900] = w[0, 5]  # exact duplicate row -> tie must resolve to id 5
    x = torch.randn(m, k)
    x[3] = w[0, 5] * 40  # make row 3 pick the tied pair
    wq, wsf, wd, npad = _quant_weights(w)
    xq, xsf, xd = _quant_act(x, _pad_rows(m))
    tiles = npad // 128
    keys = torch.zeros(m, tiles, dtype=torch.int64, device="cuda")
    gemm(C,wq, wsf, xq, xsf, k, npad, vocab, 1, m, None, None, None, EPI_ARGMAX, keys, tiles,
                None, None, None, None, 0)
    ids = torch.zeros(m, dtype=torch.int32, device="cuda")
    vals = torch.zeros(m, dtype=torch.float32, device="cuda")
    C.argmax_reduce(keys, m, tiles, ids, vals, None)
    torch.cuda.synchronize()
    logits = xd @ wd[0, :vocab].T
    assert ids[3].item() == 5
    assert torch.equal(ids.cpu().long(), logits.argmax(-1))
    torch.testing.assert_close(vals.cpu(), logits.max(-1).values, rtol=1e-4, atol=1e-3)


def test_quant_bitexact(C):
    torch.manual_seed(0)
    x = (torch.randn(300, 512) * torch.rand(300, 1) * 5).to(torch.bfloat16)
    x[7] = 0
    q = torch.zeros(300, 512, dtype=torch.uint8, device="cuda")
    sf = torch.zeros(mx.atoms_bytes(300, 512), dtype=torch.uint8, device="cuda")
    C.quant_mxf8(x.cuda(), q, sf)
    torch.cuda.synchronize()
    qr, cr = mx.quantize(x.float())
    assert torch.equal(q.cpu(), qr)
    assert torch.equal(mx.codes_from_atoms(sf.cpu(), 300, 512), cr)


def test_add_rmsnorm_quant(C):
    torch.manual_seed(0)
    rows, h, terms = 70, 2048, 3
    res = torch.randn(rows, h).to(torch.bfloat16)
    delta = torch.randn(rows, terms, h).to(torch.bfloat16)
    w = (torch.randn(h) * 0.1).to(torch.bfloat16)
    res_g = res.cuda()
    normed = torch.zeros(rows, h, dtype=torch.bfloat16, device="cuda")
    q = torch.zeros(rows, h, dtype=torch.uint8, device="cuda")
    sf = torch.zeros(mx.atoms_bytes(rows, h), dtype=torch.uint8, device="cuda")
    C.add_rmsnorm_quant(res_g, delta.cuda(), terms, terms * h, h, w.cuda(), 1.0, 1e-6, rows, normed, q, sf)
    torch.cuda.synchronize()
    r_ref, n_ref = ref.add_rmsnorm(res, delta.float().sum(1), w, 1e-6)
    torch.testing.assert_close(res_g.cpu().float(), r_ref, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(normed.cpu().float(), n_ref, rtol=2e-2, atol=2e-2)
    got = mx.dequantize(q.cpu(), mx.codes_from_atoms(sf.cpu(), rows, h))
    torch.testing.assert_close(got, n_ref, rtol=0.07, atol=0.05)


def test_add_rmsnorm_gathered_terms(C):
    """MoE combine: each row adds weighted, gathered rows of the expert output (negative
    index = pair handled elsewhere)."""
    torch.manual_seed(2)
    rows, h, k1, n_src = 40, 2048, 3, 100
    res = torch.randn(rows, h).to(torch.bfloat16)
    y = torch.randn(n_src, h).to(torch.bfloat16)
    idx = torch.randint(-1, n_src, (rows, k1), dtype=torch.int32)
    wts = torch.rand(rows, k1)
    w = (torch.randn(h) * 0.1).to(torch.bfloat16)
    res_g = res.cuda()
    q = torch.zeros(128, h, dtype=torch.uint8, device="cuda")
    sf = torch.zeros(mx.atoms_bytes(128, h), dtype=torch.uint8, device="cuda")
    C.add_rmsnorm_quant(res_g, y.cuda(), k1, h, 0, w.cuda(), 1.0, 1e-6, rows, None, q, sf, idx.cuda(), wts.cuda())
    torch.cuda.synchronize()
    delta = torch.zeros(rows, h)
    for r in range(rows):
        for t in range(k1):
            if idx[r, t] >= 0:
                delta[r] += wts[r, t] * y[idx[r, t]].float()
    r_ref, _ = ref.add_rmsnorm(res, delta, w, 1e-6)
    torch.testing.assert_close(res_g.cpu().float(), r_ref, rtol=1e-2, atol=1e-2)


def _gdn_setup(hk, hv, rows, slots_total, seed=0):
    torch.manual_seed(seed)
    dk = dv = 128
    conv_dim = 2 * hk * dk + hv * dv
    width = conv_dim + hv * dv + 2 * hv
    proj = (torch.randn(rows, width) * 0.5).to(torch.bfloat16)
    conv_w = (torch.randn(conv_dim, 4) * 0.3).to(torch.bfloat16)
    a_log = torch.rand(hv) * 2 - 1
    dt_bias = torch.rand(hv) * 0.5
    norm_w = (1 + 0.1 * torch.randn(dv)).to(torch.bfloat16)
    conv_state = (torch.randn(slots_total, 2, conv_dim, 3) * 0.5).to(torch.bfloat16)
    ssm = torch.randn(slots_total, hv, dv, dk) * 0.1
    return dict(proj=proj, conv_w=conv_w, a_log=a_log, dt_bias=dt_bias, norm_w=norm_w,
                conv_state=conv_state, ssm=ssm, conv_dim=conv_dim)


def test_gdn_decode(C):
    hk, hv, rows = 2, 4, 5
    s = _gdn_setup(hk, hv, rows, 8)
    slots = torch.tensor([3, 0, 7, 5, 1], dtype=torch.int32)
    pos = torch.tensor([10, 0, 3, 1, 6], dtype=torch.int32)
    cs, ssm = s["conv_state"].cuda(), s["ssm"].cuda()
    out = torch.zeros(rows, hv * 128, dtype=torch.bfloat16, device="cuda")
    C.gdn_decode(s["proj"].cuda(), hk, hv, s["conv_w"].cuda(), cs, ssm, s["a_log"].cuda(),
                 s["dt_bias"].cuda(), s["norm_w"].cuda(), 1e-6, slots.cuda(), pos.cuda(), rows,
                 out, None, None, None)
    torch.cuda.synchronize()
    for r in range(rows):
        sl, p = slots[r].item(), pos[r].item()
        win = s["conv_state"][sl, p & 1].float() if p > 0 else torch.zeros(s["conv_dim"], 3)
        st = s["ssm"][sl] if p > 0 else torch.zeros(hv, 128, 128)
        y, win2, st2 = ref.gdn_token(s["proj"][r].float(), win, st, hk=hk, hv=hv, conv_w=s["conv_w"],
                                     a_log=s["a_log"], dt_bias=s["dt_bias"], norm_w=s["norm_w"], eps=1e-6)
        torch.testing.assert_close(out[r].cpu().float(), y, rtol=2e-2, atol=2e-2)
        torch.testing.assert_close(ssm[sl].cpu(), st2, rtol=1e-3, atol=1e-4)
        torch.testing.assert_close(cs[sl, (p + 1) & 1].cpu().float(), win2, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("impl,lens", [(1, [5, 1, 9]), (2, [5, 1, 9]), (2, [150, 1, 70]), (1, [150, 1, 70])])
def test_gdn_prefill_matches_decode_and_checkpoints(C, impl, lens):
    """Token-sequential (impl 1) and chunked (impl 2) prefill against the fp32 per-token
    reference, with a continued sequence and checkpoints inside and across chunks."""
    hk, hv = 2, 4
    rows = sum(lens)
    s = _gdn_setup(hk, hv, rows, 8, seed=1)
    seq_slots = [2, 4, 6]
    starts = [0, 3, 0]  # second sequence continues from position 3
    slots, pos, seq_start = [], [], [0]
    for sl, st, ln in zip(seq_slots, starts, lens):
        slots += [sl] * ln
        pos += list(range(st, st + ln))
        seq_start.append(seq_start[-1] + ln)
    max_ckpt = 2
    ck_rows = torch.full((3, max_ckpt), -1, dtype=torch.int32)
    ck_slots = torch.zeros(3, max_ckpt, dtype=torch.int32)
    ck_rows[0, 0], ck_slots[0, 0] = 2, 7   # after row 2 of seq 0
    ck_rows[2, 0], ck_slots[2, 0] = seq_start[2] + 3, 1  # after the 4th token of seq 2
    if lens[0] > 100:
        ck_rows[0, 1], ck_slots[0, 1] = 127, 5  # a chunk-aligned checkpoint as well
    cs, ssm = s["conv_state"].cuda(), s["ssm"].cuda()
    out = torch.zeros(rows, hv * 128, dtype=torch.bfloat16, device="cuda")
    C.gdn_prefill(s["proj"].cuda(), hk, hv, s["conv_w"].cuda(), cs, ssm, s["a_log"].cuda(),
                  s["dt_bias"].cuda(), s["norm_w"].cuda(), 1e-6, torch.tensor(slots, dtype=torch.int32).cuda(),
                  torch.tensor(pos, dtype=torch.int32).cuda(), rows, out, None, None,
                  torch.tensor(seq_start, dtype=torch.int32).cuda(), 3, ck_rows.cuda(), ck_slots.cuda(),
                  max_ckpt, None, impl=impl)
    torch.cuda.synchronize()
    for si, (sl, st0, ln) in enumerate(zip(seq_slots, starts, lens)):
        win = s["conv_state"][sl, st0 & 1].float() if st0 > 0 else torch.zeros(s["conv_dim"], 3)
        st = s["ssm"][sl] if st0 > 0 else torch.zeros(hv, 128, 128)
        for j in range(ln):
            r = seq_start[si] + j
            y, win, st = ref.gdn_token(s["proj"][r].float(), win, st, hk=hk, hv=hv, conv_w=s["conv_w"],
                                       a_log=s["a_log"], dt_bias=s["dt_bias"], norm_w=s["norm_w"], eps=1e-6)
            torch.testing.assert_close(out[r].cpu().float(), y, rtol=3e-2, atol=3e-2)
            for c in range(max_ckpt):
                if ck_rows[si, c].item() == r:
                    cslot = ck_slots[si, c].item()
                    torch.testing.assert_close(ssm[cslot].cpu(), st, rtol=1e-3, atol=1e-4)
                    torch.testing.assert_close(cs[cslot, (st0 + j + 1) & 1].cpu().float(), win, rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(ssm[sl].cpu(), st, rtol=1e-3, atol=1e-4)


@pytest.mark.parametrize("impl", [1, 2, "rows"])
def test_gdn_prefill_continuation_with_even_rows(C, impl):
    """Sequences that continue from position 5 with an even number of new rows (a chunked
    prefill continuation, a speculative replay of 2 or 4 rows).  Their q/k conv window ends
    in the parity buffer it is read from; with 160 sequences the value heads of one q/k
    group run waves apart, so a window written by the first of them before the others had
    read it would show up here.  impl 1 token-sequential, 2 chunked, "rows" the streaming
    kernel over row groups.  Outputs, final states and every final conv window against the
    fp32 per-token reference."""
    hk, hv = 2, 4
    n, p0 = 160, 5
    lens = [2 if i % 2 else 4 for i in range(n)]
    rows = sum(lens)
    s = _gdn_setup(hk, hv, rows, n, seed=3)
    slots, pos, seq_start = [], [], [0]
    for i, ln in enumerate(lens):
        slots += [i] * ln
        pos += list(range(p0, p0 + ln))
        seq_start.append(seq_start[-1] + ln)
    cs, ssm = s["conv_state"].cuda(), s["ssm"].cuda()
    out = torch.zeros(rows, hv * 128, dtype=torch.bfloat16, device="cuda")
    C.gdn_prefill(s["proj"].cuda(), hk, hv, s["conv_w"].cuda(), cs, ssm, s["a_log"].cuda(),
                  s["dt_bias"].cuda(), s["norm_w"].cuda(), 1e-6, torch.tensor(slots, dtype=torch.int32).cuda(),
                  torch.tensor(pos, dtype=torch.int32).cuda(), rows, out, None, None,
                  torch.tensor(seq_start, dtype=torch.int32).cuda(), n, None, None, 0, None,
                  impl=0 if impl == "rows" else impl, max_seq_rows=4 if impl == "rows" else 0)
    torch.cuda.synchronize()
    out, cs, ssm = out.cpu().float(), cs.cpu().float(), ssm.cpu()
    for i, ln in enumerate(lens):
        win = s["conv_state"][i, p0 & 1].float()
        st = s["ssm"][i]
        for j in range(ln):
            r = seq_start[i] + j
            y, win, st = ref.gdn_token(s["proj"][r].float(), win, st, hk=hk, hv=hv, conv_w=s["conv_w"],
                                       a_log=s["a_log"], dt_bias=s["dt_bias"], norm_w=s["norm_w"], eps=1e-6)
            torch.testing.assert_close(out[r], y, rtol=3e-2, atol=3e-2)
        torch.testing.assert_close(ssm[i], st, rtol=1e-3, atol=1e-4)
        torch.testing.assert_close(cs[i, (p0 + ln) & 1], win, rtol=1e-2, atol=1e-2)


def test_gdn_rows_streaming_kernel_with_out_slots(C):
    """The streaming GDN kernel over row groups (a speculative verify pass: the last token +
    drafts of each sequence, 1 to 4 rows, some sequences fresh): outputs per row against the
    fp32 reference, the final state and conv windows in out_slots[seq] for the sequences
    that have one (the input slot untouched), in place for the others."""
    hk, hv = 2, 4
    lens = [1, 2, 3, 4] * 40
    n = len(lens)
    starts_pos = [0 if i % 7 == 0 else 3 + i % 5 for i in range(n)]
    rows = sum(lens)
    s = _gdn_setup(hk, hv, rows, 2 * n, seed=5)
    slots, pos, seq_start = [], [], [0]
    for i, ln in enumerate(lens):
        slots += [i] * ln
        pos += list(range(starts_pos[i], starts_pos[i] + ln))
        seq_start.append(seq_start[-1] + ln)
    out_slots = [n + i if i % 2 == 0 else i for i in range(n)]
    cs, ssm = s["conv_state"].cuda(), s["ssm"].cuda()
    out = torch.zeros(rows, hv * 128, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.gdn_prefill(s["proj"].cuda(), hk, hv, s["conv_w"].cuda(), cs, ssm, s["a_log"].cuda(),
                  s["dt_bias"].cuda(), s["norm_w"].cuda(), 1e-6, torch.tensor(slots, dtype=torch.int32).cuda(),
                  torch.tensor(pos, dtype=torch.int32).cuda(), rows, out, None, None,
                  torch.tensor(seq_start, dtype=torch.int32).cuda(), n, None, None, 0, err,
                  torch.tensor(out_slots, dtype=torch.int32).cuda(), impl=0, max_seq_rows=4)
    torch.cuda.synchronize()
    assert err.item() == 0
    out, cs, ssm = out.cpu().float(), cs.cpu().float(), ssm.cpu()
    for i, ln in enumerate(lens):
        p0 = starts_pos[i]
        win = s["conv_state"][i, p0 & 1].float() if p0 > 0 else torch.zeros(s["conv_dim"], 3)
        st = s["ssm"][i] if p0 > 0 else torch.zeros(hv, 128, 128)
        for j in range(ln):
            r = seq_start[i] + j
            y, win, st = ref.gdn_token(s["proj"][r].float(), win, st, hk=hk, hv=hv, conv_w=s["conv_w"],
                                       a_log=s["a_log"], dt_bias=s["dt_bias"], norm_w=s["norm_w"], eps=1e-6)
            torch.testing.assert_close(out[r], y, rtol=3e-2, atol=3e-2)
        o = out_slots[i]
        torch.testing.assert_close(ssm[o], st, rtol=1e-3, atol=1e-4)
        torch.testing.assert_close(cs[o, (p0 + ln) & 1], win, rtol=1e-2, atol=1e-2)
        if o != i:
            torch.testing.assert_close(ssm[i], s["ssm"][i])


def test_attention_prologue_and_decode(C):
    torch.manual_seed(0)
    hq, hkv, d, page = 8, 2, 256, 16
    rows = 3
    ctx = [40, 1, 17]
    max_pages = 4
    pages_total = 16
    qkv_w = hq * 2 * d + 2 * hkv * d
    page_table = torch.tensor([[3, 9, 5, 0], [1, 0, 0, 0], [12, 2, 0, 0]], dtype=torch.int32)
    slots = torch.arange(rows, dtype=torch.int32)
    kc = (torch.randn(pages_total, hkv, page, d) * 0.5).to(torch.bfloat16)
    vc = (torch.randn(pages_total, hkv, page, d) * 0.5).to(torch.bfloat16)
    qkv = (torch.randn(rows, qkv_w)).to(torch.bfloat16)
    qn = (0.1 * torch.randn(d)).to(torch.bfloat16)
    kn = (0.1 * torch.randn(d)).to(torch.bfloat16)
    pos = torch.tensor([c - 1 for c in ctx], dtype=torch.int32)
    kc_g, vc_g = swizzle_pages(kc).cuda(), swizzle_pages(vc).cuda()
    q_out = torch.zeros(rows, hq, d, dtype=torch.bfloat16, device="cuda")
    g_out = torch.zeros(rows, hq, d, dtype=torch.bfloat16, device="cuda")
    C.attn_prologue(qkv.cuda(), hq, hkv, 64, 1e7, qn.cuda(), kn.cuda(), 1e-6, kc_g, vc_g, page,
                    page_table.cuda(), slots.cuda(), pos.cuda(), rows, q_out, g_out)
    splits = 3
    partial = torch.zeros(rows * hq * splits * 260, device="cuda")
    out = torch.zeros(rows, hq * d, dtype=torch.bfloat16, device="cuda")
    sm = 1 / math.sqrt(d)
    C.attn_decode(q_out, g_out, hq, hkv, kc_g, vc_g, page, page_table.cuda(), slots.cuda(),
                  torch.tensor(ctx, dtype=torch.int32).cuda(), rows, partial, splits, sm, out, None, None)
    torch.cuda.synchronize()
    kc_rows, vc_rows = unswizzle_pages(kc_g.cpu()), unswizzle_pages(vc_g.cpu())
    for r in range(rows):
        q, gate, k_new, v_new = ref.attn_prologue_row(qkv[r].float(), pos[r].item(), hq=hq, hkv=hkv,
                                                      q_norm_w=qn, k_norm_w=kn, eps=1e-6, rotary_dim=64,
                                                      theta=1e7)
        torch.testing.assert_close(q_out[r].cpu().float(), q, rtol=2e-2, atol=2e-2)
        p_last = pos[r].item()
        pg = page_table[r, p_last // page].item()
        torch.testing.assert_close(kc_rows[pg, :, p_last % page].float(), k_new, rtol=2e-2, atol=2e-2)
        keys = torch.stack([kc_rows[page_table[r, t // page], :, t % page].float() for t in range(ctx[r])])
        vals = torch.stack([vc_rows[page_table[r, t // page], :, t % page].float() for t in range(ctx[r])])
        expect = ref.gated_attention(q_out[r].cpu().float(), g_out[r].cpu().float(), keys, vals, sm)
        torch.testing.assert_close(out[r].cpu().float(), expect, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("hq,hkv,splits,reps", [(16, 2, 1, 1), (16, 2, 3, 1), (2, 1, 2, 1), (16, 1, 1, 1),
                                                 (16, 2, 1, 24), (16, 2, 3, 8), (2, 1, 1, 24)])
def test_attention_decode_tensor_core(C, hq, hkv, splits, reps):
    """The tcgen05 split-KV decode (128-key tiles of bulk-copied pre-swizzled pages, online
    softmax with TMEM rescale) and the SIMT kernel (impl 1; impl 2 forces tensor cores for
    the 2-head group) against the fp32 reference, over contexts that end mid-page, mid-tile,
    on tile boundaries and inside one page, and splits without pages; group sizes 8, 2 and
    16.  reps > 1 repeats the context list for more CTAs than SMs."""
    g = torch.Generator().manual_seed(7)
    d, page = 256, 16
    ctx = [1, 16, 37, 128, 129, 300, 511] * reps
    rows = len(ctx)
    max_pages = 33
    pages_total = rows * max_pages + 1
    perm = torch.randperm(pages_total - 1, generator=g) + 1
    table = perm.view(rows, max_pages).to(torch.int32)
    kc = (torch.randn(pages_total, hkv, page, d, generator=g) * 0.5).to(torch.bfloat16)
    vc = (torch.randn(pages_total, hkv, page, d, generator=g) * 0.5).to(torch.bfloat16)
    q = torch.randn(rows, hq, d, generator=g).to(torch.bfloat16)
    gate = torch.randn(rows, hq, d, generator=g).to(torch.bfloat16)
    sm = 1 / math.sqrt(d)
    dev = lambda t: t.cuda()  # noqa: E731
    outs = {}
    for impl in ((0, 1, 2) if hq // hkv <= 8 else (0,)):
        partial = torch.zeros(rows * hq * splits * 260, device="cuda")
        out = torch.zeros(rows, hq * d, dtype=torch.bfloat16, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        C.attn_decode(dev(q), dev(gate), hq, hkv, dev(swizzle_pages(kc)), dev(swizzle_pages(vc)), page, dev(table),
                      torch.arange(rows, dtype=torch.int32, device="cuda"), torch.tensor(ctx, dtype=torch.int32).cuda(),
                      rows, partial, splits, sm, out, None, None, impl=impl, err=err)
        torch.cuda.synchronize()
        assert err.item() == 0
        outs[impl] = out.cpu().float()
    grp = hq // hkv
    for r in range(rows):
        keys = torch.stack([kc[table[r, t // page], :, t % page].float() for t in range(ctx[r])])
        vals = torch.stack([vc[table[r, t // page], :, t % page].float() for t in range(ctx[r])])
        expect = ref.gated_attention(q[r].float(), gate[r].float(), keys, vals, sm)
        for impl in outs:
            torch.testing.assert_close(outs[impl][r], expect, rtol=2e-2, atol=2e-2)
    del grp


@pytest.mark.parametrize("hq,hkv,splits,impl", [(16, 2, 1, 0), (16, 2, 3, 0), (2, 1, 2, 2), (16, 1, 1, 0),
                                                 (4, 1, 1, 0)])
def test_attention_varlen_multi_row_items(C, hq, hkv, splits, impl):
    """Varlen attention with sequence boundaries (prefill / speculative verify): the
    tensor-core kernel packs up to 32 / G consecutive query rows of a sequence into one
    work item (32 query slots sharing each K/V tile), each slot masked by its own causal
    length.  Sequences of 1, 4, 5, 37 and 130 new rows after 0 to 300 cached tokens, and
    more items than SMs, against the fp32 reference row by row, with and without the
    sequence boundaries."""
    g = torch.Generator().manual_seed(11)
    d, page = 256, 16
    seqs = [(0, 37), (300, 4), (17, 1), (128, 130), (5, 5)] * 3 + [(90, 4)] * 40  # (cached, new rows)
    max_pages = 33
    n = len(seqs)
    pages_total = n * max_pages + 1
    perm = torch.randperm(pages_total - 1, generator=g) + 1
    table = perm.view(n, max_pages).to(torch.int32)
    kc = (torch.randn(pages_total, hkv, page, d, generator=g) * 0.5).to(torch.bfloat16)
    vc = (torch.randn(pages_total, hkv, page, d, generator=g) * 0.5).to(torch.bfloat16)
    slots, lens, starts = [], [], [0]
    for i, (cached, new) in enumerate(seqs):
        slots += [i] * new
        lens += [cached + j + 1 for j in range(new)]
        starts.append(starts[-1] + new)
    rows = len(lens)
    q = torch.randn(rows, hq, d, generator=g).to(torch.bfloat16)
    gate = torch.randn(rows, hq, d, generator=g).to(torch.bfloat16)
    sm = 1 / math.sqrt(d)
    dev = lambda x: x.cuda()  # noqa: E731
    outs = {}
    for mode in ("grouped", "per_row"):
        partial = torch.zeros(rows * hq * splits * 260, device="cuda")
        out = torch.zeros(rows, hq * d, dtype=torch.bfloat16, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        ss = torch.tensor(starts, dtype=torch.int32, device="cuda") if mode == "grouped" else None
        C.attn_decode(dev(q), dev(gate), hq, hkv, dev(swizzle_pages(kc)), dev(swizzle_pages(vc)), page, dev(table),
                      torch.tensor(slots, dtype=torch.int32, device="cuda"), torch.tensor(lens, dtype=torch.int32).cuda(),
                      rows, partial, splits, sm, out, None, None, impl=impl, err=err, seq_start=ss,
                      num_seqs=n if ss is not None else 0)
        torch.cuda.synchronize()
        assert err.item() == 0
        outs[mode] = out.cpu().float()
    for i, (cached, new) in enumerate(seqs):
        tot = cached + new
        keys_all = torch.stack([kc[table[i, t // page], :, t % page].float() for t in range(tot)])
        vals_all = torch.stack([vc[table[i, t // page], :, t % page].float() for t in range(tot)])
        for r in range(starts[i], starts[i + 1]):
            L = lens[r]
            expect = ref.gated_attention(q[r].float(), gate[r].float(), keys_all[:L], vals_all[:L], sm)
            torch.testing.assert_close(outs["grouped"][r], expect, rtol=2e-2, atol=2e-2)
            torch.testing.assert_close(outs["per_row"][r], expect, rtol=2e-2, atol=2e-2)


def _sample(C, logits, temp, top_k, top_p, seeds, hist=None, pres=None, freq=None, rep=None, top_n=0):
    n, v = logits.shape
    dev = "cuda"
    f = lambda x, d=0.0: torch.full((n,), d, dtype=torch.float32, device=dev) if x is None else \
        torch.as_tensor(x, dtype=torch.float32, device=dev)  # noqa: E731
    lg = logits.clone().float().to(dev)
    tok = torch.zeros(n, dtype=torch.int32, device=dev)
    lp = torch.zeros(n, device=dev) if top_n else None
    tids = torch.zeros(n, 5, dtype=torch.int32, device=dev) if top_n else None
    tlps = torch.zeros(n, 5, device=dev) if top_n else None
    if hist is None:
        h, hl = None, None
    else:
        h = torch.zeros(n, 4096, dtype=torch.int32, device=dev)
        hl = torch.zeros(n, dtype=torch.int32, device=dev)
        for i, row in enumerate(hist):
            h[i, :len(row)] = torch.tensor(row, dtype=torch.int32)
            hl[i] = len(row)
    C.sample(lg, v, n, f(temp), torch.as_tensor(top_k, dtype=torch.int32, device=dev), f(top_p, 1.0), f(pres),
             f(freq), f(rep, 1.0), torch.as_tensor(seeds, dtype=torch.int64, device=dev), h, hl, top_n, tok, lp, tids,
             tlps)
    torch.cuda.synchronize()
    return tok.cpu(), (lp.cpu() if top_n else None), (tids.cpu() if top_n else None), (tlps.cpu() if top_n else None)


def test_sample_kernel_exact_cases(C):
    """Greedy (with penalties), top-k = 1, a tiny top-p and log-probabilities are exact."""
    from zstep_b200.sampling import apply_penalties

    g = torch.Generator().manual_seed(3)
    n, v = 6, 50000
    logits = torch.randn(n, v, generator=g) * 3
    hist = [[1, 2, 2, 7], [], [int(logits[2].argmax())] * 3, [5], [9, 9], [int(logits[5].argmax())]]
    pres, freq, rep = [0.5, 0, 2.0, 0, 0.3, 0], [0.3, 0, 1.0, 0, 0.2, 0], [1.2, 1, 1, 1.5, 1, 2.0]
    tok, lp, tids, tlps = _sample(C, logits, [0.0] * n, [0] * n, [1.0] * n, list(range(n)), hist=hist, pres=pres,
                                  freq=freq, rep=rep, top_n=5)
    for i in range(n):
        pen = apply_penalties(logits[i], hist[i], pres[i], freq[i], rep[i])
        assert int(tok[i]) == int(pen.argmax()), i
        ref_lp = torch.log_softmax(logits[i].double(), 0)
        assert abs(float(lp[i]) - float(ref_lp[int(tok[i])])) < 1e-4
        top = torch.topk(logits[i], 5)
        assert tids[i].tolist() == top.indices.tolist()
        torch.testing.assert_close(tlps[i].double(), ref_lp[top.indices], rtol=0, atol=1e-4)
    tok, *_ = _sample(C, logits, [0.8] * n, [1] * n, [1.0] * n, list(range(n)))
    assert tok.tolist() == logits.argmax(-1).tolist()
    tok, *_ = _sample(C, logits, [0.8] * n, [0] * n, [1e-6] * n, list(range(n)))
    assert tok.tolist() == logits.argmax(-1).tolist()


def test_sample_kernel_distribution_and_determinism(C):
    """Many seeds over one row: every draw lies in the top-k / top-p kept set and the
    frequencies follow the renormalised truncated softmax; a seed reproduces its draw."""
    g = torch.Generator().manual_seed(4)
    v, n = 300, 6000
    row = torch.randn(v, generator=g) * 2
    temp, k, p = 0.7, 20, 0.8
    logits = row.expand(n, v).contiguous()
    seeds = torch.arange(n, dtype=torch.int64) * 7919 + 11
    tok, *_ = _sample(C, logits, [temp] * n, [k] * n, [p] * n, seeds)
    tok2, *_ = _sample(C, logits, [temp] * n, [k] * n, [p] * n, seeds)
    assert torch.equal(tok, tok2)
    s = row / temp
    vals, idx = torch.sort(s, descending=True)
    probs = torch.softmax(vals[:k].double(), 0)
    prior = torch.cumsum(probs, 0) - probs
    keep = int((prior < p).sum())
    kept = set(idx[:keep].tolist())
    assert set(tok.tolist()) <= kept
    want = probs[:keep] / probs[:keep].sum()
    counts = torch.bincount(tok.long(), minlength=v).double()[idx[:keep]] / n
    assert float((counts - want).abs().max()) < 0.03, (counts, want)


def test_moe_route_softmax_shared(C):
    torch.manual_seed(0)
    rows, E, k, hidden = 50, 64, 4, 256
    logits = torch.randn(rows, E + 1)
    x = torch.randn(rows, hidden)
    xq, xsf, _ = _quant_act(x, _pad_rows(rows))
    G = E + 1
    max_rows = rows * (k + 1) + 128 * G
    dev = dict(device="cuda")
    topk_ids = torch.zeros(rows, k, dtype=torch.int32, **dev)
    topk_w = torch.zeros(rows, k, **dev)
    cnt = torch.zeros(G, dtype=torch.int32, **dev)
    off = torch.zeros(G, dtype=torch.int32, **dev)
    pre = torch.zeros(G + 1, dtype=torch.int32, **dev)
    pair_slot = torch.zeros(rows, k + 1, dtype=torch.int32, **dev)
    row_dst = torch.full((max_rows,), -1, dtype=torch.int32, **dev)
    row_scale = torch.zeros(max_rows, **dev)
    xg = torch.zeros(max_rows, hidden, dtype=torch.uint8, **dev)
    xg_sf = torch.zeros(mx.atoms_bytes(max_rows, hidden), dtype=torch.uint8, **dev)
    err = torch.zeros(1, dtype=torch.int32, **dev)
    route(C,logits.cuda(), rows, E, k, True, 0, None, 1, 1, 1.0, E, 0, E, True, topk_ids, topk_w,
                cnt, off, pre, pair_slot, row_dst, row_scale, xq, xsf, xg, xg_sf, err)
    torch.cuda.synchronize()
    assert err.item() == 0
    ids_ref, w_ref = ref.route(logits[:, :E], top_k=k)
    assert torch.equal(topk_ids.cpu().long(), ids_ref)
    torch.testing.assert_close(topk_w.cpu(), w_ref, rtol=1e-5, atol=1e-6)
    counts = torch.bincount(ids_ref.reshape(-1), minlength=E).tolist() + [rows]
    assert cnt.cpu().tolist() == counts
    xg_c, rd, rs = xg.cpu(), row_dst.cpu(), row_scale.cpu()
    codes = mx.codes_from_atoms(xg_sf.cpu(), max_rows, hidden)
    codes_x = mx.codes_from_atoms(xsf.cpu(), rows, hidden)
    offs = off.cpu().tolist()
    for g in range(G):
        for j in range(counts[g]):
            gr = offs[g] + j
            tok, slot = divmod(rd[gr].item(), k + 1)
            assert torch.equal(xg_c[gr], xq.cpu()[tok])
            assert torch.equal(codes[gr], codes_x[tok])
            if slot < k:
                assert ids_ref[tok, slot].item() == g
                assert abs(rs[gr].item() - w_ref[tok, slot].item()) < 1e-6
            else:
                assert g == E
                assert abs(rs[gr].item() - torch.sigmoid(logits[tok, E]).item()) < 1e-6


@pytest.mark.parametrize("scoring", ["sigmoid", "sqrtsoftplus"])
def test_moe_route_sigmoid_grouped(C, scoring):
    torch.manual_seed(1)
    rows, E, k, hidden, ng, tg = 20, 64, 6, 128, 8, 3
    logits = torch.randn(rows, E)
    bias = torch.randn(E) * 0.1
    x = torch.randn(rows, hidden)
    xq, xsf, _ = _quant_act(x, _pad_rows(rows))
    max_rows = rows * (k + 1) + 128 * E
    dev = dict(device="cuda")
    out = [torch.zeros(rows, k, dtype=torch.int32, **dev), torch.zeros(rows, k, **dev)]
    mode = {"sigmoid": 1, "sqrtsoftplus": 2}[scoring]
    route(C,logits.cuda(), rows, E, k, True, mode, bias.cuda(), ng, tg, 2.5, -1, 0, E, False, out[0], out[1],
                torch.zeros(E, dtype=torch.int32, **dev), torch.zeros(E, dtype=torch.int32, **dev),
                torch.zeros(E + 1, dtype=torch.int32, **dev), torch.zeros(rows, k + 1, dtype=torch.int32, **dev),
                torch.zeros(max_rows, dtype=torch.int32, **dev), torch.zeros(max_rows, **dev), xq, xsf,
                torch.zeros(max_rows, hidden, dtype=torch.uint8, **dev),
                torch.zeros(mx.atoms_bytes(max_rows, hidden), dtype=torch.uint8, **dev), None)
    torch.cuda.synchronize()
    ids_ref, w_ref = ref.route(logits, top_k=k, scoring=scoring, bias=bias, n_group=ng, topk_group=tg,
                               routed_scale=2.5)
    assert torch.equal(out[0].cpu().long(), ids_ref)
    torch.testing.assert_close(out[1].cpu(), w_ref, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("n,k", [(1, 1), (5, 3), (37, 7)])
def test_spec_verify_kernel(C, n, k):
    """On-device greedy verify: accept length, accepted tokens, compacted replay rows and
    the draft head's catch-up rows against a host restatement."""
    g = torch.Generator().manual_seed(n * 10 + k)
    K1 = k + 1
    R = n * K1
    targets = torch.randint(0, 50, (R,), generator=g, dtype=torch.int32)
    ids = torch.randint(0, 50, (R,), generator=g, dtype=torch.int32)
    # Make sequence i's drafts match the targets for its first i % K1 positions.
    for i in range(n):
        m = i % K1
        for j in range(m):
            ids[i * K1 + j + 1] = targets[i * K1 + j]
        if m < k:
            ids[i * K1 + m + 1] = (targets[i * K1 + m] + 1) % 50
    pos = torch.arange(R, dtype=torch.int32) + 100
    slot = torch.tensor([i for i in range(n) for _ in range(K1)], dtype=torch.int32)
    dev = lambda t: t.cuda()  # noqa: E731
    i32 = lambda m: torch.full((m,), -7, dtype=torch.int32, device="cuda")  # noqa: E731
    rec = torch.full((n, k + 2), -7, dtype=torch.int32, device="cuda")
    rep_start, rep_idx = i32(n + 1), torch.full((R,), -7, dtype=torch.int64, device="cuda")
    rep_slot, rep_pos = i32(R), i32(R)
    m_ids, m_pos, m_slot, m_len = i32(R), i32(R), i32(R), i32(R)
    last = torch.full((n,), -7, dtype=torch.int64, device="cuda")
    dummy = 999
    C.spec_verify(n, k, dummy, dev(ids), dev(targets), dev(pos), dev(slot), rec, rep_start, rep_idx, rep_slot,
                  rep_pos, m_ids, m_pos, m_slot, m_len, last)
    torch.cuda.synchronize()
    rec, rep_start, rep_idx = rec.cpu(), rep_start.cpu(), rep_idx.cpu()
    start = 0
    for i in range(n):
        acc = min(i % K1, k) + 1
        assert int(rec[i, 0]) == acc
        assert rec[i, 1:1 + acc].tolist() == targets[i * K1:i * K1 + acc].tolist()
        assert all(int(x) == -1 for x in rec[i, 1 + acc:])
        assert int(rep_start[i]) == start
        assert rep_idx[start:start + acc].tolist() == list(range(i * K1, i * K1 + acc))
        assert rep_slot.cpu()[start:start + acc].tolist() == [i] * acc
        assert rep_pos.cpu()[start:start + acc].tolist() == pos[i * K1:i * K1 + acc].tolist()
        for j in range(K1):
            r = i * K1 + j
            if j < acc:
                assert (int(m_ids[r]), int(m_pos[r]), int(m_slot[r]), int(m_len[r])) == \
                    (int(targets[r]), int(pos[r]), i, int(pos[r]) + 1)
            else:
                assert int(m_slot[r]) == dummy
        assert int(last[i]) == i * K1 + acc - 1
        start += acc
    assert int(rep_start[n]) == start
