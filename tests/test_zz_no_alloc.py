"""The allocation-free attention decode entry point, called through its C symbol.

``zs_attn_decode_noalloc`` must give the same output as ``zs_attn_decode`` (which takes a
caller-allocated scratch buffer) on the same inputs, on two calls in a row (the second
call reuses the library's fixed scratch array), and must reject a call whose scratch
need exceeds the fixed size without launching anything."""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p
I = ctypes.c_int
F = ctypes.c_float


class AttnArgs(ctypes.Structure):
    """Mirror of the C struct AttnArgs in csrc/kernels/zs_kernels.h (field order matters)."""

    _fields_ = [("qkv", P), ("ld_qkv", I), ("num_q_heads", I), ("num_kv_heads", I), ("head_dim", I),
                ("rotary_dim", I), ("rope_theta", F), ("q_norm_w", P), ("k_norm_w", P), ("eps", F),
                ("k_cache", P), ("v_cache", P), ("page_size", I), ("page_table", P), ("max_pages", I),
                ("slots", P), ("positions", P), ("rows", I), ("q_out", P), ("gate_out", P), ("seq_lens", P),
                ("partial", P), ("num_splits", I), ("sm_scale", F), ("out_bf16", P), ("out_q", P), ("out_sf", P),
                ("seq_start", P), ("num_seqs", I), ("err", P), ("impl", I)]


def _lib():
    from zstep_b200.ops import _ext

    C = _ext.load()
    lib = ctypes.CDLL(C.__file__)
    fn = lib.zs_attn_decode_noalloc
    fn.argtypes = [ctypes.POINTER(AttnArgs), P]
    fn.restype = I
    return C, fn


def _case(rows=5, hq=8, hkv=2, splits=4, seed=0, max_ctx=None):
    g = torch.Generator().manual_seed(seed)
    d, page, max_pages, pages_total = 256, 16, 8, 48
    hi = max_ctx if max_ctx is not None else max_pages * page
    ctx = [1 + int(x) for x in torch.randint(0, hi, (rows,), generator=g)]
    perm = torch.randperm(pages_total - 1, generator=g) + 1
    table = perm[: rows * max_pages].view(rows, max_pages).to(torch.int32) if rows * max_pages <= pages_total - 1 \
        else (perm.repeat((rows * max_pages) // (pages_total - 1) + 1)[: rows * max_pages]).view(rows, max_pages).to(
            torch.int32)
    t = dict(
        q=(torch.randn(rows, hq, d, generator=g)).to(torch.bfloat16).cuda(),
        gate=(torch.randn(rows, hq, d, generator=g)).to(torch.bfloat16).cuda(),
        kc=(0.5 * torch.randn(pages_total, hkv, page, d, generator=g)).to(torch.bfloat16).cuda(),
        vc=(0.5 * torch.randn(pages_total, hkv, page, d, generator=g)).to(torch.bfloat16).cuda(),
        table=table.cuda(),
        slots=torch.arange(rows, dtype=torch.int32).cuda(),
        lens=torch.tensor(ctx, dtype=torch.int32).cuda(),
    )
    return t, dict(rows=rows, hq=hq, hkv=hkv, splits=splits, page=page, max_pages=max_pages)


def _args(t, c, out, impl):
    a = AttnArgs()
    a.num_q_heads, a.num_kv_heads, a.head_dim = c["hq"], c["hkv"], 256
    a.k_cache, a.v_cache = t["kc"].data_ptr(), t["vc"].data_ptr()
    a.page_size, a.page_table, a.max_pages = c["page"], t["table"].data_ptr(), c["max_pages"]
    a.slots, a.seq_lens, a.rows = t["slots"].data_ptr(), t["lens"].data_ptr(), c["rows"]
    a.q_out, a.gate_out = t["q"].data_ptr(), t["gate"].data_ptr()
    a.num_splits, a.sm_scale = c["splits"], 1.0 / math.sqrt(256)
    a.out_bf16 = out.data_ptr()
    a.impl = impl
    return a


def _reference(C, t, c, impl):
    """The existing entry point, with a caller-allocated scratch buffer."""
    rows, hq = c["rows"], c["hq"]
    ref = torch.zeros(rows, hq * 256, dtype=torch.bfloat16, device="cuda")
    partial = torch.zeros(rows * hq * c["splits"] * 260, device="cuda")
    C.attn_decode(t["q"], t["gate"], hq, c["hkv"], t["kc"], t["vc"], c["page"], t["table"], t["slots"], t["lens"],
                  rows, partial, c["splits"], 1.0 / math.sqrt(256), ref, None, None, impl)
    return ref


def _noalloc(fn, t, c, impl):
    out = torch.full((c["rows"], c["hq"] * 256), float("nan"), dtype=torch.bfloat16, device="cuda")
    args = _args(t, c, out, impl)
    assert fn(ctypes.byref(args), P(torch.cuda.current_stream().cuda_stream)) == 0
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("impl", [0, 1], ids=["tcgen05", "simt"])
def test_noalloc_matches_existing_entry_point_twice(impl):
    C, fn = _lib()
    t, c = _case()
    ref = _reference(C, t, c, impl)
    for _ in range(2):
        torch.testing.assert_close(_noalloc(fn, t, c, impl), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("impl", [0, 1], ids=["tcgen05", "simt"])
def test_noalloc_splits_without_pages_after_a_larger_call(impl):
    """A large call fills the shared array; a smaller call whose later splits own no pages
    (short contexts, 8 splits) must not pick up the large call's records."""
    C, fn = _lib()
    big_t, big_c = _case(rows=64, splits=8, seed=3)
    torch.testing.assert_close(_noalloc(fn, big_t, big_c, impl), _reference(C, big_t, big_c, impl), rtol=1e-2,
                               atol=1e-2)
    t, c = _case(rows=7, splits=8, seed=4, max_ctx=40)  # at most 3 pages: splits 3..7 are empty
    ref = _reference(C, t, c, impl)
    for _ in range(2):
        torch.testing.assert_close(_noalloc(fn, t, c, impl), ref, rtol=1e-2, atol=1e-2)


def test_noalloc_rejects_oversized_call():
    _, fn = _lib()
    t, c = _case(rows=2)
    out = torch.zeros(2, c["hq"] * 256, dtype=torch.bfloat16, device="cuda")
    stream = P(torch.cuda.current_stream().cuda_stream)
    args = _args(t, c, out, 0)
    args.rows = 4096  # 4096 * 8 heads * 4 splits * 260 floats > the fixed 2M-float array
    assert fn(ctypes.byref(args), stream) == -3
    args.rows, args.num_q_heads, args.num_splits = 2 ** 30, 2 ** 30, 8  # products that wrap a 64-bit size
    assert fn(ctypes.byref(args), stream) == -3
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0
