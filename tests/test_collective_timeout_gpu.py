"""Bounded cross-rank waits of the fused all-reduce, on one GPU.

The kernel runs as rank 0 of a 2-rank group whose "peer" block is a second buffer on the
same GPU that nothing ever writes: every wait for the peer's data must give up after the
call's timeout, record kErrPeerTimeout (2) in the error word and return, leaving the CUDA
context usable.  No GPU fault, trap or endless loop is involved: the missing peer is a
flag that nothing sets."""

import time

import pytest
import torch

from zstep_b200.ops import _ext, mx
from zstep_b200.parallel.fused import FAR_CTAS, FAR_ONESHOT_ROWS, ONESHOT, PLAIN, TWOSHOT

pytestmark = pytest.mark.gpu

H, R, W = 2048, 32, 2


def _areas(proto):
    """Byte sizes of (part, out, flags) for one rank in a W-rank group."""
    if proto == ONESHOT:
        return 2 * W * FAR_ONESHOT_ROWS * H * 4, 0, 0
    if proto == TWOSHOT:
        return (R + W) * H * 4, R * H * 4, 0
    return (R + W) * H * 2, R * H * 2, 2 * 8 * FAR_CTAS * 4


@pytest.mark.parametrize("proto", [ONESHOT, TWOSHOT, PLAIN], ids=["oneshot", "twoshot_ll", "plain"])
def test_missing_peer_times_out_and_context_survives(proto):
    C = _ext.load()
    part_b, out_b, flag_b = _areas(proto)
    blocks = [torch.zeros(part_b + out_b + flag_b + 256, dtype=torch.uint8, device="cuda") for _ in range(W)]
    base = [b.data_ptr() for b in blocks]
    part = [p for p in base]
    out = [p + part_b for p in base] if out_b else []
    flags = [p + part_b + out_b for p in base] if flag_b else []
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    grid = torch.zeros(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    delta = torch.randn(R, H, device="cuda").to(torch.bfloat16)
    hidden = torch.zeros(R, H, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    xq = torch.zeros(128, H, dtype=torch.uint8, device="cuda")
    xsf = torch.zeros(mx.atoms_bytes(128, H), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    t0 = time.time()
    C.fused_allreduce_norm(0, W, proto, delta, 1, H, 0, part, out, flags, epoch, grid, hidden, w, 1.0, 1e-6, R,
                           None, xq, xsf, err, None, None, 50)
    torch.cuda.synchronize()
    assert time.time() - t0 < 5.0
    assert int(err.item()) == 2
    # The call finished (its epoch advanced) and the context still runs kernels: the same
    # buffers as a one-rank group reduce correctly afterwards.
    assert int(epoch.item()) == 1 and int(grid.item()) == 0
    err.zero_()
    hidden.zero_()
    C.fused_allreduce_norm(0, 1, proto, delta, 1, H, 0, part[:1], out[:1], flags[:1], epoch, grid, hidden, w, 1.0,
                           1e-6, R, None, xq, xsf, err, None, None, 50)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(hidden, delta)
