"""Storage order of the paged K/V cache of the GQA attention kernels.

A (page, kv head) block holds 16 token rows x 256 dims of bf16 (8 KiB).  It is stored as
two halves of 8 rows; each half as four 64-dim chunks of 8 rows x 128 bytes; inside a
chunk the 16-byte pieces of row r are permuted to piece ^ (r % 8).  One bulk copy of a
block is then directly a tensor-core operand in shared memory (128-byte swizzle), and the
SIMT kernels index it with the same permutation.  These helpers convert blocks between
that order and plain [16, 256] rows (tests, debugging, external tools).
"""

from __future__ import annotations

import torch


def _perm(device=None) -> torch.Tensor:
    """perm[r * 256 + d] = storage index of element (row r, dim d) within a block."""
    r = torch.arange(16).view(16, 1)
    d = torch.arange(256).view(1, 256)
    idx = (r >> 3) * 2048 + (d >> 6) * 512 + (r & 7) * 64 + ((((d & 63) >> 3) ^ (r & 7)) << 3) + (d & 7)
    return idx.reshape(-1).to(device)


def swizzle_pages(rows: torch.Tensor) -> torch.Tensor:
    """[..., 16, 256] plain rows -> the same-shaped tensor in block storage order."""
    flat = rows.reshape(*rows.shape[:-2], 16 * 256)
    out = torch.empty_like(flat)
    out[..., _perm(rows.device)] = flat
    return out.view(rows.shape)


def unswizzle_pages(blocks: torch.Tensor) -> torch.Tensor:
    """Inverse of swizzle_pages."""
    flat = blocks.reshape(*blocks.shape[:-2], 16 * 256)
    return flat[..., _perm(blocks.device)].view(blocks.shape)
