"""Tensor/expert parallel plumbing: collectives (NCCL baseline and the fused NVLink
kernels), symmetric memory, and topology checks."""

from __future__ import annotations


def make_collectives(device, group=None, kind: str | None = None):
    """Pick the collective implementation for the runner (``ZSTEP_COLLECTIVES`` =
    ``fused`` (default when available) or ``nccl``)."""
    from ..utils.env import runtime_config

    kind = kind or runtime_config().collectives
    if kind == "fused":
        try:
            from .fused import FusedCollectives

            return FusedCollectives(device, group)
        except ImportError:
            pass
    from .collectives import NcclCollectives

    return NcclCollectives(group, device)
