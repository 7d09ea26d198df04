"""Host DRAM tier of the KV cache on a worker: a pinned host arena of demoted pages.

One arena slot holds one device page of every paged cache tensor of the model (all
layers), e.g. the latent and index-key caches of the DeepSeek-style model.  The master
sends KvTransfer steps (page, slot, direction); D2H gathers the pages' rows on the device
and lands them in the pinned slots, H2D scatters slots back into pages.  Copies run on
the runner's stream, so a following step sees reloaded pages and a demoted page is read
before any later step can overwrite it.  The arena is allocated after the worker pinned
itself to its GPU's NUMA node, so its host pages are local to that GPU's root complex.

Reference parity: worker/zstep_worker/kv_dram_tier.py:38 (HostDramKvTier),
:157 (execute_transfers).
"""

from __future__ import annotations

import numpy as np
import torch


class DramKvArena:
    def __init__(self, caches: list[torch.Tensor], num_blocks: int):
        """caches: device tensors [layers, pages, ...] (page is dim 1)."""
        self.caches = caches
        self.num_blocks = num_blocks
        # Pinned so the copies are asynchronous DMA (host tensors of CPU caches need no pinning).
        self.host = [torch.empty((num_blocks, c.shape[0]) + tuple(c.shape[2:]), dtype=c.dtype,
                                 pin_memory=c.is_cuda) for c in caches]
        self.bytes_per_block = sum(h[0].numel() * h.element_size() for h in self.host)
        self.d2h_blocks = 0
        self.h2d_blocks = 0

    def transfer(self, pages: np.ndarray, slots: np.ndarray, h2d: np.ndarray) -> None:
        pages = np.asarray(pages, dtype=np.int64)
        slots = np.asarray(slots, dtype=np.int64)
        h2d = np.asarray(h2d).astype(bool)
        if len(slots) and (slots.min() < 0 or slots.max() >= self.num_blocks):
            raise ValueError(f"DRAM slot out of range (arena has {self.num_blocks} blocks)")
        down, up = ~h2d, h2d
        # Every copy is asynchronous on the runner's stream: D2H gathers the demoted pages
        # into a device staging block and copies each page's block into its pinned slot;
        # H2D copies the slots into a staging block and scatters it into the pages.  Stream
        # order makes a later step see reloaded pages and keeps a demoted page's rows from
        # being overwritten before they are copied out; the host never waits.
        d_slots = slots[down].tolist()
        u_slots = slots[up].tolist()
        for c, host in zip(self.caches, self.host):
            if d_slots:
                p = torch.from_numpy(pages[down]).to(c.device, non_blocking=True)
                staged = c[:, p].transpose(0, 1).contiguous()
                for j, sl in enumerate(d_slots):
                    host[sl].copy_(staged[j], non_blocking=True)
            if u_slots:
                p = torch.from_numpy(pages[up]).to(c.device, non_blocking=True)
                staged = torch.empty((len(u_slots),) + tuple(host.shape[1:]), dtype=c.dtype, device=c.device)
                for j, sl in enumerate(u_slots):
                    staged[j].copy_(host[sl], non_blocking=True)
                c[:, p] = staged.transpose(0, 1)
        self.d2h_blocks += len(d_slots)
        self.h2d_blocks += len(u_slots)
