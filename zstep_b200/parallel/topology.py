"""NVLink / NVSwitch topology check for the tensor-parallel group.

Before the fused collectives are enabled, every rank's GPU must reach every other over
peer-to-peer (CUDA IPC mappings are loaded and stored directly by the kernels).  On an
HGX B200 board all eight GPUs sit behind NVSwitch: every pair is peer-capable with the
same bandwidth, so there is no pair ordering or PCIe-tree classification to do (the
reference needs that for PCIe-only machines).  The check gathers:

* the all-pairs peer-access matrix (``cudaDeviceCanAccessPeer``),
* active NVLink links per GPU (NVML, read-only),
* multicast object support (``CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED``), which NVLS /
  ``multimem`` collectives need,

and recommends ``fused`` collectives when the group is fully peer-connected over NVLink
and ``nccl`` otherwise.  Query functions are injectable so the decision logic is tested
on machines without GPUs.

Reference parity: worker/zstep_worker/p2p_probe.py:70 (classify_pci_pair_relation),
:165 (IPC bandwidth probe), :370 (configure_adaptive_p2p_env).
"""

from __future__ import annotations

import dataclasses


@dataclasses.dataclass
class Topology:
    devices: list[int]
    peer: list[list[bool]]
    nvlinks: list[int]
    multicast: list[bool]

    @property
    def fully_peer(self) -> bool:
        n = len(self.devices)
        return all(self.peer[i][j] for i in range(n) for j in range(n) if i != j)

    @property
    def nvlink_fabric(self) -> bool:
        return self.fully_peer and all(n > 0 for n in self.nvlinks)

    def recommended_collectives(self) -> str:
        return "fused" if len(self.devices) == 1 or self.nvlink_fabric else "nccl"

    def summary(self) -> str:
        return (f"devices={self.devices} fully_peer={self.fully_peer} nvlinks={self.nvlinks} "
                f"multicast={self.multicast} -> collectives={self.recommended_collectives()}")


def _can_access_peer(i: int, j: int) -> bool:
    import torch

    return bool(torch.cuda.can_device_access_peer(i, j))


def _nvlink_count(i: int) -> int:
    try:
        import pynvml

        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(i)
        n = 0
        for link in range(18):
            try:
                if pynvml.nvmlDeviceGetNvLinkState(h, link) == pynvml.NVML_FEATURE_ENABLED:
                    n += 1
            except pynvml.NVMLError:
                break
        return n
    except Exception:
        return 0


def _multicast_supported(i: int) -> bool:
    try:
        from cuda.bindings import driver as cu
    except Exception:
        try:
            from cuda import cuda as cu  # older cuda-python layout
        except Exception:
            return False
    try:
        cu.cuInit(0)
        err, dev = cu.cuDeviceGet(i)
        err, v = cu.cuDeviceGetAttribute(cu.CUdevice_attribute.CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev)
        return bool(v)
    except Exception:
        return False


def probe(devices: list[int], can_access_peer=_can_access_peer, nvlink_count=_nvlink_count,
          multicast_supported=_multicast_supported) -> Topology:
    n = len(devices)
    peer = [[i == j or can_access_peer(devices[i], devices[j]) for j in range(n)] for i in range(n)]
    return Topology(devices=list(devices), peer=peer, nvlinks=[nvlink_count(d) for d in devices],
                    multicast=[multicast_supported(d) for d in devices])
