"""Pin a worker process (CPU affinity and memory policy) to its GPU's NUMA node.

The GPU's PCI address gives ``/sys/bus/pci/devices/<addr>/numa_node`` and
``local_cpulist``; the process's CPU affinity is set to that list and its memory policy
to "preferred node" (``set_mempolicy(MPOL_PREFERRED)``), so the pinned staging buffers
and the shared-memory segment pages it touches land next to the GPU.  Everything takes a
``sysfs_root`` so the logic is testable on any machine.

Reference parity: worker/zstep_worker/numa_pin.py:106 (pin_process_to_device_numa),
:155 (bind_memory_to_numa_node).
"""

from __future__ import annotations

import ctypes
import os

MPOL_PREFERRED = 1
_SYS_SET_MEMPOLICY = 238  # x86_64


def parse_cpulist(text: str) -> list[int]:
    """'0-3,8,10-11' -> [0, 1, 2, 3, 8, 10, 11]."""
    cpus: list[int] = []
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-", 1)
            cpus.extend(range(int(a), int(b) + 1))
        else:
            cpus.append(int(part))
    return cpus


def pci_address(device_index: int) -> str | None:
    """Canonical sysfs PCI address ``dddd:bb:dd.0`` of a GPU, from NVML (does not create a
    CUDA context) or else from torch; None when neither is available."""
    try:
        import pynvml

        pynvml.nvmlInit()
        bus = pynvml.nvmlDeviceGetPciInfo(pynvml.nvmlDeviceGetHandleByIndex(device_index)).busId
        bus = bus.decode() if isinstance(bus, bytes) else bus
        dom, rest = bus.split(":", 1)
        return f"{int(dom, 16):04x}:{rest.lower()}"
    except Exception:
        pass
    try:
        import torch

        if not torch.cuda.is_available():
            return None
        p = torch.cuda.get_device_properties(device_index)
        return f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    except Exception:
        return None


def device_numa_node(pci_addr: str, sysfs_root: str = "/sys") -> int:
    """NUMA node of a PCI device, -1 when unknown."""
    try:
        with open(os.path.join(sysfs_root, "bus/pci/devices", pci_addr.lower(), "numa_node")) as f:
            return int(f.read().strip())
    except (OSError, ValueError):
        return -1


def device_cpus(pci_addr: str, sysfs_root: str = "/sys") -> list[int]:
    """CPUs local to the device: its local_cpulist, else the CPUs of its NUMA node."""
    base = os.path.join(sysfs_root, "bus/pci/devices", pci_addr.lower())
    try:
        with open(os.path.join(base, "local_cpulist")) as f:
            cpus = parse_cpulist(f.read())
            if cpus:
                return cpus
    except OSError:
        pass
    node = device_numa_node(pci_addr, sysfs_root)
    if node < 0:
        return []
    try:
        with open(os.path.join(sysfs_root, f"devices/system/node/node{node}/cpulist")) as f:
            return parse_cpulist(f.read())
    except OSError:
        return []


def bind_memory_to_node(node: int) -> bool:
    """Prefer allocations of this process on `node` (best effort; False if refused)."""
    if node < 0 or node >= 64:
        return False
    try:
        libc = ctypes.CDLL(None, use_errno=True)
        mask = ctypes.c_ulong(1 << node)
        return libc.syscall(_SYS_SET_MEMPOLICY, MPOL_PREFERRED, ctypes.byref(mask), 64) == 0
    except Exception:
        return False


def pin_process_to_device(device_index: int, sysfs_root: str = "/sys", pci_addr: str | None = None,
                          set_affinity=os.sched_setaffinity, bind=bind_memory_to_node) -> dict:
    """Pin the calling process next to `device_index`.  Returns what was done."""
    addr = pci_addr or pci_address(device_index)
    if addr is None:
        return {"pinned": False, "reason": "no PCI address"}
    cpus = device_cpus(addr, sysfs_root)
    allowed = set(os.sched_getaffinity(0))
    cpus = [c for c in cpus if c in allowed] or []
    if not cpus:
        return {"pinned": False, "reason": "no local CPUs", "pci": addr}
    set_affinity(0, cpus)
    node = device_numa_node(addr, sysfs_root)
    mem = bind(node) if node >= 0 else False
    return {"pinned": True, "pci": addr, "node": node, "cpus": cpus, "membind": mem}
