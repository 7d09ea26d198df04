"""Worker runtime utilities: validated env config (and the rule that nothing else in the
package reads the environment), NUMA pinning logic on a fake sysfs, and the NVLink
topology decision on injected device queries."""

import ast
import os

import pytest

from zstep_b200.parallel import topology
from zstep_b200.utils import env, numa

PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "zstep_b200")


def test_env_defaults_and_validation():
    cfg = env.RuntimeConfig.from_env({})
    assert cfg.collectives == "fused" and cfg.coll_timeout_ms == 5000 and cfg.numa_pin
    cfg = env.RuntimeConfig.from_env({"ZSTEP_COLLECTIVES": "NCCL", "ZSTEP_NUM_SPEC_TOKENS": "3",
                                      "ZSTEP_SPEC_METHOD": "mtp", "ZSTEP_NVTX": "1"})
    assert cfg.collectives == "nccl" and cfg.spec_method == "mtp" and cfg.num_spec_tokens == 3 and cfg.nvtx
    assert "collectives=nccl" in cfg.format_log_line()
    for bad in ({"ZSTEP_COLLECTIVES": "mpi"}, {"ZSTEP_COLL_TIMEOUT_MS": "0"}, {"ZSTEP_NUMA_PIN": "maybe"},
                {"ZSTEP_TYPO": "1"}, {"ZSTEP_SPEC_METHOD": "ngram"}, {"ZSTEP_NUM_SPEC_TOKENS": "9"}):
        with pytest.raises(env.EnvError):
            env.RuntimeConfig.from_env(bad)
    assert env.RuntimeConfig.from_env({"ZSTEP_API_KEY": "x"}).collectives == "fused"  # master variable


def test_dist_env():
    d = env.dist_env({"RANK": "3", "WORLD_SIZE": "8", "LOCAL_RANK": "3", "MASTER_PORT": "1234"})
    assert (d.rank, d.world_size, d.local_rank, d.master_port) == (3, 8, 3, 1234)
    with pytest.raises(env.EnvError):
        env.dist_env({"RANK": "8", "WORLD_SIZE": "8"})


def test_own_process_group_store_drops_the_agent_store_setting():
    """A worker group started from inside a torchrun job must host its own store."""
    e = {"TORCHELASTIC_USE_AGENT_STORE": "True", "MASTER_PORT": "1234"}
    env.own_process_group_store(e)
    assert e == {"MASTER_PORT": "1234"}
    env.own_process_group_store(e)  # absent: nothing to do
    assert e == {"MASTER_PORT": "1234"}


def test_no_env_reads_outside_env_module():
    """Only zstep_b200/utils/env.py may read os.environ / os.getenv."""
    offenders = []
    for root, _, files in os.walk(PKG):
        for f in files:
            if not f.endswith(".py"):
                continue
            path = os.path.join(root, f)
            if path.endswith(os.path.join("utils", "env.py")):
                continue
            tree = ast.parse(open(path).read())
            for node in ast.walk(tree):
                if isinstance(node, ast.Attribute) and node.attr in ("environ", "getenv") and \
                        isinstance(node.value, ast.Name) and node.value.id == "os":
                    offenders.append(f"{path}:{node.lineno}")
    assert not offenders, offenders


def fake_sysfs(tmp_path, addr="0000:1b:00.0", node=1, cpulist="2-3,6"):
    dev = tmp_path / "bus/pci/devices" / addr
    dev.mkdir(parents=True)
    (dev / "numa_node").write_text(f"{node}\n")
    (dev / "local_cpulist").write_text(cpulist + "\n")
    nd = tmp_path / f"devices/system/node/node{node}"
    nd.mkdir(parents=True)
    (nd / "cpulist").write_text("0-7\n")
    return str(tmp_path)


def test_numa_pin_fake_sysfs(tmp_path):
    root = fake_sysfs(tmp_path)
    assert numa.parse_cpulist("0-3,8,10-11") == [0, 1, 2, 3, 8, 10, 11]
    assert numa.device_numa_node("0000:1b:00.0", root) == 1
    assert numa.device_cpus("0000:1B:00.0", root) == [2, 3, 6]
    calls = {}
    allowed = sorted(os.sched_getaffinity(0))
    want = [c for c in [2, 3, 6] if c in allowed]
    info = numa.pin_process_to_device(0, sysfs_root=root, pci_addr="0000:1b:00.0",
                                      set_affinity=lambda pid, cpus: calls.setdefault("cpus", cpus),
                                      bind=lambda node: calls.setdefault("node", node) is not None)
    if want:
        assert info["pinned"] and calls["cpus"] == want and calls["node"] == 1
    else:
        assert not info["pinned"]
    assert not numa.pin_process_to_device(0, sysfs_root=root, pci_addr="0000:99:00.0")["pinned"]


def test_topology_decision():
    t = topology.probe([0, 1, 2, 3], can_access_peer=lambda i, j: True, nvlink_count=lambda i: 18,
                       multicast_supported=lambda i: True)
    assert t.fully_peer and t.nvlink_fabric and t.recommended_collectives() == "fused"
    t = topology.probe([0, 1], can_access_peer=lambda i, j: False, nvlink_count=lambda i: 0,
                       multicast_supported=lambda i: False)
    assert not t.fully_peer and t.recommended_collectives() == "nccl"
    t = topology.probe([0, 1], can_access_peer=lambda i, j: True, nvlink_count=lambda i: 0,
                       multicast_supported=lambda i: False)
    assert t.fully_peer and not t.nvlink_fabric and t.recommended_collectives() == "nccl"
    assert "collectives=" in t.summary()


def test_runahead_guard_caps_in_flight_steps():
    from zstep_b200.runtime.runahead import RunAheadGuard

    class FakeEvents:
        """Events that complete only when the test says so; wait() completes one."""

        def __init__(self):
            self.created, self.pending, self.waited = 0, set(), []

        def create(self):
            self.created += 1
            return self.created

        def record(self, ev):
            self.pending.add(ev)

        def done(self, ev):
            return ev not in self.pending

        def wait(self, ev):
            self.waited.append(ev)
            self.pending.discard(ev)

    be = FakeEvents()
    g = RunAheadGuard(2, be)
    for _ in range(2):
        g.before_launch()
        g.after_launch()
    assert g.depth == 2 and not be.waited
    g.before_launch()  # third step: must wait for the oldest
    assert be.waited == [1] and g.depth == 1
    g.after_launch()
    be.pending.clear()  # everything finished on the device
    g.before_launch()
    assert g.depth == 0 and g.waits == 1
    g.after_launch()
    assert be.created == 2  # events are pooled, not re-created
    g.drain()
    assert g.depth == 0
    off = RunAheadGuard(0, be)
    off.before_launch()
    off.after_launch()
    assert off.depth == 0 and not off.enabled


def test_dram_arena_demotes_and_reloads_pages():
    """Host DRAM arena (CPU tensors here): pages demoted to slots come back bit-identical
    into other pages, one call may mix both directions, and out-of-range slots are refused."""
    import numpy as np
    import torch

    from zstep_b200.runtime.kv_dram import DramKvArena

    g = torch.Generator().manual_seed(0)
    caches = [torch.randn(3, 10, 2, 4, generator=g), torch.randint(0, 255, (3, 10, 8), generator=g).to(torch.uint8)]
    orig = [c.clone() for c in caches]
    arena = DramKvArena(caches, num_blocks=4)
    assert arena.bytes_per_block == 3 * 2 * 4 * 4 + 3 * 8
    arena.transfer(np.array([2, 5]), np.array([0, 3]), np.array([0, 0]))  # demote pages 2, 5
    for c in caches:
        c[:, 2] = 0
        c[:, 5] = 0
    # Reload slot 3 into page 7 and demote page 9 into slot 1 in the same call.
    arena.transfer(np.array([7, 9]), np.array([3, 1]), np.array([1, 0]))
    arena.transfer(np.array([1, 2]), np.array([0, 1]), np.array([1, 1]))  # slot 0 -> page 1, slot 1 -> page 2
    for c, o in zip(caches, orig):
        assert torch.equal(c[:, 7], o[:, 5])
        assert torch.equal(c[:, 1], o[:, 2])
        assert torch.equal(c[:, 2], o[:, 9])
    assert (arena.d2h_blocks, arena.h2d_blocks) == (3, 3)
    with pytest.raises(ValueError):
        arena.transfer(np.array([0]), np.array([4]), np.array([0]))
