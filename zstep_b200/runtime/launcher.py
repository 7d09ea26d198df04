"""Start the C++ engine with its shared-memory worker processes from Python.

Used by the offline ``Engine`` API, the tests and the bench.  The master picks a free
TCP port on 127.0.0.1 for the workers' torch.distributed rendezvous (gloo on CPU,
NCCL on GPU) and passes it through the environment; the transport fds travel on the
worker command line (see runtime/worker.py).
"""

from __future__ import annotations

import os
import socket
import sys

from .. import _master
from ..utils.env import python_path


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def engine_config(**kw) -> "_master.EngineConfig":
    cfg = _master.EngineConfig()
    for k, v in kw.items():
        if not hasattr(cfg, k):
            raise AttributeError(f"unknown engine option {k}")
        setattr(cfg, k, v)
    return cfg


def launch(*, model: str = "qwen3.5-tiny", world_size: int = 1, device: str = "cpu", seed: int = 0,
           max_seqs: int = 8, max_step_tokens: int = 512, page_size: int = 16, num_pages: int = 1024,
           max_model_len: int = 2048, num_ckpt_slots: int = 0, vocab_size: int = 0, engine: dict | None = None,
           ready_timeout_ms: int = 600000, step_timeout_ms: int = 300000, heartbeat_timeout_ms: int = 10000,
           extra_env: dict | None = None, dram_kv_blocks: int = 0):
    """Returns (engine, coordinator).  Call ``coordinator.shutdown()`` when done."""
    geo = _master.Geometry()
    geo.world_size = world_size
    geo.max_seqs = max_seqs
    geo.max_step_tokens = max_step_tokens
    geo.max_pages_per_seq = (max_model_len + page_size - 1) // page_size
    geo.page_size = page_size
    geo.vocab_size = vocab_size
    ecfg = engine_config(max_seqs=max_seqs, max_step_tokens=max_step_tokens, page_size=page_size,
                         num_pages=num_pages, max_model_len=max_model_len, num_ckpt_slots=num_ckpt_slots,
                         **(engine or {}))
    argv = [sys.executable, "-m", "zstep_b200.runtime.worker", "--model", model, "--device", device, "--seed",
            str(seed), "--num-pages", str(num_pages), "--max-model-len", str(max_model_len), "--num-ckpt-slots",
            str(num_ckpt_slots), "--dram-kv-blocks", str(dram_kv_blocks), "--spec-method", ecfg.spec_method,
            "--num-spec-tokens", str(ecfg.num_spec_tokens)]
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    env = {"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(free_port()),
           "PYTHONPATH": root + os.pathsep + python_path()}
    env.update(extra_env or {})
    return _master.make_shm_engine(ecfg, geo, argv, env, ready_timeout_ms, step_timeout_ms, heartbeat_timeout_ms)


def run_to_completion(engine, max_steps: int = 100000) -> dict:
    """Drive the engine until idle; returns {request_id: tokens}."""
    out = {}
    for _ in range(max_steps):
        if not engine.has_work():
            break
        for ev in engine.step():
            out.setdefault(ev["request_id"], []).extend(ev["tokens"])
        if engine.poisoned():
            raise RuntimeError(engine.error())
    return out
