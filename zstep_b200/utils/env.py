"""Typed, validated runtime knobs (the only place the package reads the environment).

Every ``ZSTEP_*`` variable the workers understand is declared here with its type,
default and allowed range; ``RuntimeConfig.from_env()`` parses and validates all of them
at once (a bad value fails at start-up with the variable's name, not deep inside a
step) and ``format_log_line()`` prints the effective configuration in one line.  Other
modules call ``runtime_config()`` instead of touching ``os.environ``; a test walks the
package's syntax trees to keep it that way.  The distributed launcher variables
(RANK, WORLD_SIZE, LOCAL_RANK, MASTER_ADDR/PORT) are read through ``dist_env()``.

Reference parity: worker/zstep_worker/env_config.py:121 (WorkerRuntimeConfig),
:166 (from_env), :307 (format_log_line).
"""

from __future__ import annotations

import dataclasses
import os
from functools import lru_cache


class EnvError(ValueError):
    pass


def _bool(name: str, raw: str) -> bool:
    v = raw.strip().lower()
    if v in ("1", "true", "yes", "on"):
        return True
    if v in ("0", "false", "no", "off", ""):
        return False
    raise EnvError(f"{name}={raw!r}: expected a boolean (0/1/true/false)")


def _int(name: str, raw: str, lo: int | None = None, hi: int | None = None) -> int:
    try:
        v = int(raw.strip(), 0)
    except ValueError as e:
        raise EnvError(f"{name}={raw!r}: expected an integer") from e
    if lo is not None and v < lo or hi is not None and v > hi:
        raise EnvError(f"{name}={v}: must be within [{lo}, {hi}]")
    return v


def _choice_int(name: str, raw: str, choices: tuple[int, ...]) -> int:
    v = _int(name, raw)
    if v not in choices:
        raise EnvError(f"{name}={v}: expected one of {', '.join(map(str, choices))}")
    return v


def _choice(name: str, raw: str, choices: tuple[str, ...]) -> str:
    v = raw.strip().lower()
    if v not in choices:
        raise EnvError(f"{name}={raw!r}: expected one of {', '.join(choices)}")
    return v


@dataclasses.dataclass(frozen=True)
class RuntimeConfig:
    collectives: str = "fused"            # ZSTEP_COLLECTIVES: fused | nccl
    coll_timeout_ms: int = 5000           # ZSTEP_COLL_TIMEOUT_MS: bound on cross-rank waits
    coll_oneshot_rows: int = 16           # ZSTEP_COLL_ONESHOT_ROWS: all-reduces up to this many rows go one-shot
    coll_ll_rows: int = 1024              # ZSTEP_COLL_LL_ROWS: two-shot LL lines up to this many rows, plain above
    coll_push: bool = True                # ZSTEP_COLL_PUSH: row-parallel GEMM epilogues push into the all-reduce
    mla_impl: int = 1                     # ZSTEP_MLA_IMPL: DeepSeek latent attention, 1 SIMT, 2 tensor cores
    coll_nvls_rows: int = 0               # ZSTEP_COLL_NVLS_ROWS: all-reduces above the one-shot size and up to
                                          # this many rows reduce in the NVSwitch (multicast object; 0: off)
    gemm_fix_splits: bool = False         # ZSTEP_GEMM_FIX_SPLITS: in-kernel split-K for small GEMMs
    gemm_dense_bn: int = 0                # ZSTEP_GEMM_DENSE_BN: dense GEMM token tile 32 | 128 (0: by shape)
    decode_graphs: bool = True            # ZSTEP_DECODE_GRAPHS: CUDA-graph decode buckets
    pdl: bool = True                      # ZSTEP_PDL: programmatic dependent launch of the kernels
    spec_method: str = "none"             # ZSTEP_SPEC_METHOD: none | ngram | mtp
    num_spec_tokens: int = 0              # ZSTEP_NUM_SPEC_TOKENS: 0..7
    num_recurrent_checkpoints: int = 0    # ZSTEP_NUM_RECURRENT_CHECKPOINTS
    dram_kv_blocks: int = 0               # ZSTEP_DRAM_KV_BLOCKS: host DRAM KV tier size (pages)
    numa_pin: bool = True                 # ZSTEP_NUMA_PIN: pin workers to their GPU's NUMA node
    nvtx: bool = False                    # ZSTEP_NVTX: NVTX ranges around runner phases
    runahead_depth: int = 2               # ZSTEP_RUNAHEAD_DEPTH: eager steps in flight per worker (0: no cap)
    log_level: str = "info"               # ZSTEP_LOG_LEVEL: debug | info | warning | error

    _VARS = {
        "ZSTEP_COLLECTIVES": ("collectives", lambda n, r: _choice(n, r, ("fused", "nccl"))),
        "ZSTEP_COLL_TIMEOUT_MS": ("coll_timeout_ms", lambda n, r: _int(n, r, 1, 600000)),
        "ZSTEP_COLL_ONESHOT_ROWS": ("coll_oneshot_rows", lambda n, r: _int(n, r, 0, 64)),
        "ZSTEP_COLL_LL_ROWS": ("coll_ll_rows", lambda n, r: _int(n, r, 0, 1 << 16)),
        "ZSTEP_COLL_PUSH": ("coll_push", _bool),
        "ZSTEP_COLL_NVLS_ROWS": ("coll_nvls_rows", lambda n, r: _int(n, r, 0, 1 << 16)),
        "ZSTEP_MLA_IMPL": ("mla_impl", lambda n, r: _choice_int(n, r, (1, 2))),
        "ZSTEP_GEMM_FIX_SPLITS": ("gemm_fix_splits", _bool),
        "ZSTEP_GEMM_DENSE_BN": ("gemm_dense_bn", lambda n, r: _choice_int(n, r, (0, 32, 128))),
        "ZSTEP_DECODE_GRAPHS": ("decode_graphs", _bool),
        "ZSTEP_PDL": ("pdl", _bool),
        "ZSTEP_SPEC_METHOD": ("spec_method", lambda n, r: _choice(n, r, ("none", "ngram", "mtp"))),
        "ZSTEP_NUM_SPEC_TOKENS": ("num_spec_tokens", lambda n, r: _int(n, r, 0, 7)),
        "ZSTEP_NUM_RECURRENT_CHECKPOINTS": ("num_recurrent_checkpoints", lambda n, r: _int(n, r, 0, 1 << 20)),
        "ZSTEP_DRAM_KV_BLOCKS": ("dram_kv_blocks", lambda n, r: _int(n, r, 0, 1 << 26)),
        "ZSTEP_NUMA_PIN": ("numa_pin", _bool),
        "ZSTEP_NVTX": ("nvtx", _bool),
        "ZSTEP_RUNAHEAD_DEPTH": ("runahead_depth", lambda n, r: _int(n, r, 0, 64)),
        "ZSTEP_LOG_LEVEL": ("log_level", lambda n, r: _choice(n, r, ("debug", "info", "warning", "error"))),
    }

    @classmethod
    def from_env(cls, env: dict | None = None) -> "RuntimeConfig":
        env = os.environ if env is None else env
        unknown = [k for k in env if k.startswith("ZSTEP_") and k not in cls._VARS and k not in _MASTER_VARS]
        if unknown:
            raise EnvError(f"unknown ZSTEP_ variable(s): {', '.join(sorted(unknown))}")
        kw = {}
        for var, (field, parse) in cls._VARS.items():
            if var in env:
                kw[field] = parse(var, env[var])
        cfg = cls(**kw)
        if cfg.spec_method != "none" and cfg.num_spec_tokens == 0:
            raise EnvError("ZSTEP_SPEC_METHOD set but ZSTEP_NUM_SPEC_TOKENS is 0")
        return cfg

    def format_log_line(self) -> str:
        parts = [f"{f.name}={getattr(self, f.name)}" for f in dataclasses.fields(self)]
        return "zstep worker config: " + " ".join(parts)


# Variables consumed by the master process (C++), accepted here so that a shared
# environment does not fail the worker's validation.
_MASTER_VARS = {"ZSTEP_API_KEY", "ZSTEP_ALLOW_REMOTE_METRICS", "ZSTEP_GIT_SHA"}


@lru_cache(maxsize=1)
def runtime_config() -> RuntimeConfig:
    return RuntimeConfig.from_env()


@dataclasses.dataclass(frozen=True)
class DistEnv:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    master_addr: str = "127.0.0.1"
    master_port: int = 29500


def dist_env(env: dict | None = None) -> DistEnv:
    """torch.distributed launcher variables (set by torchrun or the master)."""
    env = os.environ if env is None else env
    rank = _int("RANK", env.get("RANK", "0"), 0)
    world = _int("WORLD_SIZE", env.get("WORLD_SIZE", "1"), 1)
    if rank >= world:
        raise EnvError(f"RANK={rank} outside WORLD_SIZE={world}")
    return DistEnv(rank=rank, world_size=world, local_rank=_int("LOCAL_RANK", env.get("LOCAL_RANK", str(rank)), 0),
                   master_addr=env.get("MASTER_ADDR", "127.0.0.1"),
                   master_port=_int("MASTER_PORT", env.get("MASTER_PORT", "29500"), 1, 65535))


def python_path() -> str:
    return os.environ.get("PYTHONPATH", "")


def own_process_group_store(env: dict | None = None) -> None:
    """Make this process group host its own rendezvous store (rank 0 serves it).  A process
    started from inside a torchrun job inherits TORCHELASTIC_USE_AGENT_STORE=True, which
    tells torch.distributed that the launcher's agent runs the store, so every rank,
    rank 0 included, would connect as a client to a server that never starts."""
    env = os.environ if env is None else env
    env.pop("TORCHELASTIC_USE_AGENT_STORE", None)
