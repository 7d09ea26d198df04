"""Run-ahead guard: a cap on how many eager (non-graph) steps a worker keeps in flight.

An eager prefill step launches hundreds of kernels.  When a worker launches the next step
before the previous one finished (a pipelined prefill, or run-ahead steps whose results
are read later), those launches queue up in the driver; past the submission queue's depth
a launch blocks the worker's main loop, and with it the heartbeat replies the master
watches.  The guard records one completion event per launched step and, before the next
launch, waits for the oldest in-flight step whenever ``max_depth`` steps are pending, so
the queue never holds more than ``max_depth`` steps' work.  With ``max_depth = 0`` it does
nothing.  Events come from a pluggable backend (CUDA events on a GPU worker, a fake in
tests) and are pooled, so a steady stream of steps creates no new events.

Reference parity: worker/zstep_worker/runahead.py:65 (PrefillRunAheadGuard).
"""

from __future__ import annotations

from collections import deque


class TorchEventBackend:
    """CUDA events recorded on the current stream of `device`."""

    def __init__(self, device):
        self.device = device

    def create(self):
        import torch

        return torch.cuda.Event(enable_timing=False)

    def record(self, ev) -> None:
        import torch

        ev.record(torch.cuda.current_stream(self.device))

    def done(self, ev) -> bool:
        return bool(ev.query())

    def wait(self, ev) -> None:
        ev.synchronize()


class RunAheadGuard:
    def __init__(self, max_depth: int = 2, backend=None):
        if max_depth < 0:
            raise ValueError(f"max_depth must be >= 0, got {max_depth}")
        self.max_depth = max_depth
        self.backend = backend
        self._in_flight: deque = deque()
        self._pool: list = []
        self.launched = 0
        self.waits = 0

    @property
    def enabled(self) -> bool:
        return self.max_depth > 0 and self.backend is not None

    @property
    def depth(self) -> int:
        return len(self._in_flight)

    def _reap(self) -> None:
        while self._in_flight and self.backend.done(self._in_flight[0]):
            self._pool.append(self._in_flight.popleft())

    def before_launch(self) -> None:
        """Block until fewer than `max_depth` guarded steps are in flight."""
        if not self.enabled:
            return
        self._reap()
        while len(self._in_flight) >= self.max_depth:
            ev = self._in_flight.popleft()
            self.backend.wait(ev)
            self._pool.append(ev)
            self.waits += 1

    def after_launch(self) -> None:
        """Fence the step just launched."""
        if not self.enabled:
            return
        ev = self._pool.pop() if self._pool else self.backend.create()
        self.backend.record(ev)
        self._in_flight.append(ev)
        self.launched += 1

    def drain(self) -> None:
        """Wait for every guarded step (shutdown, or before reusing host-visible outputs)."""
        while self.enabled and self._in_flight:
            ev = self._in_flight.popleft()
            self.backend.wait(ev)
            self._pool.append(ev)
