"""Worker process: executes the master's step plans on one rank.

    python -m zstep_b200.runtime.worker --model qwen3.5-tiny --device cpu \
        --shm-fd N --shm-bytes B --plan-fd P --done-fd D --rank R --world-size W

Lifecycle: map the inherited shared-memory fd, validate magic / version / layout hash
against this build's own layout computation, set up torch.distributed (gloo on CPU,
NCCL on GPU; MASTER_ADDR/MASTER_PORT come from the master's environment), build the
runner, mark READY and loop: wait on the plan eventfd, read the published plan slot,
execute it, (rank 0) publish the result slot, advance ``ready_step`` and signal the done
eventfd.  A watchdog thread refreshes the heartbeat every 250 ms and stops the process
when the segment's abort word is set.  Any exception marks the rank ERROR with a code
before exiting, so the master fails fast instead of timing out.

Reference parity: worker/zstep_worker/runtime_loop.py (RuntimeLoop :338, watchdog :403,
plan-eventfd wait :442, run :480, report_error :668, main :734).
"""

from __future__ import annotations

import argparse

import numpy as np
import gc
import mmap
import os
import select
import signal
import struct
import sys
import threading
import time
import traceback

from . import wire

ERR_EXCEPTION = 1
ERR_LAYOUT = 2


def _monotonic_ns() -> int:
    return time.monotonic_ns()


def _set_pdeathsig() -> None:
    """Die with the master even if it is killed (Linux prctl PR_SET_PDEATHSIG)."""
    try:
        import ctypes

        libc = ctypes.CDLL("libc.so.6", use_errno=True)
        libc.prctl(1, signal.SIGKILL)  # PR_SET_PDEATHSIG = 1
    except OSError:
        pass


class EventFd:
    def __init__(self, fd: int):
        self.fd = fd

    def signal(self, n: int = 1) -> None:
        os.write(self.fd, struct.pack("<Q", n))

    def wait(self, timeout_s: float) -> int:
        r, _, _ = select.select([self.fd], [], [], timeout_s)
        if not r:
            return 0
        try:
            return struct.unpack("<Q", os.read(self.fd, 8))[0]
        except BlockingIOError:
            return 0


class WorkerLoop:
    def __init__(self, args):
        self.args = args
        self.rank = args.rank
        self.world = args.world_size
        self.mm = mmap.mmap(args.shm_fd, args.shm_bytes)
        sb = struct.unpack_from("<QIIIIIIII", self.mm, 0)
        self.geo = wire.Geometry(world_size=sb[3], max_seqs=sb[4], max_step_tokens=sb[5], max_pages_per_seq=sb[6],
                                 page_size=sb[7], vocab_size=sb[8])
        self.view = wire.SegmentView(self.mm, self.geo)
        self.last_tok = np.zeros(self.geo.max_seqs + 64, dtype=np.int32)  # last sampled token per slot
        self.plan_efd = EventFd(args.plan_fd)
        self.done_efd = EventFd(args.done_fd)
        self._stop = threading.Event()
        if sb[0] != wire.MAGIC or sb[1] != wire.VERSION or sb[2] != wire.layout_hash(self.geo):
            self.fail(ERR_LAYOUT, f"segment layout mismatch: magic={sb[0]:#x} version={sb[1]} hash={sb[2]:#x} "
                                  f"expected hash {wire.layout_hash(self.geo):#x}")
        self.view.set_worker(self.rank, status=wire.WORKER_STARTING, pid=os.getpid(), heartbeat_ns=_monotonic_ns())
        self.watchdog = threading.Thread(target=self._watchdog, daemon=True)
        self.watchdog.start()

    def fail(self, code: int, msg: str) -> None:
        sys.stderr.write(f"[zstep worker rank {self.rank}] {msg}\n")
        sys.stderr.flush()
        try:
            self.view.set_worker(self.rank, error=code, status=wire.WORKER_ERROR)
            self.done_efd.signal()
        finally:
            os._exit(3)

    def _watchdog(self) -> None:
        while not self._stop.is_set():
            self.view.set_worker(self.rank, heartbeat_ns=_monotonic_ns())
            if self.view.abort_word():
                sys.stderr.write(f"[zstep worker rank {self.rank}] abort requested by master\n")
                os._exit(4)
            time.sleep(0.25)

    def run(self) -> None:
        from .runners import make_runner

        try:
            self.runner = make_runner(self.args, self.rank, self.world, self.geo)
        except Exception:  # noqa: BLE001
            self.fail(ERR_EXCEPTION, "runner init failed:\n" + traceback.format_exc())
        self.view.set_worker(self.rank, status=wire.WORKER_READY)
        self.done_efd.signal()
        gc.disable()  # no collector pauses inside the step loop
        step = 0
        while True:
            want = step + 1
            if self.view.plan_step_id(want) < want:
                self.plan_efd.wait(0.2)
                continue
            step = want
            plan = self.view.read_plan(step)
            if plan["opcode"] == wire.OP_SHUTDOWN:
                self.view.set_worker(self.rank, status=wire.WORKER_EXITED, ready_step=step)
                self.done_efd.signal()
                break
            self.view.set_worker(self.rank, status=wire.WORKER_RUNNING)
            t0 = time.perf_counter()
            if plan["flags"] & wire.FLAG_DEVICE_TOKENS:
                # Run-ahead step: every row continues its slot with the token this worker
                # sampled for it in the previous step (identical on all ranks).
                plan["token_ids"] = self.last_tok[plan["row_slot"]]
            try:
                outputs = self.runner.execute(plan)
            except Exception:  # noqa: BLE001
                self.fail(ERR_EXCEPTION, f"step {step} failed:\n" + traceback.format_exc())
            for o in outputs:
                if o["num_tokens"] > 0:
                    self.last_tok[o["req_slot"]] = o["tokens"][o["num_tokens"] - 1]
            gpu_us = getattr(self.runner, "last_gpu_us", 0) or int((time.perf_counter() - t0) * 1e6)
            if self.rank == 0:
                self.view.write_result(step, outputs, 0, gpu_us)
            self.view.set_worker(self.rank, ready_step=step, status=wire.WORKER_READY, gpu_us=gpu_us)
            self.done_efd.signal()
        self._stop.set()
        self.runner.close()


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3.5-tiny", help="preset name or HF model directory")
    ap.add_argument("--device", default="cpu", choices=["cpu", "cuda"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--num-pages", type=int, default=4096)
    ap.add_argument("--max-model-len", type=int, default=4096)
    ap.add_argument("--num-ckpt-slots", type=int, default=0)
    ap.add_argument("--spec-method", default="none")
    ap.add_argument("--num-spec-tokens", type=int, default=0)
    ap.add_argument("--dram-kv-blocks", type=int, default=0, help="host DRAM tier blocks (pinned page arena)")
    ap.add_argument("--micro-hidden", type=int, default=5120, help="micro-step model: RMSNorm / GEMM input width")
    ap.add_argument("--micro-features", type=int, default=2048, help="micro-step model: GEMM output columns")
    ap.add_argument("--micro-experts", type=int, default=384, help="micro-step model: router experts")
    ap.add_argument("--micro-topk", type=int, default=6, help="micro-step model: router top-k")
    ap.add_argument("--shm-fd", type=int, required=True)
    ap.add_argument("--shm-bytes", type=int, required=True)
    ap.add_argument("--plan-fd", type=int, required=True)
    ap.add_argument("--done-fd", type=int, required=True)
    ap.add_argument("--rank", type=int, required=True)
    ap.add_argument("--world-size", type=int, required=True)
    return ap.parse_args(argv)


def main(argv=None) -> int:
    _set_pdeathsig()
    args = parse_args(argv)
    from ..utils.env import runtime_config

    cfg = runtime_config()  # validates every ZSTEP_* variable before any work
    print(f"[rank {args.rank}] {cfg.format_log_line()}", file=sys.stderr, flush=True)
    if args.device == "cuda" and cfg.numa_pin:
        # Before the shared-memory segment and CUDA are touched, so their pages and the
        # pinned staging buffers are allocated on the GPU's node.
        from ..utils.numa import pin_process_to_device

        info = pin_process_to_device(args.rank)
        print(f"[rank {args.rank}] numa: {info}", file=sys.stderr, flush=True)
    WorkerLoop(args).run()
    return 0


if __name__ == "__main__":
    sys.exit(main())
