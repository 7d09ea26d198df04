"""Python mirror of the shared-memory ABI in csrc/master/wire.h.

The worker computes the segment layout and layout hash independently and refuses a
segment whose magic / version / hash differ, so a master and worker built from
different sources never disagree silently about offsets.  ``tests/test_wire.py``
checks this module against the C++ definition (through ``zstep_b200._master``).

Reference parity: worker/zstep_worker/shm_bridge.py (constants :35-75,
compute_layout_hash :293, plan views :610).
"""

from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

MAGIC = 0x3030324253545A5A
VERSION = 1
MAX_WORKERS = 8
PLAN_SLOTS = 2
RESULT_SLOTS = 2
MAX_SPEC_TOKENS = 8
MAX_TOP_LOGPROBS = 5
SUPERBLOCK_BYTES = 4096
WORKER_REGION_BYTES = 4096
WORKER_STATE_BYTES = 64
ABORT_OFFSET = 128
ALIGN = 256

FLAG_DECODE_ONLY = 1 << 0
FLAG_DEVICE_TOKENS = 1 << 1
FLAG_NEXT_PUBLISHED = 1 << 2
FLAG_SAMPLING = 1 << 3
FLAG_PENALTY = 1 << 4
FLAG_SPEC_VERIFY = 1 << 5
FLAG_LOGPROBS = 1 << 6

OP_NORMAL, OP_WARMUP, OP_RELOAD, OP_KV_TRANSFER, OP_SHUTDOWN = 0, 1, 2, 3, 4
WORKER_STARTING, WORKER_READY, WORKER_RUNNING, WORKER_EXITED, WORKER_ERROR = 0, 1, 2, 3, 99

DECODE_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 384, 448, 512)

SIZEOF_SUPERBLOCK = 192
SIZEOF_WORKER_STATE = 64
SIZEOF_STEP_HEADER = 64
SIZEOF_SAMPLING = 40
SIZEOF_RESULT_HEADER = 64
SIZEOF_SEQ_OUTPUT = 4 * (4 + 3 * MAX_SPEC_TOKENS + 2 * MAX_TOP_LOGPROBS)

SAMPLING_DTYPE = np.dtype([("temperature", "<f4"), ("top_p", "<f4"), ("top_k", "<i4"), ("presence", "<f4"),
                           ("frequency", "<f4"), ("repetition", "<f4"), ("seed", "<u8"), ("logprobs", "<i4"),
                           ("pad", "<i4")])
SEQ_OUTPUT_DTYPE = np.dtype([("req_slot", "<i4"), ("num_tokens", "<i4"), ("tokens", "<i4", (MAX_SPEC_TOKENS,)),
                             ("logprobs", "<f4", (MAX_SPEC_TOKENS,)), ("top_ids", "<i4", (MAX_TOP_LOGPROBS,)),
                             ("top_logprobs", "<f4", (MAX_TOP_LOGPROBS,)),
                             ("next_drafts", "<i4", (MAX_SPEC_TOKENS,)), ("num_drafts", "<i4"), ("pad", "<i4")])
assert SAMPLING_DTYPE.itemsize == SIZEOF_SAMPLING
assert SEQ_OUTPUT_DTYPE.itemsize == SIZEOF_SEQ_OUTPUT


def select_bucket(n: int) -> int:
    for b in DECODE_BUCKETS:
        if b >= n:
            return b
    return 0


def align_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


@dataclass(frozen=True)
class Geometry:
    world_size: int = 1
    max_seqs: int = 256
    max_step_tokens: int = 8192
    max_pages_per_seq: int = 256
    page_size: int = 16
    vocab_size: int = 0


PLAN_FIELDS = ("header", "token_ids", "positions", "row_slot", "query_start", "seq_slot", "seq_len", "sample_row",
               "sampling", "dirty_rows", "dirty_pages", "ckpt_row", "ckpt_slot", "restore_slot", "spec_width", "kv_ops")


def plan_layout(g: Geometry) -> dict:
    max_ckpt = min(g.max_step_tokens, 4096)
    max_kv_ops = 1024
    sizes = {
        "header": SIZEOF_STEP_HEADER,
        "token_ids": 4 * g.max_step_tokens,
        "positions": 4 * g.max_step_tokens,
        "row_slot": 4 * g.max_step_tokens,
        "query_start": 4 * (g.max_seqs + 1),
        "seq_slot": 4 * g.max_seqs,
        "seq_len": 4 * g.max_seqs,
        "sample_row": 4 * g.max_seqs,
        "sampling": SIZEOF_SAMPLING * g.max_seqs,
        "dirty_rows": 4 * g.max_seqs,
        "dirty_pages": 4 * g.max_seqs * g.max_pages_per_seq,
        "ckpt_row": 4 * max_ckpt,
        "ckpt_slot": 4 * max_ckpt,
        "restore_slot": 4 * g.max_seqs,
        "spec_width": 4 * g.max_seqs,
        "kv_ops": 12 * max_kv_ops,
    }
    out, o = {}, 0
    for f in PLAN_FIELDS:
        o = align_up(o, ALIGN)
        out[f] = o
        o += sizes[f]
    out["bytes"] = align_up(o, 4096)
    out["max_ckpt"] = max_ckpt
    return out


def segment_layout(g: Geometry) -> dict:
    p = plan_layout(g)
    result_outputs = ALIGN
    result_bytes = align_up(ALIGN + SIZEOF_SEQ_OUTPUT * g.max_seqs, 4096)
    plan_offset = SUPERBLOCK_BYTES + WORKER_REGION_BYTES
    result_offset = plan_offset + PLAN_SLOTS * p["bytes"]
    total = result_offset + RESULT_SLOTS * result_bytes
    return {"plan": p, "result_outputs": result_outputs, "result_bytes": result_bytes, "plan_offset": plan_offset,
            "result_offset": result_offset, "total_bytes": total}


def _fnv1a_u64s(values) -> int:
    h = 2166136261
    for v in values:
        for b in struct.pack("<Q", v & 0xFFFFFFFFFFFFFFFF):
            h ^= b
            h = (h * 16777619) & 0xFFFFFFFF
    return h


def layout_hash(g: Geometry) -> int:
    s = segment_layout(g)
    p = s["plan"]
    vals = [VERSION, SIZEOF_SUPERBLOCK, SIZEOF_WORKER_STATE, SIZEOF_STEP_HEADER, SIZEOF_SAMPLING,
            SIZEOF_RESULT_HEADER, SIZEOF_SEQ_OUTPUT, ABORT_OFFSET, g.world_size, g.max_seqs, g.max_step_tokens,
            g.max_pages_per_seq, g.page_size]
    vals += [p[f] for f in PLAN_FIELDS[1:]]
    vals += [p["bytes"], s["result_outputs"], s["result_bytes"], s["plan_offset"], s["result_offset"],
             s["total_bytes"]]
    return _fnv1a_u64s(vals)


# Memory ordering: the master publishes a slot with a release store of its step id and
# the worker publishes results the same way.  On x86-64 (TSO) stores are not reordered
# with stores nor loads with loads, so the aligned 8-byte struct accesses below observe
# the protocol's ordering without extra fences.
class SegmentView:
    """Typed numpy views over a mapped segment (bytes-like object)."""

    def __init__(self, buf, geo: Geometry):
        self.buf = buf
        self.geo = geo
        self.lay = segment_layout(geo)
        self.u8 = np.frombuffer(buf, dtype=np.uint8)

    # -- superblock
    def superblock(self) -> dict:
        f = struct.unpack_from("<QIIIIIIII", self.buf, 0)
        return {"magic": f[0], "version": f[1], "layout_hash": f[2], "world_size": f[3], "max_seqs": f[4],
                "max_step_tokens": f[5], "max_pages_per_seq": f[6], "page_size": f[7], "vocab_size": f[8]}

    def abort_word(self) -> int:
        return struct.unpack_from("<I", self.buf, ABORT_OFFSET)[0]

    # -- worker state
    def worker_off(self, rank: int) -> int:
        return SUPERBLOCK_BYTES + rank * WORKER_STATE_BYTES

    def set_worker(self, rank: int, *, status=None, error=None, ready_step=None, heartbeat_ns=None, pid=None,
                   gpu_us=None) -> None:
        o = self.worker_off(rank)
        if pid is not None:
            struct.pack_into("<I", self.buf, o + 24, pid)
            struct.pack_into("<I", self.buf, o + 28, rank)
        if error is not None:
            struct.pack_into("<I", self.buf, o + 4, error)
        if gpu_us is not None:
            struct.pack_into("<Q", self.buf, o + 32, gpu_us)
        if heartbeat_ns is not None:
            struct.pack_into("<Q", self.buf, o + 16, heartbeat_ns)
        if ready_step is not None:
            struct.pack_into("<Q", self.buf, o + 8, ready_step)
        if status is not None:
            struct.pack_into("<I", self.buf, o, status)

    def worker(self, rank: int) -> dict:
        o = self.worker_off(rank)
        st, err, ready, hb, pid = struct.unpack_from("<IIQQI", self.buf, o)
        return {"status": st, "error": err, "ready_step": ready, "heartbeat_ns": hb, "pid": pid}

    # -- plan slots
    def plan_base(self, step_id: int) -> int:
        return self.lay["plan_offset"] + (step_id % PLAN_SLOTS) * self.lay["plan"]["bytes"]

    def plan_step_id(self, step_id: int) -> int:
        return struct.unpack_from("<Q", self.buf, self.plan_base(step_id))[0]

    def read_plan(self, step_id: int) -> dict:
        base = self.plan_base(step_id)
        p = self.lay["plan"]
        sid, opcode, flags, rows, seqs, ndirty, bucket, nckpt, nkv = struct.unpack_from("<QIIIIIIII", self.buf, base)
        g = self.geo

        def arr(field, n, dtype=np.int32):
            return np.frombuffer(self.buf, dtype=dtype, count=n, offset=base + p[field]).copy()

        plan = {"step_id": sid, "opcode": opcode, "flags": flags, "num_rows": rows, "num_seqs": seqs,
                "bucket": bucket, "token_ids": arr("token_ids", rows), "positions": arr("positions", rows),
                "row_slot": arr("row_slot", rows), "query_start": arr("query_start", seqs + 1),
                "seq_slot": arr("seq_slot", seqs), "seq_len": arr("seq_len", seqs),
                "sample_row": arr("sample_row", seqs), "sampling": arr("sampling", seqs, SAMPLING_DTYPE),
                "dirty_rows": arr("dirty_rows", ndirty),
                "dirty_pages": arr("dirty_pages", ndirty * g.max_pages_per_seq).reshape(ndirty, g.max_pages_per_seq),
                "ckpt_row": arr("ckpt_row", nckpt), "ckpt_slot": arr("ckpt_slot", nckpt),
                "restore_slot": arr("restore_slot", seqs), "spec_width": arr("spec_width", seqs)}
        return plan

    # -- result slots
    def write_result(self, step_id: int, outputs: np.ndarray, status: int = 0, gpu_us: int = 0) -> None:
        base = self.lay["result_offset"] + (step_id % RESULT_SLOTS) * self.lay["result_bytes"]
        n = len(outputs)
        dst = np.frombuffer(self.buf, dtype=SEQ_OUTPUT_DTYPE, count=n, offset=base + self.lay["result_outputs"])
        dst[:] = outputs
        struct.pack_into("<IIQ", self.buf, base + 8, status, n, gpu_us)
        struct.pack_into("<Q", self.buf, base, step_id)  # publish last
