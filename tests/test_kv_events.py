"""KV event publishing: msgpack batch encoding and the ZMTP 3.0 PUB transport, checked
against a minimal ZMTP subscriber written here (no ZeroMQ library needed)."""

import socket
import struct
import threading

import pytest

from zstep_b200 import _master as M

msgpack = pytest.importorskip("msgpack")


def test_encode_batch():
    b = msgpack.unpackb(M.encode_kv_batch(0, [1, 0x0102030405060708], 12.5), raw=False)
    assert b[0] == 12.5
    ev = b[1][0]
    assert ev["type"] == "BlockStored" and ev["medium"] == "GPU"
    assert ev["block_hashes"] == [struct.pack(">Q", 1), bytes(range(1, 9))]
    assert msgpack.unpackb(M.encode_kv_batch(1, [7], 0.0))[1][0] == {"type": "BlockRemoved",
                                                                   "block_hashes": [struct.pack(">Q", 7)]}
    assert msgpack.unpackb(M.encode_kv_batch(2, [], 0.0))[1][0] == {"type": "AllBlocksCleared"}


def _read_exact(c, n):
    b = b""
    while len(b) < n:
        chunk = c.recv(n - len(b))
        assert chunk, "peer closed"
        b += chunk
    return b


def _read_frame(c):
    flags, = _read_exact(c, 1)
    size = struct.unpack(">Q", _read_exact(c, 8))[0] if flags & 2 else _read_exact(c, 1)[0]
    return flags, _read_exact(c, size)


def _frame(body: bytes, more=False, command=False):
    return bytes([(1 if more else 0) | (4 if command else 0), len(body)]) + body


def test_zmtp_pub_delivers_to_subscriber():
    srv = socket.socket()
    srv.bind(("127.0.0.1", 0))
    srv.listen(1)
    port = srv.getsockname()[1]
    got = []

    def subscriber():
        c, _ = srv.accept()
        greeting = b"\xff" + b"\0" * 8 + b"\x7f" + bytes([3, 0]) + b"NULL".ljust(20, b"\0") + b"\0" + b"\0" * 31
        c.sendall(greeting)
        peer = _read_exact(c, 64)
        assert peer[0] == 0xFF and peer[10] == 3 and peer[12:16] == b"NULL"
        ready = b"\x05READY" + b"\x0bSocket-Type" + struct.pack(">I", 3) + b"SUB"
        c.sendall(_frame(ready, command=True))
        flags, body = _read_frame(c)
        assert flags & 4 and body[1:6] == b"READY" and b"PUB" in body
        c.sendall(_frame(b"\x01model/"))  # subscribe to the topic prefix
        while len(got) < 3:
            parts = []
            while True:
                flags, body = _read_frame(c)
                parts.append(body)
                if not flags & 1:
                    break
            got.append(parts)
        c.close()

    t = threading.Thread(target=subscriber)
    t.start()
    pub = M.KvEventPublisher(f"tcp://127.0.0.1:{port}", "model/0")
    pub.start()
    pub.publish(0, [11, 12])
    pub.publish(1, [11])
    t.join(timeout=30)
    pub.stop()
    srv.close()
    assert len(got) == 3
    topics = {p[0] for p in got}
    assert topics == {b"model/0"}
    seqs = [struct.unpack(">Q", p[1])[0] for p in got]
    assert seqs == [0, 1, 2]
    events = [msgpack.unpackb(p[2])[1][0]["type"] for p in got]
    assert events == ["AllBlocksCleared", "BlockStored", "BlockRemoved"]


def test_file_sink(tmp_path):
    path = tmp_path / "events.bin"
    pub = M.KvEventPublisher(f"file://{path}", "t")
    pub.start()
    pub.publish(0, [5])
    pub.stop()
    data = path.read_bytes()
    out = []
    while data:
        n = struct.unpack(">I", data[:4])[0]
        out.append(msgpack.unpackb(data[4:4 + n])[1][0]["type"])
        data = data[4 + n:]
    assert out == ["AllBlocksCleared", "BlockStored"] and pub.sent() == 2
