"""Snapshot format (src/persist/format.ts) on the CPU: the byte layout of the
header, metadata JSON and vector region, round trips, the v2 graph section,
and the reference's error messages."""
import json
import struct

import numpy as np
import pytest

from browservec_b200.persist import deserialize, serialize


def _entries(n):
    return [{"id": f"id{i}", "metadata": ({"lang": "en", "year": 2000 + i, "w": 0.5} if i % 3 else None)}
            for i in range(n)]


def test_layout_matches_format_ts():
    n, d = 5, 3
    v = np.arange(n * d, dtype=np.float32).reshape(n, d) / 7
    buf = serialize(d, "dot", True, _entries(n), v)
    magic, ver, dim, metric, flags, count, mlen, goff = struct.unpack_from("<8I", buf, 0)
    assert (magic, ver, dim, metric, flags, count, goff) == (0x43455642, 1, 3, 1, 1, 5, 0)
    assert buf[:4] == b"BVEC"
    meta = buf[32:32 + mlen].decode()
    # JSON.stringify form: compact, id first, metadata omitted when absent, integral numbers bare
    assert meta.startswith('[{"id":"id0"},{"id":"id1","metadata":{"lang":"en","year":2001,"w":0.5}}')
    voff = 32 + ((mlen + 3) & ~3)
    assert len(buf) == voff + n * d * 4
    assert np.array_equal(np.frombuffer(buf, "<f4", n * d, voff).reshape(n, d), v)


def test_round_trip_and_view():
    n, d = 100, 17
    v = np.random.default_rng(0).standard_normal((n, d)).astype(np.float32)
    s = deserialize(serialize(d, "cosine", True, _entries(n), v))
    assert (s.dimension, s.metric, s.normalize, s.count) == (d, "cosine", True, n)
    assert np.array_equal(s.vectors, v) and s.graph is None
    assert [e["id"] for e in s.entries] == [f"id{i}" for i in range(n)]
    assert s.entries[1]["metadata"] == {"lang": "en", "year": 2001, "w": 0.5} and "metadata" not in s.entries[0]


def test_v2_graph_section_is_read():
    n, d, M = 4, 2, 2
    v = np.ones((n, d), np.float32)
    base = bytearray(serialize(d, "l2", False, _entries(n), v))
    goff = len(base)
    levels = np.array([0, 1, 0, 0], "<i4")
    links0 = np.arange(n * (2 * M + 1), dtype="<i4")
    upper = np.array([7, 8], "<i4")
    head = struct.pack("<8I", 0x57534E48, 1, M, 1, 1, upper.size, 0, 0)
    base[4:8] = struct.pack("<I", 2)
    base[28:32] = struct.pack("<I", goff)
    buf = bytes(base) + head + levels.tobytes() + links0.tobytes() + upper.tobytes()
    s = deserialize(buf)
    assert s.graph["M"] == M and s.graph["entry"] == 1 and np.array_equal(s.graph["upper"], upper)
    assert np.array_equal(s.graph["links0"], links0) and np.array_equal(s.vectors, v)


def test_reference_errors():
    good = serialize(2, "cosine", True, _entries(2), np.zeros((2, 2), np.float32))
    with pytest.raises(ValueError, match="snapshot too small / corrupt"):
        deserialize(good[:10])
    with pytest.raises(ValueError, match="bad magic: not a BrowserVec snapshot"):
        deserialize(b"XXXX" + good[4:])
    with pytest.raises(ValueError, match=r"unsupported snapshot version 3 \(this build reads 1..2\)"):
        deserialize(good[:4] + struct.pack("<I", 3) + good[8:])
    with pytest.raises(ValueError, match="unknown metric code in snapshot"):
        deserialize(good[:12] + struct.pack("<I", 9) + good[16:])
    with pytest.raises(ValueError, match="snapshot truncated \\(vector region\\)"):
        deserialize(good[:-4])
    bad = json.dumps([{"id": "a"}]).encode()
    with pytest.raises(ValueError, match="entry count 1 != header count 2"):
        deserialize(struct.pack("<8I", 0x43455642, 1, 2, 0, 1, 2, len(bad), 0) + bad + b"\0" * 64)
