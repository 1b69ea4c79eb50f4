"""BrowserVec snapshots: the reference's versioned binary format, read and
written on the host, loaded into the device index in one bulk append.

Format (src/persist/format.ts:1-22, little-endian): a 32-byte header ("BVEC",
version, dimension, metric code, flags bit0 = normalize, count, metadata JSON
length, v2 graph offset), the metadata JSON (``[{id, metadata?}]`` in row
order), padding to 4 bytes, then count x dimension float32 vectors, already
normalized when the store normalizes; version 2 appends an HNSW graph section
(kept by ``deserialize``, unused by this flat index).  Error messages are the
reference's (format.ts:121-175), so callers see the same failures.

The reference reloads a snapshot by inserting every row through its store and
re-quantizing on the host (src/index.ts:673-700); here the vector region is
viewed in place (no copy) and handed to the index in one append, which
encodes on the GPU.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field
from typing import Any

import numpy as np

MAGIC = 0x43455642        # "BVEC"
GRAPH_MAGIC = 0x57534E48  # "HNSW"
FORMAT_VERSION = 2
HEADER_BYTES = 32
GRAPH_HEADER_WORDS = 8
GRAPH_VERSION = 1
METRIC_TO_CODE = {"cosine": 0, "dot": 1, "l2": 2}
CODE_TO_METRIC = ["cosine", "dot", "l2"]


@dataclass
class Snapshot:
    dimension: int
    metric: str
    normalize: bool
    count: int
    entries: list          # [{"id": str, "metadata"?: dict}] in row order
    vectors: np.ndarray    # (count, dimension) float32 (a view of the buffer when read)
    graph: dict | None = field(default=None)


def _js_json(obj: Any) -> bytes:
    """JSON.stringify of the entries: compact separators, NaN/Infinity as null."""
    def clean(v):
        if isinstance(v, float) and (v != v or v in (float("inf"), float("-inf"))):
            return None
        if isinstance(v, float) and v == int(v) and abs(v) < 1e21:
            return int(v)  # JS prints integral numbers without a fraction
        if isinstance(v, dict):
            return {k: clean(x) for k, x in v.items()}
        if isinstance(v, (list, tuple)):
            return [clean(x) for x in v]
        return v
    return json.dumps(clean(obj), separators=(",", ":"), ensure_ascii=False).encode("utf-8")


def serialize(dimension: int, metric: str, normalize: bool, entries: list, vectors: np.ndarray) -> bytes:
    """format.ts:64-117 without a graph section (a v1 snapshot)."""
    vectors = np.ascontiguousarray(vectors, dtype="<f4")
    count = len(entries)
    if vectors.size != count * dimension:
        raise ValueError(f"vectors length {vectors.size} != count*dim {count * dimension}")
    meta = _js_json([{"id": e["id"], "metadata": e["metadata"]} if e.get("metadata") is not None
                     else {"id": e["id"]} for e in entries])
    pad = (len(meta) + 3) & ~3
    head = struct.pack("<8I", MAGIC, 1, dimension, METRIC_TO_CODE[metric], 1 if normalize else 0, count,
                       len(meta), 0)
    return b"".join([head, meta, b"\0" * (pad - len(meta)), vectors.tobytes()])


def deserialize(buf) -> Snapshot:
    """format.ts:119-176.  The vectors are a read-only view of `buf`."""
    mv = memoryview(buf)
    if mv.nbytes < HEADER_BYTES:
        raise ValueError("snapshot too small / corrupt")
    magic, version, dimension, mcode, flags, count, meta_len, goff = struct.unpack_from("<8I", mv, 0)
    if magic != MAGIC:
        raise ValueError("bad magic: not a BrowserVec snapshot")
    if version < 1 or version > FORMAT_VERSION:
        raise ValueError(f"unsupported snapshot version {version} (this build reads 1..{FORMAT_VERSION})")
    if mcode >= len(CODE_TO_METRIC):
        raise ValueError("unknown metric code in snapshot")
    metric = CODE_TO_METRIC[mcode]
    meta_padded = (meta_len + 3) & ~3
    entries = json.loads(bytes(mv[HEADER_BYTES:HEADER_BYTES + meta_len]).decode("utf-8"))
    if len(entries) != count:
        raise ValueError(f"entry count {len(entries)} != header count {count}")
    voff = HEADER_BYTES + meta_padded
    if mv.nbytes < voff + count * dimension * 4:
        raise ValueError("snapshot truncated (vector region)")
    vectors = np.frombuffer(mv, dtype="<f4", count=count * dimension, offset=voff).reshape(count, dimension)
    snap = Snapshot(dimension, metric, (flags & 1) == 1, count, entries, vectors)
    goff = goff if version >= 2 else 0
    if goff:
        if mv.nbytes < goff + GRAPH_HEADER_WORDS * 4:
            raise ValueError("snapshot truncated (graph header)")
        head = struct.unpack_from(f"<{GRAPH_HEADER_WORDS}I", mv, goff)
        if head[0] != GRAPH_MAGIC:
            raise ValueError("bad graph section magic")
        if head[1] != GRAPH_VERSION:
            raise ValueError(f"unsupported graph section version {head[1]}")
        M, upper_len = head[2], head[5]
        links0_len = count * (2 * M + 1)
        off = goff + GRAPH_HEADER_WORDS * 4
        if mv.nbytes < off + (count + links0_len + upper_len) * 4:
            raise ValueError("snapshot truncated (graph region)")
        i32 = np.frombuffer(mv, dtype="<i4", count=count + links0_len + upper_len, offset=off)
        snap.graph = {"M": M, "entry": struct.unpack("<i", struct.pack("<I", head[3]))[0],
                      "top": struct.unpack("<i", struct.pack("<I", head[4]))[0],
                      "levels": i32[:count], "links0": i32[count:count + links0_len],
                      "upper": i32[count + links0_len:]}
    return snap
