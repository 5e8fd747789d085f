"""Writer for the reference's ``.wgpack`` container (``WGPACK02``).

The layout is the reference's, kept byte-for-byte so packs stay drop-in
(src/prepacked/format.ts:3-5,105-144): 8-byte magic, u32 little-endian JSON
header length, compact JSON header, payloads 256-byte aligned after the header.
Compact projections use the q4_0-tile32 layout (format.ts:65-99). The CUDA
library parses packs itself (csrc/wgpack.cpp); this module only writes them,
for synthetic models and tooling.
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field

import numpy as np

MAGIC = b"WGPACK02"
LAYOUT = "q4_0-tile32-compact-v2"
COMPACT = "q4_0-tile32-compact"
RAW = "raw"
F32, F16, Q4_0, Q4_K, Q6_K = 0, 1, 2, 12, 14


@dataclass
class PackedTensor:
    name: str
    dimensions: list
    type: int
    storage: str
    data: np.ndarray  # uint8 payload
    extra: dict = field(default_factory=dict)


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def build_wgpack(tensors: list[PackedTensor], metadata: dict | None = None, source_sha256: str = "",
                 source_bytes: int = 0) -> bytes:
    """buildPrepackedFile (format.ts:105-144)."""
    entries = []
    rel = 0
    for t in tensors:
        rel = _align(rel, 256)
        entries.append({"name": t.name, "dimensions": list(t.dimensions), "type": int(t.type),
                        "storage": t.storage, "offset": rel, "byteLength": int(t.data.nbytes)})
        rel += int(t.data.nbytes)
    header = {"version": 2, "sourceSha256": source_sha256, "sourceBytes": source_bytes, "layout": LAYOUT,
              "tileRows": 32, "blockValues": 32, "blockBytes": 20, "metadata": metadata or {},
              "tensors": entries}
    hb = json.dumps(header, separators=(",", ":"), ensure_ascii=False).encode("utf-8")
    data_offset = _align(12 + len(hb), 256)
    out = bytearray(data_offset + rel)
    out[0:8] = MAGIC
    out[8:12] = len(hb).to_bytes(4, "little")
    out[12:12 + len(hb)] = hb
    for t, e in zip(tensors, entries):
        o = data_offset + e["offset"]
        out[o:o + t.data.nbytes] = np.ascontiguousarray(t.data, dtype=np.uint8).tobytes()
    return bytes(out)
