"""CPU oracle for the Nemotron-3-Embed-1B forward pass (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s ``cpu_baseline``
leg may import this package: it is the checker the CUDA library is compared
against, never part of the product path.

The arithmetic lives in ``oracle.cpp`` (a C++ restatement of the reference's
``src/gguf/quantization.ts``, ``src/math/f16.ts``, ``src/prepacked/format.ts``
and the WGSL shader math of ``src/webgpu/ops.ts`` / ``quant-matmul.ts`` wired as
``src/webgpu/model.ts:73-176``). This module restates the ``.wgpack`` parser
(``src/prepacked/format.ts:146-169``) and binds the library with ctypes.

Parity pins: the quantisation/format/merge-length code is pinned against the
reference's own known-answer tests (tests/golden/reference_known_answers.json).
The forward pass has no golden vectors in the reference; it is pinned only by
this restatement.
"""
from __future__ import annotations

import ctypes
import json
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

F32, F16, Q4_0, Q4_K, Q6_K = 0, 1, 2, 12, 14
HIDDEN, INTER, QKV_WIDTH = 2048, 6144, 5120
COMPACT = "q4_0-tile32-compact"
RAW = "raw"


def build() -> str:
    """Compiles liboracle.so from oracle.cpp (make in this directory)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
            os.path.join(_HERE, "oracle.cpp")
        ):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        L.orc_half_to_float.restype = ctypes.c_double
        L.orc_half_to_float.argtypes = [ctypes.c_uint16]
        L.orc_float_to_half.restype = ctypes.c_uint16
        L.orc_float_to_half.argtypes = [ctypes.c_double]
        L.orc_f16_rne.restype = ctypes.c_uint16
        L.orc_f16_rne.argtypes = [ctypes.c_float]
        for name in ("orc_dequant_q4k_block", "orc_dequant_q40_block", "orc_dequant_q6k_block",
                     "orc_quantize_q40_block"):
            getattr(L, name).argtypes = [P, P]
            getattr(L, name).restype = None
        L.orc_requantize_to_q40.argtypes = [P, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        L.orc_pack_q40_tile32.argtypes = [P, P, ctypes.c_int, ctypes.c_int, P]
        L.orc_decode_matrix.argtypes = [P, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        ctypes.c_int, P]
        L.orc_merged_length.restype = ctypes.c_uint32
        L.orc_merged_length.argtypes = [ctypes.c_uint32]
        L.orc_model_create.restype = P
        L.orc_model_create.argtypes = [P, ctypes.c_char_p, ctypes.c_size_t]
        L.orc_model_destroy.argtypes = [P]
        L.orc_model_weights_f16.argtypes = [P, ctypes.c_int, ctypes.c_int, P]
        L.orc_forward.argtypes = [P, ctypes.c_int, ctypes.c_int, P, P, P, P, P, P, ctypes.c_char_p,
                                  ctypes.c_size_t]
        L.orc_forward_ex.argtypes = [P, ctypes.c_int, ctypes.c_int, P, P, ctypes.c_int, P, P, P, P,
                                     ctypes.c_char_p, ctypes.c_size_t]
        L.orc_embedding.argtypes = [P, ctypes.c_int, P, ctypes.c_int, P]
        L.orc_residual_rmsnorm.argtypes = [P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.orc_matmul_f16.argtypes = [P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P]
        L.orc_rope_table.argtypes = [ctypes.c_int, P]
        L.orc_rope.argtypes = [P, P, ctypes.c_int, P, P, P]
        L.orc_attention.argtypes = [P, P, P, P, P, ctypes.c_int, P]
        L.orc_swiglu.argtypes = [P, ctypes.c_int, P]
        L.orc_token_merge.argtypes = [P, P, P, P, P, ctypes.c_int, P]
        L.orc_mean_pool.argtypes = [P, P, P, ctypes.c_int, P]
        L.orc_num_threads.restype = ctypes.c_int
        L.orc_set_num_threads.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


# --- scalar / block helpers -------------------------------------------------

def half_to_float(bits: int) -> float:
    return lib().orc_half_to_float(bits)


def float_to_half(value: float) -> int:
    """f16.ts:4-25 (half-up rounding)."""
    return lib().orc_float_to_half(value)


def f16_rne(values: np.ndarray) -> np.ndarray:
    """The shader's f16() cast (round to nearest even) as u16 bit patterns."""
    v = np.ascontiguousarray(values, dtype=np.float32).ravel()
    return np.array([lib().orc_f16_rne(float(x)) for x in v], dtype=np.uint16)


def dequant_block(block: bytes | np.ndarray, gtype: int) -> np.ndarray:
    b = np.frombuffer(bytes(block), dtype=np.uint8).copy()
    out = np.zeros(32 if gtype == Q4_0 else 256, dtype=np.float32)
    fn = {Q4_K: "orc_dequant_q4k_block", Q4_0: "orc_dequant_q40_block", Q6_K: "orc_dequant_q6k_block"}[gtype]
    getattr(lib(), fn)(_p(b), _p(out))
    return out


def quantize_q40_block(values: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.float32)
    out = np.zeros(18, dtype=np.uint8)
    lib().orc_quantize_q40_block(_p(v), _p(out))
    return out


def requantize_to_q40(src: np.ndarray, gtype: int, k: int, n: int) -> np.ndarray:
    s = np.ascontiguousarray(src, dtype=np.uint8)
    out = np.zeros(n * (k // 32) * 18, dtype=np.uint8)
    rc = lib().orc_requantize_to_q40(_p(s), s.nbytes, gtype, k, n, _p(out))
    if rc:
        raise ValueError(f"requantize failed ({rc})")
    return out


def pack_q40_tile32(parts: list[tuple[np.ndarray, int]], k: int) -> np.ndarray:
    arrs = [np.ascontiguousarray(a, dtype=np.uint8) for a, _ in parts]
    rows = np.array([n for _, n in parts], dtype=np.int32)
    ptrs = (ctypes.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
    n = int(rows.sum())
    out = np.zeros(((n + 31) // 32) * (k // 32) * 32 * 20, dtype=np.uint8)
    rc = lib().orc_pack_q40_tile32(ptrs, _p(rows), len(arrs), k, _p(out))
    if rc:
        raise ValueError(f"pack failed ({rc})")
    return out


def decode_matrix(data: np.ndarray, gtype: int, compact: bool, k: int, n: int) -> np.ndarray:
    d = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.zeros((n, k), dtype=np.float32)
    rc = lib().orc_decode_matrix(_p(d), d.nbytes, gtype, int(compact), k, n, _p(out))
    if rc:
        raise ValueError(f"decode failed ({rc})")
    return out


def merged_length(sequence: int) -> int:
    return lib().orc_merged_length(sequence)


# --- .wgpack parser (format.ts:146-169) ------------------------------------

MAGIC = b"WGPACK02"


@dataclass
class PackTensor:
    name: str
    dimensions: list
    type: int
    storage: str
    offset: int
    byte_length: int
    byte_offset: int


def parse_wgpack(buf: bytes | memoryview) -> tuple[dict, dict]:
    """Restates parsePrepackedModel (format.ts:146-169)."""
    buf = memoryview(buf)
    if len(buf) < 12:
        raise ValueError("prepacked model is shorter than its prelude")
    if bytes(buf[:8]) != MAGIC:
        raise ValueError(f"invalid prepacked model magic {bytes(buf[:8])!r}")
    hlen = int.from_bytes(bytes(buf[8:12]), "little")
    if 12 + hlen > len(buf):
        raise ValueError("prepacked model header extends past end of file")
    header = json.loads(bytes(buf[12:12 + hlen]).decode("utf-8"))
    if (header.get("version") != 2 or header.get("layout") != "q4_0-tile32-compact-v2"
            or header.get("tileRows") != 32 or header.get("blockValues") != 32 or header.get("blockBytes") != 20):
        raise ValueError(f"unsupported prepacked layout {header.get('layout')}")
    data_offset = (12 + hlen + 255) // 256 * 256
    tensors = {}
    for t in header["tensors"]:
        bo = data_offset + t["offset"]
        if bo + t["byteLength"] > len(buf):
            raise ValueError(f"{t['name']} extends past end of prepacked file")
        if t["name"] in tensors:
            raise ValueError(f"duplicate prepacked tensor {t['name']}")
        if t["storage"] == COMPACT and (t["type"] != Q4_0 or len(t["dimensions"]) != 2):
            raise ValueError(f"{t['name']} has invalid compact Q4_0 metadata")
        if t["storage"] not in (COMPACT, RAW):
            raise ValueError(f"{t['name']} has unsupported storage {t['storage']}")
        tensors[t["name"]] = PackTensor(t["name"], list(t["dimensions"]), t["type"], t["storage"], t["offset"],
                                        t["byteLength"], bo)
    return header, tensors


# --- model + forward --------------------------------------------------------

class _Part(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("nbytes", ctypes.c_size_t), ("type", ctypes.c_int),
                ("compact", ctypes.c_int), ("k", ctypes.c_int), ("n", ctypes.c_int)]


class _Proj(ctypes.Structure):
    _fields_ = [("parts", _Part * 3), ("nparts", ctypes.c_int)]


class _Desc(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("vocab", ctypes.c_int), ("token_embd", ctypes.c_void_p),
                ("token_embd_bytes", ctypes.c_size_t), ("attn_norm", ctypes.c_void_p * 16),
                ("ffn_norm", ctypes.c_void_p * 16), ("output_norm", ctypes.c_void_p),
                ("qkv", _Proj * 16), ("o", _Proj * 16), ("gate_up", _Proj * 16), ("down", _Proj * 16)]


_FUSED = {
    "qkv": ("attn_qkv", ["attn_q", "attn_k", "attn_v"]),
    "o": ("attn_output", ["attn_output"]),
    "gate_up": ("ffn_gate_up", ["ffn_gate", "ffn_up"]),
    "down": ("ffn_down", ["ffn_down"]),
}


class OracleModel:
    """Effective f16 weights of a .wgpack, decoded once, plus the CPU forward."""

    def __init__(self, pack: bytes | np.ndarray):
        self._buf = np.frombuffer(bytes(pack) if not isinstance(pack, np.ndarray) else pack.tobytes(),
                                  dtype=np.uint8)
        self.header, self.tensors = parse_wgpack(self._buf.data)
        base = self._buf.ctypes.data
        d = _Desc()
        n_layers = 0
        while f"blk.{n_layers}.attn_norm.weight" in self.tensors:
            n_layers += 1
        d.n_layers = n_layers
        te = self.tensors["token_embd.weight"]
        d.vocab = te.dimensions[1]
        d.token_embd = base + te.byte_offset
        d.token_embd_bytes = te.byte_length
        d.output_norm = base + self.tensors["output_norm.weight"].byte_offset
        for l in range(n_layers):
            d.attn_norm[l] = base + self.tensors[f"blk.{l}.attn_norm.weight"].byte_offset
            d.ffn_norm[l] = base + self.tensors[f"blk.{l}.ffn_norm.weight"].byte_offset
            for field, (fused, parts) in _FUSED.items():
                proj = getattr(d, field)[l]
                fname = f"blk.{l}.{fused}.weight"
                if fname in self.tensors and self.tensors[fname].storage == COMPACT:
                    names = [fname]
                else:
                    names = [f"blk.{l}.{p}.weight" for p in parts]
                proj.nparts = len(names)
                for i, nm in enumerate(names):
                    t = self.tensors[nm]
                    proj.parts[i].data = base + t.byte_offset
                    proj.parts[i].nbytes = t.byte_length
                    proj.parts[i].type = t.type
                    proj.parts[i].compact = int(t.storage == COMPACT)
                    proj.parts[i].k = t.dimensions[0]
                    proj.parts[i].n = t.dimensions[1]
        err = ctypes.create_string_buffer(256)
        self.n_layers = n_layers
        self.vocab = d.vocab
        self._desc = d
        self._h = lib().orc_model_create(ctypes.byref(d), err, 256)
        if not self._h:
            raise ValueError(err.value.decode())

    def close(self):
        if getattr(self, "_h", None):
            lib().orc_model_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def weights_f16(self, layer: int, which: int) -> np.ndarray:
        shapes = [(QKV_WIDTH, HIDDEN), (HIDDEN, 3072), (2 * INTER, HIDDEN), (HIDDEN, INTER)]
        out = np.zeros(shapes[which], dtype=np.uint16)
        if lib().orc_model_weights_f16(self._h, layer, which, _p(out)):
            raise ValueError("bad layer/which")
        return out

    def norm_weight(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return self._buf[t.byte_offset:t.byte_offset + t.byte_length].view(np.float32)

    def token_embd(self) -> np.ndarray:
        t = self.tensors["token_embd.weight"]
        return self._buf[t.byte_offset:t.byte_offset + t.byte_length]

    def forward(self, batch: int, sequence: int, ids: np.ndarray, lengths: np.ndarray, dumps: bool = False,
                exact: bool = False):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        lengths = np.ascontiguousarray(lengths, dtype=np.uint32)
        if ids.size != batch * sequence:
            raise ValueError("token buffer does not match execution plan")
        out = np.zeros((batch, HIDDEN), dtype=np.float32)
        xd = nd = None
        tpl = np.zeros(16, dtype=np.int32)
        if dumps:
            xd = np.zeros((self.n_layers, batch * sequence, HIDDEN), dtype=np.uint16)
            nd = np.zeros_like(xd)
        err = ctypes.create_string_buffer(256)
        rc = lib().orc_forward_ex(self._h, batch, sequence, _p(ids), _p(lengths), 1 if exact else 0, _p(out),
                                  _p(xd) if dumps else None, _p(nd) if dumps else None, _p(tpl), err, 256)
        if rc:
            raise ValueError(err.value.decode())
        if dumps:
            return out, [(xd[l, :tpl[l]], nd[l, :tpl[l]]) for l in range(self.n_layers)]
        return out


# --- stage wrappers (packed valid tokens) -----------------------------------

def embedding(token_embd: np.ndarray, vocab: int, ids: np.ndarray) -> np.ndarray:
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    out = np.zeros((ids.size, HIDDEN), dtype=np.uint16)
    lib().orc_embedding(_p(np.ascontiguousarray(token_embd)), vocab, _p(ids), ids.size, _p(out))
    return out


def residual_rmsnorm(x: np.ndarray, residual, weight: np.ndarray, eps: float = 1e-5):
    x = np.ascontiguousarray(x, dtype=np.uint16).copy()
    w = np.ascontiguousarray(weight, dtype=np.float32)
    norm = np.zeros_like(x)
    r = None if residual is None else np.ascontiguousarray(residual, dtype=np.uint16)
    lib().orc_residual_rmsnorm(_p(x), None if r is None else _p(r), _p(w), _p(norm), x.shape[0], x.shape[1], eps)
    return x, norm


def matmul_f16(x: np.ndarray, w: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.uint16)
    w = np.ascontiguousarray(w, dtype=np.uint16)
    m, k = x.shape
    n = w.shape[0]
    of = np.zeros((m, n), dtype=np.float32)
    oh = np.zeros((m, n), dtype=np.uint16)
    lib().orc_matmul_f16(_p(x), _p(w), m, n, k, _p(of), _p(oh))
    return of, oh


def rope_table(sequence: int) -> np.ndarray:
    t = np.zeros((sequence, 64, 2), dtype=np.float32)
    lib().orc_rope_table(sequence, _p(t))
    return t


def rope(qkv: np.ndarray, positions: np.ndarray, table: np.ndarray):
    qkv = np.ascontiguousarray(qkv, dtype=np.uint16)
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    t = qkv.shape[0]
    q = np.zeros((t, 3072), dtype=np.uint16)
    k = np.zeros((t, 1024), dtype=np.uint16)
    lib().orc_rope(_p(qkv), _p(pos), t, _p(np.ascontiguousarray(table, dtype=np.float32)), _p(q), _p(k))
    return q, k


def attention(q: np.ndarray, k: np.ndarray, qkv: np.ndarray, lengths: np.ndarray) -> np.ndarray:
    lengths = np.ascontiguousarray(lengths, dtype=np.uint32)
    offsets = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(np.int32)
    out = np.zeros((q.shape[0], 3072), dtype=np.uint16)
    lib().orc_attention(_p(np.ascontiguousarray(q)), _p(np.ascontiguousarray(k)), _p(np.ascontiguousarray(qkv)),
                        _p(offsets), _p(lengths), lengths.size, _p(out))
    return out


def swiglu(gate_up: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(gate_up, dtype=np.uint16)
    out = np.zeros((g.shape[0], INTER), dtype=np.uint16)
    lib().orc_swiglu(_p(g), g.shape[0], _p(out))
    return out


def token_merge(x: np.ndarray, src_lengths: np.ndarray, dst_lengths: np.ndarray) -> np.ndarray:
    sl = np.ascontiguousarray(src_lengths, dtype=np.uint32)
    dl = np.ascontiguousarray(dst_lengths, dtype=np.uint32)
    so = np.concatenate([[0], np.cumsum(sl)[:-1]]).astype(np.int32)
    do = np.concatenate([[0], np.cumsum(dl)[:-1]]).astype(np.int32)
    out = np.zeros((int(dl.sum()), HIDDEN), dtype=np.uint16)
    lib().orc_token_merge(_p(np.ascontiguousarray(x, dtype=np.uint16)), _p(so), _p(sl), _p(do), _p(dl), sl.size,
                          _p(out))
    return out


def mean_pool(x: np.ndarray, lengths: np.ndarray) -> np.ndarray:
    ln = np.ascontiguousarray(lengths, dtype=np.uint32)
    off = np.concatenate([[0], np.cumsum(ln)[:-1]]).astype(np.int32)
    out = np.zeros((ln.size, HIDDEN), dtype=np.float32)
    lib().orc_mean_pool(_p(np.ascontiguousarray(x, dtype=np.uint16)), _p(off), _p(ln), ln.size, _p(out))
    return out


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(n)
