"""Seeded synthetic Nemotron-3-Embed-1B packs and inputs.

No checkpoint or GGUF can be downloaded here, so every benchmark and parity test
runs on random-init weights of the real architecture, written as real
``WGPACK02`` files in one of two flavours:

* ``"kquant"`` -- the Q4_K_M mix kept as raw GGML K-quant blocks, one tensor per
  GGUF projection (attn_q/k/v, attn_output, ffn_gate/up/down). Q6_K on
  ``token_embd``, every ``attn_v`` and ``ffn_down`` in the layers llama.cpp's
  Q4_K_M rule upgrades (0,1,4,7,10,13,14,15); Q4_K elsewhere.
* ``"q40"`` -- what the reference's offline converter emits from that GGUF
  (scripts/prepack-model.ts:28-45): every projection requantised to Q4_0
  (quantization.ts:77-131, half-up f16 scales of f16.ts:4-25), Q/K/V and
  gate/up fused, tile32-packed (format.ts:65-99).

The numpy restatements below are vectorised versions of the reference's CPU
code; tests check them bit-exactly against the C oracle.
"""
from __future__ import annotations

import hashlib
import os

import numpy as np

from .wgpack import COMPACT, F32, Q4_0, Q4_K, Q6_K, RAW, PackedTensor, build_wgpack

HIDDEN, INTER, VOCAB, LAYERS = 2048, 6144, 131072, 16
BOS, PAD = 1, 11
# llama.cpp's Q4_K_M "use more bits" layers for n_layer = 16.
Q6K_DOWN_LAYERS = frozenset({0, 1, 4, 7, 10, 13, 14, 15})
# Block scale sigmas chosen so decoded weights have std ~0.02 and mean ~0.
Q4K_D_SIGMA = 6.1e-5
Q4K_DMIN_SIGMA = 7.5 * Q4K_D_SIGMA
Q6K_D_SIGMA = 1.5e-5


# --- f16 -------------------------------------------------------------------

def float_to_half_up(values) -> np.ndarray:
    """floatToHalf (f16.ts:4-25), vectorised: f32 input, half-up rounding."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.int64)
    sign = (bits >> 16) & 0x8000
    exp = ((bits >> 23) & 0xFF) - 127 + 15
    man = bits & 0x7FFFFF
    out = np.zeros_like(bits)
    tiny = exp < -10
    sub = (exp <= 0) & ~tiny
    shift = np.where(sub, 1 - exp, 0)
    m_sub = (man | 0x800000) >> shift
    out = np.where(tiny, sign, out)
    out = np.where(sub, sign | ((m_sub + 0x1000) >> 13), out)
    normal = exp > 0
    round_up = normal & ((man & 0x1000) != 0)
    man2 = np.where(round_up, man + 0x2000, man)
    carry = (man2 & 0x800000) != 0
    man2 = np.where(carry, 0, man2)
    exp2 = np.where(carry, exp + 1, exp)
    norm_val = sign | (exp2 << 10) | (man2 >> 13)
    out = np.where(normal, norm_val, out)
    out = np.where(normal & (exp2 >= 31), sign | 0x7C00, out)
    out = np.where(exp >= 31, sign | 0x7C00, out)
    return out.astype(np.uint16)


def _f16_field(blocks: np.ndarray, at: int) -> np.ndarray:
    return np.ascontiguousarray(blocks[:, at:at + 2]).view(np.float16).astype(np.float64).reshape(-1)


# --- decoders (quantization.ts:11-74) -------------------------------------

def dequant_q4k(blocks: np.ndarray) -> np.ndarray:
    blocks = blocks.reshape(-1, 144)
    n = blocks.shape[0]
    d = _f16_field(blocks, 0)[:, None]
    dmin = _f16_field(blocks, 2)[:, None]
    s = blocks[:, 4:16].astype(np.int64)
    sc = np.empty((n, 8), np.int64)
    mn = np.empty((n, 8), np.int64)
    sc[:, :4] = s[:, :4] & 63
    mn[:, :4] = s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 0x0F) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    q = blocks[:, 16:144].reshape(n, 4, 32).astype(np.int64)
    out = np.empty((n, 4, 2, 32), np.float32)
    for g in range(4):
        out[:, g, 0] = (d * sc[:, 2 * g:2 * g + 1] * (q[:, g] & 15) - dmin * mn[:, 2 * g:2 * g + 1]).astype(np.float32)
        out[:, g, 1] = (d * sc[:, 2 * g + 1:2 * g + 2] * (q[:, g] >> 4) - dmin * mn[:, 2 * g + 1:2 * g + 2]).astype(np.float32)
    return out.reshape(n, 256)


def dequant_q6k(blocks: np.ndarray) -> np.ndarray:
    blocks = blocks.reshape(-1, 210)
    n = blocks.shape[0]
    d = _f16_field(blocks, 208)[:, None]
    ql = blocks[:, 0:128].astype(np.int64)
    qh = blocks[:, 128:192].astype(np.int64)
    sc = blocks[:, 192:208].view(np.int8).astype(np.int64)
    out = np.empty((n, 2, 4, 32), np.float32)
    lane_pair = np.arange(32) >> 4
    for h in range(2):
        la = ql[:, h * 64:h * 64 + 32]
        lb = ql[:, h * 64 + 32:h * 64 + 64]
        hi = qh[:, h * 32:h * 32 + 32]
        qs = [(la & 15) | ((hi & 3) << 4), (lb & 15) | (((hi >> 2) & 3) << 4),
              (la >> 4) | (((hi >> 4) & 3) << 4), (lb >> 4) | (((hi >> 6) & 3) << 4)]
        for j in range(4):
            scale = sc[:, h * 8 + lane_pair + 2 * j]
            out[:, h, j] = (d * scale * (qs[j] - 32)).astype(np.float32)
    return out.reshape(n, 256)


def dequant_q40(blocks: np.ndarray) -> np.ndarray:
    blocks = blocks.reshape(-1, 18)
    d = _f16_field(blocks, 0)[:, None]
    q = blocks[:, 2:18].astype(np.int64)
    return np.concatenate([(d * ((q & 15) - 8)), (d * ((q >> 4) - 8))], axis=1).astype(np.float32)


# --- encoders ---------------------------------------------------------------

def quantize_q40(values: np.ndarray) -> np.ndarray:
    """quantizeQ40Block (quantization.ts:77-98) over rows of 32 values."""
    v = values.reshape(-1, 32).astype(np.float32).astype(np.float64)
    a = np.abs(v)
    idx = np.argmax(a, axis=1)
    signed = v[np.arange(v.shape[0]), idx]
    zero = signed == 0
    scale = np.where(zero, 0.0, signed / -8.0)
    with np.errstate(divide="ignore"):
        inv = np.where(scale == 0, 0.0, 1.0 / np.where(scale == 0, 1.0, scale))
    bits = float_to_half_up(scale.astype(np.float32))
    lo = np.clip(np.floor(v[:, :16] * inv[:, None] + 8.5), 0, 15).astype(np.uint8)
    hi = np.clip(np.floor(v[:, 16:] * inv[:, None] + 8.5), 0, 15).astype(np.uint8)
    out = np.empty((v.shape[0], 18), np.uint8)
    out[:, 0] = bits & 0xFF
    out[:, 1] = bits >> 8
    out[:, 2:] = lo | (hi << 4)
    return out


def requantize_to_q40(src: np.ndarray, gtype: int, k: int, n: int) -> np.ndarray:
    """requantizeMatrixToQ40 (quantization.ts:101-131): row-major Q4_0 bytes."""
    if k % 256:
        raise ValueError(f"K={k} is not divisible by a K-quant block")
    bb = {Q4_K: 144, Q6_K: 210, Q4_0: 18}[gtype]
    bv = 32 if gtype == Q4_0 else 256
    if src.nbytes != n * (k // bv) * bb:
        raise ValueError("source has the wrong byte length")
    dec = {Q4_K: dequant_q4k, Q6_K: dequant_q6k, Q4_0: dequant_q40}[gtype]
    out = np.empty((n, k // 32, 18), np.uint8)
    rows_per_chunk = max(1, (1 << 22) // k)
    src = src.reshape(n, -1)
    for r0 in range(0, n, rows_per_chunk):
        r1 = min(n, r0 + rows_per_chunk)
        vals = dec(src[r0:r1].reshape(-1)).reshape(-1, 32)
        out[r0:r1] = quantize_q40(vals).reshape(r1 - r0, k // 32, 18)
    return out.reshape(-1)


def pack_q40_tile32(parts: list[tuple[np.ndarray, int]], k: int) -> np.ndarray:
    """packQ40Tile32 (format.ts:65-99)."""
    kb = k // 32
    rows = np.concatenate([p.reshape(n, kb, 18) for p, n in parts], axis=0)
    n = rows.shape[0]
    nt = (n + 31) // 32
    padded = np.zeros((nt * 32, kb, 18), np.uint8)
    padded[:n] = rows
    t = padded.reshape(nt, 32, kb, 18).transpose(0, 2, 1, 3)
    out = np.zeros((nt, kb, 32, 20), np.uint8)
    out[..., 0:2] = t[..., 0:2]
    out[..., 4:20] = t[..., 2:18]
    return out.reshape(-1)


# --- random blocks ------------------------------------------------------------

def pack_q4k_scales(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Inverse of scaleAndMin (quantization.ts:11-17): 8 scales + 8 mins -> 12 bytes."""
    sc = sc.astype(np.int64)
    mn = mn.astype(np.int64)
    s = np.empty((sc.shape[0], 12), np.int64)
    s[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return s.astype(np.uint8)


def gen_q4k(rng: np.random.Generator, n_blocks: int, d_sigma: float, dmin_sigma: float) -> np.ndarray:
    """Random Q4_K blocks: d=f16(|N(0,d_sigma)|), dmin=f16(|N(0,dmin_sigma)|), 6-bit scales/mins U{0..63},
    4-bit quants U{0..15} (every bit of every field exercised)."""
    b = np.empty((n_blocks, 144), np.uint8)
    d = np.abs(rng.normal(0, d_sigma, n_blocks)).astype(np.float16)
    dm = np.abs(rng.normal(0, dmin_sigma, n_blocks)).astype(np.float16)
    b[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
    b[:, 2:4] = dm.view(np.uint8).reshape(-1, 2)
    b[:, 4:16] = pack_q4k_scales(rng.integers(0, 64, (n_blocks, 8)), rng.integers(0, 64, (n_blocks, 8)))
    b[:, 16:] = rng.integers(0, 256, (n_blocks, 128), dtype=np.uint8)
    return b.reshape(-1)


def gen_q6k(rng: np.random.Generator, n_blocks: int, d_sigma: float) -> np.ndarray:
    """Random Q6_K blocks: 6-bit quants, int8 sub-block scales over the full range, d=f16(|N(0,d_sigma)|)."""
    b = np.empty((n_blocks, 210), np.uint8)
    b[:, 0:208] = rng.integers(0, 256, (n_blocks, 208), dtype=np.uint8)
    d = np.abs(rng.normal(0, d_sigma, n_blocks)).astype(np.float16)
    b[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return b.reshape(-1)


def config1_matrix(seed: int = 1, n: int = 2048, k: int = 2048) -> tuple[np.ndarray, np.ndarray]:
    """Config 1: X f16 [15 x 2048] ~ N(0,1); W Q4_K [2048 x 2048] with d~|N(0,0.002)|, dmin~|N(0,0.001)|."""
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (15, k)).astype(np.float16)
    w = gen_q4k(rng, n * (k // 256), 0.002, 0.001)
    return x, w


# --- model packs --------------------------------------------------------------

def _norm(rng: np.random.Generator) -> np.ndarray:
    return (1.0 + rng.normal(0, 0.05, HIDDEN)).astype(np.float32).view(np.uint8)


def make_model_pack(seed: int = 0, flavour: str = "kquant", n_layers: int = LAYERS, vocab: int = VOCAB) -> bytes:
    """A seeded random-init Nemotron-3-Embed-1B ``.wgpack`` (see module docstring)."""
    if flavour not in ("kquant", "q40"):
        raise ValueError("flavour must be 'kquant' or 'q40'")
    rng = np.random.default_rng(seed)
    raw: list[PackedTensor] = []
    packed: list[PackedTensor] = []
    raw.append(PackedTensor("token_embd.weight", [HIDDEN, vocab], Q6_K, RAW, gen_q6k(rng, vocab * 8, Q6K_D_SIGMA)))
    for layer in range(n_layers):
        p = f"blk.{layer}"
        raw.append(PackedTensor(f"{p}.attn_norm.weight", [HIDDEN], F32, RAW, _norm(rng)))
        raw.append(PackedTensor(f"{p}.ffn_norm.weight", [HIDDEN], F32, RAW, _norm(rng)))

        def q4k(rows, k):
            return Q4_K, gen_q4k(rng, rows * (k // 256), Q4K_D_SIGMA, Q4K_DMIN_SIGMA), k, rows

        def q6k(rows, k):
            return Q6_K, gen_q6k(rng, rows * (k // 256), Q6K_D_SIGMA), k, rows

        mats = {
            "attn_q": q4k(3072, HIDDEN), "attn_k": q4k(1024, HIDDEN), "attn_v": q6k(1024, HIDDEN),
            "attn_output": q4k(HIDDEN, 3072), "ffn_gate": q4k(INTER, HIDDEN), "ffn_up": q4k(INTER, HIDDEN),
            "ffn_down": (q6k if layer in Q6K_DOWN_LAYERS else q4k)(HIDDEN, INTER),
        }
        if flavour == "kquant":
            for name, (gt, data, k, n) in mats.items():
                raw.append(PackedTensor(f"{p}.{name}.weight", [k, n], gt, RAW, data))
        else:
            q40 = {name: (requantize_to_q40(data, gt, k, n), n, k) for name, (gt, data, k, n) in mats.items()}
            groups = [("attn_qkv", ["attn_q", "attn_k", "attn_v"]), ("attn_output", ["attn_output"]),
                      ("ffn_gate_up", ["ffn_gate", "ffn_up"]), ("ffn_down", ["ffn_down"])]
            for fused, names in groups:
                k = q40[names[0]][2]
                n = sum(q40[nm][1] for nm in names)
                data = pack_q40_tile32([(q40[nm][0], q40[nm][1]) for nm in names], k)
                packed.append(PackedTensor(f"{p}.{fused}.weight", [k, n], Q4_0, COMPACT, data))
    raw.append(PackedTensor("output_norm.weight", [HIDDEN], F32, RAW, _norm(rng)))
    meta = {"general.architecture": "mistral3", "general.name": "synthetic Nemotron-3-Embed-1B",
            "nemo.synthetic.seed": seed, "nemo.synthetic.flavour": flavour}
    return build_wgpack(raw + packed, meta, source_sha256="synthetic", source_bytes=0)


def cached_model_pack(seed: int = 0, flavour: str = "kquant", n_layers: int = LAYERS, vocab: int = VOCAB,
                      cache_dir: str | None = None) -> str:
    """Path of a generated pack, created once per (seed, flavour, layers, vocab) in ``cache_dir``."""
    cache_dir = cache_dir or os.environ.get("NEMO_PACK_CACHE", "/tmp/nemo_b200_packs")
    os.makedirs(cache_dir, exist_ok=True)
    path = os.path.join(cache_dir, f"synthetic_{flavour}_s{seed}_l{n_layers}_v{vocab}.wgpack")
    if not os.path.exists(path):
        data = make_model_pack(seed, flavour, n_layers, vocab)
        tmp = f"{path}.{os.getpid()}.tmp"
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, path)
    return path


def make_requests(seed: int, lengths: list[int], vocab: int = VOCAB) -> list[list[int]]:
    """Token id lists: BOS then ids uniform over the vocabulary."""
    rng = np.random.default_rng(seed)
    return [[BOS] + rng.integers(0, vocab, n - 1).tolist() for n in lengths]


def pad_batch(requests: list[list[int]], pad: int = PAD) -> tuple[np.ndarray, np.ndarray, int]:
    """ids [batch*sequence] padded after each request (embedding-engine.ts:70-77) and lengths."""
    seq = max(len(r) for r in requests)
    ids = np.full((len(requests), seq), pad, np.uint32)
    for i, r in enumerate(requests):
        ids[i, :len(r)] = r
    return ids.reshape(-1), np.array([len(r) for r in requests], np.uint32), seq


def sha256_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()
