"""The B200-tiled pack producer (nemo_pack_b200, host only): the output is a
WGPACK02 file the reference's parser accepts (restated in oracle.parse_wgpack,
src/prepacked/format.ts:146-169), with the token table and norms unchanged and
every projection as one raw tile-slab image whose bytes are the source blocks,
re-tiled: chunk (tile, slab) = two 64-row regions (Q4_K / Q4_0 144 B per row;
Q6_K 208 B per row then 64 f16 scales), gate/up tiles = 64 gate rows + the
matching 64 up rows. Checked here position by position against the source
tensors; the GPU test (test_gpu_forward.py) checks that a model loaded from it
gives the same embeddings."""
import numpy as np
import pytest

import oracle
from nemo_b200 import synth
from nemo_b200.runtime import NemoError, pack_b200

FUSED = ["attn_qkv", "attn_output", "ffn_gate_up", "ffn_down"]
N = [5120, 2048, 12288, 2048]
K = [2048, 3072, 2048, 6144]
TILE_ENTRY = 16  # SkinnyTile: u32 offset, u32 chunk_bytes, u8 fmt[2], 6 pad bytes


@pytest.fixture(scope="module")
def packs():
    src = synth.make_model_pack(seed=6, flavour="kquant", n_layers=5, vocab=512)
    return src, pack_b200(src)


def _rows_of(tensors, buf, names):
    """Row-major source blocks of the fused projection's parts: (fmt, bytes per row, per-row arrays)."""
    out = []
    for nm in names:
        t = tensors[nm]
        k, n = t.dimensions
        per = {oracle.Q4_K: 144, oracle.Q6_K: 210}[t.type] * (k // 256)
        data = np.frombuffer(buf, np.uint8, t.byte_length, t.byte_offset).reshape(n, per)
        out += [(t.type, data[r]) for r in range(n)]
    return out


def test_b200_pack_parses_and_keeps_raw_tensors(packs):
    src, b2 = packs
    hs, ts = oracle.parse_wgpack(src)
    hb, tb = oracle.parse_wgpack(b2)
    assert hb["metadata"]["nemo.layout"] == "b200-tile-slab-v1"
    assert hb["sourceSha256"] == hs["sourceSha256"]
    for name in ["token_embd.weight", "output_norm.weight"] + [f"blk.{l}.{w}_norm.weight" for l in range(5)
                                                                for w in ("attn", "ffn")]:
        a, b = ts[name], tb[name]
        assert b.storage == "raw" and b.type == a.type and b.dimensions == a.dimensions
        assert src[a.byte_offset:a.byte_offset + a.byte_length] == b2[b.byte_offset:b.byte_offset + b.byte_length]
    for l in range(5):
        for w, fused in enumerate(FUSED):
            t = tb[f"blk.{l}.{fused}.b200_tiles"]
            assert t.storage == "raw" and t.dimensions == [t.byte_length]


@pytest.mark.parametrize("which", range(4), ids=FUSED)
def test_b200_images_hold_the_source_blocks(packs, which):
    src, b2 = packs
    _, ts = oracle.parse_wgpack(src)
    _, tb = oracle.parse_wgpack(b2)
    parts = {0: ["attn_q", "attn_k", "attn_v"], 1: ["attn_output"], 2: ["ffn_gate", "ffn_up"], 3: ["ffn_down"]}[which]
    l = 1
    rows = _rows_of(ts, src, [f"blk.{l}.{p}.weight" for p in parts])
    n, k = N[which], K[which]
    assert len(rows) == n
    t = tb[f"blk.{l}.{FUSED[which]}.b200_tiles"]
    img = np.frombuffer(b2, np.uint8, t.byte_length, t.byte_offset)
    ntiles, slabs = n // 128, k // 256
    table = (ntiles * TILE_ENTRY + 255) // 256 * 256
    rng = np.random.default_rng(which)
    offset = 0
    for tile in range(ntiles):
        e = img[tile * TILE_ENTRY:(tile + 1) * TILE_ENTRY]
        off, chunk = int(e[0:4].view(np.uint32)[0]), int(e[4:8].view(np.uint32)[0])
        fmts = [int(e[8]), int(e[9])]
        assert off == offset
        regions = [64 * (210 if f == 1 else 144) for f in fmts]
        assert chunk == sum(regions)
        offset += chunk * slabs
        for _ in range(3):
            s, half, rr = int(rng.integers(slabs)), int(rng.integers(2)), int(rng.integers(64))
            row = (tile * 64 + rr if half == 0 else n // 2 + tile * 64 + rr) if which == 2 else tile * 128 + 64 * half + rr
            gtype, blocks = rows[row]
            region = table + off + s * chunk + (regions[0] if half else 0)
            if gtype == oracle.Q4_K:
                assert fmts[half] == 0
                assert np.array_equal(img[region + rr * 144:region + rr * 144 + 144], blocks[s * 144:(s + 1) * 144])
            else:
                assert fmts[half] == 1
                blk = blocks[s * 210:(s + 1) * 210]
                assert np.array_equal(img[region + rr * 208:region + rr * 208 + 208], blk[:208])
                assert np.array_equal(img[region + 64 * 208 + rr * 2:region + 64 * 208 + rr * 2 + 2], blk[208:210])
    assert table + offset == t.byte_length


def test_b200_pack_rejects_its_own_output_and_bad_input(packs):
    _, b2 = packs
    with pytest.raises(NemoError, match="already B200-tiled"):
        pack_b200(b2)
    with pytest.raises(NemoError, match="magic"):
        pack_b200(b"WGPACK01" + b"\0" * 64)


def test_b200_image_of_a_tile32_pack():
    """Reference-faithful packs (q4_0-tile32-compact, format.ts:84-97): each
    row's 8 blocks of a 256-column slab become 8 f16 scales then 8 x 16
    quant bytes."""
    src = synth.make_model_pack(seed=7, flavour="q40", n_layers=5, vocab=512)
    b2 = pack_b200(src)
    _, ts = oracle.parse_wgpack(src)
    _, tb = oracle.parse_wgpack(b2)
    t32 = ts["blk.2.attn_output.weight"]
    assert t32.storage == "q4_0-tile32-compact"
    k, n = t32.dimensions
    kb32 = k // 32
    tiles = np.frombuffer(src, np.uint8, t32.byte_length, t32.byte_offset)
    t = tb["blk.2.attn_output.b200_tiles"]
    img = np.frombuffer(b2, np.uint8, t.byte_length, t.byte_offset)
    table = (n // 128 * TILE_ENTRY + 255) // 256 * 256
    chunk = 2 * 64 * 144
    rng = np.random.default_rng(3)
    for _ in range(20):
        row, s = int(rng.integers(n)), int(rng.integers(k // 256))
        tile, half, rr = row // 128, (row // 64) & 1, row & 63
        dst = img[table + (tile * (k // 256) + s) * chunk + half * 64 * 144 + rr * 144:][:144]
        for b in range(8):
            blk = tiles[((row // 32 * kb32 + s * 8 + b) * 32 + row % 32) * 20:][:20]
            assert np.array_equal(dst[2 * b:2 * b + 2], blk[0:2])
            assert np.array_equal(dst[16 + 16 * b:32 + 16 * b], blk[4:20])
