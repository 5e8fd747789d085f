"""The product's format writers and synthetic-pack restatements
(nemo_b200.synth / nemo_b200.wgpack) against the oracle, bit for bit, and the
reference's .wgpack golden file case (tests/prepacked-format.test.ts:13-33)."""
import numpy as np
import pytest

import oracle
from nemo_b200 import synth
from nemo_b200.wgpack import COMPACT, F32, Q4_0, RAW, PackedTensor, build_wgpack


def test_half_up_matches_oracle(rng):
    x = np.concatenate([rng.normal(0, 1e-3, 3000), rng.normal(0, 1e4, 1000), rng.normal(0, 1e-6, 1000),
                        [0.0, -0.0, 65504.0, 65520.0, 1e9, -1e9, 6.1e-5, 2.98e-8, 5.96e-8]]).astype(np.float32)
    got = synth.float_to_half_up(x)
    want = np.array([oracle.float_to_half(float(v)) for v in x], np.uint16)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("gtype", [oracle.Q4_K, oracle.Q6_K])
def test_decoders_and_requantize_match_oracle(rng, gtype):
    k, n = 512, 96
    if gtype == oracle.Q4_K:
        src = synth.gen_q4k(rng, n * k // 256, synth.Q4K_D_SIGMA, synth.Q4K_DMIN_SIGMA)
        dec = synth.dequant_q4k(src)
    else:
        src = synth.gen_q6k(rng, n * k // 256, synth.Q6K_D_SIGMA)
        dec = synth.dequant_q6k(src)
    ref = oracle.decode_matrix(src, gtype, False, k, n)
    assert np.array_equal(dec.reshape(n, k).view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(synth.requantize_to_q40(src, gtype, k, n), oracle.requantize_to_q40(src, gtype, k, n))


def test_quantize_q40_edge_rows():
    rows = np.zeros((5, 32), np.float32)
    rows[1, 3] = -2.5            # negative maximum
    rows[2, :] = 1.0             # all equal
    rows[2, 7] = -1.0            # tie in |max|: first occurrence wins
    rows[3, :] = np.linspace(-3, 3, 32)
    rows[4, 0] = 1e-30           # tiny scale -> f16 zero
    got = synth.quantize_q40(rows)
    want = np.stack([oracle.quantize_q40_block(r) for r in rows])
    assert np.array_equal(got, want)


def test_tile32_pack_matches_oracle(rng):
    k = 256
    a = rng.integers(0, 256, (70 * k // 32 * 18,), dtype=np.uint8)
    b = rng.integers(0, 256, (33 * k // 32 * 18,), dtype=np.uint8)
    got = synth.pack_q40_tile32([(a, 70), (b, 33)], k)
    want = oracle.pack_q40_tile32([(a, 70), (b, 33)], k)
    assert np.array_equal(got, want)


def test_tile32_golden_and_file_roundtrip(golden):
    c = golden["tile32_pack"]
    parts = [(np.frombuffer(bytes.fromhex(p["bytes"]), np.uint8), p["n"]) for p in c["parts"]]
    packed = synth.pack_q40_tile32(parts, 32)
    assert packed.nbytes == c["byte_length"]
    assert list(packed[0:8]) == c["bytes_0_8"] and list(packed[20:28]) == c["bytes_20_28"]
    f = c["file"]
    raw = PackedTensor(f["raw"]["name"], f["raw"]["dimensions"], f["raw"]["type"], RAW,
                       np.frombuffer(bytes.fromhex(f["raw"]["bytes"]), np.uint8))
    fused = PackedTensor("fused", c["dimensions"], Q4_0, COMPACT, packed)
    data = build_wgpack([raw, fused], f["metadata"], f["sourceSha256"], f["sourceBytes"])
    header, tensors = oracle.parse_wgpack(data)
    assert header["sourceSha256"] == "abc123" and header["sourceBytes"] == 42
    assert header["metadata"]["general.name"] == "test"
    for name, want in (("norm", f["expect_raw"]), ("fused", f["expect_fused"])):
        t = tensors[name]
        assert t.dimensions == want["dimensions"] and t.type == want["type"]
        assert t.storage == want["storage"] and t.byte_length == want["byteLength"]
    assert tensors["fused"].byte_offset % 256 == 0


def test_parser_rejects_bad_files():
    good = build_wgpack([PackedTensor("n", [1], F32, RAW, np.zeros(4, np.uint8))])
    with pytest.raises(ValueError, match="magic"):
        oracle.parse_wgpack(b"WGPACK01" + good[8:])
    with pytest.raises(ValueError, match="prelude"):
        oracle.parse_wgpack(good[:8])
    with pytest.raises(ValueError, match="past end"):
        oracle.parse_wgpack(good[:-2])


def test_q4k_scale_packing_inverts_scale_and_min(rng):
    sc = rng.integers(0, 64, (200, 8))
    mn = rng.integers(0, 64, (200, 8))
    s = synth.pack_q4k_scales(sc, mn)
    blocks = np.zeros((200, 144), np.uint8)
    blocks[:, 0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    blocks[:, 2:4] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    blocks[:, 4:16] = s
    blocks[:, 16:] = 0x11  # every quant = 1
    v = synth.dequant_q4k(blocks.reshape(-1))
    # value = sc * 1 - mn for sub-block j: elements j*32..j*32+31
    want = np.repeat(sc - mn, 32, axis=1).astype(np.float32)
    order = [0, 1, 2, 3, 4, 5, 6, 7]
    assert np.array_equal(v, want[:, np.concatenate([np.arange(j * 32, j * 32 + 32) for j in order])])
