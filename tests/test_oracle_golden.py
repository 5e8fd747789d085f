"""Pins the CPU oracle against the reference's own known-answer tests
(tests/golden/reference_known_answers.json, transcribed from the reference's
tests/quantization.test.ts, tests/prepacked-format.test.ts and
tests/model-config.test.ts)."""
import numpy as np

import oracle


def test_half_to_float(golden):
    for bits, value in golden["half_to_float"]["pairs"]:
        assert oracle.half_to_float(bits) == value


def test_q4k_block(golden):
    c = golden["q4k_block"]
    v = oracle.dequant_block(bytes.fromhex(c["block"]), oracle.Q4_K)
    for idx, want in c["expect"].items():
        assert v[int(idx)] == want


def test_q40_block(golden):
    c = golden["q40_block"]
    v = oracle.dequant_block(bytes.fromhex(c["block"]), oracle.Q4_0)
    for idx, want in c["expect"].items():
        assert v[int(idx)] == want


def test_q6k_block(golden):
    c = golden["q6k_block"]
    v = oracle.dequant_block(bytes.fromhex(c["block"]), oracle.Q6_K)
    assert np.all(v == c["expect_all"])


def test_q40_roundtrip(golden):
    c = golden["q40_roundtrip"]
    values = np.array(c["values"], np.float32)
    enc = oracle.quantize_q40_block(values)
    dec = oracle.dequant_block(enc.tobytes(), oracle.Q4_0)
    assert np.max(np.abs(dec - values)) < c["max_abs_error_below"]


def test_requantize_q6k(golden):
    c = golden["requantize_q6k"]
    src = np.frombuffer(bytes.fromhex(c["block"]), np.uint8)
    out = oracle.requantize_to_q40(src, c["type"], c["k"], c["n"])
    assert out.nbytes == c["byte_length"]
    dec = oracle.decode_matrix(out, oracle.Q4_0, False, c["k"], c["n"])
    assert np.all(dec == c["decoded_all"])


def test_tile32_pack_golden_bytes(golden):
    c = golden["tile32_pack"]
    parts = [(np.frombuffer(bytes.fromhex(p["bytes"]), np.uint8), p["n"]) for p in c["parts"]]
    packed = oracle.pack_q40_tile32(parts, c["parts"][0]["k"])
    assert packed.nbytes == c["byte_length"]
    assert list(packed[0:8]) == c["bytes_0_8"]
    assert list(packed[20:28]) == c["bytes_20_28"]


def test_merged_length(golden):
    for source, expected in golden["merged_length"]["pairs"]:
        assert oracle.merged_length(source) == expected


def test_requantize_rejects_bad_k():
    import pytest
    with pytest.raises(ValueError):
        oracle.requantize_to_q40(np.zeros(144, np.uint8), oracle.Q4_K, 128, 1)
