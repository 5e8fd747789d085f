"""Writes reference_known_answers.json: the known-answer cases of the reference's
own unit tests, restated as data so the oracle (and the CUDA path) can be pinned
against them without a JS engine.

Every case names the reference test it comes from. The inputs are built exactly
as the TypeScript test builds them; the expected values are the ones the test
asserts. Run: python tests/golden/make_known_answers.py
"""
import json
import os


def hexs(b: bytes) -> str:
    return bytes(b).hex()


def main() -> None:
    cases = {}
    # tests/quantization.test.ts:5-9
    cases["half_to_float"] = {
        "source": "tests/quantization.test.ts:5-9",
        "pairs": [[0x3C00, 1.0], [0xC000, -2.0], [0x0000, 0.0]],
    }
    # tests/quantization.test.ts:11-22
    q4k = bytearray(144)
    q4k[0:2] = (0x3C00).to_bytes(2, "little")
    q4k[4:12] = bytes([1] * 8)
    q4k[12:16] = bytes([0x11] * 4)
    q4k[16:144] = bytes([0x72] * 128)
    cases["q4k_block"] = {
        "source": "tests/quantization.test.ts:11-22",
        "block": hexs(q4k),
        "expect": {"0": 2.0, "31": 2.0, "32": 7.0, "255": 7.0},
    }
    # tests/quantization.test.ts:24-33
    q40 = bytearray(18)
    q40[0:2] = (0x3C00).to_bytes(2, "little")
    q40[2:18] = bytes([0xF0] * 16)
    cases["q40_block"] = {
        "source": "tests/quantization.test.ts:24-33",
        "block": hexs(q40),
        "expect": {"0": -8.0, "15": -8.0, "16": 7.0, "31": 7.0},
    }
    # tests/quantization.test.ts:35-42
    q6k = bytearray(210)
    q6k[192:208] = bytes([1] * 16)
    q6k[208:210] = (0x3C00).to_bytes(2, "little")
    cases["q6k_block"] = {
        "source": "tests/quantization.test.ts:35-42",
        "block": hexs(q6k),
        "expect_all": -32.0,
    }
    # tests/quantization.test.ts:44-49
    cases["q40_roundtrip"] = {
        "source": "tests/quantization.test.ts:44-49",
        "values": [(i - 16) / 4 for i in range(32)],
        "max_abs_error_below": 0.55,
    }
    # tests/quantization.test.ts:51-58
    cases["requantize_q6k"] = {
        "source": "tests/quantization.test.ts:51-58",
        "block": hexs(q6k),
        "type": 14,
        "k": 256,
        "n": 1,
        "byte_length": 8 * 18,
        "decoded_all": -32.0,
    }
    # tests/prepacked-format.test.ts:5-33
    def q40_block(scale_bits, quants):
        b = bytearray(18)
        b[0:2] = bytes(scale_bits)
        for i in range(16):
            b[2 + i] = quants[i] | (quants[i + 16] << 4)
        return b

    first = q40_block([0x00, 0x3C], [i & 15 for i in range(32)])
    second = q40_block([0x00, 0x40], [15 - (i & 15) for i in range(32)])
    cases["tile32_pack"] = {
        "source": "tests/prepacked-format.test.ts:13-33",
        "parts": [{"name": "first", "k": 32, "n": 1, "bytes": hexs(first)},
                  {"name": "second", "k": 32, "n": 1, "bytes": hexs(second)}],
        "dimensions": [32, 2],
        "byte_length": 640,
        "bytes_0_8": [0x00, 0x3C, 0x00, 0x00, 0x00, 0x11, 0x22, 0x33],
        "bytes_20_28": [0x00, 0x40, 0x00, 0x00, 0xFF, 0xEE, 0xDD, 0xCC],
        "file": {"sourceSha256": "abc123", "sourceBytes": 42, "metadata": {"general.name": "test"},
                 "raw": {"name": "norm", "dimensions": [1], "type": 0, "bytes": "01020304"},
                 "expect_raw": {"dimensions": [1], "type": 0, "storage": "raw", "byteLength": 4},
                 "expect_fused": {"dimensions": [32, 2], "type": 2, "storage": "q4_0-tile32-compact",
                                  "byteLength": 640}},
    }
    # tests/model-config.test.ts:5-15
    cases["merged_length"] = {
        "source": "tests/model-config.test.ts:5-15",
        "pairs": [[1, 1], [15, 10], [50, 32], [150, 96], [500, 320], [1500, 960], [5000, 3200]],
    }
    # tests/embedding-engine.test.ts:5-50
    cases["engine"] = {
        "source": "tests/embedding-engine.test.ts:5-50",
        "coalesce": {"requests": 16, "bos": 99, "expect_calls": 1, "expect_batch": 16, "expect_sequence": 2,
                     "expect_lengths": [2] * 16},
        "padding": {"bos": 99, "pad": 99, "texts": ["1", "2,3"], "expect_ids": [99, 1, 99, 99, 2, 3]},
        "storage_split": {"max_storage": 2 * 6144 * 2 * 2, "requests": 5, "expect_batches": [2, 2, 1]},
    }
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_known_answers.json")
    with open(out, "w") as f:
        json.dump(cases, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
