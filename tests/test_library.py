"""The C-ABI library loads and exports every symbol include/*.h declares (no
compute calls: runs without a GPU)."""
import ctypes
import os
import re

from conftest import REPO


def declared_functions():
    names = set()
    for h in ("nemo.h", "nemo_ops.h"):
        with open(os.path.join(REPO, "include", h)) as f:
            text = f.read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(nemo_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    from nemo_b200 import runtime
    lib = runtime.load_library()
    names = declared_functions()
    assert len(names) >= 20
    for n in sorted(names):
        assert hasattr(lib, n), n


def test_host_only_entry_points():
    from nemo_b200 import runtime
    lib = runtime.load_library()
    assert runtime.merged_length(5000) == 3200
    assert lib.nemo_stage_name(0) == b"embedding_norm" and lib.nemo_stage_name(10) == b"pool"
    import numpy as np
    import oracle
    t = np.zeros((7, 64, 2), np.float32)
    assert lib.nemo_rope_table(7, t.ctypes.data_as(ctypes.c_void_p)) == 0
    assert np.array_equal(t, oracle.rope_table(7))
    # tile-slab image size of the standalone quantised matmul: 256-byte tile
    # table + 128 x 256 chunks (Q4_K / Q4_0: 2 x 64 x 144 B; Q6_K: 2 x 64 x 210 B)
    assert lib.nemo_op_qmatmul_image_bytes(0, 2048, 2048) == 256 + 16 * 8 * 18432
    assert lib.nemo_op_qmatmul_image_bytes(1, 256, 6144) == 256 + 2 * 24 * 26880
    assert lib.nemo_op_qmatmul_image_bytes(0, 200, 2048) == 0
    # the image decode rejects bad arguments before touching a device
    assert lib.nemo_op_qmatmul_image_decode(0, None, 256, 2048, None) == -1
    assert b"nemo_op_qmatmul_image_decode" in lib.nemo_last_error()
    fake = ctypes.c_void_p(256)
    assert lib.nemo_op_qmatmul_image_decode(0, fake, 200, 2048, fake) == -1
    assert lib.nemo_op_qmatmul_image_decode(0, fake, 256, 2000, fake) == -1
