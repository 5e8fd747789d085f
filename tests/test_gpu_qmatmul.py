"""Op-level parity of the quantised projection kernels through the standalone
matmul entry points (include/nemo_ops.h nemo_op_qmatmul*): the device re-tile
into the tile-slab image, the fused-dequant split-K kernel (m <= 64) and the
dequant-fused batched GEMM (m > 64), each against the CPU oracle's decode and
f32-accumulated matmul on the same seeded blocks.

Config 1 of the benchmark is the first case: X f16 [15 x 2048] ~ N(0,1), W a
2048 x 2048 Q4_K matrix with d ~ |N(0,0.002)|, dmin ~ |N(0,0.001)|, 6-bit
scales/mins U[0,63] and quants U[0,15], Y f32 [15 x 2048]. The decode is
checked bit-exact, the matmul within an f16-scale tolerance.

Reference: src/gguf/quantization.ts:19-74 (decode), src/webgpu/quant-matmul.ts
:37-154 (the GGUF dequant-fused pipelines), :438-563 (QuantMatmulKernel)."""
import numpy as np
import pytest

import oracle
from gpu_util import dev, empty, f16_bits, host, ptr, rel_err
from nemo_b200 import synth
from nemo_b200.runtime import NemoError, check, load_library

pytestmark = pytest.mark.gpu

FMT_IDS = ["q4_k", "q6_k", "q4_0", "q4_0_tile32"]
# max|Y - Y_oracle| / max|Y_oracle|: both accumulate f16 products in f32 (the
# order differs), so the bound is far inside the f16 output rounding (2^-11).
TOL = 1e-3


def L():
    return load_library()


def blocks(rng, fmt, rows, k):
    """Seeded quantised matrix [rows x k] in format fmt (NEMO_FMT_*), with the
    oracle's type code and layout flag."""
    if fmt == 0:
        return synth.gen_q4k(rng, rows * k // 256, 0.002, 0.001), oracle.Q4_K, False
    if fmt == 1:
        return synth.gen_q6k(rng, rows * k // 256, 1e-3), oracle.Q6_K, False
    q6 = synth.gen_q6k(rng, rows * k // 256, 1e-3)
    q40 = synth.requantize_to_q40(q6, oracle.Q6_K, k, rows)
    if fmt == 2:
        return q40, oracle.Q4_0, False
    return synth.pack_q40_tile32([(q40, rows)], k), oracle.Q4_0, True


def run_qmatmul(fmt, w, x_bits, n, k):
    t = __import__("torch")
    m = x_bits.shape[0]
    y = empty((m, n), t.float32)
    d_w, d_x = dev(w), dev(x_bits.view(np.float16))
    check(L().nemo_op_qmatmul(fmt, ptr(d_w), ptr(d_x), m, n, k, ptr(y)))
    return host(y)


def oracle_matmul(fmt_code, compact, w, x_bits, n, k):
    w32 = oracle.decode_matrix(w, fmt_code, compact, k, n)
    ref32, _ = oracle.matmul_f16(x_bits, w32.astype(np.float16).view(np.uint16))
    return w32, ref32


def test_config1_q4k_dequant_matmul():
    x, w = synth.config1_matrix(seed=1)
    n = k = 2048
    x_bits = x.view(np.uint16)
    # decode bit-exact against the oracle (quantization.ts:19-38)
    t = __import__("torch")
    d_w = dev(w)
    o16 = empty((n, k), t.float16)
    o32 = empty((n, k), t.float32)
    check(L().nemo_op_decode(0, ptr(d_w), n, k, ptr(o16), ptr(o32)))
    w32, ref32 = oracle_matmul(oracle.Q4_K, False, w, x_bits, n, k)
    assert np.array_equal(host(o32).view(np.uint32), w32.view(np.uint32))
    assert np.array_equal(host(o16).view(np.uint16), w32.astype(np.float16).view(np.uint16))
    got = run_qmatmul(0, w, x_bits, n, k)
    assert got.shape == (15, 2048) and got.dtype == np.float32
    assert rel_err(got, ref32) < TOL


@pytest.mark.parametrize("m", [1, 15, 16, 17, 64, 65, 333])
@pytest.mark.parametrize("fmt", [0, 1, 2, 3], ids=FMT_IDS)
def test_qmatmul_formats_and_token_counts(rng, fmt, m):
    n, k = 512, 2048
    w, code, compact = blocks(rng, fmt, n, k)
    x_bits = f16_bits(rng.normal(0, 1, (m, k)))
    _, ref32 = oracle_matmul(code, compact, w, x_bits, n, k)
    got = run_qmatmul(fmt, w, x_bits, n, k)
    assert rel_err(got, ref32) < TOL


@pytest.mark.parametrize("shape", [(2048, 6144, 40), (256, 3072, 9), (1024, 6144, 200)],
                         ids=["down_k6144_m40", "o_k3072_m9", "down_k6144_m200"])
def test_qmatmul_projection_shapes(rng, shape):
    n, k, m = shape
    w, code, compact = blocks(rng, 1, n, k)  # Q6_K: the ffn_down / attn_v format of the Q4_K_M mix
    x_bits = f16_bits(rng.normal(0, 1, (m, k)))
    _, ref32 = oracle_matmul(code, compact, w, x_bits, n, k)
    assert rel_err(run_qmatmul(1, w, x_bits, n, k), ref32) < TOL


def test_qmatmul_enqueue_on_image_repeats_bit_identically(rng):
    """The image path (re-tile once, enqueue many times) gives the same bits
    on every call, at both kernel families."""
    t = __import__("torch")
    n, k = 1024, 2048
    w, code, compact = blocks(rng, 0, n, k)
    d_w = dev(w)
    nbytes = L().nemo_op_qmatmul_image_bytes(0, n, k)
    assert nbytes == 256 + (n // 128) * (k // 256) * 2 * 64 * 144
    image = t.zeros(nbytes, dtype=t.uint8, device="cuda")
    check(L().nemo_op_qmatmul_image(0, ptr(d_w), n, k, ptr(image)))
    err = t.zeros(1, dtype=t.int32, device="cuda")
    for m in (15, 129):
        x_bits = f16_bits(rng.normal(0, 1, (m, k)))
        d_x = dev(x_bits.view(np.float16))
        outs = []
        for _ in range(3):
            y = t.full((m, n), float("nan"), dtype=t.float32, device="cuda")
            check(L().nemo_op_qmatmul_enqueue(0, ptr(image), ptr(d_x), m, n, k, ptr(y), ptr(err), None))
            t.cuda.synchronize()
            outs.append(host(y))
        assert int(host(err)[0]) == 0
        assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
        assert np.array_equal(outs[0].view(np.uint32), outs[2].view(np.uint32))
        _, ref32 = oracle_matmul(code, compact, w, x_bits, n, k)
        assert rel_err(outs[0], ref32) < TOL


def signed_blocks(rng, fmt, rows, k):
    """blocks() with the sign of d (and of dmin for Q4_K) flipped on random
    blocks and the scales of a quarter of the blocks zeroed, so that zero
    products of either sign occur."""
    w, code, compact = blocks(rng, fmt, rows, k)
    b = w.reshape(-1, 144 if fmt == 0 else 210).copy()
    flip = rng.random(len(b)) < 0.5
    zero = rng.random(len(b)) < 0.25
    if fmt == 0:
        b[flip, 1] |= 0x80
        b[rng.random(len(b)) < 0.5, 3] |= 0x80
        b[zero, 4:16] = 0
        b[rng.random(len(b)) < 0.25, 8:12] = 0  # mins of sub-blocks 0-3
    else:
        b[flip, 209] |= 0x80
        b[zero, 192:208] = 0
    return b.reshape(-1), code, compact


@pytest.mark.parametrize("case", ["q4_k", "q6_k", "q4_0", "q4_0_tile32", "q4_k_signed", "q6_k_signed"])
def test_tile_slab_decoders_bit_exact(rng, case):
    """The per-row decoders every projection kernel runs on the tile-slab
    image (single-launch forward, split-K small-token kernel, dequant-fused
    GEMM, and model load's f16 weights) give f16(decode(blocks)) bit for bit,
    zero signs included (quantization.ts:19-74, f16 rounding as
    quant-matmul.ts:106)."""
    t = __import__("torch")
    fmt = FMT_IDS.index(case.replace("_signed", ""))
    n, k = 384, 2048
    w, code, compact = (signed_blocks if case.endswith("signed") else blocks)(rng, fmt, n, k)
    d_w = dev(w)
    image = t.zeros(L().nemo_op_qmatmul_image_bytes(fmt, n, k), dtype=t.uint8, device="cuda")
    check(L().nemo_op_qmatmul_image(fmt, ptr(d_w), n, k, ptr(image)))
    w16 = t.full((n, k), float("nan"), dtype=t.float16, device="cuda")
    check(L().nemo_op_qmatmul_image_decode(fmt, ptr(image), n, k, ptr(w16)))
    want = oracle.decode_matrix(w, code, compact, k, n).astype(np.float16)
    assert np.array_equal(host(w16).view(np.uint16), want.view(np.uint16))


def test_qmatmul_rejects_bad_shapes(rng):
    t = __import__("torch")
    w = dev(np.zeros(256 * 144, np.uint8))
    x = empty((4, 2000), t.float16)
    y = empty((4, 256), t.float32)
    with pytest.raises(NemoError, match="divisible by 256"):
        check(L().nemo_op_qmatmul(0, ptr(w), ptr(x), 4, 256, 2000, ptr(y)))
    with pytest.raises(NemoError):
        check(L().nemo_op_qmatmul(0, ptr(w), ptr(x), 4, 200, 2048, ptr(y)))
    assert L().nemo_op_qmatmul_image_bytes(0, 200, 2048) == 0
    assert L().nemo_op_qmatmul_image_bytes(7, 256, 2048) == 0
