"""Kernel-level parity on the GPU: every CUDA kernel of the forward pass,
called through the C ABI (include/nemo_ops.h), against the CPU oracle on the
same seeded inputs. Bit-exact where the arithmetic is deterministic (decode,
embedding, residual add, RoPE, merge); within stated f16 tolerances elsewhere."""
import ctypes

import numpy as np
import pytest

import oracle
from gpu_util import dev, empty, f16_bits, f16_of_bits, host, ptr, rel_err, ulp_diff
from nemo_b200 import synth
from nemo_b200.runtime import check, load_library

pytestmark = pytest.mark.gpu


def L():
    return load_library()


def meta_for(lengths, seq):
    t = __import__("torch")
    lengths = np.asarray(lengths, np.uint32)
    d_len = dev(lengths)
    d_meta = t.zeros(L().nemo_op_meta_bytes(), dtype=t.uint8, device="cuda")
    check(L().nemo_op_meta(ptr(d_len), lengths.size, seq, ptr(d_meta)))
    return d_len, d_meta


def tokens_ptr(d_meta, merged):
    return L().nemo_op_meta_tokens(ptr(d_meta), merged)


# --- decode -----------------------------------------------------------------

def _blocks(rng, fmt, rows, k):
    if fmt == 0:
        return synth.gen_q4k(rng, rows * k // 256, 0.002, 0.001), oracle.Q4_K, False
    if fmt == 1:
        return synth.gen_q6k(rng, rows * k // 256, 1e-3), oracle.Q6_K, False
    q6 = synth.gen_q6k(rng, rows * k // 256, 1e-3)
    q40 = synth.requantize_to_q40(q6, oracle.Q6_K, k, rows)
    if fmt == 2:
        return q40, oracle.Q4_0, False
    return synth.pack_q40_tile32([(q40, rows)], k), oracle.Q4_0, True


@pytest.mark.parametrize("fmt", [0, 1, 2, 3], ids=["q4_k", "q6_k", "q4_0", "q4_0_tile32"])
def test_decode_bit_exact(rng, fmt):
    rows, k = 192, 2048
    src, gtype, compact = _blocks(rng, fmt, rows, k)
    t = __import__("torch")
    d_src = dev(src)
    o16 = empty((rows, k), t.float16)
    o32 = empty((rows, k), t.float32)
    check(L().nemo_op_decode(fmt, ptr(d_src), rows, k, ptr(o16), ptr(o32)))
    want = oracle.decode_matrix(src, gtype, compact, k, rows)
    assert np.array_equal(host(o32).view(np.uint32), want.view(np.uint32))
    assert np.array_equal(host(o16).view(np.uint16), want.astype(np.float16).view(np.uint16))


# --- elementwise kernels ------------------------------------------------------------

def test_embedding_bit_exact(rng):
    vocab, seq = 3000, 9
    table = synth.gen_q6k(rng, vocab * 8, 1e-3)
    lengths = [9, 4, 1]
    ids = rng.integers(0, vocab, (3, seq)).astype(np.uint32)
    d_len, d_meta = meta_for(lengths, seq)
    t = __import__("torch")
    x = empty((3 * seq, 2048), t.float16)
    d_ids, d_table = dev(ids), dev(table)  # held: the kernel reads them after ptr() returns
    check(L().nemo_op_embedding(ptr(d_ids), ptr(d_table), vocab, ptr(d_meta), 3 * seq, ptr(x)))
    packed = np.concatenate([ids[b, :n] for b, n in enumerate(lengths)])
    want = oracle.embedding(table, vocab, packed)
    got = host(x).view(np.uint16)[:packed.size]
    assert np.array_equal(got, want)


def test_residual_rmsnorm(rng):
    rows = 37
    x = f16_bits(rng.normal(0, 2, (rows, 2048)))
    r = f16_bits(rng.normal(0, 1, (rows, 2048)))
    w = (1 + rng.normal(0, 0.1, 2048)).astype(np.float32)
    t = __import__("torch")
    for residual in (None, r):
        dx = dev(x.view(np.float16))
        dn = empty((rows, 2048), t.float16)
        d_rows = dev(np.array([rows], np.int32))
        dr = dev(residual.view(np.float16)) if residual is not None else None
        dw = dev(w)
        check(L().nemo_op_rmsnorm(ptr(dx), ptr(dr) if dr is not None else None, ptr(dw), ptr(dn), ptr(d_rows),
                                  rows + 5))
        wx, wn = oracle.residual_rmsnorm(x, residual, w)
        assert np.array_equal(host(dx).view(np.uint16), wx)  # residual add is exact
        assert ulp_diff(host(dn).view(np.uint16), wn) <= 1


def test_rope_bit_exact(rng):
    seq = 40
    lengths = [40, 17]
    T = sum(lengths)
    qkv = f16_bits(rng.normal(0, 1, (T, 5120)))
    table = oracle.rope_table(seq)
    d_len, d_meta = meta_for(lengths, seq)
    t = __import__("torch")
    q = empty((T, 3072), t.float16)
    k = empty((T, 1024), t.float16)
    d_qkv, d_table = dev(qkv.view(np.float16)), dev(table)
    check(L().nemo_op_rope(ptr(d_qkv), ptr(d_table), ptr(d_meta), 0, 2 * seq, ptr(q), ptr(k)))
    pos = np.concatenate([np.arange(n) for n in lengths]).astype(np.int32)
    wq, wk = oracle.rope(qkv, pos, table)
    assert np.array_equal(host(q).view(np.uint16), wq)
    assert np.array_equal(host(k).view(np.uint16), wk)


def test_swiglu(rng):
    rows = 23
    gu = f16_bits(rng.normal(0, 3, (rows, 12288)))
    t = __import__("torch")
    out = empty((rows, 6144), t.float16)
    d_gu, d_rows = dev(gu.view(np.float16)), dev(np.array([rows], np.int32))
    check(L().nemo_op_swiglu(ptr(d_gu), ptr(d_rows), rows, ptr(out)))
    assert ulp_diff(host(out).view(np.uint16), oracle.swiglu(gu)) <= 1


@pytest.mark.parametrize("lengths", [[15, 150, 1, 2], [5000], [33, 64, 1000]])
def test_merge_bit_exact(rng, lengths):
    seq = max(lengths)
    T = sum(lengths)
    x = f16_bits(rng.normal(0, 1, (T, 2048)))
    n = f16_bits(rng.normal(0, 1, (T, 2048)))
    d_len, d_meta = meta_for(lengths, seq)
    mseq = oracle.merged_length(seq)
    tgt = np.array([min(mseq, oracle.merged_length(l)) for l in lengths], np.uint32)
    t = __import__("torch")
    xm = empty((len(lengths) * mseq, 2048), t.float16)
    nm = empty((len(lengths) * mseq, 2048), t.float16)
    d_x, d_n = dev(x.view(np.float16)), dev(n.view(np.float16))
    check(L().nemo_op_merge(ptr(d_x), ptr(d_n), ptr(d_meta), len(lengths) * mseq, ptr(xm), ptr(nm)))
    T1 = int(tgt.sum())
    assert np.array_equal(host(xm).view(np.uint16)[:T1], oracle.token_merge(x, lengths, tgt))
    assert np.array_equal(host(nm).view(np.uint16)[:T1], oracle.token_merge(n, lengths, tgt))


def test_mean_pool(rng):
    src = [30, 5, 1]
    seq = 30
    tgt = [oracle.merged_length(s) for s in src]
    T1 = sum(tgt)
    x = f16_bits(rng.normal(0, 1, (T1, 2048)))
    d_len, d_meta = meta_for(src, seq)
    t = __import__("torch")
    out = empty((3, 2048), t.float32)
    d_x = dev(x.view(np.float16))
    check(L().nemo_op_pool(ptr(d_x), ptr(d_meta), 3, ptr(out)))
    want = oracle.mean_pool(x, np.array(tgt, np.uint32))
    np.testing.assert_allclose(host(out), want, rtol=2e-5, atol=1e-7)


@pytest.mark.parametrize("impl", ["simt", "tcgen05"])
@pytest.mark.parametrize("lengths", [[15], [40, 3, 17], [2100, 300], [129, 255, 1]],
                         ids=["15", "ragged", "stride3", "tiles"])
def test_attention(rng, lengths, impl):
    seq = max(lengths)
    T = sum(lengths)
    qkv = f16_bits(rng.normal(0, 1, (T, 5120)))
    q = f16_bits(rng.normal(0, 1.5, (T, 3072)))
    k = f16_bits(rng.normal(0, 1.5, (T, 1024)))
    d_len, d_meta = meta_for(lengths, seq)
    t = __import__("torch")
    out = empty((T, 3072), t.float16)
    d_q, d_k, d_qkv = dev(q.view(np.float16)), dev(k.view(np.float16)), dev(qkv.view(np.float16))
    if impl == "simt":
        check(L().nemo_op_attention(ptr(d_q), ptr(d_k), ptr(d_qkv), ptr(d_meta), 0, len(lengths), seq, ptr(out)))
    else:
        check(L().nemo_op_attention_tc(ptr(d_q), ptr(d_k), ptr(d_qkv), ptr(d_meta), 0, len(lengths), seq, T,
                                       ptr(out)))
    want = oracle.attention(q, k, qkv, np.array(lengths, np.uint32))
    got = host(out).view(np.uint16)
    assert rel_err(f16_of_bits(got), f16_of_bits(want)) < 2e-3


# --- projection GEMM ----------------------------------------------------------------

@pytest.mark.parametrize("m", [15, 128, 333])
@pytest.mark.parametrize("impl_bn", [(0, 0), (1, 64), (1, 128), (1, 256)], ids=["simt", "tc64", "tc128", "tc256"])
def test_gemm(rng, m, impl_bn):
    impl, bn = impl_bn
    n, k = 512, 2048
    rows_pad = (m + 127) // 128 * 128
    x = np.zeros((rows_pad, k), np.uint16)
    x[:m] = f16_bits(rng.normal(0, 1, (m, k)))
    w = f16_bits(rng.normal(0, 0.02, (n, k)))
    t = __import__("torch")
    y = empty((rows_pad, n), t.float16)
    d_x, d_w, d_m = dev(x.view(np.float16)), dev(w.view(np.float16)), dev(np.array([m], np.int32))
    check(L().nemo_op_gemm(impl, ptr(d_x), ptr(d_w), ptr(y), ptr(d_m), m, n, k, bn))
    ref32, ref16 = oracle.matmul_f16(x[:m], w)
    got = host(y).view(np.uint16)[:m]
    assert rel_err(f16_of_bits(got), ref32) < 2e-3
