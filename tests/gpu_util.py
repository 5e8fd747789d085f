"""Helpers shared by the GPU tests: device buffers through torch, f16 views."""
import numpy as np


def torch():
    import torch as t
    return t


def dev(a: np.ndarray):
    t = torch()
    return t.from_numpy(np.ascontiguousarray(a)).cuda()


def empty(shape, dtype):
    t = torch()
    return t.zeros(shape, dtype=dtype, device="cuda")


def host(t_):
    return t_.cpu().numpy()


def ptr(t_) -> int:
    return t_.data_ptr()


def f16_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)


def f16_of_bits(b: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(b, np.uint16).view(np.float16).astype(np.float32)


def ulp_diff(a_bits: np.ndarray, b_bits: np.ndarray) -> int:
    """Max distance in f16 units in the last place between two f16 bit arrays."""
    def key(b):
        b = b.astype(np.int32)
        return np.where(b & 0x8000, -(b & 0x7FFF), b)
    return int(np.max(np.abs(key(a_bits) - key(b_bits)))) if a_bits.size else 0


def rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max|got - ref| / max|ref| over a tensor (the per-layer parity measure)."""
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(np.asarray(got, np.float64) - ref)) / max(np.max(np.abs(ref)), 1e-30))
