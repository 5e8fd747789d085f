"""ctypes binding of libnemo_b200.so (include/nemo.h, include/nemo_ops.h).

Mirrors the reference's runtime interface so the engine and tests read like the
reference's own code:

* ``NemotronB200Model`` stands where ``NemotronWebGPUModel`` stands
  (src/webgpu/model.ts:236-329) and implements ``EmbeddingRuntime``
  (src/webgpu/embedding-engine.ts:11-14): ``create_plan(batch, sequence)``.
* ``NemotronExecutionPlan`` stands where the reference's plan of the same name
  stands (model.ts:58-234): ``run(ids, lengths) -> list of float32[2048]``,
  ``profile(ids, lengths) -> {stage: ms}``, ``destroy()``.

There is no CPU path: if the CUDA library is missing the import fails.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HIDDEN = 2048
EXACT_ATTENTION = 1  # NEMO_PLAN_EXACT_ATTENTION: no token merge, no key sampling
NUM_STAGES = 12
_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "libnemo_b200.so")

_lib = None


class NemoError(RuntimeError):
    """A failed libnemo call: ``status`` is the negative nemo_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class ModelInfo(ctypes.Structure):
    _fields_ = [("n_layers", ctypes.c_int), ("vocab", ctypes.c_int), ("n_devices", ctypes.c_int),
                ("compact_matrices", ctypes.c_int), ("kquant_matrices", ctypes.c_int),
                ("packed_weight_bytes", ctypes.c_uint64), ("device_bytes", ctypes.c_uint64)]


def load_library() -> ctypes.CDLL:
    """Loads the in-tree CUDA library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {os.path.dirname(LIB_PATH)}`")
    L = ctypes.CDLL(LIB_PATH)
    P, S, I, U32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_uint32
    sig = {
        "nemo_model_load": (I, [P, S, P, I, ctypes.POINTER(P)]),
        "nemo_model_destroy": (None, [P]),
        "nemo_pack_b200": (I, [P, S, P, S, ctypes.POINTER(S)]),
        "nemo_model_info_get": (I, [P, ctypes.POINTER(ModelInfo)]),
        "nemo_plan_create": (I, [P, U32, U32, ctypes.POINTER(P)]),
        "nemo_plan_create_ex": (I, [P, U32, U32, U32, ctypes.POINTER(P)]),
        "nemo_plan_run": (I, [P, P, S, P, S, P]),
        "nemo_plan_run_device": (I, [P, P, P, P]),
        "nemo_plan_stream": (P, [P]),
        "nemo_plan_single_launch": (I, [P]),
        "nemo_plan_head_parallel": (I, [P]),
        "nemo_plan_synchronize": (I, [P]),
        "nemo_plan_profile": (I, [P, P, S, P, S, P]),
        "nemo_stage_name": (ctypes.c_char_p, [I]),
        "nemo_plan_run_debug": (I, [P, P, S, P, S, P, P, P, P]),
        "nemo_plan_destroy": (None, [P]),
        "nemo_merged_length": (U32, [U32]),
        "nemo_last_error": (ctypes.c_char_p, []),
        "nemo_op_decode": (I, [I, P, I, I, P, P]),
        "nemo_op_meta_bytes": (S, []),
        "nemo_op_meta": (I, [P, I, I, P]),
        "nemo_op_meta_tokens": (P, [P, I]),
        "nemo_op_embedding": (I, [P, P, I, P, I, P]),
        "nemo_op_rmsnorm": (I, [P, P, P, P, P, I]),
        "nemo_rope_table": (I, [I, P]),
        "nemo_op_rope": (I, [P, P, P, I, I, P, P]),
        "nemo_op_attention": (I, [P, P, P, P, I, I, I, P]),
        "nemo_op_attention_tc": (I, [P, P, P, P, I, I, I, I, P]),
        "nemo_op_attention_tc_noalloc": (I, [P, P, P, P, I, I, I, I, P]),
        "nemo_op_swiglu": (I, [P, P, I, P]),
        "nemo_op_merge": (I, [P, P, P, I, P, P]),
        "nemo_op_pool": (I, [P, P, I, P]),
        "nemo_op_gemm": (I, [I, P, P, P, P, I, I, I, I]),
        "nemo_op_qmatmul_image_bytes": (S, [I, I, I]),
        "nemo_op_qmatmul_image": (I, [I, P, I, I, P]),
        "nemo_op_qmatmul_enqueue": (I, [I, P, P, I, I, I, P, P, P]),
        "nemo_op_qmatmul_image_decode": (I, [I, P, I, I, P]),
        "nemo_op_qmatmul": (I, [I, P, P, I, I, I, P]),
        "nemo_hp_qkv_route": (I, [I, P, P, P]),
        "nemo_hp_row_owner": (I, [I, I, I, P]),
        "nemo_tokenizer_load": (I, [P, S, ctypes.POINTER(P)]),
        "nemo_tokenizer_encode": (I, [P, P, S, P, S, ctypes.POINTER(S)]),
        "nemo_tokenizer_destroy": (None, [P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != 0:
        raise NemoError(rc, load_library().nemo_last_error().decode())


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def pack_b200(wgpack: bytes) -> bytes:
    """A B200-tiled copy of a .wgpack (nemo_pack_b200; host only): projections
    stored as the tile-slab images the kernels stream, loaded without re-tiling."""
    src = np.frombuffer(wgpack, dtype=np.uint8)
    need = ctypes.c_size_t()
    L = load_library()
    check(L.nemo_pack_b200(_ptr(src), src.size, None, 0, ctypes.byref(need)))
    out = np.empty(need.value, np.uint8)
    check(L.nemo_pack_b200(_ptr(src), src.size, _ptr(out), out.size, ctypes.byref(need)))
    return out.tobytes()


class NemotronTokenizer:
    """The host tokenizer (nemo_tokenizer_*) over a Hugging Face tokenizer.json.
    Called like the browser tokenizer the reference's engine uses
    (src/webgpu/embedding-engine.ts:41): tokenizer(text)["input_ids"] is a
    [1 x n] array whose first id is the post-processor's BOS."""

    def __init__(self, tokenizer_json: bytes | str):
        if isinstance(tokenizer_json, str):
            with open(tokenizer_json, "rb") as f:
                tokenizer_json = f.read()
        buf = np.frombuffer(tokenizer_json, dtype=np.uint8)
        h = ctypes.c_void_p()
        check(load_library().nemo_tokenizer_load(_ptr(buf), buf.size, ctypes.byref(h)))
        self._h = h

    def encode(self, text: str) -> list[int]:
        raw = text.encode("utf-8")
        n = ctypes.c_size_t()
        L = load_library()
        check(L.nemo_tokenizer_encode(self._h, raw, len(raw), None, 0, ctypes.byref(n)))
        ids = np.empty(max(n.value, 1), np.uint32)
        check(L.nemo_tokenizer_encode(self._h, raw, len(raw), _ptr(ids), ids.size, ctypes.byref(n)))
        return ids[:n.value].tolist()

    def __call__(self, text: str) -> dict:
        return {"input_ids": np.array([self.encode(text)], dtype=np.int64)}

    def close(self) -> None:
        if getattr(self, "_h", None):
            load_library().nemo_tokenizer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def merged_length(sequence: int) -> int:
    """contextualMergedLength (model.ts:30-32)."""
    return load_library().nemo_merged_length(sequence)


class NemotronExecutionPlan:
    """One (batch, sequence) plan: buffers + captured CUDA graphs on every device."""

    def __init__(self, model: "NemotronB200Model", batch: int, sequence: int, exact: bool = False):
        self.model = model
        self.batch = batch
        self.input_sequence = sequence
        self.exact = exact
        self.sequence = sequence if exact else merged_length(sequence)
        h = ctypes.c_void_p()
        check(load_library().nemo_plan_create_ex(model._h, batch, sequence, EXACT_ATTENTION if exact else 0,
                                                 ctypes.byref(h)))
        self._h = h

    def _inputs(self, ids, lengths):
        ids = np.ascontiguousarray(ids, dtype=np.uint32).reshape(-1)
        lengths = np.ascontiguousarray(lengths, dtype=np.uint32).reshape(-1)
        return ids, lengths

    def run(self, ids, lengths) -> list[np.ndarray]:
        """EmbeddingPlan.run: ids [batch*sequence] padded rows, lengths [batch] -> batch arrays of 2048 f32."""
        ids, lengths = self._inputs(ids, lengths)
        out = np.empty((self.batch, HIDDEN), np.float32)
        check(load_library().nemo_plan_run(self._h, _ptr(ids), ids.size, _ptr(lengths), lengths.size, _ptr(out)))
        return [out[i].copy() for i in range(self.batch)]

    def run_array(self, ids, lengths, out: np.ndarray | None = None) -> np.ndarray:
        """Like run() but fills and returns one [batch x 2048] array."""
        ids, lengths = self._inputs(ids, lengths)
        if out is None:
            out = np.empty((self.batch, HIDDEN), np.float32)
        check(load_library().nemo_plan_run(self._h, _ptr(ids), ids.size, _ptr(lengths), lengths.size, _ptr(out)))
        return out

    def run_device(self, d_ids: int, d_lengths: int, d_out: int) -> None:
        """Asynchronous forward on device-resident inputs (raw device pointers)."""
        check(load_library().nemo_plan_run_device(self._h, d_ids, d_lengths, d_out))

    def stream(self) -> int:
        return load_library().nemo_plan_stream(self._h) or 0

    @property
    def head_parallel_min(self) -> int:
        """Request length from which runs go head-parallel over the plan's
        devices (0: the plan has no head-parallel path)."""
        r = load_library().nemo_plan_head_parallel(self._h)
        if r < 0:
            check(r)
        return r

    @property
    def fused(self) -> bool:
        """True when the plan runs the forward as one persistent launch."""
        r = load_library().nemo_plan_single_launch(self._h)
        if r < 0:
            check(r)
        return r == 1

    def synchronize(self) -> None:
        check(load_library().nemo_plan_synchronize(self._h))

    def profile(self, ids, lengths) -> dict[str, float]:
        """Per-stage device milliseconds, summed over layers (model.ts:178-224)."""
        ids, lengths = self._inputs(ids, lengths)
        ms = np.zeros(NUM_STAGES, np.float32)
        check(load_library().nemo_plan_profile(self._h, _ptr(ids), ids.size, _ptr(lengths), lengths.size, _ptr(ms)))
        L = load_library()
        return {L.nemo_stage_name(i).decode(): float(ms[i]) for i in range(NUM_STAGES)}

    def run_debug(self, ids, lengths):
        """Forward with per-layer dumps: (embeddings, [(x_f16_bits, norm_f16_bits) per layer])."""
        ids, lengths = self._inputs(ids, lengths)
        n_layers = self.model.info().n_layers
        out = np.empty((self.batch, HIDDEN), np.float32)
        xd = np.zeros((n_layers, self.batch * self.input_sequence, HIDDEN), np.uint16)
        nd = np.zeros_like(xd)
        tpl = np.zeros(16, np.int32)
        check(load_library().nemo_plan_run_debug(self._h, _ptr(ids), ids.size, _ptr(lengths), lengths.size, _ptr(out),
                                                 _ptr(xd), _ptr(nd), _ptr(tpl)))
        return out, [(xd[l, :tpl[l]], nd[l, :tpl[l]]) for l in range(n_layers)]

    def destroy(self) -> None:
        if getattr(self, "_h", None):
            load_library().nemo_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


class NemotronB200Model:
    """A loaded .wgpack with one replica per device; an EmbeddingRuntime."""

    # The B200 build has no storage-binding cap (embedding-engine.ts:65-67).
    max_storage_buffer_binding_size = None

    def __init__(self, wgpack: bytes | str, devices: list[int] | None = None):
        if isinstance(wgpack, str):
            with open(wgpack, "rb") as f:
                wgpack = f.read()
        buf = np.frombuffer(wgpack, dtype=np.uint8)
        devs = np.asarray(devices if devices else [0], dtype=np.int32)
        h = ctypes.c_void_p()
        check(load_library().nemo_model_load(_ptr(buf), buf.size, _ptr(devs), devs.size, ctypes.byref(h)))
        self._h = h
        self.plans: list[NemotronExecutionPlan] = []

    def info(self) -> ModelInfo:
        i = ModelInfo()
        check(load_library().nemo_model_info_get(self._h, ctypes.byref(i)))
        return i

    def create_plan(self, batch: int, sequence: int, exact: bool = False) -> NemotronExecutionPlan:
        """EmbeddingRuntime.createPlan; exact=True drops the token merge and the
        stride-3 key sampling (a build-specific mode, not the reference's)."""
        plan = NemotronExecutionPlan(self, batch, sequence, exact)
        self.plans.append(plan)
        return plan

    def destroy(self) -> None:
        for p in self.plans:
            p.destroy()
        self.plans = []
        if getattr(self, "_h", None):
            load_library().nemo_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass
