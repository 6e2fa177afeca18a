"""ctypes binding of libpurebee_b200.so (the C ABI in include/purebee_cuda.h).

The library is built in-tree by purebee_b200/build.py.  There is no CPU
fallback: if the library is missing or no sm_100 device is present, the
calls raise.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpurebee_b200.so")

PB_OK, PB_ERR_ARG, PB_ERR_OOM, PB_ERR_CUDA, PB_ERR_TIMEOUT, PB_ERR_DEVICE, PB_ERR_STATE, PB_ERR_NOTFOUND = range(8)
TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q4_1, TYPE_Q8_0 = 0, 1, 2, 3, 8
QMAT_TABLE = 0x100  # OR into the type: LM-head table layout (pb_qmat_head)
MODEL_STREAMING_Q4, MODEL_LLAMA_Q8A = 0, 1
MATVEC_FAST, MATVEC_EXACT = 0, 1  # pb_set_matvec_mode

_ERRNAMES = {1: "PB_ERR_ARG", 2: "PB_ERR_OOM", 3: "PB_ERR_CUDA", 4: "PB_ERR_TIMEOUT", 5: "PB_ERR_DEVICE",
             6: "PB_ERR_STATE", 7: "PB_ERR_NOTFOUND"}


class PureBeeError(RuntimeError):
    """A non-zero status from the C ABI (the reference throws Error with the message)."""

    def __init__(self, code, msg):
        super().__init__(f"{_ERRNAMES.get(code, code)}: {msg}")
        self.code = code


class ModelConfig(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("emb_type", ctypes.c_int), ("dim", ctypes.c_int),
                ("hidden_dim", ctypes.c_int), ("n_layers", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("vocab", ctypes.c_int),
                ("seq_len", ctypes.c_int), ("rope_theta", ctypes.c_double), ("eps", ctypes.c_double)]


class SplitPlan(ctypes.Structure):
    """pb_split_plan: the rows rank `rank` of `world` holds in a row-split batch."""
    _fields_ = [(n, ctypes.c_int) for n in ("world", "rank", "n_heads", "n_kv_heads", "q_row0", "k_row0", "v_row0",
                                           "qkv_rows", "dim_chunk", "hidden_chunk", "vocab_row0", "vocab_rows",
                                           "vocab_chunk")]


COMM_ID_BYTES = 128

V = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
U64 = ctypes.c_uint64
D = ctypes.c_double
SZ = ctypes.c_size_t

# name: (restype, argtypes)
SIGNATURES = {
    "pb_init": (I, [I, ctypes.POINTER(V)]),
    "pb_shutdown": (I, [V]),
    "pb_last_error": (ctypes.c_char_p, [V]),
    "pb_abi_version": (I, []),
    "pb_set_timeout_ms": (I, [V, I]),
    "pb_sync": (I, [V]),
    "pb_stream": (V, [V]),
    "pb_device_error": (I, [V, ctypes.POINTER(I)]),
    "pb_launch_count": (I64, [V]),
    "pb_capture_begin": (I, [V]),
    "pb_capture_end": (I, [V, ctypes.POINTER(V)]),
    "pb_graph_launch": (I, [V, V]),
    "pb_graph_free": (I, [V]),
    "pb_malloc": (I, [V, SZ, ctypes.POINTER(V)]),
    "pb_free": (I, [V, V]),
    "pb_upload": (I, [V, V, V, SZ]),
    "pb_download": (I, [V, V, V, SZ]),
    "pb_memset": (I, [V, V, I, SZ]),
    "pb_memcpy_d2d": (I, [V, V, V, SZ]),
    "pb_qmat_upload": (I, [V, I, V, I, I, ctypes.POINTER(V)]),
    "pb_qmat_from_device": (I, [V, I, V, I, I, ctypes.POINTER(V)]),
    "pb_qmat_download_gguf": (I, [V, V, V]),
    "pb_qmat_free": (I, [V, V]),
    "pb_qmat_info": (I, [V, ctypes.POINTER(I), ctypes.POINTER(I), ctypes.POINTER(I)]),
    "pb_qmat_matvec": (I, [V, V, V, V, I, I]),
    "pb_q4_0_matvec": (I, [V, V, V, I, I, V]),
    "pb_q4_1_matvec": (I, [V, V, V, I, I, V]),
    "pb_lm_head": (I, [V, V, V, I, I, V]),
    "pb_q4_gemm": (I, [V, V, V, I, I, V, I]),
    "pb_qmat_head": (I, [V, V, V, V, V]),
    "pb_argmax": (I, [V, V, I, V]),
    "pb_matmul_f32": (I, [V, V, I, I, V, I, V, V]),
    "pb_matmul_q8a": (I, [V, V, I, I, V, V, I, V, V]),
    "pb_rmsnorm": (I, [V, V, I, I, V, D, V]),
    "pb_softmax": (I, [V, V, I, I, V]),
    "pb_layernorm": (I, [V, V, I, I, V, V, D, V]),
    "pb_gelu": (I, [V, V, I64, V]),
    "pb_silu": (I, [V, V, I64, V]),
    "pb_elementmul": (I, [V, V, V, I64, V]),
    "pb_tensoradd": (I, [V, V, V, I64, V]),
    "pb_attention": (I, [V, V, V, V, I, I, I, I, I, V]),
    "pb_attention_noalloc": (I, [V, V, V, V, I, I, I, I, I, V]),
    "pb_rope": (I, [V, V, V, I, I, I, I, I, D]),
    "pb_attn_cached": (I, [V, V, V, V, I, I, I, I, I, V]),
    "pb_attn_decode": (I, [V, V, V, V, I, I, I, I, I, V]),
    "pb_set_matvec_mode": (I, [V, I]),
    "pb_matvec_mode": (I, [V]),
    "pb_set_mvi_min_rows": (I, [V, I]),
    "pb_set_mvt": (I, [V, I]),
    "pb_set_fuse_attn": (I, [V, I]),
    "pb_swiglu": (I, [V, V, V, I, V]),
    "pb_quantize_q8a": (I, [V, V, I64, V, V]),
    "pb_quantize_q4a": (I, [V, V, I64, V, V]),
    "pb_dequantize_q8a": (I, [V, V, V, I64, V]),
    "pb_dequantize_q4a": (I, [V, V, V, I64, V]),
    "pb_gguf_dequant": (I, [V, I, V, I64, V]),
    "pb_gguf_quantize": (I, [V, I, V, I64, V]),
    "pb_synth_weights": (I, [V, V, I64, U64, U64, D]),
    "pb_synth_activation": (I, [V, V, I64, U64, U64]),
    "pb_synth_tokens": (I, [V, I, U64, I, I]),
    "pb_model_create": (I, [V, ctypes.POINTER(ModelConfig), ctypes.POINTER(V)]),
    "pb_model_free": (I, [V]),
    "pb_model_init_synthetic": (I, [V, U64, D]),
    "pb_model_set_tensor": (I, [V, I, I, V, SZ]),
    "pb_model_attach_head": (I, [V, I]),
    "pb_model_forward_ex": (I, [V, V, I, I, I, V, ctypes.POINTER(I)]),
    "pb_model_decode_ex": (I, [V, I, I, I, ctypes.POINTER(I), V, ctypes.POINTER(I)]),
    "pb_model_set_early_exit": (I, [V, D, I]),
    "pb_model_exit_stats": (I, [V, ctypes.POINTER(I), ctypes.POINTER(I), ctypes.POINTER(I)]),
    "pb_model_sample": (I, [V, I, D, U64, U64, ctypes.POINTER(I)]),
    "pb_sample_topk": (I, [V, V, I, I, D, U64, U64, V]),
    "pb_sample_uniform": (D, [U64, U64]),
    "pb_model_generate_sampled": (I, [V, V, I, I, I, I, D, U64, V, I, ctypes.POINTER(I)]),
    "pb_gguf_last_error": (ctypes.c_char_p, []),
    "pb_gguf_open": (I, [ctypes.c_char_p, ctypes.POINTER(V)]),
    "pb_gguf_close": (I, [V]),
    "pb_gguf_version": (I, [V]),
    "pb_gguf_data_start": (I64, [V]),
    "pb_gguf_alignment": (I64, [V]),
    "pb_gguf_meta_count": (I, [V]),
    "pb_gguf_meta_find": (I, [V, ctypes.c_char_p]),
    "pb_gguf_meta_key": (I, [V, I, ctypes.POINTER(ctypes.c_char_p)]),
    "pb_gguf_meta_type": (I, [V, I, ctypes.POINTER(I), ctypes.POINTER(I), ctypes.POINTER(I64)]),
    "pb_gguf_meta_int": (I, [V, I, ctypes.POINTER(I64)]),
    "pb_gguf_meta_float": (I, [V, I, ctypes.POINTER(D)]),
    "pb_gguf_meta_string": (I, [V, I, ctypes.POINTER(V), ctypes.POINTER(I64)]),
    "pb_gguf_meta_array_string": (I, [V, I, I64, ctypes.POINTER(V), ctypes.POINTER(I64)]),
    "pb_gguf_meta_array_number": (I, [V, I, I64, ctypes.POINTER(D)]),
    "pb_gguf_tensor_count": (I, [V]),
    "pb_gguf_tensor_find": (I, [V, ctypes.c_char_p]),
    "pb_gguf_tensor_info": (I, [V, I, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(I), ctypes.POINTER(I),
                                ctypes.POINTER(I64), ctypes.POINTER(I64), ctypes.POINTER(I64)]),
    "pb_gguf_tensor_read": (I, [V, I, V, SZ]),
    "pb_gguf_config": (I, [V, ctypes.POINTER(ModelConfig)]),
    "pb_model_load_gguf": (I, [V, V, I, ctypes.POINTER(V)]),
    "pb_model_get_tensor": (I, [V, I, I, V, SZ]),
    "pb_model_forward": (I, [V, V, I, I, V]),
    "pb_model_decode": (I, [V, I, I, ctypes.POINTER(I), V]),
    "pb_model_generate": (I, [V, V, I, I, I, V, I, ctypes.POINTER(I)]),
    "pb_model_decode_loop": (I, [V, I, I, V]),
    "pb_model_set_token": (I, [V, I]),
    "pb_model_reset_cache": (I, [V]),
    "pb_model_rollback_cache": (I, [V, I]),
    "pb_model_kv": (I, [V, I, I, V, SZ]),
    "pb_model_set_rope_scaling": (I, [V, D, D, D, I]),
    "pb_model_rope_scaling": (I, [V, ctypes.POINTER(D)]),
    "pb_rope_freqs": (I, [D, I, D, D, D, I, V]),
    "pb_model_decode_bytes": (I64, [V, I]),
    "pb_model_decode_launches": (I, [V]),
    "pb_q4_gemm_f16": (I, [V, V, V, I, V, I]),
    "pb_q4_gemm_ex": (I, [V, V, V, I, I, V, I, I]),
    "pb_q4_gemm_hl": (I, [V, V, V, I, V, I]),
    "pb_batch_create": (I, [V, I, ctypes.POINTER(V)]),
    "pb_batch_free": (I, [V]),
    "pb_batch_prefill": (I, [V, V, I, V, V]),
    "pb_batch_decode": (I, [V, I, V, V]),
    "pb_batch_set_precision": (I, [V, I]),
    "pb_batch_split_plan": (I, [ctypes.POINTER(ModelConfig), I, I, ctypes.POINTER(SplitPlan)]),
    "pb_batch_create_split": (I, [V, I, V, ctypes.POINTER(V)]),
    "pb_batch_create_group": (I, [V, I, I, ctypes.POINTER(V)]),
    "pb_comm_id": (I, [V]),
    "pb_comm_init": (I, [V, I, I, V, ctypes.POINTER(V)]),
    "pb_comm_free": (I, [V]),
    "pb_comm_rank": (I, [V]),
    "pb_comm_world": (I, [V]),
    "pb_comm_allgather": (I, [V, V, V, SZ]),
    "pb_comm_peer_access": (I, [V]),
    "pb_comm_register": (I, [V, V, ctypes.POINTER(V)]),
    "pb_comm_deregister": (I, [V, V]),
    "pb_comm_allgather_inplace": (I, [V, V, SZ]),
    "pb_comm_selftest_wait": (I, [V, I, ctypes.POINTER(I)]),
}

_lib = None


def lib():
    """Load the library (raises if it was not built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing; build it with `python purebee_b200/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ptr(a) -> int:
    """Address of a host numpy array's data."""
    return a.ctypes.data


class DeviceBuffer:
    """A device allocation owned by a Context."""

    def __init__(self, ctx: "Context", nbytes: int):
        self.ctx = ctx
        self.nbytes = int(nbytes)
        p = V()
        ctx._check(lib().pb_malloc(ctx.h, self.nbytes, ctypes.byref(p)))
        self.ptr = p.value

    def upload(self, arr: np.ndarray) -> None:
        a = np.ascontiguousarray(arr)
        if a.nbytes > self.nbytes:
            raise ValueError("upload larger than buffer")
        self.ctx._check(lib().pb_upload(self.ctx.h, self.ptr, ptr(a), a.nbytes))

    def download(self, dtype=np.float32, count=None) -> np.ndarray:
        dt = np.dtype(dtype)
        n = self.nbytes // dt.itemsize if count is None else int(count)
        out = np.empty(n, dt)
        self.ctx._check(lib().pb_download(self.ctx.h, ptr(out), self.ptr, out.nbytes))
        return out

    def free(self) -> None:
        if self.ptr and self.ctx.h:
            lib().pb_free(self.ctx.h, self.ptr)
        self.ptr = None

    def __del__(self):
        try:
            if self.ptr and self.ctx.h:
                lib().pb_free(self.ctx.h, self.ptr)
        except Exception:
            pass


class Context:
    """One device, one stream (pb_init / pb_shutdown)."""

    def __init__(self, device: int = 0):
        h = V()
        rc = lib().pb_init(device, ctypes.byref(h))
        if rc != PB_OK:
            raise PureBeeError(rc, f"pb_init(device={device}) failed (no sm_100 device, or the self-test failed)")
        self.h = h.value
        self.device = device

    def _check(self, rc: int) -> None:
        if rc != PB_OK:
            raise PureBeeError(rc, lib().pb_last_error(self.h).decode(errors="replace"))

    def close(self) -> None:
        if self.h:
            lib().pb_shutdown(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def sync(self) -> None:
        self._check(lib().pb_sync(self.h))

    def set_matvec_mode(self, mode: int) -> None:
        """MATVEC_FAST (default) or MATVEC_EXACT (the reference's lane order, bit for bit)."""
        self._check(lib().pb_set_matvec_mode(self.h, int(mode)))

    @property
    def matvec_mode(self) -> int:
        return int(lib().pb_matvec_mode(self.h))

    def set_mvi_min_rows(self, rows: int) -> None:
        """Fast mode: matrix rows from which Q4_0 matvecs take the int8 tensor-core kernel."""
        self._check(lib().pb_set_mvi_min_rows(self.h, int(rows)))

    def set_fuse_attn(self, on: bool) -> None:
        """Fast mode: one-sequence decode projection + attention in one kernel (default off; same bits)."""
        self._check(lib().pb_set_fuse_attn(self.h, 1 if on else 0))

    def set_mvt(self, on: bool) -> None:
        """Fast mode: the tcgen05 int8 matvec for the Q4_0 matrices uploaded while it is on (default off)."""
        self._check(lib().pb_set_mvt(self.h, 1 if on else 0))

    def set_timeout_ms(self, ms: int) -> None:
        self._check(lib().pb_set_timeout_ms(self.h, ms))

    @property
    def launches(self) -> int:
        return int(lib().pb_launch_count(self.h))

    def alloc(self, nbytes: int) -> DeviceBuffer:
        return DeviceBuffer(self, nbytes)

    def to_device(self, arr: np.ndarray) -> DeviceBuffer:
        a = np.ascontiguousarray(arr)
        b = DeviceBuffer(self, max(a.nbytes, 16))
        b.upload(a)
        return b

    def capture(self, fn) -> "Graph":
        """Record the device-pointer calls fn() makes into a replayable graph."""
        self._check(lib().pb_capture_begin(self.h))
        try:
            fn()
        finally:
            g = V()
            rc = lib().pb_capture_end(self.h, ctypes.byref(g))
        self._check(rc)
        return Graph(self, g.value)

    def device_error(self) -> int:
        c = I()
        self._check(lib().pb_device_error(self.h, ctypes.byref(c)))
        return c.value


class QMat:
    """A quantized matrix resident on the device (pb_qmat)."""

    def __init__(self, ctx: Context, type_: int, gguf: np.ndarray, N: int, K: int):
        self.ctx = ctx
        g = np.ascontiguousarray(gguf, np.uint8)
        h = V()
        ctx._check(lib().pb_qmat_upload(ctx.h, type_, ptr(g), N, K, ctypes.byref(h)))
        self.h = h.value
        self.type, self.N, self.K = type_ & ~QMAT_TABLE, N, K

    def gguf_bytes(self) -> np.ndarray:
        bb = {TYPE_Q4_0: 18, TYPE_Q4_1: 20, TYPE_Q8_0: 34}[self.type]
        out = np.empty(self.N * (self.K // 32) * bb, np.uint8)
        self.ctx._check(lib().pb_qmat_download_gguf(self.ctx.h, self.h, ptr(out)))
        return out

    def free(self):
        if self.h and self.ctx.h:
            lib().pb_qmat_free(self.ctx.h, self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Graph:
    """A recorded sequence of calls (pb_capture_begin / pb_capture_end)."""

    def __init__(self, ctx: Context, h):
        self.ctx, self.h = ctx, h

    def launch(self) -> None:
        self.ctx._check(lib().pb_graph_launch(self.ctx.h, self.h))

    def free(self) -> None:
        if self.h:
            lib().pb_graph_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
