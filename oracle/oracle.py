"""ctypes binding of the CPU oracle (oracle/pb_oracle.c).

TEST INFRASTRUCTURE ONLY.  tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg import this module as the parity checker or the timed CPU
restatement of the reference.  The product package never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "pb_oracle.c")
LIB_PATH = os.path.join(HERE, "_build", "libpb_oracle.so")
SYNTH_DIR = os.path.join(os.path.dirname(HERE), "purebee_b200", "csrc")

F32P = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
U8P = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
I8P = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    """Compile the oracle with gcc (separate float multiply and add kept)."""
    srcs = [SRC, os.path.join(HERE, "pb_oracle.h"), os.path.join(SYNTH_DIR, "pb_synth.h")]
    if not force and os.path.exists(LIB_PATH):
        lib_t = os.path.getmtime(LIB_PATH)
        if all(os.path.getmtime(s) <= lib_t for s in srcs):
            return LIB_PATH
    os.makedirs(os.path.dirname(LIB_PATH), exist_ok=True)
    cmd = ["gcc", "-O2", "-std=c11", "-D_GNU_SOURCE", "-ffp-contract=off", "-fno-fast-math",
           "-fPIC", "-shared", "-pthread", "-I" + SYNTH_DIR, "-o", LIB_PATH, SRC, "-lm"]
    subprocess.check_call(cmd)
    return LIB_PATH


class _Cfg(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("emb_type", ctypes.c_int), ("dim", ctypes.c_int),
                ("hidden_dim", ctypes.c_int), ("n_layers", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("vocab", ctypes.c_int),
                ("seq_len", ctypes.c_int), ("rope_theta", ctypes.c_double), ("eps", ctypes.c_double)]


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    L = ctypes.CDLL(build())
    c_i64 = ctypes.c_int64
    sig = {
        "orc_set_threads": (None, [ctypes.c_int]),
        "orc_get_threads": (ctypes.c_int, []),
        "orc_f16_exact": (ctypes.c_float, [ctypes.c_uint16]),
        "orc_f16_wasm": (ctypes.c_float, [ctypes.c_uint16]),
        "orc_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
        "orc_dequant_q4_0": (None, [U8P, c_i64, F32P]),
        "orc_dequant_q4_1": (None, [U8P, c_i64, F32P]),
        "orc_dequant_q8_0": (None, [U8P, c_i64, F32P]),
        "orc_dequant_f16": (None, [U8P, c_i64, F32P]),
        "orc_dequant_q6_k": (None, [U8P, c_i64, F32P]),
        "orc_quantize_gguf_q4_0": (None, [F32P, c_i64, U8P]),
        "orc_quantize_gguf_q8_0": (None, [F32P, c_i64, U8P]),
        "orc_q4_0_matvec_wasm": (None, [F32P, U8P, ctypes.c_int, ctypes.c_int, F32P]),
        "orc_q4_1_matvec_wasm": (None, [F32P, U8P, ctypes.c_int, ctypes.c_int, F32P]),
        "orc_q4_0_matvec_js": (None, [F32P, U8P, ctypes.c_int, ctypes.c_int, F32P]),
        "orc_q4_1_matvec_js": (None, [F32P, U8P, ctypes.c_int, ctypes.c_int, F32P]),
        "orc_batch_dot": (None, [F32P, F32P, ctypes.c_int, ctypes.c_int, F32P]),
        "orc_matmul_wasm": (None, [F32P, ctypes.c_int, ctypes.c_int, F32P, ctypes.c_int, ctypes.c_void_p, F32P]),
        "orc_quantize_q8a": (None, [F32P, c_i64, F32P, I8P]),
        "orc_quantize_q4a": (None, [F32P, c_i64, F32P, U8P]),
        "orc_dequantize_q8a": (None, [F32P, I8P, c_i64, F32P]),
        "orc_dequantize_q4a": (None, [F32P, U8P, c_i64, F32P]),
        "orc_matmul_q8": (None, [F32P, ctypes.c_int, ctypes.c_int, F32P, I8P, ctypes.c_int, ctypes.c_void_p, F32P]),
        "orc_rmsnorm": (None, [F32P, ctypes.c_int, ctypes.c_int, F32P, ctypes.c_double, F32P]),
        "orc_softmax": (None, [F32P, ctypes.c_int, ctypes.c_int, F32P]),
        "orc_layernorm": (None, [F32P, ctypes.c_int, ctypes.c_int, F32P, ctypes.c_void_p, ctypes.c_double, F32P]),
        "orc_gelu": (None, [F32P, c_i64, F32P]),
        "orc_silu": (None, [F32P, c_i64, F32P]),
        "orc_elementmul": (None, [F32P, F32P, c_i64, F32P]),
        "orc_tensoradd": (None, [F32P, F32P, c_i64, F32P]),
        "orc_attention": (None, [F32P, F32P, F32P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_int, F32P]),
        "orc_rope": (None, [F32P, F32P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                            ctypes.c_int, ctypes.c_double]),
        "orc_attn_cached": (None, [F32P, F32P, F32P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_int, ctypes.c_int, F32P]),
        "orc_swiglu_fused": (None, [F32P, F32P, ctypes.c_int, F32P]),
        "orc_argmax": (ctypes.c_int, [F32P, ctypes.c_int]),
        "orc_synth_weights": (None, [F32P, c_i64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_double]),
        "orc_synth_activation": (None, [F32P, c_i64, ctypes.c_uint64, ctypes.c_uint64]),
        "orc_synth_tokens": (None, [I32P, ctypes.c_int, ctypes.c_uint64, ctypes.c_int, ctypes.c_int]),
        "orc_model_create": (ctypes.c_void_p, [ctypes.POINTER(_Cfg)]),
        "orc_model_free": (None, [ctypes.c_void_p]),
        "orc_model_init_synthetic": (None, [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_double]),
        "orc_model_tensor": (ctypes.POINTER(ctypes.c_uint8), [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                                              ctypes.POINTER(c_i64)]),
        "orc_model_q8a_scales": (ctypes.POINTER(ctypes.c_float), [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                                                  ctypes.POINTER(c_i64)]),
        "orc_model_refresh": (None, [ctypes.c_void_p]),
        "orc_model_set_head": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
        "orc_sample": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_double]),
        "orc_sample_uniform": (ctypes.c_double, [ctypes.c_uint64, ctypes.c_uint64]),
        "orc_forward_ex": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_double, ctypes.c_int, ctypes.c_void_p,
                                          ctypes.POINTER(ctypes.c_int)]),
        "orc_exit_prob": (ctypes.c_double, [ctypes.c_void_p, ctypes.c_int]),
        "orc_forward": (ctypes.c_int, [ctypes.c_void_p, I32P, ctypes.c_int, ctypes.c_int, F32P]),
        "orc_generate": (ctypes.c_int, [ctypes.c_void_p, I32P, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                        I32P, ctypes.c_int]),
        "orc_reset_cache": (None, [ctypes.c_void_p]),
        "orc_rollback_cache": (None, [ctypes.c_void_p, ctypes.c_int]),
        "orc_kv": (ctypes.POINTER(ctypes.c_float), [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a):
    return np.ascontiguousarray(a, dtype=np.uint8)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


# ---- elementwise / kernels -------------------------------------------------

def f16_exact(bits: int) -> float:
    return lib().orc_f16_exact(int(bits))


def f16_wasm(bits: int) -> float:
    return lib().orc_f16_wasm(int(bits))


def f32_to_f16(v: float) -> int:
    return lib().orc_f32_to_f16(float(v))


def dequant_q4_0(raw, n):
    out = np.empty(n, np.float32)
    lib().orc_dequant_q4_0(_u8(raw), n, out)
    return out


def dequant_q4_1(raw, n):
    out = np.empty(n, np.float32)
    lib().orc_dequant_q4_1(_u8(raw), n, out)
    return out


def dequant_q6_k(raw, n):
    out = np.empty(n, np.float32)
    lib().orc_dequant_q6_k(_u8(raw), n, out)
    return out


def dequant_q8_0(raw, n):
    out = np.empty(n, np.float32)
    lib().orc_dequant_q8_0(_u8(raw), n, out)
    return out


def quantize_gguf_q4_0(x):
    x = _f32(x).ravel()
    out = np.zeros(x.size // 32 * 18, np.uint8)
    lib().orc_quantize_gguf_q4_0(x, x.size, out)
    return out


def quantize_gguf_q8_0(x):
    x = _f32(x).ravel()
    out = np.zeros(x.size // 32 * 34, np.uint8)
    lib().orc_quantize_gguf_q8_0(x, x.size, out)
    return out


def q4_0_matvec(x, raw, N, K):
    y = np.empty(N, np.float32)
    lib().orc_q4_0_matvec_wasm(_f32(x), _u8(raw), N, K, y)
    return y


def q4_1_matvec(x, raw, N, K):
    y = np.empty(N, np.float32)
    lib().orc_q4_1_matvec_wasm(_f32(x), _u8(raw), N, K, y)
    return y


def q4_0_matvec_js(x, raw, N, K):
    y = np.empty(N, np.float32)
    lib().orc_q4_0_matvec_js(_f32(x), _u8(raw), N, K, y)
    return y


def q4_1_matvec_js(x, raw, N, K):
    y = np.empty(N, np.float32)
    lib().orc_q4_1_matvec_js(_f32(x), _u8(raw), N, K, y)
    return y


def batch_dot(x, W, N, K):
    out = np.empty(N, np.float32)
    lib().orc_batch_dot(_f32(x), _f32(W).ravel(), N, K, out)
    return out


def matmul_wasm(A, M, K, B, N, bias=None):
    out = np.empty(M * N, np.float32)
    b = _f32(bias) if bias is not None else None
    lib().orc_matmul_wasm(_f32(A).ravel(), M, K, _f32(B).ravel(), N,
                          b.ctypes.data if b is not None else None, out)
    return out


def quantize_q8a(data):
    data = _f32(data).ravel()
    nb = (data.size + 31) // 32
    scales = np.zeros(nb, np.float32)
    q = np.zeros(nb * 32, np.int8)
    lib().orc_quantize_q8a(data, data.size, scales, q)
    return scales, q


def quantize_q4a(data):
    data = _f32(data).ravel()
    nb = (data.size + 31) // 32
    scales = np.zeros(nb, np.float32)
    q = np.zeros((nb * 32 + 1) // 2, np.uint8)
    lib().orc_quantize_q4a(data, data.size, scales, q)
    return scales, q


def dequantize_q8a(scales, q, n):
    out = np.empty(n, np.float32)
    lib().orc_dequantize_q8a(_f32(scales), np.ascontiguousarray(q, np.int8), n, out)
    return out


def dequantize_q4a(scales, q, n):
    out = np.empty(n, np.float32)
    lib().orc_dequantize_q4a(_f32(scales), _u8(q), n, out)
    return out


def matmul_q8(a, M, K, scales, q, N, bias=None):
    out = np.empty(M * N, np.float32)
    b = _f32(bias) if bias is not None else None
    lib().orc_matmul_q8(_f32(a).ravel(), M, K, _f32(scales), np.ascontiguousarray(q, np.int8), N,
                        b.ctypes.data if b is not None else None, out)
    return out


def rmsnorm(x, seq, dim, w, eps=1e-5):
    out = np.empty(seq * dim, np.float32)
    lib().orc_rmsnorm(_f32(x).ravel(), seq, dim, _f32(w), eps, out)
    return out


def softmax(x, rows, cols):
    out = np.empty(rows * cols, np.float32)
    lib().orc_softmax(_f32(x).ravel(), rows, cols, out)
    return out


def layernorm(x, seq, dim, w, b=None, eps=1e-5):
    out = np.empty(seq * dim, np.float32)
    bb = _f32(b) if b is not None else None
    lib().orc_layernorm(_f32(x).ravel(), seq, dim, _f32(w), bb.ctypes.data if bb is not None else None, eps, out)
    return out


def gelu(x):
    x = _f32(x).ravel()
    out = np.empty_like(x)
    lib().orc_gelu(x, x.size, out)
    return out


def silu(x):
    x = _f32(x).ravel()
    out = np.empty_like(x)
    lib().orc_silu(x, x.size, out)
    return out


def elementmul(a, b):
    a = _f32(a).ravel()
    out = np.empty_like(a)
    lib().orc_elementmul(a, _f32(b).ravel(), a.size, out)
    return out


def tensoradd(a, b):
    a = _f32(a).ravel()
    out = np.empty_like(a)
    lib().orc_tensoradd(a, _f32(b).ravel(), a.size, out)
    return out


def attention(Q, K, V, seqQ, seqK, dK, dV, causal=True):
    out = np.empty(seqQ * dV, np.float32)
    lib().orc_attention(_f32(Q).ravel(), _f32(K).ravel(), _f32(V).ravel(), seqQ, seqK, dK, dV, int(causal), out)
    return out


def rope(q, k, seq, start_pos, dim, n_heads, n_kv, head_dim, theta):
    q = _f32(q).ravel().copy()
    k = _f32(k).ravel().copy()
    lib().orc_rope(q, k, seq, start_pos, dim, n_heads, n_kv, head_dim, theta)
    return q, k


def attn_cached(q, kc, vc, seq, start_pos, dim, n_heads, n_kv, head_dim):
    out = np.empty(seq * dim, np.float32)
    lib().orc_attn_cached(_f32(q).ravel(), _f32(kc).ravel(), _f32(vc).ravel(), seq, start_pos, dim, n_heads,
                          n_kv, head_dim, out)
    return out


def swiglu_fused(g, u):
    g = _f32(g).ravel()
    out = np.empty_like(g)
    lib().orc_swiglu_fused(g, _f32(u).ravel(), g.size, out)
    return out


def argmax(logits):
    l = _f32(logits).ravel()
    return int(lib().orc_argmax(l, l.size))


def sample(logits, topK, temperature, r):
    """llama-streaming.js:868-894 with the uniform draw r given."""
    x = _f32(logits)
    return int(lib().orc_sample(x.ctypes.data, x.size, topK, temperature, r))


def exit_prob(logits):
    x = _f32(logits)
    return float(lib().orc_exit_prob(x.ctypes.data, x.size))


def sample_uniform(seed, counter):
    return float(lib().orc_sample_uniform(seed, counter))


def synth_weights(n, seed, tensor_id, stdev=0.02):
    out = np.empty(n, np.float32)
    lib().orc_synth_weights(out, n, seed, tensor_id, stdev)
    return out


def synth_activation(n, seed, stream):
    out = np.empty(n, np.float32)
    lib().orc_synth_activation(out, n, seed, stream)
    return out


def synth_tokens(n, seed, lo, hi):
    out = np.empty(n, np.int32)
    lib().orc_synth_tokens(out, n, seed, lo, hi)
    return out


# ---- model ------------------------------------------------------------------

KIND_STREAMING_Q4 = 0
KIND_LLAMA_Q8A = 1
EMB_F32, EMB_Q4_0, EMB_Q8_0 = 0, 2, 8


@dataclass
class Config:
    kind: int
    emb_type: int
    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    seq_len: int
    rope_theta: float = 10000.0
    eps: float = 1e-5

    def c(self):
        return _Cfg(self.kind, self.emb_type, self.dim, self.hidden_dim, self.n_layers, self.n_heads,
                    self.n_kv_heads, self.head_dim, self.vocab, self.seq_len, self.rope_theta, self.eps)


class Model:
    """The reference runtime restated: llama-streaming.js (GGUF Q4_0) or llama.js (quantize.js Q8)."""

    def __init__(self, cfg: Config):
        self.cfg = cfg
        self._c = cfg.c()
        self.h = lib().orc_model_create(ctypes.byref(self._c))
        if not self.h:
            raise RuntimeError("orc_model_create failed")

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_free(self.h)
            self.h = None

    def init_synthetic(self, seed, stdev=0.02):
        lib().orc_model_init_synthetic(self.h, seed, stdev)

    def tensor(self, layer, which) -> np.ndarray:
        n = ctypes.c_int64()
        p = lib().orc_model_tensor(self.h, layer, which, ctypes.byref(n))
        return np.ctypeslib.as_array(p, shape=(n.value,))

    def q8a_scales(self, layer, which) -> np.ndarray:
        n = ctypes.c_int64()
        p = lib().orc_model_q8a_scales(self.h, layer, which, ctypes.byref(n))
        return np.ctypeslib.as_array(p, shape=(n.value,))

    def refresh(self):
        lib().orc_model_refresh(self.h)

    def set_head(self, emb_type, raw):
        """Untied LM head (GGUF Q4_0 / Q8_0 bytes of output.weight)."""
        raw = np.ascontiguousarray(raw, np.uint8)
        if lib().orc_model_set_head(self.h, emb_type, raw.ctypes.data) != 0:
            raise ValueError("orc_model_set_head: unsupported type")

    def forward(self, tokens, start_pos):
        toks = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.cfg.vocab, np.float32)
        rc = lib().orc_forward(self.h, toks, toks.size, start_pos, logits)
        if rc != 0:
            raise ValueError(f"orc_forward failed ({rc})")
        return logits

    def forward_ex(self, tokens, start_pos, max_layers=0, exit_threshold=0.0, exit_interval=4):
        """forward(tokens, startPos, {maxLayers}) with the early exit; returns (logits, layersUsed)."""
        toks = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.cfg.vocab, np.float32)
        used = ctypes.c_int()
        rc = lib().orc_forward_ex(self.h, toks.ctypes.data, toks.size, start_pos, max_layers, exit_threshold,
                                  exit_interval, logits.ctypes.data, ctypes.byref(used))
        if rc != 0:
            raise ValueError(f"orc_forward_ex failed ({rc})")
        return logits, used.value

    def generate(self, prompt, max_tokens, eos_id=2):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(p.size + max_tokens + 1, np.int32)
        n = lib().orc_generate(self.h, p, p.size, max_tokens, eos_id, out, out.size)
        if n < 0:
            raise ValueError("orc_generate failed")
        return out[:n].tolist()

    def reset_cache(self):
        lib().orc_reset_cache(self.h)

    def rollback_cache(self, pos):
        lib().orc_rollback_cache(self.h, pos)

    def kv(self, layer, which_v):
        p = lib().orc_kv(self.h, layer, which_v)
        kvd = self.cfg.n_kv_heads * self.cfg.head_dim
        return np.ctypeslib.as_array(p, shape=(self.cfg.seq_len, kvd))
