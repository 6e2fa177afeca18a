"""The wasm-q4.js module API (wasm-q4.js:841-847) on the B200.

    init()                          -> bool        (wasm-q4.js:647-668)
    q4_0_matvec(x, rawBuf, N, K)    -> float32[N]  (wasm-q4.js:716-747)
    q4_1_matvec(x, rawBuf, N, K)    -> float32[N]  (wasm-q4.js:758-785)
    lmHead(hidden, embData, V, D)   -> float32[V]  (wasm-q4.js:798-839)
    supported                                     (wasm-q4.js:846)

Inputs are host arrays, as in the reference (which copies them into WASM
memory on every call); results are bit-identical to the reference kernels'
f32 lane order.  Errors raise (the reference throws `WASM Q4 not available`).
"""
from __future__ import annotations

import numpy as np

from . import _native as N

_ctx = None
_supported = False


def context() -> N.Context:
    global _ctx
    if _ctx is None and not init():
        raise RuntimeError("WASM Q4 not available")  # wasm-q4.js:718 wording
    return _ctx


def init(device: int = 0) -> bool:
    """Create the device context; pb_init runs the [32, 128] self-test."""
    global _ctx, _supported
    if _ctx is not None:
        return True
    try:
        _ctx = N.Context(device)
        _supported = True
    except (N.PureBeeError, ImportError, OSError):
        _ctx = None
        _supported = False
    return _supported


def __getattr__(name):
    if name == "supported":
        return _supported
    raise AttributeError(name)


def _call(fn, x, raw, n, k, out_len):
    ctx = context()
    xa = np.ascontiguousarray(x, np.float32)
    ra = np.ascontiguousarray(np.frombuffer(memoryview(raw), np.uint8) if not isinstance(raw, np.ndarray) else raw,
                              np.uint8)
    if xa.size < k:
        raise ValueError(f"x has {xa.size} values, K={k}")
    out = np.empty(out_len, np.float32)
    ctx._check(fn(ctx.h, N.ptr(xa), N.ptr(ra), int(n), int(k), N.ptr(out)))
    return out


def q4_0_matvec(x, rawBuf, N_: int, K: int) -> np.ndarray:
    return _call(N.lib().pb_q4_0_matvec, x, rawBuf, N_, K, N_)


def q4_1_matvec(x, rawBuf, N_: int, K: int) -> np.ndarray:
    return _call(N.lib().pb_q4_1_matvec, x, rawBuf, N_, K, N_)


def lmHead(hidden, embData, vocabSize: int, dim: int) -> np.ndarray:
    ctx = context()
    h = np.ascontiguousarray(hidden, np.float32)
    e = np.ascontiguousarray(embData, np.float32)
    if e.size < vocabSize * dim:
        raise ValueError("embedding smaller than vocabSize * dim")
    out = np.empty(vocabSize, np.float32)
    ctx._check(N.lib().pb_lm_head(ctx.h, N.ptr(h), N.ptr(e), int(vocabSize), int(dim), N.ptr(out)))
    return out
