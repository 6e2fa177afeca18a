"""The PureBee instruction set (purebee.js:27-211) over device-resident tensors.

`Tensor` and `PureBeeMemory` mirror memory.js:11-155: named, shaped f32
tensors, reallocated when a write changes the size.  The data lives in device
memory; `Tensor.data` reads it back as a numpy float32 array (the reference's
Float32Array).  `QuantizedTensor` mirrors quantize.js:30-65 (format (a): f32
scales per 32-value block plus int8 codes or packed nibbles) and is produced by
the device quantizers.

Every instruction runs a CUDA kernel through the C ABI, reads its inputs by
name and writes its result back under the output name, returning the result
tensor, as the reference does.  PARALLEL_MAP takes a Python callable, which
cannot run on the device: it raises instead of silently running on the CPU.
"""
from __future__ import annotations

import time
from typing import Dict, List, Optional

import numpy as np

from . import _native as N


def _size(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


class Tensor:
    """memory.js:11-81: name, shape, f32 data (on the device)."""

    def __init__(self, ctx: N.Context, name: str, shape, data: Optional[np.ndarray] = None):
        self.ctx = ctx
        self.name = name
        self.shape = [int(s) for s in shape]
        self.size = _size(self.shape)
        self.buf = ctx.alloc(max(self.size * 4, 16))
        if data is not None:
            self.write(data)
        else:
            ctx._check(N.lib().pb_memset(ctx.h, self.buf.ptr, 0, self.size * 4))

    @property
    def ptr(self) -> int:
        return self.buf.ptr

    def write(self, data) -> None:
        a = np.ascontiguousarray(np.asarray(data, np.float32).ravel())
        if a.size > self.size:
            raise ValueError(f"{self.name}: {a.size} values for {self.size} elements")
        self.buf.upload(a)

    @property
    def data(self) -> np.ndarray:
        return self.buf.download(np.float32, self.size)

    def fill(self, value: float) -> "Tensor":
        self.write(np.full(self.size, value, np.float32))
        return self

    @property
    def bytes(self) -> int:
        return self.size * 4

    def __repr__(self):
        return f"Tensor({self.name}, shape={self.shape}, size={self.size}, {self.bytes / 1048576:.2f}MB)"


class QuantizedTensor:
    """quantize.js:30-65 format (a): scales f32[numBlocks], data int8 / packed uint8."""

    def __init__(self, ctx: N.Context, name: str, shape, type_: str = "q8_0"):
        self.ctx = ctx
        self.name = name
        self.shape = [int(s) for s in shape]
        self.type = type_
        self.size = _size(self.shape)
        self.numBlocks = (self.size + 31) // 32
        self.scales = ctx.alloc(self.numBlocks * 4)
        nbytes = self.numBlocks * 32 if type_ == "q8_0" else (self.numBlocks * 32 + 1) // 2
        self.qdata = ctx.alloc(max(nbytes, 16))
        self.qbytes = nbytes

    @property
    def bytes(self) -> int:
        return self.numBlocks * 4 + self.qbytes

    def host(self):
        s = self.scales.download(np.float32, self.numBlocks)
        q = self.qdata.download(np.int8 if self.type == "q8_0" else np.uint8, self.qbytes)
        return s, q


class PureBeeMemory:
    """memory.js:87-155: the name -> tensor registry."""

    def __init__(self, ctx: N.Context):
        self.ctx = ctx
        self._store: Dict[str, object] = {}

    def alloc(self, name, shape) -> Tensor:
        t = Tensor(self.ctx, name, shape)
        self._store[name] = t
        return t

    def write(self, name, shape, data) -> Tensor:
        t = self._store.get(name)
        if not isinstance(t, Tensor) or t.size != _size(shape):
            t = Tensor(self.ctx, name, shape)
            self._store[name] = t
        else:
            t.shape = [int(s) for s in shape]
        if data is not None:
            t.write(data)
        return t

    def read(self, name) -> Tensor:
        t = self._store.get(name)
        if t is None:
            raise KeyError(f"PureBee: tensor '{name}' not found in memory")  # memory.js:126
        return t

    def has(self, name) -> bool:
        return name in self._store

    def free(self, name) -> None:
        self._store.pop(name, None)

    def stats(self):
        total = sum(getattr(t, "bytes", 0) for t in self._store.values())
        return {"tensors": len(self._store), "totalMB": f"{total / 1048576:.1f}", "keys": list(self._store)}


def quantize_q8(ctx: N.Context, name, shape, data) -> QuantizedTensor:
    """quantize.js:79-109 on the device."""
    x = Tensor(ctx, name + "_src", shape, data) if not isinstance(data, Tensor) else data
    qt = QuantizedTensor(ctx, name, shape, "q8_0")
    ctx._check(N.lib().pb_quantize_q8a(ctx.h, x.ptr, qt.size, qt.scales.ptr, qt.qdata.ptr))
    return qt


def quantize_q4(ctx: N.Context, name, shape, data) -> QuantizedTensor:
    """quantize.js:124-161 on the device."""
    x = Tensor(ctx, name + "_src", shape, data) if not isinstance(data, Tensor) else data
    qt = QuantizedTensor(ctx, name, shape, "q4_0")
    ctx._check(N.lib().pb_quantize_q4a(ctx.h, x.ptr, qt.size, qt.scales.ptr, qt.qdata.ptr))
    return qt


def dequantize(qt: QuantizedTensor) -> np.ndarray:
    """quantize.js:170-208 on the device."""
    ctx = qt.ctx
    out = ctx.alloc(qt.size * 4)
    fn = N.lib().pb_dequantize_q8a if qt.type == "q8_0" else N.lib().pb_dequantize_q4a
    ctx._check(fn(ctx.h, qt.scales.ptr, qt.qdata.ptr, qt.size, out.ptr))
    return out.download(np.float32, qt.size)


class PureBee:
    """purebee.js:27-211 instruction set."""

    def __init__(self, options: Optional[dict] = None, ctx: Optional[N.Context] = None):
        options = options or {}
        self.ctx = ctx or N.Context(options.get("device", 0))
        self.mem = PureBeeMemory(self.ctx)
        self._log = options.get("log", False)
        self._opLog: List[dict] = []
        self._ops = 0
        self._flops = 0

    def _emit(self, instruction, details=""):
        if self._log:
            print(f"  [PureBee] {instruction}{' ' + details if details else ''}")
        self._opLog.append({"instruction": instruction, "details": details, "t": time.time()})

    def _out(self, name, shape) -> Tensor:
        return self.mem.write(name, shape, None)

    # -- memory -------------------------------------------------------------
    def GRID_ALLOC(self, name, shape):
        self._emit("GRID_ALLOC", f"{name} {list(shape)}")
        return self.mem.alloc(name, shape)

    def GRID_WRITE(self, name, shape, data):
        self._emit("GRID_WRITE", f"{name} {list(shape)}")
        return self.mem.write(name, shape, data)

    def GRID_READ(self, name):
        self._emit("GRID_READ", name)
        return self.mem.read(name)

    def GRID_WRITE_RAW(self, name, obj):
        self._emit("GRID_WRITE_RAW", name)
        self.mem._store[name] = obj
        return obj

    def FREE(self, name):
        self.mem.free(name)

    def SYNC(self):
        """purebee.js:193-197: wait for all queued device work (bounded)."""
        self._emit("SYNC")
        self.ctx.sync()
        return True

    # -- compute ------------------------------------------------------------
    def TENSOR_MUL(self, aName, bName, outName):
        """engine.js:119-167 -> the WASM matmul order (wasm-simd.js:71-91)."""
        self._emit("TENSOR_MUL", f"{aName} x {bName} -> {outName}")
        A, B = self.mem.read(aName), self.mem.read(bName)
        (M, K), (K2, Nn) = A.shape, B.shape
        if K != K2:
            raise ValueError(f"TENSOR_MUL: dimension mismatch A[{M},{K}] x B[{K2},{Nn}]")
        out = self._out(outName, [M, Nn])
        self.ctx._check(N.lib().pb_matmul_f32(self.ctx.h, A.ptr, M, K, B.ptr, Nn, None, out.ptr))
        self._flops += 2 * M * Nn * K
        return out

    def LINEAR(self, xName, wName, bName, outName):
        """purebee.js:74-88: y = x @ W + b, QuantizedTensor weights go to matmul_q8."""
        self._emit("LINEAR", f"{xName} @ {wName} + {bName} -> {outName}")
        x = self.mem.read(xName)
        W = self.mem._store.get(wName)
        if W is None:
            raise KeyError(f"PureBee: '{wName}' not found in memory")
        b = self.mem.read(bName) if bName else None
        M, K = x.shape if len(x.shape) == 2 else (1, x.shape[0])
        Nn = W.shape[1]
        out = self._out(outName, [M, Nn])
        if isinstance(W, QuantizedTensor):
            if W.type != "q8_0":
                raise ValueError("LINEAR: quantize.js matmul_q8 takes q8_0 weights")
            self.ctx._check(N.lib().pb_matmul_q8a(self.ctx.h, x.ptr, M, K, W.scales.ptr, W.qdata.ptr, Nn,
                                                  b.ptr if b else None, out.ptr))
        else:
            self.ctx._check(N.lib().pb_matmul_f32(self.ctx.h, x.ptr, M, K, W.ptr, Nn, b.ptr if b else None,
                                                  out.ptr))
        self._flops += 2 * M * Nn * K
        return out

    def TENSOR_ADD(self, aName, bName, outName):
        self._emit("TENSOR_ADD", f"{aName} + {bName} -> {outName}")
        A, B = self.mem.read(aName), self.mem.read(bName)
        if A.size != B.size:
            raise ValueError(f"TENSOR_ADD: size mismatch {A.size} vs {B.size}")  # engine.js:97
        out = self._out(outName, A.shape)
        self.ctx._check(N.lib().pb_tensoradd(self.ctx.h, A.ptr, B.ptr, A.size, out.ptr))
        return out

    def ELEMENT_MUL(self, aName, bName, outName):
        self._emit("ELEMENT_MUL", f"{aName} * {bName} -> {outName}")
        A, B = self.mem.read(aName), self.mem.read(bName)
        if A.size != B.size:
            raise ValueError(f"ELEMENT_MUL: size mismatch {A.size} vs {B.size}")
        out = self._out(outName, A.shape)
        self.ctx._check(N.lib().pb_elementmul(self.ctx.h, A.ptr, B.ptr, A.size, out.ptr))
        return out

    def SOFTMAX(self, inputName, outName):
        """engine.js:279-303: rows = shape[0], cols = shape[1] (or the size for 1-D)."""
        self._emit("SOFTMAX", f"{inputName} -> {outName}")
        t = self.mem.read(inputName)
        cols = t.shape[1] if len(t.shape) > 1 else t.size
        rows = t.shape[0] if len(t.shape) > 1 else 1
        out = self._out(outName, t.shape)
        self.ctx._check(N.lib().pb_softmax(self.ctx.h, t.ptr, rows, cols, out.ptr))
        return out

    def RMS_NORM(self, xName, weightName, outName, eps=1e-5):
        self._emit("RMS_NORM", f"{xName} -> {outName}")
        x, w = self.mem.read(xName), self.mem.read(weightName)
        seq, dim = (x.shape if len(x.shape) == 2 else (1, x.shape[0]))
        out = self._out(outName, x.shape)
        self.ctx._check(N.lib().pb_rmsnorm(self.ctx.h, x.ptr, seq, dim, w.ptr, float(eps), out.ptr))
        return out

    def LAYER_NORM(self, xName, weightName, biasName, outName, eps=1e-5):
        self._emit("LAYER_NORM", f"{xName} -> {outName}")
        x, w = self.mem.read(xName), self.mem.read(weightName)
        b = self.mem.read(biasName) if biasName else None
        seq, dim = (x.shape if len(x.shape) == 2 else (1, x.shape[0]))
        out = self._out(outName, x.shape)
        self.ctx._check(N.lib().pb_layernorm(self.ctx.h, x.ptr, seq, dim, w.ptr, b.ptr if b else None, float(eps),
                                             out.ptr))
        return out

    def GELU(self, inputName, outName):
        self._emit("GELU", f"{inputName} -> {outName}")
        t = self.mem.read(inputName)
        out = self._out(outName, t.shape)
        self.ctx._check(N.lib().pb_gelu(self.ctx.h, t.ptr, t.size, out.ptr))
        return out

    def SILU(self, inputName, outName):
        self._emit("SILU", f"{inputName} -> {outName}")
        t = self.mem.read(inputName)
        out = self._out(outName, t.shape)
        self.ctx._check(N.lib().pb_silu(self.ctx.h, t.ptr, t.size, out.ptr))
        return out

    def ATTENTION(self, qName, kName, vName, outName, causal=True):
        """engine.js:374-415."""
        self._emit("ATTENTION", f"Q={qName} K={kName} V={vName} -> {outName}")
        Q, K, Vt = self.mem.read(qName), self.mem.read(kName), self.mem.read(vName)
        seqQ, dK = Q.shape
        seqK = K.shape[0]
        dV = Vt.shape[1]
        out = self._out(outName, [seqQ, dV])
        self.ctx._check(N.lib().pb_attention(self.ctx.h, Q.ptr, K.ptr, Vt.ptr, seqQ, seqK, dK, dV, int(bool(causal)),
                                             out.ptr))
        return out

    def PARALLEL_MAP(self, inputName, fn, outName):
        raise NotImplementedError("PARALLEL_MAP takes a host callable; the device backend has no JS/Python "
                                  "interpreter, and it does not fall back to the CPU")

    def stats(self):
        return {"memory": self.mem.stats(), "engine": {"ops": len(self._opLog), "flops": self._flops},
                "ops": len(self._opLog), "launches": self.ctx.launches}
