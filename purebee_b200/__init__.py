"""purebee_b200 - B200 (sm_100a) backend for PureBee's quantized Llama inference.

The compute path is the CUDA library libpurebee_b200.so (C ABI in
include/purebee_cuda.h); this package is the host side that mirrors the
reference's JavaScript interfaces:

  - wasm_q4: the wasm-q4.js module (q4_0_matvec, q4_1_matvec, lmHead)
  - runtime: StreamingLlamaRuntime (llama-streaming.js), LlamaRuntime (llama.js)
  - purebee: the PureBee instruction set (purebee.js) over device tensors
"""
from . import _native
from ._native import Context, PureBeeError, QMat

__all__ = ["Context", "PureBeeError", "QMat", "_native"]
