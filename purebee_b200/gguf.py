"""GGUF model files: the reference's gguf.js parser and streaming-loader.js
header pass, over the library's host-side parser (pb_gguf_* in the C ABI).

`GGUFFile(path)` parses the header, metadata and tensor index once
(gguf.js:76-194 GGUFParser; streaming-loader.js:35-87 parseHeader) and reads
tensor bytes on demand (streaming-loader.js:245-262 loadTensorRaw).
`parseHeader(path)` returns the reference's dictionary shape.  Model loading
(`StreamingLlamaRuntime.fromGGUF`) sends every tensor once into the packed
device layout instead of re-reading and dequantizing per call.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional

import numpy as np

from . import _native as N

# GGUF metadata value types (gguf.js:24-27) and ggml tensor types (:30-33)
GGUF_TYPE = dict(UINT8=0, INT8=1, UINT16=2, INT16=3, UINT32=4, INT32=5, FLOAT32=6, BOOL=7, STRING=8, ARRAY=9,
                 UINT64=10, INT64=11, FLOAT64=12)
GGML_TYPE = dict(F32=0, F16=1, Q4_0=2, Q4_1=3, Q5_0=6, Q5_1=7, Q8_0=8, Q8_1=9, Q2_K=10, Q3_K=11, Q4_K=12, Q5_K=13,
                 Q6_K=14, Q8_K=15)
_INT_TYPES = {0, 1, 2, 3, 4, 5, 10, 11}
_FLOAT_TYPES = {6, 12}


class GGUFError(ValueError):
    """A malformed or unsupported file (the reference throws Error with a message)."""


def _err(rc: int) -> None:
    if rc != N.PB_OK:
        raise GGUFError(N.lib().pb_gguf_last_error().decode(errors="replace"))


def mapTensorName(ggufName: str) -> Dict[str, object]:
    """gguf.js:376-404: GGUF tensor name -> PureBee name (and whether the
    reference transposes it for its own matmul convention)."""
    if ggufName == "token_embd.weight":
        return {"name": "token_embedding", "transpose": False}
    if ggufName == "output.weight":
        return {"name": "lm_head", "transpose": False}
    if ggufName == "output_norm.weight":
        return {"name": "rms_final", "transpose": False}
    if ggufName.startswith("blk."):
        parts = ggufName.split(".", 2)
        if len(parts) == 3 and parts[1].isdigit():
            prefix = f"layer{parts[1]}"
            table = {"attn_norm.weight": ("rms_att", False), "ffn_norm.weight": ("rms_ffn", False),
                     "attn_q.weight": ("wq", True), "attn_k.weight": ("wk", True), "attn_v.weight": ("wv", True),
                     "attn_output.weight": ("wo", True), "ffn_gate.weight": ("w1", True),
                     "ffn_down.weight": ("w2", True), "ffn_up.weight": ("w3", True)}
            if parts[2] in table:
                name, tr = table[parts[2]]
                return {"name": f"{prefix}.{name}", "transpose": tr}
    return {"name": ggufName, "transpose": False}


class GGUFFile:
    """One parsed GGUF v2/v3 file."""

    def __init__(self, path: str):
        self.path = path
        h = ctypes.c_void_p()
        _err(N.lib().pb_gguf_open(str(path).encode(), ctypes.byref(h)))
        self.h = h.value
        L = N.lib()
        self.version = L.pb_gguf_version(self.h)
        self.alignment = L.pb_gguf_alignment(self.h)
        self.dataStart = L.pb_gguf_data_start(self.h)
        self._meta: Optional[Dict[str, object]] = None
        self._infos: Optional[List[dict]] = None

    # -- metadata (gguf.js:159-167 readMetadata) ------------------------
    def _value(self, i: int):
        L = N.lib()
        t, at, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
        _err(L.pb_gguf_meta_type(self.h, i, ctypes.byref(t), ctypes.byref(at), ctypes.byref(n)))
        t = t.value
        if t == GGUF_TYPE["STRING"]:
            p, ln = ctypes.c_void_p(), ctypes.c_int64()
            _err(L.pb_gguf_meta_string(self.h, i, ctypes.byref(p), ctypes.byref(ln)))
            return ctypes.string_at(p, ln.value).decode("utf-8", errors="replace")
        if t == GGUF_TYPE["ARRAY"]:
            out = []
            if at.value == GGUF_TYPE["STRING"]:
                p, ln = ctypes.c_void_p(), ctypes.c_int64()
                for j in range(n.value):
                    _err(L.pb_gguf_meta_array_string(self.h, i, j, ctypes.byref(p), ctypes.byref(ln)))
                    out.append(ctypes.string_at(p, ln.value).decode("utf-8", errors="replace"))
            else:
                d = ctypes.c_double()
                for j in range(n.value):
                    _err(L.pb_gguf_meta_array_number(self.h, i, j, ctypes.byref(d)))
                    v = d.value
                    out.append(int(v) if at.value in _INT_TYPES else bool(v) if at.value == 7 else v)
            return out
        if t in _FLOAT_TYPES:
            d = ctypes.c_double()
            _err(L.pb_gguf_meta_float(self.h, i, ctypes.byref(d)))
            return d.value
        v = ctypes.c_int64()
        _err(L.pb_gguf_meta_int(self.h, i, ctypes.byref(v)))
        return bool(v.value) if t == GGUF_TYPE["BOOL"] else v.value

    @property
    def metadata(self) -> Dict[str, object]:
        if self._meta is None:
            L = N.lib()
            meta = {}
            for i in range(L.pb_gguf_meta_count(self.h)):
                k = ctypes.c_char_p()
                _err(L.pb_gguf_meta_key(self.h, i, ctypes.byref(k)))
                meta[k.value.decode("utf-8", errors="replace")] = self._value(i)
            self._meta = meta
        return self._meta

    # -- tensor index (gguf.js:169-183 readTensorInfos) ------------------
    @property
    def tensorInfos(self) -> List[dict]:
        if self._infos is None:
            L = N.lib()
            infos = []
            dims = (ctypes.c_int64 * 4)()
            for i in range(L.pb_gguf_tensor_count(self.h)):
                name, t, nd, off, nb = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
                _err(L.pb_gguf_tensor_info(self.h, i, ctypes.byref(name), ctypes.byref(t), ctypes.byref(nd), dims,
                                           ctypes.byref(off), ctypes.byref(nb)))
                infos.append({"name": name.value.decode("utf-8", errors="replace"), "dims": [dims[d] for d in range(nd.value)],
                              "type": t.value, "offset": off.value, "byteSize": nb.value})
            self._infos = infos
        return self._infos

    def readTensorRaw(self, name: str) -> np.ndarray:
        """streaming-loader.js:245-262: a tensor's raw bytes."""
        L = N.lib()
        i = L.pb_gguf_tensor_find(self.h, name.encode())
        if i < 0:
            raise GGUFError(f"StreamingLoader: tensor '{name}' not found in index")
        out = np.empty(self.tensorInfos[i]["byteSize"], np.uint8)
        _err(L.pb_gguf_tensor_read(self.h, i, out.ctypes.data, out.nbytes))
        return out

    # -- config (gguf.js:402-424 extractConfig) ---------------------------
    def modelConfig(self) -> N.ModelConfig:
        c = N.ModelConfig()
        _err(N.lib().pb_gguf_config(self.h, ctypes.byref(c)))
        return c

    def config(self):
        from .runtime import LlamaConfig
        c = self.modelConfig()
        m = self.metadata
        arch = m.get("general.architecture", "llama") or "llama"
        return LlamaConfig(dim=c.dim, hiddenDim=c.hidden_dim, nLayers=c.n_layers, nHeads=c.n_heads,
                           nKvHeads=c.n_kv_heads, vocabSize=c.vocab, seqLen=c.seq_len, headDim=c.head_dim,
                           ropeTheta=c.rope_theta, rmsNormEps=c.eps), {"arch": arch,
                                                                      "name": m.get("general.name", "unknown"),
                                                                      "embType": c.emb_type}

    def tokenizer(self):
        """gguf.js:486-548 GGUFTokenizer from this file's metadata."""
        from .tokenizer import GGUFTokenizer
        return GGUFTokenizer(self.metadata)

    def close(self):
        if self.h:
            N.lib().pb_gguf_close(self.h)
        self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def parseHeader(path: str) -> dict:
    """streaming-loader.js:35-87: config, tensor index (PureBee names ->
    absolute offset, type, dims, byteSize, transpose, ggufName), dataStart,
    alignment, sharedWeights, plus the metadata."""
    with GGUFFile(path) as f:
        cfg, extra = f.config()
        index = {}
        shared = True
        for info in f.tensorInfos:
            mapped = mapTensorName(info["name"])
            if info["name"] == "output.weight":
                shared = False
            index[mapped["name"]] = {"offset": info["offset"], "type": info["type"], "dims": info["dims"],
                                     "byteSize": info["byteSize"], "transpose": mapped["transpose"],
                                     "ggufName": info["name"]}
        return {"config": cfg, "arch": extra["arch"], "tensorIndex": index, "dataStart": f.dataStart,
                "alignment": f.alignment, "sharedWeights": shared, "metadata": f.metadata}
