"""The Llama runtimes of the reference, backed by the device model (pb_model).

StreamingLlamaRuntime mirrors llama-streaming.js:182-1002 (GGUF Q4_0 layer
weights, raw Q4 matvecs for decode, dequantized f32 matmuls for prefill, the
batch_dot LM head).  LlamaRuntime mirrors llama.js:36-511 (quantize.js Q8
layer weights through matmul_q8, double-precision head over the f32
embedding).  Weights live on the device for the whole session (the
reference's raw SharedArrayBuffer cache, streaming-loader.js:119-162); the
decode step is one replayed CUDA graph.
"""
from __future__ import annotations

import ctypes
import os
import time
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import _native as N


@dataclass
class LlamaConfig:
    """llama.js:22-34 LlamaConfig (plus the GGUF fields of gguf.js:429-450)."""
    dim: int
    hiddenDim: int
    nLayers: int
    nHeads: int
    nKvHeads: int
    vocabSize: int
    seqLen: int
    headDim: int = 0
    ropeTheta: float = 10000.0
    rmsNormEps: float = 1e-5

    def __post_init__(self):
        if not self.headDim:
            self.headDim = self.dim // self.nHeads  # llama.js:31


class _DeviceModel:
    def __init__(self, ctx: N.Context, cfg: LlamaConfig, kind: int, emb_type: int, handle: Optional[int] = None,
                 head_type: Optional[int] = None):
        self.ctx = ctx
        self.cfg = cfg
        self.kind = kind
        self.emb_type = emb_type
        self.head_type = head_type  # untied LM head table type, None when tied
        if handle is None:
            c = N.ModelConfig(kind, emb_type, cfg.dim, cfg.hiddenDim, cfg.nLayers, cfg.nHeads, cfg.nKvHeads,
                              cfg.headDim, cfg.vocabSize, cfg.seqLen, float(cfg.ropeTheta), float(cfg.rmsNormEps))
            h = ctypes.c_void_p()
            ctx._check(N.lib().pb_model_create(ctx.h, ctypes.byref(c), ctypes.byref(h)))
            handle = h.value
        self.h = handle

    def free(self):
        # a model lives inside its context: once the context is closed the
        # device memory is gone with it and the handle must not be touched
        if self.h and self.ctx.h:
            N.lib().pb_model_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def init_synthetic(self, seed: int, stdev: float = 0.02):
        self.ctx._check(N.lib().pb_model_init_synthetic(self.h, seed, stdev))

    def tensor_bytes(self, layer: int, which: int) -> int:
        c = self.cfg
        if which == 11:
            if self.head_type is None:
                raise ValueError("the model has no untied head")
            if self.head_type == N.TYPE_F32:
                return c.vocabSize * c.dim * 4
            return c.vocabSize * c.dim // 32 * (18 if self.head_type == N.TYPE_Q4_0 else 34)
        if which >= 8:
            return c.dim * 4
        if which == 0:
            ne = c.vocabSize * c.dim
            if self.kind == N.MODEL_LLAMA_Q8A or self.emb_type == N.TYPE_F32:
                return ne * 4
            return ne // 32 * (18 if self.emb_type == N.TYPE_Q4_0 else 34)
        kv = c.nKvHeads * c.headDim
        rows, cols = {1: (c.dim, c.dim), 2: (kv, c.dim), 3: (kv, c.dim), 4: (c.dim, c.dim),
                      5: (c.hiddenDim, c.dim), 6: (c.dim, c.hiddenDim), 7: (c.hiddenDim, c.dim)}[which]
        n = rows * cols
        if self.kind == N.MODEL_STREAMING_Q4:
            return n // 32 * 18
        nb = (n + 31) // 32
        return nb * 36

    def set_tensor(self, layer: int, which: int, data: np.ndarray):
        a = np.ascontiguousarray(data)
        self.ctx._check(N.lib().pb_model_set_tensor(self.h, layer, which, N.ptr(a), a.nbytes))

    def get_tensor(self, layer: int, which: int) -> np.ndarray:
        out = np.empty(self.tensor_bytes(layer, which), np.uint8)
        self.ctx._check(N.lib().pb_model_get_tensor(self.h, layer, which, N.ptr(out), out.nbytes))
        return out

    def forward_ex(self, tokens, start_pos: int, max_layers: int = 0):
        t = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.cfg.vocabSize, np.float32)
        used = ctypes.c_int()
        self.ctx._check(N.lib().pb_model_forward_ex(self.h, N.ptr(t), t.size, int(start_pos), int(max_layers),
                                                    N.ptr(logits), ctypes.byref(used)))
        return logits, used.value

    def step(self, token: int, pos: int, max_layers: int = 0) -> int:
        """One decode step (graph replay); the greedy next token, no logits copy."""
        nxt = ctypes.c_int()
        self.ctx._check(N.lib().pb_model_decode_ex(self.h, int(token), int(pos), int(max_layers), ctypes.byref(nxt),
                                                   None, None))
        return nxt.value

    def sample_last(self, top_k: int, temperature: float, seed: int, counter: int) -> int:
        tok = ctypes.c_int()
        self.ctx._check(N.lib().pb_model_sample(self.h, int(top_k), float(temperature), seed & (2 ** 64 - 1),
                                                int(counter), ctypes.byref(tok)))
        return tok.value

    def set_early_exit(self, threshold: float, interval: int):
        self.ctx._check(N.lib().pb_model_set_early_exit(self.h, float(threshold), int(interval)))

    def exit_stats(self):
        u, l, e = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        self.ctx._check(N.lib().pb_model_exit_stats(self.h, ctypes.byref(u), ctypes.byref(l), ctypes.byref(e)))
        return u.value, l.value, e.value

    def forward_logits(self, tokens, start_pos: int) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.cfg.vocabSize, np.float32)
        self.ctx._check(N.lib().pb_model_forward(self.h, N.ptr(t), t.size, int(start_pos), N.ptr(logits)))
        return logits

    def decode(self, token: int, pos: int, want_logits: bool = False):
        nxt = ctypes.c_int()
        logits = np.empty(self.cfg.vocabSize, np.float32) if want_logits else None
        self.ctx._check(N.lib().pb_model_decode(self.h, int(token), int(pos), ctypes.byref(nxt),
                                                N.ptr(logits) if logits is not None else None))
        return nxt.value, logits

    def generate_greedy(self, prompt, max_tokens: int, eos_id: int):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(p.size + max_tokens + 1, np.int32)
        n = ctypes.c_int()
        self.ctx._check(N.lib().pb_model_generate(self.h, N.ptr(p), p.size, int(max_tokens), int(eos_id),
                                                  N.ptr(out), out.size, ctypes.byref(n)))
        return out[:n.value].tolist()

    def generate_sampled(self, prompt, max_tokens: int, eos_id: int, top_k: int, temperature: float, seed: int):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(p.size + max_tokens + 1, np.int32)
        n = ctypes.c_int()
        self.ctx._check(N.lib().pb_model_generate_sampled(self.h, N.ptr(p), p.size, int(max_tokens), int(eos_id),
                                                          int(top_k), float(temperature), seed & (2 ** 64 - 1),
                                                          N.ptr(out), out.size, ctypes.byref(n)))
        return out[:n.value].tolist()

    def reset_cache(self):
        self.ctx._check(N.lib().pb_model_reset_cache(self.h))

    def rollback_cache(self, pos: int):
        self.ctx._check(N.lib().pb_model_rollback_cache(self.h, int(pos)))

    def set_rope_scaling(self, factor: float, low_freq_factor: float = 1.0, high_freq_factor: float = 4.0,
                         original_max_pos: int = 8192):
        """Llama-3 RoPE frequency scaling on (factor > 0) or off (factor <= 0,
        the default and the reference's behaviour)."""
        self.ctx._check(N.lib().pb_model_set_rope_scaling(self.h, float(factor), float(low_freq_factor),
                                                          float(high_freq_factor), int(original_max_pos)))

    @property
    def rope_scaling_factor(self) -> float:
        f = ctypes.c_double()
        self.ctx._check(N.lib().pb_model_rope_scaling(self.h, ctypes.byref(f)))
        return f.value

    def kv(self, layer: int, which_v: int) -> np.ndarray:
        c = self.cfg
        kvd = c.nKvHeads * c.headDim
        out = np.empty(c.seqLen * kvd, np.float32)
        self.ctx._check(N.lib().pb_model_kv(self.h, layer, which_v, N.ptr(out), out.size))
        return out.reshape(c.seqLen, kvd)


def argmax(logits) -> int:
    """llama-streaming.js:899-909: first index of the strict maximum."""
    best, idx = -np.inf, 0
    arr = np.asarray(logits, np.float32)
    finite = np.where(np.isnan(arr), -np.inf, arr)
    m = finite.max() if finite.size else -np.inf
    if m > best:
        idx = int(np.argmax(finite == m))
    return idx


def sample(ctx: N.Context, logits, topK: int = 40, temperature: float = 0.8, seed: Optional[int] = None,
           counter: int = 0) -> int:
    """llama-streaming.js:868-894 top-K + temperature sampling, on the device
    (pb_sample_topk).  The reference draws r from the unseeded Math.random;
    here r = pb_sample_uniform(seed, counter), a fresh seed when none is given."""
    arr = np.ascontiguousarray(logits, np.float32)
    if seed is None:
        seed = int.from_bytes(os.urandom(8), "little")
    d = ctx.to_device(arr)
    t = ctx.alloc(16)
    ctx._check(N.lib().pb_sample_topk(ctx.h, d.ptr, arr.size, int(topK), float(temperature), int(seed) & (2 ** 64 - 1),
                                      int(counter), t.ptr))
    tok = int(t.download(np.int32, 1)[0])
    d.free()
    t.free()
    return tok


class _RuntimeBase:
    KIND = N.MODEL_STREAMING_Q4

    def __init__(self, config: LlamaConfig, options: Optional[dict] = None, ctx: Optional[N.Context] = None,
                 emb_type: Optional[int] = None):
        options = options or {}
        self.config = config
        self.ctx = ctx or N.Context(options.get("device", 0))
        if emb_type is None:
            emb_type = N.TYPE_F32 if self.KIND == N.MODEL_LLAMA_Q8A else N.TYPE_Q4_0
        self.model = _DeviceModel(self.ctx, config, self.KIND, emb_type)
        self._loaded = False
        self._layersUsed = 0
        self._totalForwards = 0
        self._applyOptions(options)

    def _applyOptions(self, options: dict):
        """llama-streaming.js:202-203: earlyExitThreshold (0: off), earlyExitInterval (4)."""
        self.model.set_early_exit(options.get("earlyExitThreshold") or 0.0, options.get("earlyExitInterval") or 4)

    # -- weights --------------------------------------------------------
    def loadSynthetic(self, seed: int, stdev: float = 0.02):
        """Random-init weights N(0, stdev) from the seed; norm gains 1."""
        self.model.init_synthetic(seed, stdev)
        self._loaded = True

    def setTensor(self, layer: int, which: int, data: np.ndarray):
        self.model.set_tensor(layer, which, data)
        self._loaded = True

    def getTensor(self, layer: int, which: int) -> np.ndarray:
        return self.model.get_tensor(layer, which)

    # -- inference ------------------------------------------------------
    def forward(self, tokenIds, startPos: int = 0, options: Optional[dict] = None):
        """llama-streaming.js:738-815 forward(tokenIds, startPos, {maxLayers})."""
        if not self._loaded:
            raise RuntimeError("Resident weights not loaded")  # llama-streaming.js:739
        options = options or {}
        logits, used = self.model.forward_ex(tokenIds, startPos, int(options.get("maxLayers") or 0))
        self._layersUsed += used
        self._totalForwards += 1
        return {"logits": logits, "layersUsed": used}

    def step(self, token: int, pos: int, maxLayers: int = 0) -> int:
        """forward([token], pos, {maxLayers}) followed by argmax, both on the
        device: the greedy next token without copying the logits."""
        nxt = self.model.step(token, pos, maxLayers)
        used, _, _ = self.model.exit_stats()
        self._layersUsed += used
        self._totalForwards += 1
        return nxt

    def sampleLast(self, topK: int, temperature: float, seed: int, counter: int) -> int:
        """sample(logits of the last forward, topK, temperature) on the device."""
        return self.model.sample_last(topK, temperature, seed, counter)

    def argmax(self, logits) -> int:
        return argmax(logits)

    def sample(self, logits, topK: int = 40, temperature: float = 0.8) -> int:
        return sample(self.ctx, logits, topK, temperature)

    def generate(self, promptTokens, maxTokens: int = 50, opts: Optional[dict] = None):
        """llama-streaming.js:914-970.  Greedy runs the device loop (argmax on
        the device); sampling reads logits back every step."""
        opts = opts or {}
        eos = opts.get("eosId") or 2
        greedy = opts.get("greedy", False)
        on_token = opts.get("onToken")
        t0 = time.perf_counter()
        if greedy and on_token is None:
            toks = self.model.generate_greedy(promptTokens, maxTokens, eos)
            dt = time.perf_counter() - t0
            generated = len(toks) - len(promptTokens)
            return {"tokens": toks, "generated": generated, "prefillTime": None,
                    "decodeTime": dt * 1000, "tokPerSec": max(generated - 1, 1) / max(dt, 1e-9),
                    "avgLayers": self.config.nLayers, "earlyExits": 0}
        temperature = opts.get("temperature") or 0.8
        topK = opts.get("topK") or 40
        if not greedy and on_token is None and self.KIND == N.MODEL_STREAMING_Q4:
            seed = opts.get("seed")
            if seed is None:
                seed = int.from_bytes(os.urandom(8), "little")
            toks = self.model.generate_sampled(promptTokens, maxTokens, eos, int(topK), float(temperature), int(seed))
            dt = time.perf_counter() - t0
            generated = len(toks) - len(promptTokens)
            return {"tokens": toks, "generated": generated, "prefillTime": None,
                    "decodeTime": dt * 1000, "tokPerSec": max(generated - 1, 1) / max(dt, 1e-9),
                    "avgLayers": self.config.nLayers, "earlyExits": 0}
        self.resetCache()
        allTokens = list(promptTokens)
        out = self.forward(promptTokens, 0)
        prefill = time.perf_counter() - t0
        pos = len(promptTokens)
        nxt = self.argmax(out["logits"]) if greedy else self.sample(out["logits"], topK, temperature)
        allTokens.append(nxt)
        if on_token:
            on_token(nxt, 0)
        d0 = time.perf_counter()
        generated = 1
        for i in range(1, maxTokens):
            if nxt == eos:
                break
            step = self.forward([nxt], pos)
            pos += 1
            nxt = self.argmax(step["logits"]) if greedy else self.sample(step["logits"], topK, temperature)
            allTokens.append(nxt)
            generated += 1
            if on_token:
                on_token(nxt, i, step["layersUsed"])
            if nxt == eos:
                break
        dt = time.perf_counter() - d0
        return {"tokens": allTokens, "generated": generated, "prefillTime": prefill * 1000,
                "decodeTime": dt * 1000, "tokPerSec": max(generated - 1, 1) / max(dt, 1e-9),
                "avgLayers": self.config.nLayers, "earlyExits": 0}

    async def forwardAsync(self, tokenIds, startPos: int = 0, options: Optional[dict] = None):
        """llama-streaming.js:821-823, kept there for API compatibility: forward()."""
        return self.forward(tokenIds, startPos, options)

    async def generateAsync(self, promptTokens, maxTokens: int = 50, opts: Optional[dict] = None):
        """llama-streaming.js:976-978, kept there for API compatibility: generate()."""
        return self.generate(promptTokens, maxTokens, opts)

    async def initThreadPool(self, numWorkers: Optional[int] = None) -> bool:
        """llama-streaming.js:230-244 starts host worker threads for the
        row-split matvecs and resolves false when it cannot start them.  Every
        matvec here runs on the device, so there is no host pool: false, the
        reference's answer without one (the row split over several GPUs is
        purebee_b200.thread_pool's)."""
        return False

    def resetCache(self):
        self.model.reset_cache()

    def rollbackCache(self, pos: int):
        self.model.rollback_cache(pos)

    @property
    def stats(self):
        _, last, exits = self.model.exit_stats()
        return {"totalForwards": self._totalForwards,
                "avgLayers": (self._layersUsed / self._totalForwards) if self._totalForwards else 0,
                "earlyExits": exits, "lastExitLayer": last, "launches": self.ctx.launches}

    def shutdown(self):
        self.model.free()


class StreamingLlamaRuntime(_RuntimeBase):
    """llama-streaming.js StreamingLlamaRuntime over GGUF Q4_0 layer weights and
    a Q4_0 or Q8_0 tied embedding (emb_type), or an f32 one (TYPE_F32: the
    dequantized table of a Q6_K / F16 / F32 token_embd.weight)."""
    KIND = N.MODEL_STREAMING_Q4

    @classmethod
    def fromGGUF(cls, path: str, options: Optional[dict] = None, ctx: Optional[N.Context] = None):
        """A runtime over a GGUF file (streaming-loader.js:35-87 parseHeader,
        :119-162 resident raw weights, llama-streaming.js constructor): every
        tensor goes once into the packed device layout; output.weight, when
        the file has one, becomes an untied head.  options.seqLen overrides
        the file's context length."""
        from .gguf import GGUFFile
        options = options or {}
        ctx = ctx or N.Context(options.get("device", 0))
        seq = int(options.get("seqLen") or 0)
        with GGUFFile(path) as f:
            cfg, extra = f.config()
            if seq:
                cfg.seqLen = seq
            head = next((i for i in f.tensorInfos if i["name"] == "output.weight"), None)
            h = ctypes.c_void_p()
            ctx._check(N.lib().pb_model_load_gguf(ctx.h, f.h, seq, ctypes.byref(h)))
            meta = f.metadata
            tok = f.tokenizer()
        rt = cls.__new__(cls)
        rt.config = cfg
        rt.ctx = ctx
        # Q4_0 / Q8_0 tables stay quantized; any other type is held as a
        # dequantized f32 table (streaming-loader.js:324-335)
        head_type = None if head is None else {2: N.TYPE_Q4_0, 8: N.TYPE_Q8_0}.get(head["type"], N.TYPE_F32)
        rt.model = _DeviceModel(ctx, cfg, cls.KIND, extra["embType"], handle=h.value, head_type=head_type)
        rt._loaded = True
        rt._layersUsed = 0
        rt._totalForwards = 0
        rt._applyOptions(options)
        rt.sharedWeights = head is None
        rt.tokenizer = tok
        rt.bosId = tok.bosId
        rt.eosId = tok.eosId
        return rt


class LlamaRuntime(_RuntimeBase):
    """llama.js LlamaRuntime over quantize.js Q8 layer weights and an f32
    embedding (the `run.js --q8` path)."""
    KIND = N.MODEL_LLAMA_Q8A


class BatchedLlamaRuntime:
    """n_seqs sequences decoded together over one StreamingLlamaRuntime's
    weights (the batched configuration).  The projections and the LM head
    run as tensor-core GEMMs over f16 hi/lo operand pairs, so logits agree
    with the one-sequence runtime within a relative tolerance, not bit for
    bit.

    comm (thread_pool.NcclComm): this process is one rank of a row split
    over comm's GPUs (pb_batch_create_split); every rank calls prefill and
    decode with the same arguments and gets the same tokens and logits.
    group=w: all w ranks of a row split in this process on one device
    (pb_batch_create_group), the split's arithmetic without a second GPU.
    Both give the same bits as the unsplit batch."""

    def __init__(self, base: StreamingLlamaRuntime, n_seqs: int, comm=None, group: int = 0):
        self.base = base
        self.ctx = base.ctx
        self.n_seqs = n_seqs
        self.comm = comm
        h = ctypes.c_void_p()
        if comm is not None:
            self.world = comm.world
            self.ctx._check(N.lib().pb_batch_create_split(base.model.h, n_seqs, comm.h, ctypes.byref(h)))
        elif group:
            self.world = int(group)
            self.ctx._check(N.lib().pb_batch_create_group(base.model.h, n_seqs, self.world, ctypes.byref(h)))
        else:
            self.world = 1
            self.ctx._check(N.lib().pb_batch_create(base.model.h, n_seqs, ctypes.byref(h)))
        self.h = h.value
        self.n_prompt = 0

    def set_precision(self, terms: int) -> None:
        """3 (default): hi/lo f16 operand pairs, three tensor-core products per
        GEMM; 1: each operand rounded to f16 once (faster, about 3e-3)."""
        self.ctx._check(N.lib().pb_batch_set_precision(self.h, int(terms)))

    def prefill(self, prompts, want_logits: bool = False):
        """prompts: [n_seqs][n_prompt] token ids -> next greedy token per sequence."""
        t = np.ascontiguousarray(prompts, np.int32)
        if t.ndim != 2 or t.shape[0] != self.n_seqs:
            raise ValueError(f"prompts must be [{self.n_seqs}][n_prompt]")
        nxt = np.zeros(self.n_seqs, np.int32)
        lg = np.empty((self.n_seqs, self.base.config.vocabSize), np.float32) if want_logits else None
        self.ctx._check(N.lib().pb_batch_prefill(self.h, N.ptr(t), t.shape[1], N.ptr(nxt),
                                                 N.ptr(lg) if lg is not None else None))
        self.n_prompt = t.shape[1]
        return (nxt, lg) if want_logits else nxt

    def decode(self, steps: int = 1, want_logits: bool = False):
        """`steps` greedy steps of every sequence -> tokens [steps][n_seqs]."""
        toks = np.zeros((steps, self.n_seqs), np.int32)
        lg = np.empty((self.n_seqs, self.base.config.vocabSize), np.float32) if want_logits else None
        self.ctx._check(N.lib().pb_batch_decode(self.h, int(steps), N.ptr(toks),
                                                N.ptr(lg) if lg is not None else None))
        return (toks, lg) if want_logits else toks

    def free(self):
        if self.h and self.ctx.h:
            N.lib().pb_batch_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
