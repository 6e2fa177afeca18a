"""Generate tests/golden/golden.npz from the CPU oracle (oracle/pb_oracle.c).

The reference (JavaScript) cannot run in this image, so its arithmetic is
pinned two ways: the reference's own known-answer tests (replayed in
tests/test_oracle_kat.py) and these seeded vectors, which freeze the oracle's
outputs on small cases that exercise ragged shapes, scalar tails, zero and
subnormal scales and the quantize.js tie rule.  The GPU parity tests compare
the CUDA kernels against the same vectors.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

OUT = os.path.join(HERE, "golden.npz")

TINY_STREAMING = dict(kind=O.KIND_STREAMING_Q4, emb_type=O.EMB_Q4_0, dim=64, hidden_dim=128, n_layers=2, n_heads=4,
                      n_kv_heads=2, head_dim=16, vocab=96, seq_len=32, rope_theta=10000.0, eps=1e-5)
TINY_STREAMING_Q8E = dict(TINY_STREAMING, emb_type=O.EMB_Q8_0, vocab=128)
TINY_LLAMA_Q8A = dict(kind=O.KIND_LLAMA_Q8A, emb_type=O.EMB_F32, dim=64, hidden_dim=96, n_layers=2, n_heads=4,
                      n_kv_heads=4, head_dim=16, vocab=80, seq_len=32, rope_theta=10000.0, eps=1e-5)


def gguf_q4_0_raw(rng, N, K, special=True):
    """Random GGUF Q4_0 rows; a few blocks get zero / subnormal / large scales."""
    nb = K // 32
    raw = rng.integers(0, 256, size=(N, nb, 18), dtype=np.uint8)
    d = (rng.standard_normal((N, nb)) * 0.01).astype(np.float16)
    raw[:, :, 0:2] = d.view(np.uint8).reshape(N, nb, 2)
    if special and N * nb >= 4:
        flat = raw.reshape(-1, 18)
        flat[0, 0:2] = np.array([0, 0], np.uint8)              # d = +0
        flat[1, 0:2] = np.array([0x01, 0x00], np.uint8)        # subnormal (WASM decode -> 0)
        flat[2, 0:2] = np.array([0x00, 0x80], np.uint8)        # d = -0
        flat[3, 0:2] = np.array([0xff, 0x7b], np.uint8)        # 65504
    return raw.reshape(-1)


def gguf_q4_1_raw(rng, N, K):
    nb = K // 32
    raw = rng.integers(0, 256, size=(N, nb, 20), dtype=np.uint8)
    d = (rng.random((N, nb)) * 0.01).astype(np.float16)
    m = (rng.standard_normal((N, nb)) * 0.01).astype(np.float16)
    raw[:, :, 0:2] = d.view(np.uint8).reshape(N, nb, 2)
    raw[:, :, 2:4] = m.view(np.uint8).reshape(N, nb, 2)
    return raw.reshape(-1)


def model_case(cfg_kw, seed, n_prompt, n_steps):
    cfg = O.Config(**cfg_kw)
    m = O.Model(cfg)
    m.init_synthetic(seed, 0.02)
    prompt = O.synth_tokens(n_prompt, seed, 1, cfg.vocab)
    toks = m.generate(prompt, n_steps, eos_id=-1)
    # teacher-forced logits of the final step
    m.reset_cache()
    m.forward(prompt, 0)
    logits = None
    for i, t in enumerate(toks[n_prompt:-1]):
        logits = m.forward([t], n_prompt + i)
    return np.array(prompt, np.int32), np.array(toks, np.int32), logits


def main():
    rng = np.random.default_rng(20261201)
    g = {}
    # --- Q4_0 / Q4_1 matvec (wasm-q4.js order) -----------------------------
    for tag, (N, K) in {"a": (7, 64), "b": (33, 96), "c": (64, 256)}.items():
        x = rng.standard_normal(K).astype(np.float32)
        raw = gguf_q4_0_raw(rng, N, K)
        g[f"q4_0_{tag}_x"], g[f"q4_0_{tag}_raw"] = x, raw
        g[f"q4_0_{tag}_y"] = O.q4_0_matvec(x, raw, N, K)
        g[f"q4_0_{tag}_shape"] = np.array([N, K], np.int32)
    N, K = 9, 64
    x = rng.standard_normal(K).astype(np.float32)
    raw = gguf_q4_1_raw(rng, N, K)
    g["q4_1_x"], g["q4_1_raw"], g["q4_1_y"] = x, raw, O.q4_1_matvec(x, raw, N, K)
    g["q4_1_shape"] = np.array([N, K], np.int32)
    # --- batch_dot with a scalar tail (K % 4 == 2) --------------------------
    N, K = 37, 70
    x = rng.standard_normal(K).astype(np.float32)
    W = rng.standard_normal((N, K)).astype(np.float32)
    g["bd_x"], g["bd_W"], g["bd_y"] = x, W, O.batch_dot(x, W, N, K)
    # --- f32 WASM matmul with bias ------------------------------------------
    M, K, N = 3, 5, 7
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    g["mm_A"], g["mm_B"], g["mm_bias"] = A, B, bias
    g["mm_C"] = O.matmul_wasm(A, M, K, B, N, bias)
    # --- quantize.js format (a), including exact .5 ties --------------------
    data = (rng.standard_normal(100) * 0.05).astype(np.float32)
    # block 0: max 127 -> Q8 inv = 1, exact .5 ties (Math.round(-2.5) = -2, not -3)
    data[0:32] = np.array([127.0, -2.5, 2.5, -0.5, 0.5, -1.5, 1.5, -126.5] + [3.25] * 24, np.float32)
    # block 1: max 7 -> Q4 inv = 1, exact ties and clamping at -8
    data[32:64] = np.array([7.0, -7.0, -2.5, 2.5, -0.5, 0.5, 6.5, -6.5] + [1.0] * 24, np.float32)
    data[64:96] = 0.0                                   # scale 0 block
    s8, q8 = O.quantize_q8a(data)
    s4, q4 = O.quantize_q4a(data)
    g["qa_data"], g["q8a_scales"], g["q8a_q"], g["q4a_scales"], g["q4a_q"] = data, s8, q8, s4, q4
    g["q8a_deq"] = O.dequantize_q8a(s8, q8, data.size)
    g["q4a_deq"] = O.dequantize_q4a(s4, q4, data.size)
    # --- matmul_q8 with N % 32 != 0 (block straddles rows) and zero acts ----
    M, K, N = 2, 40, 40
    a = rng.standard_normal((M, K)).astype(np.float32)
    a[0, 3] = 0.0
    w = (rng.standard_normal(K * N) * 0.05).astype(np.float32)
    ws, wq = O.quantize_q8a(w)
    g["mq_a"], g["mq_scales"], g["mq_q"] = a, ws, wq
    g["mq_out"] = O.matmul_q8(a, M, K, ws, wq, N)
    # --- GGUF encoders -------------------------------------------------------
    x = (rng.standard_normal(256) * 0.02).astype(np.float32)
    x[32:64] = 0.0
    g["gg_x"], g["gg_q4_0"], g["gg_q8_0"] = x, O.quantize_gguf_q4_0(x), O.quantize_gguf_q8_0(x)
    # --- engine ops ----------------------------------------------------------
    x = rng.standard_normal((3, 48)).astype(np.float32)
    w = rng.standard_normal(48).astype(np.float32)
    b = rng.standard_normal(48).astype(np.float32)
    g["op_x"], g["op_w"], g["op_b"] = x, w, b
    g["op_rmsnorm"] = O.rmsnorm(x, 3, 48, w)
    g["op_softmax"] = O.softmax(x, 3, 48)
    g["op_layernorm"] = O.layernorm(x, 3, 48, w, b)
    g["op_gelu"] = O.gelu(x)
    g["op_silu"] = O.silu(x)
    # --- RoPE + cached attention --------------------------------------------
    seq, start, nh, nkv, hd = 3, 5, 4, 2, 16
    q = rng.standard_normal(seq * nh * hd).astype(np.float32)
    k = rng.standard_normal(seq * nkv * hd).astype(np.float32)
    qr, kr = O.rope(q, k, seq, start, nh * hd, nh, nkv, hd, 500000.0)
    g["rope_q"], g["rope_k"], g["rope_qr"], g["rope_kr"] = q, k, qr, kr
    cache_len = start + seq
    kc = rng.standard_normal((cache_len, nkv * hd)).astype(np.float32)
    vc = rng.standard_normal((cache_len, nkv * hd)).astype(np.float32)
    g["att_q"], g["att_kc"], g["att_vc"] = qr, kc, vc
    g["att_out"] = O.attn_cached(qr, kc, vc, seq, start, nh * hd, nh, nkv, hd)
    # --- whole tiny models ---------------------------------------------------
    for tag, kw in {"ms": TINY_STREAMING, "mq8e": TINY_STREAMING_Q8E, "ml": TINY_LLAMA_Q8A}.items():
        p, t, lg = model_case(kw, 7, 5, 10)
        g[f"{tag}_prompt"], g[f"{tag}_tokens"], g[f"{tag}_logits"] = p, t, lg
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(g)} arrays)")


if __name__ == "__main__":
    main()
