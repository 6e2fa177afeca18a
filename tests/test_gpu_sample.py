"""Device top-K sampling (pb_sample_topk, pb_model_generate_sampled) against
the oracle's restatement of llama-streaming.js:868-894 with the same uniform
draws: identical tokens, the sampled frequencies follow the softmax, and
sampled generation follows the oracle step by step."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _draw(native, ctx, logits, K, T, seed, counters):
    L = native.lib()
    d = ctx.to_device(np.ascontiguousarray(logits, np.float32))
    t = ctx.alloc(16 * len(counters))
    for j, c in enumerate(counters):
        ctx._check(L.pb_sample_topk(ctx.h, d.ptr, len(logits), K, T, seed, c, t.ptr + 4 * j))
    out = t.download(np.int32, len(counters))
    return out.tolist()


@pytest.mark.parametrize("V,K,T", [(7, 3, 0.8), (2048, 40, 0.8), (2049, 256, 1.0), (32000, 40, 2.5),
                                   (128256, 40, 0.8), (128256, 1, 1.0), (5000, 100, 0.1)])
def test_device_sample_equals_oracle(native, ctx, oracle, V, K, T):
    rng = np.random.default_rng(V + K)
    # coarse values make ties; a few -inf; the top is sharp enough to matter
    lg = (np.round(rng.standard_normal(V) * 4) / 2).astype(np.float32)
    lg[rng.integers(0, V, max(1, V // 100))] = -np.inf
    seed = 1234 + V
    counters = list(range(24))
    got = _draw(native, ctx, lg, K, T, seed, counters)
    want = [oracle.sample(lg, K, T, oracle.sample_uniform(seed, c)) for c in counters]
    assert got == want


def test_device_sample_nan_and_small_vocab(native, ctx, oracle):
    lg = np.array([1.0, np.nan, 3.0, np.nan, 2.0], np.float32)
    got = _draw(native, ctx, lg, 10, 1.0, 9, list(range(40)))
    want = [oracle.sample(lg, 10, 1.0, oracle.sample_uniform(9, c)) for c in range(40)]
    assert got == want and 1 not in got and 3 not in got
    L = native.lib()
    d, t = ctx.to_device(lg), ctx.alloc(16)
    for K, T in ((0, 1.0), (257, 1.0), (5, 0.0), (5, -1.0)):
        assert L.pb_sample_topk(ctx.h, d.ptr, 5, K, T, 1, 0, t.ptr) == native.PB_ERR_ARG


def test_device_sample_frequencies(native, ctx):
    rng = np.random.default_rng(3)
    lg = rng.standard_normal(300).astype(np.float32) * 2
    K, T, n = 12, 0.7, 6000
    got = np.array(_draw(native, ctx, lg, K, T, 77, list(range(n))))
    v = lg.astype(np.float64) / T
    top = np.argsort(-v, kind="stable")[:K]
    p = np.exp(v[top] - v[top[0]])
    p /= p.sum()
    freq = np.array([(got == i).mean() for i in top])
    assert set(got.tolist()) <= set(top.tolist())
    # within 5 standard errors of the softmax probability
    assert np.all(np.abs(freq - p) <= 5 * np.sqrt(p * (1 - p) / n) + 1e-3)


def test_sampled_generation_follows_oracle(native, ctx, oracle):
    from purebee_b200.runtime import LlamaConfig, StreamingLlamaRuntime
    kw = dict(kind=0, emb_type=2, dim=128, hidden_dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=32,
              vocab=512, seq_len=160, rope_theta=10000.0, eps=1e-5)
    cfg = LlamaConfig(dim=128, hiddenDim=256, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=512, seqLen=160, headDim=32)
    rt = StreamingLlamaRuntime(cfg, ctx=ctx, emb_type=native.TYPE_Q4_0)
    rt.loadSynthetic(21, 0.05)
    om = oracle.Model(oracle.Config(**kw))
    om.init_synthetic(21, 0.05)
    prompt = oracle.synth_tokens(9, 4, 1, 512).tolist()
    K, T, seed = 20, 1.3, 555
    out = rt.generate(prompt, 30, {"temperature": T, "topK": K, "seed": seed, "eosId": -1})["tokens"]
    again = rt.generate(prompt, 30, {"temperature": T, "topK": K, "seed": seed, "eosId": -1})["tokens"]
    assert out == again and len(out) == len(prompt) + 30
    # the oracle along the same sequence: draw i uses sample_uniform(seed, i)
    om.reset_cache()
    lg = om.forward(prompt, 0)
    seq = list(prompt)
    for i in range(30):
        tok = oracle.sample(lg, K, T, oracle.sample_uniform(seed, i))
        assert tok == out[len(prompt) + i], f"draw {i}"
        seq.append(tok)
        lg = om.forward([tok], len(seq) - 1)
    rt.shutdown()
