"""forward(..., {maxLayers}), the early exit and self-speculative decoding
(speculative.js) on the device against the oracle: layer-limited logits,
the same exits, speculative greedy output equal to plain greedy output, and
speculative sampling equal to the reference algorithm replayed over the
oracle with the same draws."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
RTOL = 1e-5
KW = dict(kind=0, emb_type=2, dim=128, hidden_dim=256, n_layers=4, n_heads=4, n_kv_heads=2, head_dim=32, vocab=512,
          seq_len=200, rope_theta=10000.0, eps=1e-5)


def pair(native, ctx, oracle, seed, options=None):
    from purebee_b200.runtime import LlamaConfig, StreamingLlamaRuntime
    cfg = LlamaConfig(dim=128, hiddenDim=256, nLayers=4, nHeads=4, nKvHeads=2, vocabSize=512, seqLen=200, headDim=32)
    rt = StreamingLlamaRuntime(cfg, options, ctx=ctx, emb_type=native.TYPE_Q4_0)
    rt.loadSynthetic(seed, 0.05)
    om = oracle.Model(oracle.Config(**KW))
    om.init_synthetic(seed, 0.05)
    return rt, om


def close(a, b):
    return np.max(np.abs(np.asarray(a, np.float64) - b)) <= RTOL * np.max(np.abs(b))


@pytest.mark.parametrize("max_layers", [1, 2, 3])
def test_max_layers_matches_oracle(native, ctx, oracle, max_layers):
    rt, om = pair(native, ctx, oracle, 31)
    prompt = oracle.synth_tokens(7, 2, 1, 512).tolist()
    out = rt.forward(prompt, 0, {"maxLayers": max_layers})
    want, used = om.forward_ex(prompt, 0, max_layers)
    assert out["layersUsed"] == used == max_layers and close(out["logits"], want)
    for i, t in enumerate([11, 12, 13]):  # decode steps through the layer-limited graph
        out = rt.forward([t], len(prompt) + i, {"maxLayers": max_layers})
        want, used = om.forward_ex([t], len(prompt) + i, max_layers)
        assert out["layersUsed"] == used and close(out["logits"], want)
    rt.shutdown()


@pytest.mark.parametrize("threshold,interval,expect_used", [(1e-9, 1, 1), (1e-9, 2, 2), (0.999, 1, 4)])
def test_early_exit_matches_oracle(native, ctx, oracle, threshold, interval, expect_used):
    rt, om = pair(native, ctx, oracle, 32, {"earlyExitThreshold": threshold, "earlyExitInterval": interval})
    prompt = oracle.synth_tokens(6, 3, 1, 512).tolist()
    rt.forward(prompt, 0)  # prefill: no early exit for more than one token
    om.forward(prompt, 0)
    for i, t in enumerate([21, 22]):
        out = rt.forward([t], len(prompt) + i)
        want, used = om.forward_ex([t], len(prompt) + i, 0, threshold, interval)
        assert out["layersUsed"] == used == expect_used and close(out["logits"], want)
    st = rt.stats
    assert st["earlyExits"] == (2 if expect_used < 4 else 0)
    assert st["lastExitLayer"] == expect_used - 1
    rt.shutdown()


def test_speculative_greedy_equals_greedy(native, ctx, oracle):
    from purebee_b200.speculative import SelfSpeculativeDecoder
    rt, om = pair(native, ctx, oracle, 33)
    prompt = oracle.synth_tokens(8, 4, 1, 512).tolist()
    want = rt.generate(prompt, 40, {"greedy": True, "eosId": -1})["tokens"]
    sd = SelfSpeculativeDecoder(rt, {"draftLayers": 2, "draftCount": 4})
    got = sd.generate(prompt, 40, {"greedy": True, "eosIds": [-1]})
    assert got["tokens"] == want
    st = sd.stats
    assert st["totalRounds"] > 0 and 0 <= st["totalAccepted"] <= st["totalDrafted"]
    rt.shutdown()


def _reference_speculative(oracle, om, prompt, max_tokens, draft_layers, draft_count, top_k, temp, seed):
    """speculative.js:58-189 over the oracle, draw i = sample_uniform(seed, i)."""
    draws = [0]

    def samp(lg):
        t = oracle.sample(lg, top_k, temp, oracle.sample_uniform(seed, draws[0]))
        draws[0] += 1
        return t

    om.reset_cache()
    toks = list(prompt)
    nxt = samp(om.forward(prompt, 0))
    toks.append(nxt)
    pos, gen = len(prompt), 1
    while gen < max_tokens:
        drafts, dpos, d = [nxt], pos, 0
        while d < draft_count and gen + d < max_tokens:
            lg, _ = om.forward_ex([drafts[-1]], dpos, draft_layers)
            dpos += 1
            drafts.append(samp(lg))
            d += 1
        n = len(drafts) - 1
        om.rollback_cache(pos)
        acc = 0
        for d in range(n):
            v = samp(om.forward([drafts[d]], pos + d))
            if v == drafts[d + 1]:
                acc += 1
                toks.append(v)
                gen += 1
            else:
                toks.append(v)
                gen += 1
                om.rollback_cache(pos + d + 2)
                break
        if acc == n:
            b = samp(om.forward([drafts[-1]], pos + n))
            toks.append(b)
            gen += 1
            pos += n + 1
            nxt = b
        else:
            pos += acc + 1
            nxt = toks[-1]
    return toks


def test_speculative_sampling_follows_reference(native, ctx, oracle):
    from purebee_b200.speculative import SelfSpeculativeDecoder
    rt, om = pair(native, ctx, oracle, 34)
    prompt = oracle.synth_tokens(8, 5, 1, 512).tolist()
    sd = SelfSpeculativeDecoder(rt, {"draftLayers": 2, "draftCount": 3})
    got = sd.generate(prompt, 30, {"temperature": 0.9, "topK": 20, "seed": 4242, "eosIds": [-1]})["tokens"]
    want = _reference_speculative(oracle, om, prompt, 30, 2, 3, 20, 0.9, 4242)
    assert got == want
    rt.shutdown()
