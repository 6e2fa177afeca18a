"""Batched serving (pb_batch_*): every sequence's prefill and decode logits
match the one-sequence device path (which matches the reference oracle) within
the batched GEMMs' tolerance; greedy tokens follow those logits."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
# relative to the largest logit of the row: the north star's per-op bar with
# the three-term GEMMs (the default), and the bound of the one-rounding form
RTOL_LOGITS = 1e-3
RTOL_LOGITS_ONE_TERM = 2e-2


def make(native, ctx, seed=5, **kw):
    from purebee_b200.runtime import LlamaConfig, StreamingLlamaRuntime
    cfg = dict(dim=128, hiddenDim=256, nLayers=2, nHeads=4, nKvHeads=2, vocabSize=512, seqLen=160, headDim=32,
               ropeTheta=10000.0)
    cfg.update(kw)
    rt = StreamingLlamaRuntime(LlamaConfig(**cfg), ctx=ctx, emb_type=native.TYPE_Q4_0)
    rt.loadSynthetic(seed, 0.05)
    return rt


def close(a, b, rtol=RTOL_LOGITS):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    err = np.max(np.abs(a - b)) / np.max(np.abs(b))
    return err <= rtol, err


@pytest.mark.parametrize("n_seqs,n_prompt,hd,dim,terms", [(3, 5, 32, 128, 3), (4, 130, 32, 128, 3),
                                                          (3, 70, 64, 128, 3), (2, 300, 64, 128, 3),
                                                          (4, 9, 64, 512, 3), (3, 70, 64, 128, 1),
                                                          (2, 300, 64, 128, 1), (16, 256, 64, 128, 3)])
def test_batch_matches_single_sequence(native, ctx, n_seqs, n_prompt, hd, dim, terms):
    """15 / 210 rows run the fused-dequant GEMM, 520 / 600 the TMA one; head_dim 64
    takes the tiled prefill attention, 32 the per-query kernel; dim 512
    makes the decode GEMMs split K over CTAs; 4096 rows take the prefill-size
    RMSNorm (a warp per row) and, with three terms, the attention writing the
    wo GEMM's hi/lo operand.  terms: the GEMM precision."""
    from purebee_b200.runtime import BatchedLlamaRuntime
    rt = make(native, ctx, dim=dim, hiddenDim=2 * dim, headDim=hd, nHeads=dim // hd, nKvHeads=max(1, dim // (2 * hd)),
              seqLen=400)
    rng = np.random.default_rng(n_seqs * 100 + n_prompt)
    prompts = rng.integers(1, 512, (n_seqs, n_prompt)).astype(np.int32)
    bt = BatchedLlamaRuntime(rt, n_seqs)
    bt.set_precision(terms)
    rtol = RTOL_LOGITS if terms == 3 else RTOL_LOGITS_ONE_TERM
    nxt, lg = bt.prefill(prompts, want_logits=True)
    errs = []
    for s in range(n_seqs):
        rt.resetCache()
        want = rt.forward(prompts[s].tolist(), 0)["logits"]
        ok, err = close(lg[s], want, rtol)
        errs.append(err)
        assert ok, f"prefill seq {s}: rel err {err:.2e}"
        assert nxt[s] == int(np.argmax(lg[s]))
    # teacher-forced decode: the one-sequence path fed the batch's own tokens
    fed = [nxt.copy()]
    for step in range(3):
        toks, lgd = bt.decode(1, want_logits=True)
        for s in range(n_seqs):
            rt.resetCache()
            seq = prompts[s].tolist() + [int(t[s]) for t in fed]
            want = rt.forward(seq, 0)["logits"]
            ok, err = close(lgd[s], want, rtol)
            errs.append(err)
            assert ok, f"decode step {step} seq {s}: rel err {err:.2e}"
            assert toks[0][s] == int(np.argmax(lgd[s]))
        fed.append(toks[0].copy())
    print(f"\n[batched parity] {n_seqs}x{n_prompt} hd {hd} dim {dim} terms {terms}: max rel logit err {max(errs):.3e}")
    bt.free()
    rt.shutdown()


def test_batch_llama1b_shape(native, ctx):
    """configs[4] at its real shape: Llama-3.2-1B-shaped weights (N(0, 0.02),
    Q4_0), 4 sequences of 512-token prompts (the prefill GEMMs take the same
    persistent TMA path as 64 x 512, the decode steps the decode-size GEMM),
    then teacher-forced decode steps; every sequence's logits against the
    one-sequence exact path.  The relative error is printed."""
    from purebee_b200.runtime import BatchedLlamaRuntime, LlamaConfig, StreamingLlamaRuntime
    cfg = LlamaConfig(dim=2048, hiddenDim=8192, nLayers=16, nHeads=32, nKvHeads=8, vocabSize=128256, seqLen=640,
                      headDim=64, ropeTheta=500000.0)
    rt = StreamingLlamaRuntime(cfg, ctx=ctx, emb_type=native.TYPE_Q4_0)
    rt.loadSynthetic(20261201, 0.02)
    n_seqs, n_prompt = 4, 512
    prompts = np.random.default_rng(9).integers(1, cfg.vocabSize, (n_seqs, n_prompt)).astype(np.int32)
    bt = BatchedLlamaRuntime(rt, n_seqs)
    nxt, lg = bt.prefill(prompts, want_logits=True)
    errs = []
    for s in range(n_seqs):
        rt.resetCache()
        want = rt.forward(prompts[s].tolist(), 0)["logits"]
        ok, err = close(lg[s], want)
        errs.append(err)
        assert ok, f"prefill seq {s}: rel err {err:.2e}"
    fed = [nxt.copy()]
    for step in range(3):
        toks, lgd = bt.decode(1, want_logits=True)
        for s in range(n_seqs):
            rt.resetCache()
            rt.forward(prompts[s].tolist(), 0)
            for i, t in enumerate(fed[:-1]):
                rt.forward([int(t[s])], n_prompt + i)
            want = rt.forward([int(fed[-1][s])], n_prompt + len(fed) - 1)["logits"]
            ok, err = close(lgd[s], want)
            errs.append(err)
            assert ok, f"decode step {step} seq {s}: rel err {err:.2e}"
        fed.append(toks[0].copy())
    print(f"\n[batched parity] llama1B shape {n_seqs}x{n_prompt}: max rel logit err prefill "
          f"{max(errs[:n_seqs]):.3e}, decode {max(errs[n_seqs:]):.3e}")
    bt.free()
    rt.shutdown()


def test_batch_rejects(native, ctx):
    from purebee_b200.runtime import BatchedLlamaRuntime
    rt = make(native, ctx)
    bt = BatchedLlamaRuntime(rt, 2)
    with pytest.raises(native.PureBeeError):
        bt.decode(1)  # before prefill
    with pytest.raises(ValueError):
        bt.prefill(np.ones((3, 4), np.int32))
    bt.free()
    rt.shutdown()
