"""GGUF files into the device model (pb_model_load_gguf /
StreamingLlamaRuntime.fromGGUF): a file written from the oracle's weights
loads into a model whose greedy tokens equal the oracle's, with a tied or an
untied (output.weight) head, Q4_0 or Q8_0 embedding, F32 or F16 norm gains,
any tensor order; malformed models are rejected before any upload."""
import numpy as np
import pytest

import gguf_writer as W

pytestmark = pytest.mark.gpu

KW = dict(kind=0, emb_type=2, dim=128, hidden_dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=32, vocab=512,
          seq_len=160, rope_theta=10000.0, eps=1e-5)
NAMES = {1: "attn_q", 2: "attn_k", 3: "attn_v", 4: "attn_output", 5: "ffn_gate", 6: "ffn_down", 7: "ffn_up"}


def oracle_model(oracle, kw, seed):
    om = oracle.Model(oracle.Config(**kw))
    om.init_synthetic(seed, 0.05)
    return om


def write_model(path, om, kw, norm_type=0, head=None, order_seed=None, drop=None, retype=None):
    dim, hid, kv, V = kw["dim"], kw["hidden_dim"], kw["n_kv_heads"] * kw["head_dim"], kw["vocab"]
    shapes = {1: [dim, dim], 2: [dim, kv], 3: [dim, kv], 4: [dim, dim], 5: [dim, hid], 6: [hid, dim], 7: [dim, hid]}
    ones = np.ones(dim, np.float32)
    norm = (ones.tobytes(), 0) if norm_type == 0 else (ones.astype(np.float16).tobytes(), 1)
    t = [("token_embd.weight", [dim, V], kw["emb_type"], om.tensor(0, 0).tobytes()),
         ("output_norm.weight", [dim], norm[1], norm[0])]
    for l in range(kw["n_layers"]):
        for w in range(1, 8):
            t.append((f"blk.{l}.{NAMES[w]}.weight", shapes[w], 2, om.tensor(l, w).tobytes()))
        t.append((f"blk.{l}.attn_norm.weight", [dim], norm[1], norm[0]))
        t.append((f"blk.{l}.ffn_norm.weight", [dim], norm[1], norm[0]))
    if head is not None:
        t.append(("output.weight", [dim, V], head[0], head[1].tobytes()))
    if drop:
        t = [x for x in t if x[0] != drop]
    if retype:
        t = [(n, d, retype[1], b) if n == retype[0] else (n, d, ty, b) for n, d, ty, b in t]
    if order_seed is not None:
        perm = np.random.default_rng(order_seed).permutation(len(t))
        t = [t[i] for i in perm]
    md = W.llama_metadata(dim, hid, kw["n_layers"], kw["n_heads"], kw["n_kv_heads"], kw["seq_len"], V,
                          theta=kw["rope_theta"], eps=kw["eps"])
    W.write_gguf(path, md, t)
    return t


@pytest.mark.parametrize("emb_type,norm_type,order_seed", [(2, 0, None), (8, 1, 7)])
def test_gguf_model_matches_oracle(native, ctx, oracle, tmp_path, emb_type, norm_type, order_seed):
    from purebee_b200.runtime import StreamingLlamaRuntime
    kw = dict(KW, emb_type=emb_type)
    om = oracle_model(oracle, kw, 11)
    p = str(tmp_path / "m.gguf")
    write_model(p, om, kw, norm_type=norm_type, order_seed=order_seed)
    rt = StreamingLlamaRuntime.fromGGUF(p, ctx=ctx)
    assert rt.sharedWeights and rt.config.vocabSize == kw["vocab"] and rt.config.headDim == kw["head_dim"]
    # the device holds exactly the file's bytes
    for l, w in [(0, 0), (0, 1), (1, 5), (1, 6), (1, 7)]:
        assert np.array_equal(rt.getTensor(l, w), om.tensor(l, w).view(np.uint8)), (l, w)
    assert np.array_equal(rt.getTensor(1, 9).view(np.float32), np.ones(kw["dim"], np.float32))
    prompt = oracle.synth_tokens(12, 99, 1, kw["vocab"]).tolist()
    want = om.generate(prompt, 40, eos_id=2)
    got = rt.generate(prompt, 40, {"greedy": True, "eosId": 2})["tokens"]
    assert got == want
    rt.shutdown()


def test_gguf_untied_head(native, ctx, oracle, tmp_path):
    from purebee_b200.runtime import StreamingLlamaRuntime
    om = oracle_model(oracle, KW, 12)
    table = oracle.synth_weights(KW["vocab"] * KW["dim"], 12, 999, 0.05)
    head = oracle.quantize_gguf_q8_0(table)
    om.set_head(8, head)
    p = str(tmp_path / "u.gguf")
    write_model(p, om, KW, head=(8, head))
    rt = StreamingLlamaRuntime.fromGGUF(p, ctx=ctx)
    assert not rt.sharedWeights
    assert np.array_equal(rt.getTensor(0, 11), np.asarray(head, np.uint8))
    prompt = oracle.synth_tokens(10, 5, 1, KW["vocab"]).tolist()
    want = om.generate(prompt, 32, eos_id=2)
    got = rt.generate(prompt, 32, {"greedy": True, "eosId": 2})["tokens"]
    assert got == want
    # the untied head is what the logits come from: a tied model differs
    rt.resetCache()
    lg = rt.forward(prompt, 0)["logits"]
    om.reset_cache()
    ref = om.forward(prompt, 0)
    assert np.max(np.abs(lg - ref)) <= 1e-5 * np.max(np.abs(ref))
    rt.shutdown()


def _q6k_raw(rng, n):
    raw = rng.integers(0, 256, n // 256 * 210, dtype=np.uint8)
    d = (np.abs(rng.standard_normal(n // 256)) * 2e-4 + 1e-4).astype(np.float16)
    raw.reshape(-1, 210)[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return raw


@pytest.mark.parametrize("untied", [False, True])
def test_gguf_q6_k_tables(native, ctx, oracle, tmp_path, untied):
    """A Q6_K token_embd.weight (and a Q6_K output.weight when untied), the
    type llama.cpp's quantizer commonly writes for these tables: the device
    keeps them dequantized to f32, as streaming-loader.js:324-335 does, and
    the head runs batch_dot over the f32 table.  Logits and greedy tokens
    equal the oracle's, which holds the same dequantized tables."""
    from purebee_b200.runtime import StreamingLlamaRuntime
    rng = np.random.default_rng(7 + untied)
    kw = dict(KW, emb_type=0)  # the oracle's f32 embedding (streaming kind)
    om = oracle_model(oracle, dict(KW), 15)
    n = kw["vocab"] * kw["dim"]
    emb_q6 = _q6k_raw(rng, n)
    emb_f32 = oracle.dequant_q6_k(emb_q6, n)
    omf = oracle.Model(oracle.Config(**kw))
    for l in range(kw["n_layers"]):
        for w in range(1, 8):
            omf.tensor(l, w)[:] = om.tensor(l, w)
    omf.tensor(0, 0)[:] = emb_f32.view(np.uint8)
    omf.refresh()
    head = None
    if untied:
        head_q6 = _q6k_raw(rng, n)
        omf.set_head(0, oracle.dequant_q6_k(head_q6, n).view(np.uint8))
        head = (14, head_q6)
    p = str(tmp_path / "q6.gguf")
    t = write_model(p, om, KW, head=head)
    t = [(nm, d, 14, emb_q6.tobytes()) if nm == "token_embd.weight" else (nm, d, ty, b) for nm, d, ty, b in t]
    md = W.llama_metadata(kw["dim"], kw["hidden_dim"], kw["n_layers"], kw["n_heads"], kw["n_kv_heads"],
                          kw["seq_len"], kw["vocab"], theta=kw["rope_theta"], eps=kw["eps"])
    W.write_gguf(p, md, t)
    rt = StreamingLlamaRuntime.fromGGUF(p, ctx=ctx)
    assert rt.sharedWeights == (not untied)
    # the device table is the decoded f32 table
    assert np.array_equal(rt.getTensor(0, 0).view(np.float32), emb_f32)
    prompt = oracle.synth_tokens(10, 21, 1, kw["vocab"]).tolist()
    lg = rt.forward(prompt, 0)["logits"]
    ref = omf.forward(prompt, 0)
    assert np.max(np.abs(lg - ref)) <= 1e-5 * np.max(np.abs(ref))
    rt.resetCache()
    omf.reset_cache()
    want = omf.generate(prompt, 24, eos_id=2)
    got = rt.generate(prompt, 24, {"greedy": True, "eosId": 2})["tokens"]
    assert got == want
    rt.shutdown()


def test_gguf_seq_len_override(native, ctx, oracle, tmp_path):
    from purebee_b200.runtime import StreamingLlamaRuntime
    om = oracle_model(oracle, KW, 13)
    p = str(tmp_path / "s.gguf")
    write_model(p, om, KW)
    rt = StreamingLlamaRuntime.fromGGUF(p, {"seqLen": 64}, ctx=ctx)
    assert rt.config.seqLen == 64
    with pytest.raises(native.PureBeeError):
        rt.forward(list(range(1, 66)), 0)  # longer than the overridden context
    rt.shutdown()


def test_gguf_load_rejects(native, ctx, oracle, tmp_path):
    from purebee_b200.runtime import StreamingLlamaRuntime
    om = oracle_model(oracle, KW, 14)
    p = str(tmp_path / "r.gguf")
    launches = ctx.launches
    write_model(p, om, KW, drop="blk.1.ffn_up.weight")
    with pytest.raises(native.PureBeeError, match="lacks"):
        StreamingLlamaRuntime.fromGGUF(p, ctx=ctx)
    write_model(p, om, KW, retype=("blk.0.attn_k.weight", 3))  # Q4_1 layer weight
    with pytest.raises(native.PureBeeError, match="ggml type 3"):
        StreamingLlamaRuntime.fromGGUF(p, ctx=ctx)
    assert ctx.launches == launches  # nothing uploaded
