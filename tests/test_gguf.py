"""GGUF parsing on the host (no GPU): the library's parser against files the
test writes, following gguf.js:76-194 (GGUFParser), :204-211
(tensorByteSize), :376-404 (mapTensorName), :402-424 (extractConfig) and
streaming-loader.js:35-87 (parseHeader: aligned data start, tensor index,
sharedWeights)."""
import os

import numpy as np
import pytest

import gguf_writer as W


@pytest.fixture
def gg(native):
    from purebee_b200 import gguf
    return gguf


def _tiny_tensors(rng, dim=64, vocab=40, types=(2, 2)):
    emb_bytes = vocab * dim // 32 * (18 if types[0] == 2 else 34)
    return [("token_embd.weight", [dim, vocab], types[0], rng.integers(0, 256, emb_bytes, dtype=np.uint8).tobytes()),
            ("output_norm.weight", [dim], 0, W.f32_bytes(np.ones(dim)))]


def test_metadata_every_value_type(tmp_path, gg):
    md = [("a.u8", W.U8, 200), ("a.i8", W.I8, -5), ("a.u16", W.U16, 60000), ("a.i16", W.I16, -30000),
          ("a.u32", W.U32, 4000000000), ("a.i32", W.I32, -2000000000), ("a.f32", W.F32, 1.5),
          ("a.bool", W.BOOL, 1), ("a.str", W.STRING, "héllo"), ("a.u64", W.U64, 2 ** 40 + 3),
          ("a.i64", W.I64, -(2 ** 40)), ("a.f64", W.F64, 0.1),
          ("a.arr_i", W.ARRAY, (W.I32, [1, -2, 3])), ("a.arr_f", W.ARRAY, (W.F32, [0.5, -0.25])),
          ("a.arr_s", W.ARRAY, (W.STRING, ["x", "", "yz"])), ("a.empty", W.ARRAY, (W.U8, []))]
    p = str(tmp_path / "m.gguf")
    W.write_gguf(p, md, [])
    with gg.GGUFFile(p) as f:
        m = f.metadata
        assert f.version == 3
        assert m["a.u8"] == 200 and m["a.i8"] == -5 and m["a.u16"] == 60000 and m["a.i16"] == -30000
        assert m["a.u32"] == 4000000000 and m["a.i32"] == -2000000000
        assert m["a.f32"] == 1.5 and m["a.bool"] is True and m["a.str"] == "héllo"
        assert m["a.u64"] == 2 ** 40 + 3 and m["a.i64"] == -(2 ** 40) and m["a.f64"] == 0.1
        assert m["a.arr_i"] == [1, -2, 3] and m["a.arr_f"] == [0.5, -0.25] and m["a.arr_s"] == ["x", "", "yz"]
        assert m["a.empty"] == []
        assert f.tensorInfos == []


@pytest.mark.parametrize("version,alignment", [(2, 32), (3, 32), (3, 64), (3, 256)])
def test_tensor_index_offsets_and_sizes(tmp_path, gg, version, alignment):
    rng = np.random.default_rng(3)
    # one tensor of every block geometry the reference's size table knows (gguf.js:36-51)
    specs = [("f32", [5, 3], 0, 15 * 4), ("f16", [7], 1, 14), ("q4_0", [64, 3], 2, 6 * 18),
             ("q4_1", [32, 2], 3, 2 * 20), ("q8_0", [96], 8, 3 * 34), ("q6_k", [256, 2], 14, 2 * 210),
             ("q4_k", [512], 12, 2 * 144)]
    tensors = [(n, d, t, rng.integers(0, 256, nb, dtype=np.uint8).tobytes()) for n, d, t, nb in specs]
    md = [("general.alignment", W.U32, alignment)] if alignment != 32 else []
    p = str(tmp_path / "t.gguf")
    W.write_gguf(p, md, tensors, version=version, alignment=alignment)
    with gg.GGUFFile(p) as f:
        assert f.version == version and f.alignment == alignment
        assert f.dataStart % alignment == 0
        infos = f.tensorInfos
        assert [i["name"] for i in infos] == [t[0] for t in tensors]
        raw = open(p, "rb").read()
        for info, (name, dims, t, data), (_, _, _, nb) in zip(infos, tensors, specs):
            assert info["dims"] == list(dims) and info["type"] == t and info["byteSize"] == nb
            assert (info["offset"] - f.dataStart) % alignment == 0
            assert raw[info["offset"]:info["offset"] + nb] == data
            assert f.readTensorRaw(name).tobytes() == data
        with pytest.raises(gg.GGUFError, match="not found"):
            f.readTensorRaw("nope")


def test_extract_config_values_and_defaults(tmp_path, gg):
    rng = np.random.default_rng(4)
    p = str(tmp_path / "c.gguf")
    W.write_gguf(p, W.llama_metadata(64, 160, 3, 4, 2, 96, 40, theta=5e5, eps=1e-6), _tiny_tensors(rng))
    with gg.GGUFFile(p) as f:
        cfg, extra = f.config()
        assert (cfg.dim, cfg.hiddenDim, cfg.nLayers, cfg.nHeads, cfg.nKvHeads, cfg.seqLen) == (64, 160, 3, 4, 2, 96)
        assert cfg.headDim == 16 and cfg.vocabSize == 40 and cfg.ropeTheta == 5e5
        assert abs(cfg.rmsNormEps - 1e-6) < 1e-12 and extra["arch"] == "llama" and extra["name"] == "test-model"
    # missing or zero values take extractConfig's defaults (JS `||`): kv heads = heads,
    # context 2048, eps 1e-5, theta 1e4; another architecture prefix; floor(dim / heads)
    md = [("general.architecture", W.STRING, "qwen2"), ("qwen2.embedding_length", W.U32, 66),
          ("qwen2.feed_forward_length", W.U64, 96), ("qwen2.block_count", W.I32, 2),
          ("qwen2.attention.head_count", W.U32, 4), ("qwen2.rope.freq_base", W.F32, 0.0),
          ("tokenizer.ggml.tokens", W.ARRAY, (W.STRING, ["a"] * 40))]
    p2 = str(tmp_path / "d.gguf")
    W.write_gguf(p2, md, _tiny_tensors(rng, dim=64))
    with gg.GGUFFile(p2) as f:
        cfg, extra = f.config()
        assert extra["arch"] == "qwen2"
        assert (cfg.dim, cfg.hiddenDim, cfg.nLayers, cfg.nHeads, cfg.nKvHeads) == (66, 96, 2, 4, 4)
        assert cfg.seqLen == 2048 and cfg.rmsNormEps == 1e-5 and cfg.ropeTheta == 10000.0 and cfg.headDim == 16
    # no token list: the embedding's row count is the vocabulary
    md3 = [m for m in W.llama_metadata(64, 160, 3, 4, 2, 96, 40) if m[0] != "tokenizer.ggml.tokens"]
    p3 = str(tmp_path / "e.gguf")
    W.write_gguf(p3, md3, _tiny_tensors(rng, vocab=40, types=(8, 0)))
    with gg.GGUFFile(p3) as f:
        cfg, extra = f.config()
        assert cfg.vocabSize == 40 and extra["embType"] == 8


def test_parse_header_index(tmp_path, gg):
    rng = np.random.default_rng(5)
    t = _tiny_tensors(rng) + [("blk.0.attn_q.weight", [64, 64], 2, bytes(64 * 2 * 18)),
                              ("blk.0.ffn_norm.weight", [64], 0, W.f32_bytes(np.ones(64))),
                              ("blk.11.ffn_up.weight", [64, 32], 2, bytes(32 * 2 * 18)),
                              ("custom.thing", [4], 0, bytes(16))]
    p = str(tmp_path / "h.gguf")
    W.write_gguf(p, W.llama_metadata(64, 160, 12, 4, 2, 96, 40), t)
    h = gg.parseHeader(p)
    idx = h["tensorIndex"]
    assert set(idx) == {"token_embedding", "rms_final", "layer0.wq", "layer0.rms_ffn", "layer11.w3", "custom.thing"}
    assert idx["layer0.wq"]["transpose"] is True and idx["rms_final"]["transpose"] is False
    assert idx["layer11.w3"]["ggufName"] == "blk.11.ffn_up.weight" and idx["layer11.w3"]["dims"] == [64, 32]
    assert h["sharedWeights"] is True and h["dataStart"] % 32 == 0
    t2 = t + [("output.weight", [64, 40], 2, bytes(40 * 2 * 18))]
    W.write_gguf(p, W.llama_metadata(64, 160, 12, 4, 2, 96, 40), t2)
    h = gg.parseHeader(p)
    assert h["sharedWeights"] is False and "lm_head" in h["tensorIndex"]


def test_malformed_files_raise(tmp_path, gg):
    rng = np.random.default_rng(6)
    md = W.llama_metadata(64, 160, 3, 4, 2, 96, 40)
    t = _tiny_tensors(rng)
    p = str(tmp_path / "bad.gguf")
    with pytest.raises(gg.GGUFError, match="cannot open"):
        gg.GGUFFile(str(tmp_path / "missing.gguf"))
    open(p, "wb").write(b"GGML" + bytes(60))
    with pytest.raises(gg.GGUFError, match="bad magic"):
        gg.GGUFFile(p)
    for v in (1, 4):
        W.write_gguf(p, md, t, version=v)
        with pytest.raises(gg.GGUFError, match="version"):
            gg.GGUFFile(p)
    # truncated inside the metadata, inside the tensor index, and inside the data
    W.write_gguf(p, md, t)
    size = os.path.getsize(p)
    for cut in (size - 100, 60, 200):
        data = open(p, "rb").read()
        open(str(tmp_path / "cut.gguf"), "wb").write(data[:cut] if cut < size else data)
        with pytest.raises(gg.GGUFError):
            gg.GGUFFile(str(tmp_path / "cut.gguf"))
    # an unknown metadata value type
    import struct
    raw = struct.pack("<IIQQ", 0x46554747, 3, 0, 1) + struct.pack("<Q", 1) + b"k" + struct.pack("<I", 13) + bytes(8)
    open(p, "wb").write(raw)
    with pytest.raises(gg.GGUFError, match="metadata value"):
        gg.GGUFFile(p)
    # a string array claiming more elements than the rest of the file can
    # encode (8 bytes per string at least): rejected before any element is
    # allocated
    raw = (struct.pack("<IIQQ", 0x46554747, 3, 0, 1) + struct.pack("<Q", 1) + b"k"
           + struct.pack("<IIQ", 9, 8, 1 << 20) + bytes(1 << 20))
    open(p, "wb").write(raw)
    with pytest.raises(gg.GGUFError, match="metadata array"):
        gg.GGUFFile(p)
    # config needs the llama keys and an embedding type the device model takes
    W.write_gguf(p, [("general.architecture", W.STRING, "llama")], t)
    with gg.GGUFFile(p) as f, pytest.raises(gg.GGUFError, match="embedding_length"):
        f.config()
    W.write_gguf(p, md, [("token_embd.weight", [256, 40], 12, bytes(40 * 144))])  # Q4_K: not decoded
    with gg.GGUFFile(p) as f, pytest.raises(gg.GGUFError, match="Q4_0, Q8_0, Q6_K"):
        f.config()
    W.write_gguf(p, md, [("token_embd.weight", [256, 40], 14, bytes(40 * 210))])  # Q6_K: a dequantized f32 table
    with gg.GGUFFile(p) as f:
        assert f.config()[1]["embType"] == 0
    W.write_gguf(p, md, [("output_norm.weight", [64], 0, bytes(256))])
    with gg.GGUFFile(p) as f, pytest.raises(gg.GGUFError, match="token_embd"):
        f.config()


_FUZZ = r'''
import os, sys, struct
import numpy as np
sys.path.insert(0, os.path.join(os.environ["PB_ROOT"], "tests"))
sys.path.insert(0, os.environ["PB_ROOT"])
import gguf_writer as W
from purebee_b200 import gguf as gg

rng = np.random.default_rng(int(os.environ["PB_SEED"]))
dim, vocab = 64, 40
md = W.llama_metadata(dim, 160, 3, 4, 2, 96, vocab)
tensors = [("token_embd.weight", [dim, vocab], 2, rng.integers(0, 256, vocab * dim // 32 * 18, dtype=np.uint8).tobytes()),
           ("output_norm.weight", [dim], 0, W.f32_bytes(np.ones(dim)))]
path = os.path.join(os.environ["PB_TMP"], "fuzz.gguf")
W.write_gguf(path, md, tensors)
good = open(path, "rb").read()
huge = [2**63 - 1, 2**62, 2**40, 2**32, 2**31, 2**24, 0xFFFFFFFF, 1 << 20]
outcomes = {"ok": 0, "error": 0}
for it in range(int(os.environ["PB_ITERS"])):
    b = bytearray(good)
    kind = it % 3
    if kind == 0:    # a few random bytes anywhere before the tensor data
        for _ in range(int(rng.integers(1, 9))):
            b[int(rng.integers(0, len(b) - vocab * dim // 32 * 18))] = int(rng.integers(0, 256))
    elif kind == 1:  # an 8-byte field set to a large value
        off = int(rng.integers(0, len(b) - 8))
        b[off:off + 8] = struct.pack("<Q", huge[int(rng.integers(0, len(huge)))])
    else:            # truncated
        b = b[:int(rng.integers(0, len(b)))]
    open(path, "wb").write(bytes(b))
    try:
        with gg.GGUFFile(path) as f:
            f.metadata
            for t in f.tensorInfos:
                try:
                    f.readTensorRaw(t["name"])
                except gg.GGUFError:
                    pass
            try:
                f.config()
                f.tokenizer()
            except gg.GGUFError:
                pass
        outcomes["ok"] += 1
    except gg.GGUFError:
        outcomes["error"] += 1
print(outcomes)
'''


def test_corrupted_files_error_or_parse(tmp_path, native):
    """Random corruption of a valid file (flipped bytes, 8-byte fields set to
    huge counts, offsets or sizes, truncation) either parses or raises
    GGUFError: the parser never crashes, hangs or allocates without bound.  It
    runs in a child process so that a crash fails this test alone."""
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PB_ROOT=root, PB_TMP=str(tmp_path), PB_SEED="17", PB_ITERS="600")
    r = subprocess.run([sys.executable, "-c", _FUZZ], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, f"parser crashed (rc {r.returncode}): {r.stderr[-2000:]}"
    assert "'error'" in r.stdout


def test_metadata_round_trip_property(tmp_path, gg):
    """Any metadata the format can hold reads back as written: every scalar
    type over its whole range, Unicode keys (without NUL: keys are C strings
    at the ABI) and strings (with NUL: values carry their length), arrays of
    scalars and of strings."""
    from hypothesis import given, settings, strategies as st
    ints = {W.U8: (0, 2**8 - 1), W.I8: (-2**7, 2**7 - 1), W.U16: (0, 2**16 - 1), W.I16: (-2**15, 2**15 - 1),
            W.U32: (0, 2**32 - 1), W.I32: (-2**31, 2**31 - 1), W.U64: (0, 2**53), W.I64: (-2**53, 2**53)}
    text = st.text(st.characters(blacklist_categories=("Cs",)), max_size=12)
    keys = st.text(st.characters(blacklist_categories=("Cs",), blacklist_characters="\x00"), max_size=12)

    def value(t):
        if t in ints:
            return st.integers(*ints[t])
        if t == W.F32:
            return st.floats(width=32, allow_nan=False)
        if t == W.F64:
            return st.floats(allow_nan=False)
        if t == W.BOOL:
            return st.booleans().map(int)
        return text

    scalar_t = st.sampled_from(sorted(ints) + [W.F32, W.F64, W.BOOL, W.STRING])
    entry = scalar_t.flatmap(lambda t: st.one_of(
        value(t).map(lambda v: (t, v)),
        st.lists(value(t), max_size=5).map(lambda vs: (W.ARRAY, (t, vs)))))
    path = str(tmp_path / "p.gguf")

    @settings(max_examples=150, deadline=None)
    @given(st.dictionaries(keys, entry, max_size=8))
    def check(md):
        W.write_gguf(path, [(k, t, v) for k, (t, v) in md.items()], [])
        with gg.GGUFFile(path) as f:
            got = f.metadata
        assert set(got) == set(md)
        for k, (t, v) in md.items():
            if t == W.ARRAY:
                et, vs = v
                want = [bool(x) for x in vs] if et == W.BOOL else vs
                assert got[k] == want, (k, et)
            elif t == W.BOOL:
                assert got[k] is bool(v)
            else:
                assert got[k] == v, (k, t)

    check()
