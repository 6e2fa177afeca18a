"""The GGUF tokenizer (purebee_b200/tokenizer.py) on hand-built vocabularies,
following gguf.js:461-762: GPT-2 byte-level BPE by merge rank, SentencePiece
spaces and byte fallback, special-token splitting, control tokens skipped on
decode, byte tokens decoded to the character with that code point."""
import numpy as np

from purebee_b200.tokenizer import GGUFTokenizer, buildByteToUnicode

import gguf_writer as W


def gpt2_vocab(extra, merges, types=None):
    b2u, _ = buildByteToUnicode()
    vocab = list(b2u) + list(extra)
    md = {"tokenizer.ggml.model": "gpt2", "tokenizer.ggml.tokens": vocab, "tokenizer.ggml.merges": merges}
    if types is not None:
        md["tokenizer.ggml.token_type"] = types
    return GGUFTokenizer(md), vocab


def test_byte_to_unicode_table():
    b2u, u2b = buildByteToUnicode()
    assert len(set(b2u)) == 256 and b2u[ord("a")] == "a" and b2u[32] == "Ġ" and b2u[10] == "Ċ"
    assert all(u2b[b2u[b]] == b for b in range(256))


def test_gpt2_merges_by_rank():
    extra = ["he", "ll", "hell", "hello", "Ġh", "lo"]
    merges = ["l l", "h e", "he ll", "hell o", "Ġ h", "l o"]
    tk, vocab = gpt2_vocab(extra, merges)
    ids = tk.encode("hello hello")
    # every "l l" (rank 0) first, then every "h e" (1): the second "h" pairs with "e"
    # before "Ġ h" (4) is reached, and "l o" (5) loses to "ll"
    assert [vocab[i] for i in ids] == ["hello", "Ġ", "hello"]
    assert tk.decode(ids) == "hello hello"
    # leftmost wins among equal ranks; the merged string must be in the vocabulary
    tk2, v2 = gpt2_vocab(["aa"], ["a a", "aa a"])
    assert [v2[i] for i in tk2.encode("aaaaa")] == ["aa", "aa", "a"]


def test_gpt2_round_trip_and_per_token_decoding():
    tk, _ = gpt2_vocab(["he", "ll", "Ã¯"], ["h e", "l l", "Ã ¯"])
    for text in ["", "hello", "\x00\x01 tabs\tand\nnewlines"]:
        assert tk.decode(tk.encode(text)) == text
    # decode works token by token (Buffer.toString per token): a character whose
    # UTF-8 bytes sit in one merged token survives, one split over byte tokens
    # becomes one U+FFFD per byte
    assert tk.decode(tk.encode("naïve")) == "naïve"
    assert tk.decode(tk.encode("café")) == "caf\ufffd\ufffd"


def test_special_tokens_split_the_text():
    extra = ["<|im_start|>", "<|im_end|>", "<|im_start|>x|>", "us", "use", "user"]
    tk, vocab = gpt2_vocab(extra, ["u s", "us e", "use r"])
    ids = tk.encode("<|im_start|>x|>user<|im_end|>")
    # the longest special token matches first
    assert vocab[ids[0]] == "<|im_start|>x|>" and vocab[ids[1]] == "user" and vocab[ids[2]] == "<|im_end|>"
    assert tk.getSpecialToken("<|im_end|>") == vocab.index("<|im_end|>")
    # control tokens (type 3) are dropped when decoding
    types = [1] * len(vocab)
    types[vocab.index("<|im_end|>")] = 3
    tk3, _ = gpt2_vocab(extra, ["u s", "us e", "use r"], types)
    assert tk3.decode(ids) == "<|im_start|>x|>user"
    assert tk3.decode([-1, len(vocab)]) == ""


def test_sentencepiece_spaces_merges_and_byte_fallback():
    vocab = ["<unk>", "<s>", "</s>", "▁", "h", "i", "▁h", "▁hi", "▁t"]
    types = [2, 3, 3] + [1] * 6
    vocab += [f"<0x{b:02X}>" for b in range(256)]
    types += [6] * 256
    md = {"tokenizer.ggml.model": "llama", "tokenizer.ggml.tokens": vocab, "tokenizer.ggml.token_type": types,
          "tokenizer.ggml.merges": ["▁ h", "▁h i"], "tokenizer.ggml.scores": [0.0] * len(vocab)}
    tk = GGUFTokenizer(md)
    assert tk.bosId == 1 and tk.eosId == 2
    # a leading U+2581, then merges by rank
    assert tk.encode("hi") == [vocab.index("▁hi")]
    # spaces become U+2581; é falls back to its UTF-8 byte tokens; <s> splits
    ids = tk.encode("<s>hi é")
    want = [1, vocab.index("▁hi"), vocab.index("▁"), vocab.index("<0xC3>"), vocab.index("<0xA9>")]
    assert ids == want
    # decode: <s> is a control token; U+2581 -> space; byte tokens -> the character with that code point
    assert tk.decode(ids) == " hi " + "Ã©"
    # a text starting with a space gets no extra U+2581
    assert tk.encode(" hi") == [vocab.index("▁hi")]


def test_repeated_entries_keep_the_last():
    md = {"tokenizer.ggml.model": "llama", "tokenizer.ggml.tokens": ["▁", "a", "a", "▁a"],
          "tokenizer.ggml.merges": ["▁ a", "▁ a"]}
    tk = GGUFTokenizer(md)
    assert tk.encode("a") == [3]
    assert tk._tokenToId["a"] == 2 and tk._mergeRank[(0, 2)] == 1


def test_tokenizer_from_gguf_file(native, tmp_path):
    from purebee_b200.gguf import GGUFFile
    vocab = ["<unk>", "<s>", "</s>", "▁", "h", "i", "▁h", "▁hi"]
    md = [("tokenizer.ggml.model", W.STRING, "llama"), ("tokenizer.ggml.tokens", W.ARRAY, (W.STRING, vocab)),
          ("tokenizer.ggml.token_type", W.ARRAY, (W.I32, [2, 3, 3, 1, 1, 1, 1, 1])),
          ("tokenizer.ggml.merges", W.ARRAY, (W.STRING, ["▁ h", "▁h i"])),
          ("tokenizer.ggml.bos_token_id", W.U32, 1), ("tokenizer.ggml.eos_token_id", W.U32, 2)]
    p = str(tmp_path / "tok.gguf")
    W.write_gguf(p, md, [])
    with GGUFFile(p) as f:
        tk = f.tokenizer()
    assert tk.encode("hi hi") == [7, 7] and tk.decode([1, 7, 7, 2]) == " hi hi"


def test_gpt2_encoding_is_lossless_at_the_byte_level():
    """Byte-level BPE keeps every byte: for any text the tokens' strings
    concatenate to the byte-to-unicode image of its UTF-8 bytes, every merge
    yields a vocabulary entry, and ASCII text decodes back exactly."""
    from hypothesis import given, settings, strategies as st
    b2u, _ = buildByteToUnicode()
    extra = ["th", "he", "the", "Ġt", "Ġthe", "in", "ing", "Ã©", "ll", "ĠĠ"]
    merges = ["t h", "h e", "th e", "Ġ t", "Ġt he", "i n", "in g", "Ã ©", "l l", "Ġ Ġ"]
    tk, vocab = gpt2_vocab(extra, merges)

    @settings(max_examples=300, deadline=None)
    @given(st.text(max_size=40))
    def check(text):
        ids = tk.encode(text)
        assert all(0 <= i < len(vocab) for i in ids)
        assert "".join(vocab[i] for i in ids) == "".join(b2u[b] for b in text.encode("utf-8", "surrogatepass"))
        if text.isascii():
            assert tk.decode(ids) == text

    check()
