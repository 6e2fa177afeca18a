"""The GGUF tokenizer (gguf.js:461-762 buildByteToUnicode, GGUFTokenizer), host side.

Built from a GGUF file's `tokenizer.ggml.*` metadata.  encode() splits on
special tokens (`<s>`, `</s>`, and every `<|...|>` token), encodes each
segment either GPT-2 style (UTF-8 bytes through the byte-to-unicode table) or
SentencePiece style (spaces to U+2581, a leading U+2581, byte-token fallback),
then merges adjacent pairs by the rank of `tokenizer.ggml.merges`, lowest
rank first, leftmost on ties, while the merged string is in the vocabulary.
decode() skips control tokens (type 3), maps GPT-2 unicode back to bytes, a
leading U+2581 to a space, and `<0xNN>` byte tokens to the character NN.

Behaviour kept from the reference as it is:
- the merge loop uses the merges list only, so a SentencePiece vocabulary
  without merges encodes to single characters and byte tokens (its scores
  are read but not used, gguf.js:673-703);
- lookups built from lists keep the last entry for a repeated key (JS
  `Map.set`), and the special-token pattern prefers the longest token;
- byte tokens decode one by one to the character with that code point.
"""
from __future__ import annotations

import re
from typing import Dict, List, Optional


def buildByteToUnicode():
    """gguf.js:461-484: GPT-2's byte <-> unicode table."""
    self_map = set(range(33, 127)) | set(range(161, 173)) | set(range(174, 256))
    byte_to_uni: List[str] = [""] * 256
    uni_to_byte: Dict[str, int] = {}
    nxt = 256
    for b in range(256):
        if b in self_map:
            byte_to_uni[b] = chr(b)
        else:
            byte_to_uni[b] = chr(nxt)
            nxt += 1
        uni_to_byte[byte_to_uni[b]] = b
    return byte_to_uni, uni_to_byte


_BYTE_TOKEN = re.compile(r"^<0x([0-9A-Fa-f]{2})>$")


class GGUFTokenizer:
    def __init__(self, metadata: dict):
        self.model = metadata.get("tokenizer.ggml.model") or "llama"
        self.vocab: List[str] = list(metadata.get("tokenizer.ggml.tokens") or [])
        self.scores = list(metadata.get("tokenizer.ggml.scores") or [])
        self.tokenTypes = list(metadata.get("tokenizer.ggml.token_type") or [])
        bos = metadata.get("tokenizer.ggml.bos_token_id")
        eos = metadata.get("tokenizer.ggml.eos_token_id")
        self.bosId = 1 if bos is None else bos  # `?? 1`
        self.eosId = 2 if eos is None else eos  # `?? 2`
        self._tokenToId: Dict[str, int] = {}
        for i, t in enumerate(self.vocab):
            self._tokenToId[t] = i
        self._mergeRank: Dict[tuple, int] = {}
        for i, m in enumerate(metadata.get("tokenizer.ggml.merges") or []):
            sp = m.find(" ")
            if sp == -1:
                continue
            a, b = self._tokenToId.get(m[:sp]), self._tokenToId.get(m[sp + 1:])
            if a is not None and b is not None:
                self._mergeRank[(a, b)] = i
        if self.model == "gpt2":
            self._byteToUni, self._uniToByte = buildByteToUnicode()
        self._byteTokens: Dict[int, int] = {}
        for i, t in enumerate(self.vocab):
            if i < len(self.tokenTypes) and self.tokenTypes[i] == 6:
                mm = _BYTE_TOKEN.match(t)
                if mm:
                    self._byteTokens[int(mm.group(1), 16)] = i
        self._specialTokens: Dict[str, int] = {}
        for i, t in enumerate(self.vocab):
            if t in ("<s>", "</s>") or (t.startswith("<|") and t.endswith("|>")):
                self._specialTokens[t] = i
        self._specialPattern = None
        if self._specialTokens:
            # stable, longest first by UTF-16 length (JS string length)
            keys = sorted(self._specialTokens, key=lambda k: len(k.encode("utf-16-le")) // 2, reverse=True)
            self._specialPattern = re.compile("(" + "|".join(re.escape(k) for k in keys) + ")")

    # -- encode -----------------------------------------------------------
    def encode(self, text: str) -> List[int]:
        """gguf.js:554-563."""
        if self._specialTokens:
            return self._encodeWithSpecials(text)
        return self._encodeSegment(text)

    def _encodeSegment(self, text: str) -> List[int]:
        return self._encodeGPT2(text) if self.model == "gpt2" else self._encodeSentencePiece(text)

    def _encodeWithSpecials(self, text: str) -> List[int]:
        """gguf.js:568-606."""
        tokens: List[int] = []
        last = 0
        for m in self._specialPattern.finditer(text):
            before = text[last:m.start()]
            if before:
                tokens.extend(self._encodeSegment(before))
            tokens.append(self._specialTokens[m.group(0)])
            last = m.end()
        rest = text[last:]
        if rest:
            tokens.extend(self._encodeSegment(rest))
        return tokens

    def _encodeGPT2(self, text: str) -> List[int]:
        """gguf.js:611-635."""
        uni = "".join(self._byteToUni[b] for b in text.encode("utf-8"))
        unk = self._tokenToId.get("<unk>") or 0
        tokens = [self._tokenToId.get(ch, unk) for ch in uni]
        return self._bpeMerge(tokens)

    def _encodeSentencePiece(self, text: str) -> List[int]:
        """gguf.js:640-668."""
        processed = text.replace(" ", "▁")
        sp = "▁" + processed if text and text[0] != " " else processed
        tokens: List[int] = []
        for ch in sp:
            i = self._tokenToId.get(ch)
            if i is not None:
                tokens.append(i)
            else:  # byte fallback
                for b in ch.encode("utf-8", errors="surrogatepass"):
                    bi = self._byteTokens.get(b)
                    if bi is not None:
                        tokens.append(bi)
        return self._bpeMerge(tokens)

    def _bpeMerge(self, tokens: List[int]) -> List[int]:
        """gguf.js:673-703: merge the lowest-rank adjacent pair (leftmost on
        ties) whose concatenation is a vocabulary entry, until none is left."""
        tokens = list(tokens)
        if len(tokens) < 2:
            return tokens
        while True:
            best_rank, best_i, best_id = None, -1, -1
            for i in range(len(tokens) - 1):
                r = self._mergeRank.get((tokens[i], tokens[i + 1]))
                if r is not None and (best_rank is None or r < best_rank):
                    mid = self._tokenToId.get(self.vocab[tokens[i]] + self.vocab[tokens[i + 1]])
                    if mid is not None:
                        best_rank, best_i, best_id = r, i, mid
            if best_i == -1:
                return tokens
            tokens[best_i:best_i + 2] = [best_id]

    # -- decode -----------------------------------------------------------
    def decode(self, tokenIds) -> str:
        """gguf.js:708-714."""
        return "".join(self._decodeToken(int(t)) for t in tokenIds)

    def decodeToken(self, tokenId: int, prevTokenId: Optional[int] = None) -> str:
        return self._decodeToken(int(tokenId))

    def _decodeToken(self, tokenId: int) -> str:
        """gguf.js:723-754."""
        if tokenId < 0 or tokenId >= len(self.vocab):
            return ""
        token = self.vocab[tokenId]
        if tokenId < len(self.tokenTypes) and self.tokenTypes[tokenId] == 3:
            return ""  # control token
        if self.model == "gpt2":
            data = bytes(self._uniToByte[ch] for ch in token if ch in self._uniToByte)
            return data.decode("utf-8", errors="replace")
        if token.startswith("▁"):
            return " " + token[1:]
        mm = _BYTE_TOKEN.match(token)
        if mm:
            return chr(int(mm.group(1), 16))
        return token

    def getSpecialToken(self, name: str) -> Optional[int]:
        return self._specialTokens.get(name)
