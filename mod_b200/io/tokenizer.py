"""Tokenizers.

* :class:`ByteBPETokenizer` - byte-level BPE from ``vocab.json`` + ``merges.txt``
  (or an HF ``tokenizer.json``), the scheme of GPT-2 / Qwen: UTF-8 bytes are
  mapped to printable code points, text is pre-split with a Unicode-aware
  pattern, and each piece is merged greedily by merge rank.
* :class:`SimpleTokenizer` - byte values as ids (fallback when no vocab exists).
* :func:`load_tokenizer` picks one for a model directory.

Counterparts: ``pio/common/custom_components/tokenizer.py:32-199`` (the
reference's pre-tokeniser lacks ``\\p{L}`` classes and returns the unknown id
for pad/eos).  Benchmarks use synthetic token ids, so this is off the timed path.
"""
from __future__ import annotations

import json
import os
from functools import lru_cache
from typing import Dict, List, Optional, Tuple

try:
    import regex as _re
except ImportError:  # pragma: no cover
    import re as _re

# Qwen2/Qwen3 pre-tokenisation pattern (letters, single digits, punctuation runs, whitespace).
_PAT = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+")


@lru_cache()
def byte_to_unicode() -> Dict[int, str]:
    """Bijective map of the 256 byte values onto printable characters: printable
    Latin-1 bytes map to themselves, the rest to code points from 256 upward."""
    keep = list(range(ord("!"), ord("~") + 1)) + list(range(0xA1, 0xAD)) + list(range(0xAE, 0x100))
    table = {}
    extra = 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


class SimpleTokenizer:
    """Ids are byte values (0-255); ``eos`` is 256."""

    def __init__(self, vocab_size: int = 257):
        self.vocab_size = vocab_size
        self.eos_token_id = 256
        self.pad_token_id = 256

    def encode(self, text: str) -> List[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids: List[int]) -> str:
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")


class ByteBPETokenizer:
    def __init__(self, vocab: Dict[str, int], merges: List[Tuple[str, str]], special: Optional[Dict[str, int]] = None,
                 eos_token: str = "<|im_end|>", pad_token: str = "<|endoftext|>"):
        self.encoder = dict(vocab)
        self.special = dict(special or {})
        self.encoder.update(self.special)
        self.decoder = {v: k for k, v in self.encoder.items()}
        self.ranks = {pair: i for i, pair in enumerate(merges)}
        self.b2u = byte_to_unicode()
        self.u2b = {v: k for k, v in self.b2u.items()}
        self.pat = _re.compile(_PAT)
        self.cache: Dict[str, List[str]] = {}
        self.eos_token_id = self.encoder.get(eos_token)
        self.pad_token_id = self.encoder.get(pad_token, self.eos_token_id)
        self.vocab_size = max(self.encoder.values()) + 1 if self.encoder else 0
        if self.special:
            self.special_pat = _re.compile("(" + "|".join(_re.escape(s) for s in
                                                          sorted(self.special, key=len, reverse=True)) + ")")
        else:
            self.special_pat = None

    @classmethod
    def from_files(cls, vocab_json: str, merges_txt: str, special: Optional[Dict[str, int]] = None):
        with open(vocab_json, encoding="utf-8") as f:
            vocab = json.load(f)
        merges = []
        with open(merges_txt, encoding="utf-8") as f:
            for line in f:
                line = line.rstrip("\n")
                if not line or line.startswith("#version"):
                    continue
                a, b = line.split(" ")
                merges.append((a, b))
        return cls(vocab, merges, special)

    @classmethod
    def from_tokenizer_json(cls, path: str):
        with open(path, encoding="utf-8") as f:
            tj = json.load(f)
        model = tj["model"]
        merges = [tuple(m.split(" ")) if isinstance(m, str) else tuple(m) for m in model["merges"]]
        special = {t["content"]: t["id"] for t in tj.get("added_tokens", [])}
        return cls(model["vocab"], merges, special)

    def _bpe(self, piece: str) -> List[str]:
        if piece in self.cache:
            return self.cache[piece]
        word = list(piece)
        while len(word) > 1:
            best, best_rank = None, None
            for i in range(len(word) - 1):
                r = self.ranks.get((word[i], word[i + 1]))
                if r is not None and (best_rank is None or r < best_rank):
                    best, best_rank = i, r
            if best is None:
                break
            a, b = word[best], word[best + 1]
            merged, i = [], 0
            while i < len(word):
                if i < len(word) - 1 and word[i] == a and word[i + 1] == b:
                    merged.append(a + b)
                    i += 2
                else:
                    merged.append(word[i])
                    i += 1
            word = merged
        if len(self.cache) < 100000:
            self.cache[piece] = word
        return word

    def _encode_plain(self, text: str) -> List[int]:
        ids = []
        for m in self.pat.findall(text):
            mapped = "".join(self.b2u[b] for b in m.encode("utf-8"))
            for tok in self._bpe(mapped):
                if tok in self.encoder:
                    ids.append(self.encoder[tok])
                else:  # unknown merge result: fall back to single byte-characters
                    ids.extend(self.encoder[c] for c in tok if c in self.encoder)
        return ids

    def encode(self, text: str) -> List[int]:
        if not self.special_pat:
            return self._encode_plain(text)
        ids = []
        for part in self.special_pat.split(text):
            if not part:
                continue
            if part in self.special:
                ids.append(self.special[part])
            else:
                ids.extend(self._encode_plain(part))
        return ids

    def decode(self, ids: List[int]) -> str:
        out = bytearray()
        for i in ids:
            tok = self.decoder.get(int(i))
            if tok is None:
                continue
            if tok in self.special:
                out += tok.encode("utf-8")
            else:
                out += bytes(self.u2b[c] for c in tok if c in self.u2b)
        return out.decode("utf-8", errors="replace")


def load_tokenizer(path: Optional[str]):
    """``tokenizer.json`` or ``vocab.json``+``merges.txt`` under ``path``; else SimpleTokenizer."""
    if path and os.path.isdir(path):
        tj = os.path.join(path, "tokenizer.json")
        if os.path.exists(tj):
            return ByteBPETokenizer.from_tokenizer_json(tj)
        v, m = os.path.join(path, "vocab.json"), os.path.join(path, "merges.txt")
        if os.path.exists(v) and os.path.exists(m):
            return ByteBPETokenizer.from_files(v, m)
    return SimpleTokenizer()
