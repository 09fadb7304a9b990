"""Byte-level BPE tokenizer read from a GGUF file's ``tokenizer.ggml.*`` metadata.

The reference hands GGUF models text prompts through llama-cli (``mocha-llm:38-47``:
Llama-3 and ChatML templates built as text); this module gives the GGUF engine the same
text interface without llama.cpp.  What it reads:

* ``tokenizer.ggml.model`` -- must be ``gpt2`` (byte-level BPE, the kind Llama 3 and
  Qwen2 ship);
* ``tokenizer.ggml.pre`` -- the pre-tokenizer: ``qwen2`` (single digits),
  ``llama-bpe`` (digit runs of up to three), anything else the GPT-2 rule;
* ``tokenizer.ggml.tokens`` / ``token_type`` / ``merges`` -- the vocabulary in id order
  (strings over the GPT-2 byte alphabet), token kinds (3 control, 4 user-defined: both
  are matched literally in prompt text) and the merge list in rank order;
* ``tokenizer.ggml.bos_token_id`` / ``eos_token_id`` / ``add_bos_token``.

Encoding follows the usual llama.cpp prompt rules: special tokens written in the text
are recognised (longest first), every other span is split by the pre-tokenizer pattern,
mapped to the byte alphabet and merged by rank; with ``add_special`` a BOS is prepended
when the model asks for one, even if the text already starts with the BOS text (llama.cpp
then warns about a doubled BOS, and so does this module).  The byte alphabet and the
merge loop are the same as the reference's own BPE (``src/tokenizer.py:12-21, 95-112``);
the Qwen2 pattern is the one ``src/tokenizer.py:48-80`` restates by hand.
"""
from __future__ import annotations

import sys
from functools import lru_cache

import regex

CONTROL, USER_DEFINED = 3, 4

# Pre-tokenizer patterns (the published regular expressions of these tokenizers).
PATTERNS = {
    "qwen2": r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+"
             r"|\s+(?!\S)|\s+",
    "llama-bpe": r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*"
                 r"|\s*[\r\n]+|\s+(?!\S)|\s+",
    "gpt2": r"'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+",
}


def byte_alphabet() -> dict[int, str]:
    """GPT-2's reversible byte -> printable character map."""
    values = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    chars = values[:]
    n = 0
    for b in range(256):
        if b not in values:
            values.append(b)
            chars.append(256 + n)
            n += 1
    return dict(zip(values, map(chr, chars)))


def _field(reader, key):
    f = reader.fields.get(key)
    return None if f is None else f.contents()


class GgufTokenizer:
    def __init__(self, tokens, types, merges, pre="gpt2", bos=None, eos=None, add_bos=False):
        self.tokens = list(tokens)
        self.types = list(types) if types is not None else [1] * len(self.tokens)
        self.ids = {t: i for i, t in enumerate(self.tokens)}
        self.ranks = {tuple(m.split(" ", 1)): i for i, m in enumerate(merges)}
        self.pre = pre if pre in PATTERNS else "gpt2"
        self.pattern = regex.compile(PATTERNS[self.pre])
        self.bos, self.eos, self.add_bos = bos, eos, bool(add_bos)
        self.byte_chars = byte_alphabet()
        self.char_bytes = {v: k for k, v in self.byte_chars.items()}
        special = sorted((t for t, k in zip(self.tokens, self.types) if k in (CONTROL, USER_DEFINED) and t),
                         key=len, reverse=True)
        self.special = regex.compile("|".join(regex.escape(t) for t in special)) if special else None
        self._bpe = lru_cache(maxsize=65536)(self._bpe_uncached)

    @classmethod
    def from_gguf(cls, path: str) -> "GgufTokenizer":
        from gguf import GGUFReader
        r = GGUFReader(path)
        model = _field(r, "tokenizer.ggml.model")
        if model != "gpt2":
            raise ValueError(f"tokenizer.ggml.model {model!r}: only byte-level BPE (gpt2) is supported")
        return cls(_field(r, "tokenizer.ggml.tokens"), _field(r, "tokenizer.ggml.token_type"),
                   _field(r, "tokenizer.ggml.merges") or [], _field(r, "tokenizer.ggml.pre") or "gpt2",
                   _field(r, "tokenizer.ggml.bos_token_id"), _field(r, "tokenizer.ggml.eos_token_id"),
                   _field(r, "tokenizer.ggml.add_bos_token"))

    def _bpe_uncached(self, word: str) -> tuple:
        parts = list(word)
        while len(parts) > 1:
            best, rank = None, None
            for pair in zip(parts, parts[1:]):
                r = self.ranks.get(pair)
                if r is not None and (rank is None or r < rank):
                    best, rank = pair, r
            if best is None:
                break
            out, i = [], 0
            while i < len(parts):
                if i + 1 < len(parts) and (parts[i], parts[i + 1]) == best:
                    out.append(parts[i] + parts[i + 1])
                    i += 2
                else:
                    out.append(parts[i])
                    i += 1
            parts = out
        ids = []
        for p in parts:
            if p in self.ids:
                ids.append(self.ids[p])
            else:  # not in the vocabulary: fall back to its single byte-characters
                ids.extend(self.ids[c] for c in p)
        return tuple(ids)

    def _encode_plain(self, text: str) -> list[int]:
        out = []
        for piece in self.pattern.findall(text):
            out.extend(self._bpe("".join(self.byte_chars[b] for b in piece.encode("utf-8"))))
        return out

    def encode(self, text: str, add_special: bool = True, parse_special: bool = True) -> list[int]:
        out = []
        if add_special and self.add_bos and self.bos is not None:
            out.append(self.bos)
        pos = 0
        if parse_special and self.special is not None:
            for m in self.special.finditer(text):
                out.extend(self._encode_plain(text[pos:m.start()]))
                out.append(self.ids[m.group(0)])
                pos = m.end()
        out.extend(self._encode_plain(text[pos:]))
        if add_special and self.add_bos and len(out) > 1 and out[0] == out[1] == self.bos:
            print("gguf_tokenizer: the prompt starts with a BOS token and one was added: two BOS tokens",
                  file=sys.stderr)
        return out

    def token_bytes(self, token: int) -> bytes:
        """Bytes a token prints; control tokens print nothing."""
        if self.types[token] == CONTROL:
            return b""
        t = self.tokens[token]
        if self.types[token] == USER_DEFINED:
            return t.encode("utf-8")
        return bytes(self.char_bytes[c] for c in t if c in self.char_bytes)

    def decode(self, ids) -> str:
        return b"".join(self.token_bytes(int(t)) for t in ids).decode("utf-8", "replace")
