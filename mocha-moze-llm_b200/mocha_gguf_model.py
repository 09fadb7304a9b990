"""Seeded random-init GGUF models with the reference's two large architectures.

* ``llama1b``: Llama-3.2-1B shapes (16 layers, 2048 hidden, 32/8 heads of 64, FFN 8192,
  vocab 128256, tied embeddings, RoPE base 5e5 with llama3 frequency factors --
  factor 32, low/high frequency factors 1/4, original context 8192 -- stored as the
  ``rope_freqs.weight`` tensor, RMSNorm eps 1e-5).
* ``qwen15b``: Qwen2.5-1.5B shapes (28 layers, 1536 hidden, 12/2 heads of 128, FFN 8960,
  vocab 151936, tied embeddings, QKV biases, RoPE base 1e6, RMSNorm eps 1e-6).

Each file also carries a small byte-level BPE tokenizer in the ``tokenizer.ggml.*``
metadata (``synthetic_tokenizer``): the 256 byte tokens, merges that spell a list of
common English words, and the architecture's special tokens at their usual ids (Llama 3:
``<|begin_of_text|>`` 128000 ... ``<|eot_id|>`` 128009, pre-tokenizer ``llama-bpe``, BOS
added; Qwen2: ``<|endoftext|>`` 151643, ``<|im_start|>`` 151644, ``<|im_end|>`` 151645,
pre-tokenizer ``qwen2``), so text prompts reach these random models the way they reach
real ones.

Tensor types follow the Q4_K_M mix of the benchmark configuration: Q4_K everywhere,
Q6_K for ``token_embd`` and for ``attn_v`` / ``ffn_down`` of even layers, and (Qwen)
Q8_0 for the bias-carrying ``attn_k``.  Norm gains are 1 + N(0, 0.01) and biases
N(0, 0.02) in fp32.  Quantised blocks are drawn directly from a seeded generator
(random quants, scales chosen so the weights span about +-0.04, i.e. a standard
deviation near 0.02) instead of quantising fp32 weights, so a 1-1.5B-parameter file
is written in seconds.  The files are standard GGUF v3 written with gguf-py.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np

Q8_0, Q4_K, Q6_K = 8, 12, 14
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


@dataclass(frozen=True)
class Arch:
    name: str
    gguf_arch: str
    layers: int
    dim: int
    heads: int
    kv_heads: int
    ffn: int
    vocab: int
    rope_base: float
    eps: float
    bias: bool
    llama3_rope: bool
    context: int = 1024

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads


ARCHS = {
    "llama1b": Arch("llama1b", "llama", 16, 2048, 32, 8, 8192, 128256, 500000.0, 1e-5, False, True),
    "qwen15b": Arch("qwen15b", "qwen2", 28, 1536, 12, 2, 8960, 151936, 1000000.0, 1e-6, True, False),
}


def f16_bytes(values) -> np.ndarray:
    return np.asarray(values, dtype=np.float16).view(np.uint8).reshape(-1, 2)


def random_q4k(rng, nblocks: int) -> np.ndarray:
    blk = np.empty((nblocks, 144), dtype=np.uint8)
    d = (8.5e-5 * rng.uniform(0.8, 1.2, nblocks)).astype(np.float32)
    blk[:, 0:2] = f16_bytes(d)
    blk[:, 2:4] = f16_bytes(d * 8)
    sc = rng.integers(32, 64, size=(nblocks, 8))
    mn = np.rint(sc * 0.9375).astype(np.int64)  # dmin*m ~ d*sc*7.5: centred weights
    s = np.zeros((nblocks, 12), dtype=np.int64)
    s[:, 0:4] = sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = mn[:, 0:4] | ((mn[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    blk[:, 4:16] = s.astype(np.uint8)
    blk[:, 16:144] = rng.integers(0, 256, size=(nblocks, 128), dtype=np.uint8)
    return blk


def random_q6k(rng, nblocks: int) -> np.ndarray:
    blk = np.empty((nblocks, 210), dtype=np.uint8)
    blk[:, 0:192] = rng.integers(0, 256, size=(nblocks, 192), dtype=np.uint8)
    sc = rng.integers(20, 128, size=(nblocks, 16)) * rng.choice([-1, 1], size=(nblocks, 16))
    blk[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    blk[:, 208:210] = f16_bytes(np.full(nblocks, 1e-5, dtype=np.float32) * rng.uniform(0.8, 1.2, nblocks))
    return blk


def random_q80(rng, nblocks: int) -> np.ndarray:
    blk = np.empty((nblocks, 34), dtype=np.uint8)
    blk[:, 0:2] = f16_bytes(np.full(nblocks, 0.04 / 127, dtype=np.float32) * rng.uniform(0.8, 1.2, nblocks))
    blk[:, 2:34] = rng.integers(0, 256, size=(nblocks, 32), dtype=np.uint8)
    return blk


def random_matrix(rng, qtype: int, rows: int, cols: int) -> np.ndarray:
    per, size = BLOCK[qtype]
    nb = rows * (cols // per)
    gen = {Q4_K: random_q4k, Q6_K: random_q6k, Q8_0: random_q80}[qtype]
    return gen(rng, nb).reshape(rows, (cols // per) * size)


def llama3_rope_factors(head_dim: int, base: float, factor: float = 32.0, low: float = 1.0, high: float = 4.0,
                        original: int = 8192) -> np.ndarray:
    """Per-frequency divisors of the llama3 RoPE scaling rule (published with
    Llama 3.1): keep high frequencies, divide low frequencies by `factor`, blend
    smoothly in between."""
    out = []
    low_wavelen, high_wavelen = original / low, original / high
    for i in range(0, head_dim, 2):
        freq = 1.0 / (base ** (i / head_dim))
        wavelen = 2 * math.pi / freq
        if wavelen < high_wavelen:
            out.append(1.0)
        elif wavelen > low_wavelen:
            out.append(factor)
        else:
            smooth = (original / wavelen - low) / (high - low)
            out.append(1.0 / ((1 - smooth) / factor + smooth))
    return np.asarray(out, dtype=np.float32)


def tensor_types(arch: Arch, layer: int) -> dict:
    even = layer % 2 == 0
    return {
        "attn_q": Q4_K,
        "attn_k": Q8_0 if arch.bias else Q4_K,
        "attn_v": Q6_K if even else Q4_K,
        "attn_output": Q4_K,
        "ffn_gate": Q4_K,
        "ffn_up": Q4_K,
        "ffn_down": Q6_K if even else Q4_K,
    }


WORDS = ("the of and to in a is that for it as was with be by on not he this are or his from at which but "
         "have an they you were her she there had been one all we can has their will would who more if no when "
         "out so what up said about into than them only other time new some could these two may first then do "
         "any like my now over such our man me even most made after also did many before must through back "
         "years where much your way well down should because each just those people how too little state good "
         "very make world still own see men work long get here between both life being under never day same "
         "another know while last might us great old year off come since against go came right used take three "
         "please introduce yourself briefly hello assistant user system model language answer question").split()

LLAMA3_SPECIAL = {128000: "<|begin_of_text|>", 128001: "<|end_of_text|>", 128004: "<|finetune_right_pad_id|>",
                  128006: "<|start_header_id|>", 128007: "<|end_header_id|>", 128008: "<|eom_id|>",
                  128009: "<|eot_id|>", 128010: "<|python_tag|>"}
QWEN2_SPECIAL = {151643: "<|endoftext|>", 151644: "<|im_start|>", 151645: "<|im_end|>"}


def synthetic_tokenizer(arch: Arch):
    """(tokens, token types, merges, {pre, bos, eos, add_bos}) of the models' tokenizer:
    byte tokens 0..255 in GPT-2's byte alphabet, then one token per merge (the words of
    WORDS and their space-prefixed forms, spelled left to right), unused fillers, and
    the architecture's special tokens (type 3) at their usual ids."""
    from gguf_tokenizer import byte_alphabet
    alpha = byte_alphabet()
    tokens = [alpha[b] for b in range(256)]
    seen = set(tokens)
    merges = []
    for w in WORDS:
        for form in (w, " " + w):
            chars = "".join(alpha[b] for b in form.encode("utf-8"))
            for k in range(1, len(chars)):
                left, right = chars[:k], chars[k]
                if chars[:k + 1] in seen:
                    continue
                merges.append(f"{left} {right}")
                tokens.append(chars[:k + 1])
                seen.add(chars[:k + 1])
    types = [1] * len(tokens)
    special = LLAMA3_SPECIAL if arch.gguf_arch == "llama" else QWEN2_SPECIAL
    first = min(special)
    tokens += [f"<|unused_{i}|>" for i in range(len(tokens), arch.vocab)]
    types += [5] * (arch.vocab - len(types))
    for i in range(first, arch.vocab):
        if arch.gguf_arch == "llama" and i not in special:
            tokens[i], types[i] = f"<|reserved_special_token_{i - first}|>", 3
    for i, t in special.items():
        tokens[i], types[i] = t, 3
    if arch.gguf_arch == "llama":
        meta = {"pre": "llama-bpe", "bos": 128000, "eos": 128009, "add_bos": True}
    else:
        meta = {"pre": "qwen2", "bos": 151643, "eos": 151645, "add_bos": False}
    return tokens, types, merges, meta


def write_model(path: str, arch_name: str, seed: int = 1) -> str:
    from gguf import GGMLQuantizationType, GGUFWriter

    arch = ARCHS[arch_name]
    rng = np.random.default_rng(seed)
    w = GGUFWriter(path + ".tmp", arch.gguf_arch)
    w.add_name(f"mocha-random-{arch.name}")
    w.add_context_length(arch.context)
    w.add_embedding_length(arch.dim)
    w.add_block_count(arch.layers)
    w.add_feed_forward_length(arch.ffn)
    w.add_head_count(arch.heads)
    w.add_head_count_kv(arch.kv_heads)
    w.add_rope_freq_base(arch.rope_base)
    w.add_layer_norm_rms_eps(arch.eps)
    w.add_rope_dimension_count(arch.head_dim)
    w.add_vocab_size(arch.vocab)
    w.add_file_type(15)  # MOSTLY_Q4_K_M
    tokens, types, merges, meta = synthetic_tokenizer(arch)
    w.add_tokenizer_model("gpt2")
    w.add_tokenizer_pre(meta["pre"])
    w.add_token_list(tokens)
    w.add_token_types(types)
    w.add_token_merges(merges)
    w.add_bos_token_id(meta["bos"])
    w.add_eos_token_id(meta["eos"])
    w.add_add_bos_token(meta["add_bos"])

    def add_q(name, qtype, rows, cols):
        w.add_tensor(name, random_matrix(rng, qtype, rows, cols), raw_dtype=GGMLQuantizationType(qtype))

    def add_f32(name, values):
        w.add_tensor(name, np.asarray(values, dtype=np.float32))

    kv = arch.kv_heads * arch.head_dim
    add_q("token_embd.weight", Q6_K, arch.vocab, arch.dim)
    if arch.llama3_rope:
        add_f32("rope_freqs.weight", llama3_rope_factors(arch.head_dim, arch.rope_base))
    for l in range(arch.layers):
        t = tensor_types(arch, l)
        p = f"blk.{l}."
        add_f32(p + "attn_norm.weight", 1 + 0.01 * rng.standard_normal(arch.dim, dtype=np.float32))
        add_q(p + "attn_q.weight", t["attn_q"], arch.dim, arch.dim)
        add_q(p + "attn_k.weight", t["attn_k"], kv, arch.dim)
        add_q(p + "attn_v.weight", t["attn_v"], kv, arch.dim)
        if arch.bias:
            add_f32(p + "attn_q.bias", 0.02 * rng.standard_normal(arch.dim, dtype=np.float32))
            add_f32(p + "attn_k.bias", 0.02 * rng.standard_normal(kv, dtype=np.float32))
            add_f32(p + "attn_v.bias", 0.02 * rng.standard_normal(kv, dtype=np.float32))
        add_q(p + "attn_output.weight", t["attn_output"], arch.dim, arch.dim)
        add_f32(p + "ffn_norm.weight", 1 + 0.01 * rng.standard_normal(arch.dim, dtype=np.float32))
        add_q(p + "ffn_gate.weight", t["ffn_gate"], arch.ffn, arch.dim)
        add_q(p + "ffn_up.weight", t["ffn_up"], arch.ffn, arch.dim)
        add_q(p + "ffn_down.weight", t["ffn_down"], arch.dim, arch.ffn)
    add_f32("output_norm.weight", 1 + 0.01 * rng.standard_normal(arch.dim, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    os.replace(path + ".tmp", path)
    return path


def model_path(arch_name: str, seed: int = 1, cache_dir: str | None = None) -> str:
    cache_dir = cache_dir or os.environ.get("MOCHA_MODEL_CACHE") or "/tmp/mocha-b200-models"
    os.makedirs(cache_dir, exist_ok=True)
    path = os.path.join(cache_dir, f"{arch_name}-q4km-seed{seed}-tok.gguf")
    if not os.path.exists(path):
        write_model(path, arch_name, seed)
    return path


def weight_bytes_per_token(path: str) -> int:
    """Bytes a decode step reads once: every tensor except the embedding rows not
    selected (the tied embedding is read in full by the vocabulary head)."""
    from gguf import GGUFReader
    r = GGUFReader(path)
    return int(sum(int(t.n_bytes) for t in r.tensors))
