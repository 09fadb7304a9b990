"""Grouped-Q8 model file: layout constants, reader and seeded random-init writer.

The file format is the reference engine's own (unchanged):

* an 8192-byte header: ``magic 0x384D4D4D, version 1, bytes, dim, hidden, layers,
  vocab, group`` (eight little-endian u32) followed by 290 tensor records
  ``{data, scales, rows, cols}`` (u32 byte offsets), ``src/minimind.h:5,15``;
* tensor order ``t[0]`` embedding / tied head, then per layer ``l`` at ``1+12*l``:
  attn norm, q, k, v, o, gate, up, down, ffn norm, q bias, k bias, v bias, and
  ``t[289]`` the final norm (``tools/convert-qwen.py:46-55``);
* matrices are int8 row-major followed by fp32 scales, one per 64 consecutive
  weights; norms and biases are plain fp32 with ``scales == 0``.

The writer quantises exactly as ``tools/convert-qwen.py:34-39`` does (symmetric,
``scale = max(max|w|/127, 1e-12)`` in float32, ``rint`` then clip to +-127), but
draws the fp32 weights from a seeded generator instead of reading a checkpoint:
weights N(0, 0.02), norm gains 1 + N(0, 0.01), biases N(0, 0.02).
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass

import numpy as np

MAGIC = 0x384D4D4D
VERSION = 1
DIM, HIDDEN, KV, HEAD_DIM, VOCAB, CONTEXT, LAYERS = 896, 4864, 128, 64, 151936, 1024, 24
STRIDE, TENSORS, HEADER_BYTES, GROUP = 12, 290, 8192, 64
BOS, EOS = 151644, 151645
CONTROL_FIRST = 151643          # ids >= this (except EOS) are masked before sampling
FILE_BYTES = 525_128_192

# per-layer tensor slots, relative to 1 + 12*layer
ATTN_NORM, WQ, WK, WV, WO, WGATE, WUP, WDOWN, FFN_NORM, BQ, BK, BV = range(12)
FINAL_NORM = TENSORS - 1


@dataclass(frozen=True)
class Tensor:
    data: int
    scales: int
    rows: int
    cols: int


def tensor_shapes():
    """(rows, cols, quantised, kind) for every tensor slot in file order."""
    out = [(VOCAB, DIM, True, "w")]
    for _ in range(LAYERS):
        out.append((DIM, DIM, False, "norm"))
        out += [(DIM, DIM, True, "w"), (KV, DIM, True, "w"), (KV, DIM, True, "w"),
                (DIM, DIM, True, "w"), (HIDDEN, DIM, True, "w"), (HIDDEN, DIM, True, "w"),
                (DIM, HIDDEN, True, "w")]
        out.append((DIM, DIM, False, "norm"))
        out += [(DIM, DIM, False, "bias"), (KV, KV, False, "bias"), (KV, KV, False, "bias")]
    out.append((DIM, DIM, False, "norm"))
    assert len(out) == TENSORS
    return out


def quantize_groups(w: np.ndarray):
    """Symmetric int8 per group of 64 with float32 scales (convert-qwen.py:34-39)."""
    g = np.ascontiguousarray(w, dtype=np.float32).reshape(-1, GROUP)
    scale = np.maximum(np.abs(g).max(axis=1) / np.float32(127), np.float32(1e-12)).astype(np.float32)
    q = np.rint(g / scale[:, None]).clip(-127, 127).astype(np.int8)
    return q, scale


def write_model(path: str, tensors) -> str:
    """Write a grouped-Q8 file from fp32 tensors given in file order; returns ``path``.

    ``tensors`` yields ``(values, quantised)`` per tensor slot: ``values`` an fp32 array
    of shape (rows, cols) or (n,) -- or, for large matrices, an iterable of row blocks
    that are quantised and written one after the other -- and ``quantised`` whether it is
    stored as int8 + per-64 scales.  The record is (data, scales, rows, cols) with
    rows = shape[0] and cols = shape[-1] (n and n for vectors), like
    ``tools/convert-qwen.py:45``; the header's shape fields are the Qwen2.5-0.5B ones.
    """
    records = []
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(bytes(HEADER_BYTES))
        count = 0
        for values, quant in tensors:
            blocks = [values] if isinstance(values, np.ndarray) else values
            rows, cols = 0, 0
            offset = f.tell()
            scale_parts = []
            for b in blocks:
                rows += b.shape[0]
                cols = b.shape[-1]
                if quant:
                    q, sc = quantize_groups(b)
                    f.write(q.tobytes())
                    scale_parts.append(sc)
                else:
                    f.write(np.ascontiguousarray(b, dtype="<f4").tobytes())
            scale_offset = f.tell() if quant else 0
            for sc in scale_parts:
                f.write(sc.astype("<f4").tobytes())
            records.append((offset, scale_offset, rows, cols))
            count += 1
        if count != TENSORS:
            raise ValueError(f"{count} tensors, the format has {TENSORS}")
        size = f.tell()
        f.seek(0)
        f.write(struct.pack("<8I", MAGIC, VERSION, size, DIM, HIDDEN, LAYERS, VOCAB, GROUP))
        for rec in records:
            f.write(struct.pack("<4I", *rec))
    os.replace(tmp, path)
    return path


def random_tensors(seed: int = 1):
    """Seeded random-init fp32 tensors of the Qwen2.5-0.5B shapes in file order:
    weights N(0, 0.02) (the embedding in row blocks, to bound temporaries), norm gains
    1 + N(0, 0.01), biases N(0, 0.02)."""
    rng = np.random.default_rng(seed)

    def blocks(rows, cols):  # drawn lazily, in file order
        step = max(1, (1 << 24) // cols)
        for r0 in range(0, rows, step):
            yield rng.standard_normal((min(step, rows - r0), cols), dtype=np.float32) * np.float32(0.02)

    for rows, cols, quant, kind in tensor_shapes():
        if quant:
            yield blocks(rows, cols), True
        else:
            v = rng.standard_normal(rows, dtype=np.float32)
            v = (np.float32(1) + np.float32(0.01) * v) if kind == "norm" else np.float32(0.02) * v
            yield v, False


def write_random_model(path: str, seed: int = 1) -> str:
    """Write a random-init Qwen2.5-0.5B-shaped grouped-Q8 file; returns ``path``."""
    return write_model(path, random_tensors(seed))


def model_path(seed: int = 1, cache_dir: str | None = None) -> str:
    """Path of the cached random model for ``seed``, writing it on first use."""
    cache_dir = cache_dir or os.environ.get("MOCHA_MODEL_CACHE") or "/tmp/mocha-b200-models"
    os.makedirs(cache_dir, exist_ok=True)
    path = os.path.join(cache_dir, f"qwen05b-q8-seed{seed}.bin")
    if not os.path.exists(path) or os.path.getsize(path) != FILE_BYTES:
        write_random_model(path, seed)
    return path


def read_header(buf) -> tuple[dict, list[Tensor]]:
    """Parse and validate the header like ``src/minimind.cpp:89-93``."""
    mv = memoryview(buf)
    magic, version, nbytes, dim, hidden, layers, vocab, group = struct.unpack_from("<8I", mv, 0)
    hdr = dict(magic=magic, version=version, bytes=nbytes, dim=dim, hidden=hidden,
               layers=layers, vocab=vocab, group=group)
    if (len(mv) < HEADER_BYTES or magic != MAGIC or version != VERSION or nbytes != len(mv)
            or dim != DIM or hidden != HIDDEN or layers != LAYERS or vocab != VOCAB or group != GROUP):
        raise ValueError("not a Qwen2.5-0.5B grouped-Q8 file")
    ts = [Tensor(*struct.unpack_from("<4I", mv, 32 + 16 * i)) for i in range(TENSORS)]
    for t in ts:
        size = t.rows * (t.cols if t.scales else 4)
        if t.data < HEADER_BYTES or t.data + size > len(mv):
            raise ValueError("tensor out of range")
        if t.scales and (t.cols % 64 or t.scales + size // 64 * 4 > len(mv)):
            raise ValueError("scales out of range")
    return hdr, ts


def random_prompt(n: int, seed: int, vocab: int = VOCAB) -> list[int]:
    """Uniform random token ids in [0, vocab)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n).astype(np.int64).tolist()
