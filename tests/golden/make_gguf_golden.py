"""Generate GGUF dequantisation golden vectors with the gguf Python package 0.19.0.

ggml (the reference bridge's own test dependency, tests/gguf-cuda-check.cpp) is not
available here; gguf-py's numpy dequantisers implement the same block formulas and
serve as the independent pin.  Blocks are seeded random bytes with bounded fp16
scales plus hand-picked edge blocks (zero, negative and subnormal scales, extreme
quants).

Usage: python tests/golden/make_gguf_golden.py   (writes tests/golden/gguf_golden.npz)
"""
import os

import numpy as np
from gguf import GGMLQuantizationType as T
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))
ROWS, COLS = 6, 512


def fp16_bytes(vals):
    return np.asarray(vals, dtype=np.float16).view(np.uint8).reshape(-1, 2)


def make_q4k(rng):
    nb = ROWS * COLS // 256
    blk = rng.integers(0, 256, size=(nb, 144), dtype=np.uint8)
    blk[:, 0:2] = fp16_bytes(rng.uniform(0, 2e-3, nb))
    blk[:, 2:4] = fp16_bytes(rng.uniform(0, 2e-3, nb))
    blk[0, 0:2] = fp16_bytes([0.0])
    blk[1, 0:2] = fp16_bytes([-1.5e-3])
    blk[2, 0:4] = np.array([0x01, 0x00, 0x07, 0x00], dtype=np.uint8)  # subnormal d and dmin
    blk[3, 4:16] = 0xFF                                               # all scales/mins at 63
    return blk.reshape(ROWS, -1)


def make_q6k(rng):
    nb = ROWS * COLS // 256
    blk = rng.integers(0, 256, size=(nb, 210), dtype=np.uint8)
    blk[:, 208:210] = fp16_bytes(rng.uniform(-4e-4, 4e-4, nb))
    blk[0, 208:210] = np.array([0x03, 0x00], dtype=np.uint8)  # subnormal
    blk[1, 192:208] = np.array([0x80] * 8 + [0x7F] * 8, dtype=np.uint8)  # scales -128 / 127
    blk[2, 0:192] = 0xFF  # q = 63 everywhere
    return blk.reshape(ROWS, -1)


def make_q80(rng):
    nb = ROWS * COLS // 32
    blk = rng.integers(0, 256, size=(nb, 34), dtype=np.uint8)
    blk[:, 0:2] = fp16_bytes(rng.uniform(-2e-3, 2e-3, nb))
    blk[0, 0:2] = np.array([0x00, 0x80], dtype=np.uint8)  # -0.0
    blk[1, 2:34] = 0x80                                     # q = -128
    return blk.reshape(ROWS, -1)


def main():
    rng = np.random.default_rng(20261201)
    out = {}
    for name, make, qt in (("q4_k", make_q4k, T.Q4_K), ("q6_k", make_q6k, T.Q6_K), ("q8_0", make_q80, T.Q8_0)):
        raw = make(rng)
        deq = quants.dequantize(raw, qt).astype(np.float32)
        assert deq.shape == (ROWS, COLS)
        out[name + "_raw"] = raw
        out[name + "_deq"] = deq
    out["shape"] = np.array([ROWS, COLS])
    np.savez_compressed(os.path.join(HERE, "gguf_golden.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
