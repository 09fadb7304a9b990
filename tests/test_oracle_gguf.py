"""GGUF dequant oracle (C restatement of src/gguf-cuda.cu:23-44) against gguf-py 0.19.0
golden vectors (tests/golden/make_gguf_golden.py)."""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden", "gguf_golden.npz")
TYPES = (("q4_k", 12), ("q6_k", 14), ("q8_0", 8))


@pytest.mark.parametrize("name,t", TYPES)
def test_dequant_bit_exact(oracle_lib, name, t):
    g = np.load(GOLD)
    rows, cols = g["shape"]
    got = oracle_lib.gguf_dequant(t, g[name + "_raw"].tobytes(), rows, cols)
    assert np.array_equal(got.view(np.uint32), g[name + "_deq"].view(np.uint32))


@pytest.mark.parametrize("name,t", TYPES)
def test_matmul_matches_float64(oracle_lib, name, t):
    g = np.load(GOLD)
    rows, cols = g["shape"]
    x = np.cos(np.arange(3 * cols).reshape(3, cols) * 0.23).astype(np.float32) * 0.21
    y = oracle_lib.gguf_matmul(t, g[name + "_raw"].tobytes(), cols, rows, x)
    exp = x.astype(np.float64) @ g[name + "_deq"].astype(np.float64).T
    assert np.all(np.abs(y - exp) <= 0.002 * (1 + np.abs(exp)))  # tests/gguf-cuda-check.cpp:29


def test_matmul_argument_checks(oracle_lib):
    raw = bytes(144 * 2)
    with pytest.raises(ValueError):
        oracle_lib.gguf_matmul(12, raw, 256, 2, np.zeros((33, 256), np.float32))  # vectors > 32
    with pytest.raises(ValueError):
        oracle_lib.gguf_matmul(13, raw, 256, 2, np.zeros((1, 256), np.float32))   # type
    assert oracle_lib.lib().gguf_o_row_bytes(8, 100) == 0


def test_half_conversion_edges(oracle_lib):
    L = oracle_lib.lib()
    for bits in (0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0xFBFF, 0x7C00, 0xFC00):
        exp = np.array([bits], dtype=np.uint16).view(np.float16).astype(np.float32)[0]
        assert np.float32(L.gguf_o_half(bits)).view(np.uint32) == exp.view(np.uint32)
