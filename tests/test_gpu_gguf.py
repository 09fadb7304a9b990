"""mocha_gguf_matmul on B200 against the oracle, after tests/gguf-cuda-check.cpp:
Q4_K/Q6_K/Q8_0 at cols=512 rows=17 vectors=3 with padded strides and a sentinel,
and Q4_K 4096x4097x2; tolerance 0.002*(1+|e|) (tests/gguf-cuda-check.cpp:29)."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "gguf_golden.npz")
BYTES = {12: 144, 14: 210, 8: 34}
ELEMS = {12: 256, 14: 256, 8: 32}


def random_rows(t, rows, cols, rng):
    nb = cols // ELEMS[t]
    blk = rng.integers(0, 256, size=(rows * nb, BYTES[t]), dtype=np.uint8)
    f16 = lambda v: np.asarray(v, np.float16).view(np.uint8).reshape(-1, 2)
    if t == 12:
        blk[:, 0:2] = f16(rng.uniform(0, 2e-3, rows * nb))
        blk[:, 2:4] = f16(rng.uniform(0, 2e-3, rows * nb))
    elif t == 14:
        blk[:, 208:210] = f16(rng.uniform(-4e-4, 4e-4, rows * nb))
    else:
        blk[:, 0:2] = f16(rng.uniform(-2e-3, 2e-3, rows * nb))
    return blk.reshape(rows, -1)


def check(native, oracle_lib, t, cols, rows, vectors, seed):
    lib = native.load()
    rng = np.random.default_rng(seed)
    base = random_rows(t, 3, cols, rng)
    packed = np.ascontiguousarray(base[np.arange(rows) % 3])            # rows repeat r % 3
    deq = oracle_lib.gguf_dequant(t, base.tobytes(), 3, cols).astype(np.float64)
    xs = cols + 8
    x = np.zeros(vectors * xs, np.float32)
    for v in range(vectors):
        x[v * xs: v * xs + cols] = np.cos(np.arange(cols) * 0.23 + v) * 0.21
    ys = rows + 7
    y = np.full(vectors * ys, 321.0, np.float32)
    rc = lib.mocha_gguf_matmul(t, packed.ctypes.data, cols, rows, x.ctypes.data, vectors, xs * 4, y.ctypes.data, ys * 4)
    assert rc == 0
    for v in range(vectors):
        exp = deq[np.arange(rows) % 3] @ x[v * xs: v * xs + cols].astype(np.float64)
        got = y[v * ys: v * ys + rows]
        assert np.all(np.isfinite(got))
        assert np.all(np.abs(got - exp) <= 0.002 * (1 + np.abs(exp)))
        assert np.all(y[v * ys + rows: (v + 1) * ys] == 321.0)


@pytest.mark.parametrize("t", [12, 14, 8])
def test_matmul_small(native, oracle_lib, t):
    check(native, oracle_lib, t, 512, 17, 3, t)


def test_matmul_q4k_large(native, oracle_lib):
    check(native, oracle_lib, 12, 4096, 4097, 2, 99)


@pytest.mark.parametrize("t", [12, 14, 8])
def test_matmul_model_shapes(native, oracle_lib, t):
    check(native, oracle_lib, t, 8960 if t != 8 else 1536, 256, 1, 5 + t)


@pytest.mark.parametrize("name,t", [("q4_k", 12), ("q6_k", 14), ("q8_0", 8)])
def test_device_dequant_bit_exact(native, name, t):
    g = np.load(GOLD)
    rows, cols = (int(v) for v in g["shape"])
    raw = np.ascontiguousarray(g[name + "_raw"])
    out = np.empty((rows, cols), np.float32)
    assert native.load().mocha_gguf_dequant(t, raw.ctypes.data, cols, rows, out.ctypes.data) == 0
    assert np.array_equal(out.view(np.uint32), g[name + "_deq"].view(np.uint32))


def test_argument_errors(native):
    lib = native.load()
    w = np.zeros(144, np.uint8)
    x = np.zeros(256, np.float32)
    y = np.zeros(1, np.float32)
    assert lib.mocha_gguf_matmul(13, w.ctypes.data, 256, 1, x.ctypes.data, 1, 1024, y.ctypes.data, 4) == 1
    assert lib.mocha_gguf_matmul(12, w.ctypes.data, 255, 1, x.ctypes.data, 1, 1024, y.ctypes.data, 4) == 1
    assert lib.mocha_gguf_matmul(12, w.ctypes.data, 256, 1, x.ctypes.data, 33, 1024, y.ctypes.data, 4) == 1
