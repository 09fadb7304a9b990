"""tcgen05 GEMM of the batched paths against an fp64 numpy product of the same
grouped-Q8 weights: y = x . dequant(q, s)^T with |err| <= 2e-5 * sum_k |w x|."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def run(native, rows, n, cols, splits, seed=0, entry="mocha_tc_gemm_check"):
    rng = np.random.default_rng(seed)
    q = rng.integers(-127, 128, size=(rows, cols), dtype=np.int8)
    s = (rng.uniform(0.5, 1.5, size=rows * cols // 64) * 0.02 / 127).astype(np.float32)
    x = rng.standard_normal((n, cols)).astype(np.float32)
    y = np.empty((n, rows), np.float32)
    rc = getattr(native.load(), entry)(0, rows, n, cols, q.ctypes.data, s.ctypes.data, x.ctypes.data,
                                       y.ctypes.data, splits)
    assert rc == 0
    w = (q.astype(np.float32) * np.repeat(s, 64).reshape(rows, cols)).astype(np.float64)
    ref = x.astype(np.float64) @ w.T
    bound = np.abs(x).astype(np.float64) @ np.abs(w).T
    return y, ref, bound


@pytest.mark.parametrize("rows,n,cols,splits", [
    (128, 64, 64, 1),       # one tile, one K step
    (256, 64, 896, 0),      # K split chosen by the plan
    (1152, 64, 896, 1),     # fused q/k/v rows, decode batch
    (896, 37, 4864, 0),     # down projection, ragged batch
    (384, 200, 896, 2),     # BN=128 tiles, ragged last tile
    (128, 1024, 128, 1),    # prefill-sized batch
])
def test_gemm_matches_fp64(native, rows, n, cols, splits):
    y, ref, bound = run(native, rows, n, cols, splits)
    err = np.abs(y - ref)
    assert np.all(np.isfinite(y))
    assert np.all(err <= 2e-5 * bound + 1e-30), float((err / bound).max())


@pytest.mark.parametrize("rows,n,cols,splits", [
    (128, 64, 128, 1),      # one tile, one stage
    (1152, 64, 896, 0),     # fused q/k/v rows, decode batch, K split by the plan
    (896, 37, 4864, 0),     # down projection, ragged batch
    (9728, 200, 896, 1),    # gate|up rows, several token tiles, ragged last tile
    (384, 1024, 896, 2),    # prefill-sized batch
])
def test_int8_limb_gemm_matches_fp64(native, rows, n, cols, splits):
    """int8 weights x three int8 limbs of x: exact int32 group sums, fp32 promotion."""
    y, ref, bound = run(native, rows, n, cols, splits, seed=1, entry="mocha_tq_gemm_check")
    err = np.abs(y - ref)
    assert np.all(np.isfinite(y))
    assert np.all(err <= 2e-5 * bound + 1e-30), float((err / bound).max())

