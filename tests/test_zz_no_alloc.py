"""mocha_topk_static: candidate selection with every device buffer in a fixed
__device__ array, for callers that cannot allocate GPU memory when they call it (a
host owning the whole memory budget in its own pool, or a latency-critical loop that
must not take cudaMalloc's implicit device synchronisation).  Checked against
gpu_collect, which runs the same selection with buffers the library allocated, on two
calls in a row (the shared array keeps the previous call's contents, which must not
leak into the next result); then a much shorter call after the full-vocabulary ones,
whose stale tail must not leak either, against a numpy selection."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
VOCAB = 151936


def test_static_topk_matches_collect(native, q8_model_bytes, golden_q8):
    lib = native.load()
    buf = q8_model_bytes
    assert lib.gpu_init(buf.ctypes.data, buf.nbytes) == 0
    try:
        prompt = golden_q8["cases"]["sampled64"]["prompt"]
        logits = np.empty(VOCAB, np.float32)
        for pos, tok in enumerate(prompt[:-1]):
            assert lib.gpu_forward(logits.ctypes.data, tok, pos, 0, 0) == 0
        hist = np.asarray(prompt[-64:], np.int32)
        for call, (k, pen) in enumerate(((40, 1.12), (1, 1.0))):
            # gpu_collect selects from the engine's last projected logits
            assert lib.gpu_forward(logits.ctypes.data, prompt[-1], len(prompt) - 1 + call, 1, 1) == 0
            ref = np.empty(VOCAB, np.float32)
            assert lib.gpu_collect(ref.ctypes.data, hist.ctypes.data, len(hist), pen, k, VOCAB) == 0
            ref_ids = np.flatnonzero(ref > -3.0e38)
            vals = np.empty(k, np.float32)
            ids = np.empty(k, np.int32)
            rc = lib.mocha_topk_static(logits.ctypes.data, VOCAB, hist.ctypes.data, len(hist), pen, k,
                                       vals.ctypes.data, ids.ctypes.data, None)
            assert rc == 0
            assert sorted(ids.tolist()) == sorted(ref_ids.tolist())
            assert np.array_equal(vals, ref[ids])                      # same penalised values
            assert np.all(np.diff(vals) <= 0)                           # best first
        # a far shorter call after the full-vocabulary ones: the array still holds the
        # earlier logits past `rows`, which must not reach the result
        rows, k, pen = 1000, 40, 1.12
        short = np.ascontiguousarray(logits[:rows] * 0.5 - 3.0)  # below the stale values
        hs = np.asarray([5, 17, 5, 999, 1000, 151645] + hist[:20].tolist(), np.int32)  # repeats, ids >= rows
        short[17] = -short[17]                                   # one negative penalised value
        vals = np.empty(k, np.float32)
        ids = np.empty(k, np.int32)
        assert lib.mocha_topk_static(short.ctypes.data, rows, hs.ctypes.data, len(hs), pen, k,
                                     vals.ctypes.data, ids.ctypes.data, None) == 0
        assert np.all((ids >= 0) & (ids < rows))
        exp = short.copy()
        for i in dict.fromkeys(int(x) for x in hs):     # distinct ids, penalised once
            if i < rows:
                exp[i] = exp[i] * np.float32(pen) if exp[i] < 0 else exp[i] / np.float32(pen)
        order = sorted(range(rows), key=lambda i: (-float(exp[i]), i))[:k]
        assert ids.tolist() == order
        assert np.array_equal(vals, exp[order])
        # k above the row count: rejected (there are fewer candidates than asked for)
        assert lib.mocha_topk_static(short.ctypes.data, 8, hist.ctypes.data, 0, 1.0, 40, vals.ctypes.data,
                                     ids.ctypes.data, None) == 1
        # beyond the fixed size: rejected, nothing launched
        big = np.zeros(VOCAB + 1, np.float32)
        assert lib.mocha_topk_static(big.ctypes.data, VOCAB + 1, hist.ctypes.data, 0, 1.0, 1, vals.ctypes.data,
                                     ids.ctypes.data, None) == 1
    finally:
        assert lib.gpu_finish() == 0


def test_static_topk_refuses_a_capturing_stream(native):
    """A call on a stream that is being captured fails with a message instead of
    synchronising the stream and invalidating the capture."""
    import ctypes

    import torch
    lib = native.load()
    logits = np.zeros(1000, np.float32)
    vals = np.empty(4, np.float32)
    ids = np.empty(4, np.int32)
    x = torch.zeros(4, device="cuda")
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        g.capture_begin()
        try:
            x.add_(1.0)  # the captured graph is not empty
            rc = lib.mocha_topk_static(logits.ctypes.data, 1000, None, 0, 1.0, 4, vals.ctypes.data,
                                       ids.ctypes.data, ctypes.c_void_p(s.cuda_stream))
        finally:
            g.capture_end()
    assert rc == 1
    g.replay()
    torch.cuda.synchronize()
    assert x.tolist() == [1.0, 1.0, 1.0, 1.0]
