"""Grouped-Q8 CUDA path against the oracle and the reference's golden tokens (B200)."""
import ctypes
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
VOCAB = 151936
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def masked_choice(logits):
    l = np.array(logits, dtype=np.float32)
    l[151643:] = -1e30
    l[151645] = logits[151645]
    return int(np.argmax(l))


@pytest.fixture(scope="module", params=["persistent", "graph"])
def handle(request, native, q8_model_bytes):
    """Both decode paths: one persistent launch per token, or the per-phase graph."""
    old = os.environ.pop("MOCHA_B200_DECODE", None)
    if request.param == "graph":
        os.environ["MOCHA_B200_DECODE"] = "graph"
    try:
        h = native.Q8Handle(0, q8_model_bytes)
    finally:
        os.environ.pop("MOCHA_B200_DECODE", None)
        if old is not None:
            os.environ["MOCHA_B200_DECODE"] = old
    yield h
    h.close()


@pytest.fixture(scope="module")
def teacher_forced(golden_q8, q8_model_bytes, oracle_lib):
    c = golden_q8["cases"]["greedy256"]
    seq = c["prompt"] + c["tokens"][:6]
    o = oracle_lib.Q8Oracle(q8_model_bytes)
    ref = {}
    for pos, tok in enumerate(seq):
        project = pos >= len(c["prompt"]) - 1
        out = o.forward(tok, pos, project)
        if project:
            ref[pos] = out
    return seq, ref


def test_forward_logits_match_oracle(handle, teacher_forced):
    seq, ref = teacher_forced
    worst = 0.0
    for pos, tok in enumerate(seq):
        got = handle.forward(tok, pos, pos in ref)
        if pos in ref:
            r = ref[pos]
            err = np.abs(got - r)
            assert np.all(np.isfinite(got))
            assert np.all(err <= 0.003 * (1 + np.abs(r))), pos          # src/minimind.cpp:154
            assert err.max() <= 2e-3 * (r.max() - r.min()), pos          # max-abs 2e-3 x logit range
            assert masked_choice(got) == masked_choice(r)
            worst = max(worst, err.max())
    print("max abs logit error", worst)


@pytest.mark.parametrize("case", ["greedy256", "greedy_penalty32", "sampled64"])
def test_token_loop_matches_reference(handle, golden_q8, case):
    c = golden_q8["cases"][case]
    toks, t = handle.generate(c["prompt"], c["n"], c["temperature"], c["top_k"], c["top_p"], c["penalty"], c["seed"])
    assert toks == c["tokens"]
    assert t.generated == len(c["tokens"])


def test_reference_abi_collect_and_head(native, q8_model_bytes, oracle_lib, golden_q8):
    lib = native.load()
    buf = q8_model_bytes
    assert lib.gpu_init(buf.ctypes.data, buf.nbytes) == 0
    try:
        c = golden_q8["cases"]["greedy256"]
        logits = np.empty(VOCAB, np.float32)
        for pos, tok in enumerate(c["prompt"]):
            last = pos == len(c["prompt"]) - 1
            assert lib.gpu_forward(logits.ctypes.data, tok, pos, int(last), int(last)) == 0
        hist = np.asarray(c["prompt"][-64:], np.int32)
        for k, pen in ((1, 1.0), (40, 1.12), (64, 1.3)):
            out = np.empty(VOCAB, np.float32)
            assert lib.gpu_collect(out.ctypes.data, hist.ctypes.data, len(hist), pen, k, VOCAB) == 0
            ref = oracle_lib.collect(logits, hist, pen, k, VOCAB)
            got_ids = np.flatnonzero(out > -3.0e38)
            assert len(got_ids) == k
            assert np.array_equal(out[got_ids], ref[got_ids])  # same candidates, same penalised values
            for temp in (0.0, 0.7):
                a = oracle_lib.sample(out, hist, temp, k, 0.9, pen, 7, skip_penalty=True)[0]
                b = oracle_lib.sample(logits, hist, temp, k, 0.9, pen, 7)[0]
                assert a == b
        assert lib.gpu_collect(logits.ctypes.data, hist.ctypes.data, len(hist), 1.0, 65, VOCAB) == 1
        assert lib.gpu_forward(logits.ctypes.data, VOCAB, 0, 1, 1) == 1  # token out of range
    finally:
        assert lib.gpu_finish() == 0
    # hybrid head: GPU rows [0, rows) of an already normalised hidden vector
    o = oracle_lib.Q8Oracle(buf)
    hidden = o.forward(c["prompt"][0], 0, True, hidden_only=True)
    assert lib.gpu_head_init(buf.ctypes.data) == 0
    try:
        rows = VOCAB * 90 // 100
        got = np.empty(rows, np.float32)
        assert lib.gpu_head_start(hidden.ctypes.data, rows) == 0
        assert lib.gpu_head_finish(got.ctypes.data, rows, 1) == 0
        full = o.forward(c["prompt"][0], 0, True)
        assert np.all(np.abs(got - full[:rows]) <= 0.003 * (1 + np.abs(full[:rows])))
    finally:
        lib.gpu_finish()


def _run_ref_host(binary, model, prompt, n, backend, check, penalty=1.0, temp=0.0, top_k=1, top_p=1.0, env=None):
    with tempfile.NamedTemporaryFile("w", suffix=".txt", delete=False) as f:
        f.write(" ".join(map(str, prompt)))
    try:
        p = subprocess.run([binary, model, f.name, str(n), backend, str(temp), "42", str(check), str(penalty),
                            str(top_k), str(top_p)], capture_output=True, text=True, timeout=900,
                           env=dict(os.environ, **(env or {})))
    finally:
        os.unlink(f.name)
    return p, dict(re.findall(r"(\w+)=([^\s]+)", p.stderr))


def test_reference_host_drop_in(golden_q8, q8_model_path):
    """The reference's own host (src/minimind.cpp) linked against libmocha_b200.so:
    --check compares every GPU logit with its CPU path (tolerance 0.003*(1+|ref|))."""
    binary = os.path.join(ROOT, "oracle", "_ref", "minimind_b200")
    if not os.path.exists(binary):
        pytest.skip("oracle/_ref/minimind_b200 not built")
    c = golden_q8["cases"]["greedy256"]
    p, m = _run_ref_host(binary, q8_model_path, c["prompt"], 8, "cuda", 1)
    assert p.returncode == 0, p.stderr[-2000:]
    assert int(m["CHECKED"]) == VOCAB * (len(c["prompt"]) + 7)
    assert float(m["MAX_ABS_ERROR"]) < 3e-3
    assert [int(t) for t in p.stdout.split()] == c["tokens"][:8]
    # sparse candidate path with the reference's own candidate verification
    p, m = _run_ref_host(binary, q8_model_path, c["prompt"], 64, "cuda", 0,
                         env={"MOCHA_LLM_VERIFY_CANDIDATES": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert [int(t) for t in p.stdout.split()] == c["tokens"][:64]
    s = golden_q8["cases"]["sampled64"]
    p, m = _run_ref_host(binary, q8_model_path, s["prompt"], 64, "cuda", 0, s["penalty"], s["temperature"],
                         s["top_k"], s["top_p"])
    assert p.returncode == 0, p.stderr[-2000:]
    assert [int(t) for t in p.stdout.split()] == s["tokens"]


def test_stream_api_matches_generate(native, handle, golden_q8):
    lib = native.load()
    c = golden_q8["cases"]["sampled64"]
    p = np.asarray(c["prompt"], np.int32)
    s = native.MochaSampling(c["temperature"], c["top_k"], c["top_p"], c["penalty"], c["seed"])
    assert lib.mocha_q8_stream_begin(handle.h, p.ctypes.data, len(p), c["n"], ctypes.byref(s)) == 0
    got, t = [], ctypes.c_int()
    while True:
        assert lib.mocha_q8_stream_next(handle.h, ctypes.byref(t)) == 0
        if t.value < 0 or t.value == 151645:
            break
        got.append(t.value)
    assert lib.mocha_q8_stream_end(handle.h) == 0
    assert got == c["tokens"]


def test_engine_binary_matches_reference(golden_q8, q8_model_path):
    """mocha-qwen-engine keeps the reference engine's argv protocol and output lines."""
    binary = os.path.join(ROOT, "mocha-moze-llm_b200", "bin", "mocha-qwen-engine")
    for case in ("greedy256", "sampled64"):
        c = golden_q8["cases"][case]
        p, m = _run_ref_host(binary, q8_model_path, c["prompt"], c["n"], "cuda", 0, c["penalty"], c["temperature"],
                             c["top_k"], c["top_p"])
        assert p.returncode == 0, p.stderr[-2000:]
        assert [int(t) for t in p.stdout.split()] == c["tokens"]
        assert int(m["GENERATED"]) == len(c["tokens"]) and float(m["DECODE_TPS"]) > 0
        assert "CUDA_FORWARD_STEPS" in m
    # argument errors keep the reference's exit code 2
    p, _ = _run_ref_host(binary, q8_model_path, [1, 2], 2000, "cuda", 0)
    assert p.returncode == 2
    p, _ = _run_ref_host(binary, q8_model_path, [1, 2], 4, "cuda", 1)
    assert p.returncode == 2
