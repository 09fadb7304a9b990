"""The grouped-Q8 oracle (C restatement of src/minimind.cpp) against the reference.

Golden vectors come from the reference engine compiled from its own sources
(tests/golden/make_q8_golden.py); the restatement pin is the reference host's own
--check run with the restatement behind its gpu_* entry points."""
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest


def test_restatement_pin_recorded(golden_q8):
    pin = golden_q8["restatement_pin"]
    assert pin["checked"] >= 151936 * 30
    assert pin["max_abs_error"] == 0.0
    assert pin["tokens"] == golden_q8["cases"]["greedy256"]["tokens"][: len(pin["tokens"])]


def test_restatement_pin_live(golden_q8, q8_model_path):
    """Reference host + restatement with --check: every logit bit-identical."""
    binary = os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref", "minimind_oracle")
    if not os.path.exists(binary):
        pytest.skip("oracle/_ref not built (needs the reference sources)")
    case = golden_q8["cases"]["greedy256"]
    with tempfile.NamedTemporaryFile("w", suffix=".txt", delete=False) as f:
        f.write(" ".join(map(str, case["prompt"])))
    try:
        p = subprocess.run([binary, q8_model_path, f.name, "3", "cuda", "0", "42", "1", "1.0", "1", "1.0"],
                           capture_output=True, text=True, timeout=600)
    finally:
        os.unlink(f.name)
    assert p.returncode == 0, p.stderr
    m = dict(re.findall(r"(\w+)=([^\s]+)", p.stderr))
    assert int(m["CHECKED"]) == 151936 * (len(case["prompt"]) + 2)
    assert float(m["MAX_ABS_ERROR"]) == 0.0
    assert [int(t) for t in p.stdout.split()] == case["tokens"][:3]


@pytest.mark.parametrize("case,n", [("greedy256", 12), ("sampled64", 10), ("greedy_penalty32", 8)])
def test_oracle_token_loop_matches_reference(golden_q8, q8_model_bytes, oracle_lib, case, n):
    c = golden_q8["cases"][case]
    o = oracle_lib.Q8Oracle(q8_model_bytes)
    toks, _ = o.generate(c["prompt"], n, c["temperature"], c["top_k"], c["top_p"], c["penalty"], c["seed"])
    assert toks == c["tokens"][:n]


def test_oracle_collect_contains_host_choice(oracle_lib):
    """Candidate path == full-vocabulary sampling (the reference's
    MOCHA_LLM_VERIFY_CANDIDATES property, src/minimind.cpp:138-150)."""
    rng = np.random.default_rng(3)
    for trial in range(4):
        logits = rng.standard_normal(151936).astype(np.float32) * 2
        logits[rng.integers(0, 151936, 5)] = logits.max()  # ties
        hist = rng.integers(0, 151936, 64).tolist() + [int(np.argmax(logits))]
        hist = hist[-64:]
        for temp, k in ((0.0, 1), (0.7, 40)):
            full_tok, full_seed, _ = oracle_lib.sample(logits, hist, temp, k, 0.9, 1.12, 42 + trial)
            cand = oracle_lib.collect(logits, hist, 1.12, k, 151936)
            sparse_tok, sparse_seed, _ = oracle_lib.sample(cand, hist, temp, k, 0.9, 1.12, 42 + trial,
                                                            skip_penalty=True)
            assert (full_tok, full_seed) == (sparse_tok, sparse_seed)


def test_oracle_collect_argument_checks(oracle_lib):
    with pytest.raises(ValueError):
        oracle_lib.collect(np.zeros(151936, np.float32), [], 1.0, 65, 151936)
    with pytest.raises(ValueError):
        oracle_lib.collect(np.zeros(151936, np.float32), list(range(65)), 1.0, 1, 151936)
