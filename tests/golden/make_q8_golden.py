"""Generate the grouped-Q8 golden fixtures from the reference engine itself.

Runs the reference CPU engine (src/minimind.cpp compiled from the reference
sources by ``make -C oracle ref`` into oracle/_ref/minimind_cpu) on the seeded
random-init model and records its output token streams, and runs the reference
host with the restatement behind its gpu_* entry points and --check, recording
the logit comparison count and maximum error (which pins the restatement).

Usage: python tests/golden/make_q8_golden.py   (writes tests/golden/q8_golden.json)
"""
import hashlib
import json
import os
import re
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "mocha-moze-llm_b200"))
import mocha_q8  # noqa: E402

MODEL_SEED = 1
CASES = [
    # name, prompt length, prompt seed, new tokens, temperature, seed, penalty, top_k, top_p
    ("greedy256", 34, 7, 256, 0.0, 42, 1.0, 1, 1.0),
    ("sampled64", 34, 11, 64, 0.7, 42, 1.12, 40, 0.9),
    ("greedy_penalty32", 20, 5, 32, 0.0, 42, 1.12, 40, 0.9),
]


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def run(binary, model, ids, n, backend, temp, seed, check, penalty, top_k, top_p):
    with tempfile.NamedTemporaryFile("w", suffix=".txt", delete=False) as f:
        f.write(" ".join(map(str, ids)))
        path = f.name
    try:
        p = subprocess.run([binary, model, path, str(n), backend, str(temp), str(seed), str(check),
                            str(penalty), str(top_k), str(top_p)], capture_output=True, text=True,
                           env=dict(os.environ, OMP_NUM_THREADS=str(os.cpu_count())))
    finally:
        os.unlink(path)
    if p.returncode != 0:
        raise RuntimeError(f"{binary} failed rc={p.returncode}: {p.stderr}")
    tokens = [int(x) for x in p.stdout.split()]
    metrics = dict(re.findall(r"(\w+)=([^\s]+)", p.stderr))
    return tokens, metrics


def main():
    model = mocha_q8.model_path(MODEL_SEED)
    ref_cpu = os.path.join(ROOT, "oracle", "_ref", "minimind_cpu")
    ref_oracle = os.path.join(ROOT, "oracle", "_ref", "minimind_oracle")
    out = {"model_seed": MODEL_SEED, "model_sha256": sha256(model), "cases": {}}
    for name, plen, pseed, n, temp, seed, pen, k, tp in CASES:
        ids = mocha_q8.random_prompt(plen, pseed)
        tokens, _ = run(ref_cpu, model, ids, n, "cpu", temp, seed, 0, pen, k, tp)
        out["cases"][name] = dict(prompt=ids, n=n, temperature=temp, seed=seed, penalty=pen,
                                  top_k=k, top_p=tp, tokens=tokens)
        print(name, len(tokens), tokens[:8], flush=True)
    # restatement pin: reference host --check against gpu_* served by the restatement
    ids = out["cases"]["greedy256"]["prompt"]
    tokens, metrics = run(ref_oracle, model, ids, 24, "cuda", 0.0, 42, 1, 1.0, 1, 1.0)
    out["restatement_pin"] = dict(prompt="greedy256", n=24, checked=int(metrics["CHECKED"]),
                                  max_abs_error=float(metrics["MAX_ABS_ERROR"]), tokens=tokens)
    print("pin", out["restatement_pin"]["checked"], out["restatement_pin"]["max_abs_error"])
    with open(os.path.join(ROOT, "tests", "golden", "q8_golden.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
