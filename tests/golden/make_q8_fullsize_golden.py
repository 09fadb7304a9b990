"""Golden fixtures of the grouped-Q8 model at the benchmarked sizes.

* Prefill (one 1023/1024-token prompt, head on the last position).  The reference
  engine caps prompt + new tokens at 1024 (src/minimind.cpp:98), so its own run is the
  1023-token prompt with one generated token: the token it emits is recorded.  The
  last-position logits of the 1023- and 1024-token prompts come from the restatement
  (oracle/q8_oracle.c, pinned bit for bit to the reference's cpu() by its --check); a
  sample of them is kept -- the 256 largest and every 17th id -- in
  q8_prefill_logits.npz.
* Batched serving.  Four sequences of the 512-sequence job (128-token prompts drawn
  from numpy's default_rng(2024), 384 tokens, T 0.7, top-k 40, top-p 0.9, penalty 1.12
  over the last 64 tokens, seed 7 + sequence index) run through the reference engine
  itself (oracle/_ref/minimind_cpu); their token streams are recorded.

Writes tests/golden/q8_fullsize.json and tests/golden/q8_prefill_logits.npz.
Usage: python tests/golden/make_q8_fullsize_golden.py   (needs oracle/_ref built)
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [HERE, os.path.join(ROOT, "mocha-moze-llm_b200"), os.path.join(ROOT, "oracle")]
import make_q8_golden as base  # noqa: E402
import mocha_q8  # noqa: E402
import oracle_py  # noqa: E402

PREFILL_SEED = 1234
SERVE_PROMPT_SEED, SERVE_SEQS, SERVE_PROMPT, SERVE_NEW, SERVE_SEED_BASE = 2024, 512, 128, 384, 7
SERVE_PICK = (0, 17, 42, 63)          # all in the first 64-sequence wave


def serve_prompts():
    return np.random.default_rng(SERVE_PROMPT_SEED).integers(0, mocha_q8.VOCAB, (SERVE_SEQS, SERVE_PROMPT))


def main():
    model = mocha_q8.model_path(base.MODEL_SEED)
    ref_cpu = os.path.join(ROOT, "oracle", "_ref", "minimind_cpu")
    out = {"model_seed": base.MODEL_SEED, "model_sha256": base.sha256(model)}
    prompt = mocha_q8.random_prompt(1024, PREFILL_SEED)
    toks, metrics = base.run(ref_cpu, model, prompt[:1023], 1, "cpu", 0.0, 42, 0, 1.0, 1, 1.0)
    out["prefill"] = {"prompt_seed": PREFILL_SEED, "prompt_len": 1024, "reference_tokens_1023": toks,
                      "reference_prefill_s_1023": float(metrics["PREFILL_S"])}
    print("prefill 1023 token", toks, metrics.get("PREFILL_S"), flush=True)
    o = oracle_py.Q8Oracle(np.fromfile(model, dtype=np.uint8))
    o.reset()
    logits = {}
    for pos, tok in enumerate(prompt):
        proj = pos >= 1022
        r = o.forward(tok, pos, proj)
        if proj:
            logits[pos + 1] = r
    arrays = {}
    for n, lg in logits.items():
        top = np.argsort(-lg, kind="stable")[:256]
        ids = np.union1d(top, np.arange(0, mocha_q8.VOCAB, 17)).astype(np.int32)
        arrays[f"ids_{n}"] = ids
        arrays[f"values_{n}"] = lg[ids].astype(np.float32)
        arrays[f"range_{n}"] = np.float32(lg.max() - lg.min())
        masked = lg.copy()
        masked[mocha_q8.CONTROL_FIRST:] = -1e30
        masked[mocha_q8.EOS] = lg[mocha_q8.EOS]
        arrays[f"argmax_{n}"] = np.int32(np.argmax(masked))
    assert int(arrays["argmax_1023"]) == toks[0], (int(arrays["argmax_1023"]), toks)
    np.savez_compressed(os.path.join(HERE, "q8_prefill_logits.npz"), **arrays)
    prompts = serve_prompts()
    serve = {"prompt_seed": SERVE_PROMPT_SEED, "prompt_len": SERVE_PROMPT, "n": SERVE_NEW, "temperature": 0.7,
             "top_k": 40, "top_p": 0.9, "penalty": 1.12, "seed_base": SERVE_SEED_BASE, "streams": {}}
    for i in SERVE_PICK:
        toks, _ = base.run(ref_cpu, model, prompts[i].tolist(), SERVE_NEW, "cpu", 0.7, SERVE_SEED_BASE + i, 0,
                           1.12, 40, 0.9)
        serve["streams"][str(i)] = toks
        print("serve", i, len(toks), toks[:6], flush=True)
    out["serve"] = serve
    with open(os.path.join(HERE, "q8_fullsize.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
