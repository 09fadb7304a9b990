"""Greedy token streams of the two random-init GGUF models at the benchmarked sizes,
from the C restatement of the llama / qwen2 forward (oracle/gguf_model_oracle.c).

llama.cpp, the reference's CPU path for these models, is not vendored, so the streams
are the restatement's (parity unpinned): Llama-3.2-1B shapes with a 32-token prompt and
128 generated tokens, Qwen2.5-1.5B shapes with 64 + 256, prompts from numpy's
default_rng(11) as the bench draws them.  The smallest greedy margin (top-1 minus top-2
logit) met along each stream is recorded with it.

Writes tests/golden/gguf_streams.json.
Usage: python tests/golden/make_gguf_stream_golden.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(ROOT, "mocha-moze-llm_b200"), os.path.join(ROOT, "oracle")]
import mocha_gguf_model  # noqa: E402
import oracle_py  # noqa: E402

WORKLOADS = (("llama1b", 32, 128), ("qwen15b", 64, 256))
PROMPT_SEED = 11


def stream(o, prompt, n):
    out, margins = [], []
    tok = prompt[0]
    for pos in range(len(prompt) + n - 1):
        project = pos + 1 >= len(prompt)
        logits = o.forward(tok, pos, project)
        if pos + 1 < len(prompt):
            tok = prompt[pos + 1]
            continue
        top2 = np.partition(logits, -2)[-2:]
        margins.append(float(top2[1] - top2[0]))
        tok = int(np.argmax(logits))
        out.append(tok)
    return out, margins


def main():
    res = {"prompt_seed": PROMPT_SEED, "source": "oracle/gguf_model_oracle.c (restatement; parity unpinned)",
           "models": {}}
    for arch, plen, n in WORKLOADS:
        path = mocha_gguf_model.model_path(arch)
        o = oracle_py.GGUFOracle(path)
        vocab = o.vocab
        prompt = np.random.default_rng(PROMPT_SEED).integers(0, vocab, plen).tolist()
        toks, margins = stream(o, prompt, n)
        res["models"][arch] = {"prompt": prompt, "n": n, "tokens": toks, "min_margin": min(margins),
                               "min_margin_step": int(np.argmin(margins))}
        print(arch, len(toks), toks[:6], "min margin", min(margins), flush=True)
        del o
    with open(os.path.join(HERE, "gguf_streams.json"), "w") as f:
        json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
