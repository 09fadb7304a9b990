"""Greedy decode of a synthetic GGUF model (Llama-3.2-1B or Qwen2.5-1.5B shapes, Q4_K_M mix).

    python mocha-moze-llm_b200/gguf_decode.py [llama1b|qwen15b] [prompt tokens] [new tokens]

Prints the generated ids, the library's launches per token and the timed decode rate
(positions after the prompt, tokens fed back on the device).  Small defaults keep a
profiler's launch list short.
"""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import mocha_gguf_model  # noqa: E402
import mocha_native as N  # noqa: E402


def main() -> int:
    arch = sys.argv[1] if len(sys.argv) > 1 else "llama1b"
    plen = int(sys.argv[2]) if len(sys.argv) > 2 else 4
    nnew = int(sys.argv[3]) if len(sys.argv) > 3 else 6
    data = np.fromfile(mocha_gguf_model.model_path(arch), dtype=np.uint8)
    h = N.GgufHandle(0, data)
    prompt = np.random.default_rng(11).integers(0, h.info.vocab, plen).tolist()
    toks, _ = h.generate(prompt, nnew)
    print(arch, "tokens", toks, "launches/token", N.load().mocha_gguf_launches_per_step(h.h))
    h.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
