"""Phase timeline of one persistent b=1 decode step (grouped-Q8 Qwen2.5-0.5B).

    python mocha-moze-llm_b200/q8_trace.py [pos]

Opens the synthetic seed-1 model, runs a 34-token prompt and four decode steps, then
traces one step at `pos` (default 150) with mocha_q8_trace_step and prints, for a few
layers, the median and last CTA time (us after the layer's x_in is gathered) of every
phase boundary, the per-layer average and the head; then times 512 decode steps.
"""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import mocha_native as N  # noqa: E402
import mocha_q8  # noqa: E402

# stamp offsets within a layer (2 + 12 * layer + offset), in the order they are reached
PHASES = [(0, "x_in"), (1, "qkv"), (2, "attn"), (3, "combine"), (4, "o"), (5, "x_mid"), (9, "gu_chunks"),
          (10, "gu_quant"), (7, "swiglu"), (6, "down"), (8, "x_out")]


def main() -> int:
    pos = int(sys.argv[1]) if len(sys.argv) > 1 else 150
    data = np.fromfile(mocha_q8.model_path(1), dtype=np.uint8)
    h = N.Q8Handle(0, data)
    toks, _ = h.generate(mocha_q8.random_prompt(34, 7), 4)
    st = h.trace_step(toks[0], pos).astype(np.int64)
    rel = (st - st[:, 0].min()) / 1000.0
    rel[st == 0] = np.nan
    for layer in (0, 12, 23):
        base = np.nanmedian(rel[:, 2 + 12 * layer])
        cells = [f"{name}={np.nanmedian(rel[:, 2 + 12 * layer + k]) - base:.2f}/"
                 f"{np.nanmax(rel[:, 2 + 12 * layer + k]) - base:.2f}" for k, name in PHASES]
        print(f"layer {layer:2d} (median/last CTA, us):", " ".join(cells))
    xin = [np.nanmedian(rel[:, 2 + 12 * layer]) for layer in range(24)]
    print(f"layer average {(xin[23] - xin[1]) / 22:.2f} us; head {np.nanmedian(rel[:, 300]):.1f} -> "
          f"{np.nanmax(rel[:, 301]):.1f} us; step {np.nanmax(rel[:, 302]):.1f} us")
    ms = h.bench_decode(toks[0], 33, 289, 256, 512)
    print(f"decode positions 33..288: {ms * 1000 / 512:.1f} us/token")
    h.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
