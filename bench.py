"""Benchmark: grouped-Q8 Qwen2.5-0.5B batch-1 greedy decode on B200.

One step = one decode pass of the reference's headline workload: 256 generated
tokens after a 34-token random prompt (positions 33..288 of a 1024 context), greedy,
repeat penalty 1.0, random-init weights (seed 1).  `value` is device-timed (CUDA
events on the library's stream) with the sampled token fed back on the device;
`e2e` goes through the public C ABI call with host buffers (prompt in, tokens out).
With --gpus N (torchrun) every rank runs an independent replica on its own GPU
(weak scaling, no data-path collective); the timing is the max over ranks.

--impl reference times the reference's own CPU engine (src/minimind.cpp built from
the reference sources into oracle/_ref/minimind_cpu) on the host cores.
"""
import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mocha-moze-llm_b200")
ORACLE = os.path.join(ROOT, "oracle")
sys.path.insert(0, PKG)

METRIC = "Qwen0.5B-Q8 decode tok/s (b=1, b=64) + prefill tok/s; % of HBM/TC roofline"
PUBLISHED_TOKS = 7.75          # reference CUDA decode on GK20A (docs/performance.md:43)
PROMPT_LEN, NEW_TOKENS, PROMPT_SEED, MODEL_SEED = 34, 256, 7, 1
WEIGHT_BYTES = 525_120_000     # int8 + fp32 scales + fp32 norms/biases per token
KV_BYTES_PER_POS = 24_576      # 24 layers x (K+V) x 128 x fp32
ONE_THREAD_TOKENS = 16         # bounded 1-thread sample of the reference engine
SERVE_REF_SEQS = 2             # sequences of the batched job timed on the reference engine
TRAFFIC_PER_TOKEN = 539_311_872  # DRAM read + write per k_step launch (538.71 + 0.60 MB), ncu, positions 40-42
# prefill workload: one 1024-token prompt, head on the last position
PREFILL_LEN = 1024
PREFILL_FLOP = 2 * 357_826_560 * 1024 + 45.1e9 + 2 * 136_134_656   # algorithmic FLOP per prompt
# batched serving workload: 512 sequences, 128-token prompts, 384 generated, 64 per GPU at a time
SERVE_SEQS, SERVE_PROMPT, SERVE_NEW, SERVE_BATCH = 512, 128, 384, 64
# GGUF decode workloads: (architecture, prompt tokens, generated tokens, weight bytes per token, KV bytes per position)
GGUF_WORKLOADS = (("llama1b", 32, 128, 799_862_784, 65_536), ("qwen15b", 64, 256, 980_097_536, 57_344))


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class Group:
    """Host-side barrier / gather for N independent replicas (gloo, CPU only)."""

    def __init__(self):
        self.rank, self.world, self.local = dist_env()
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            self.dist = dist

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def gather(self, obj):
        if self.world == 1:
            return [obj]
        out = [None] * self.world
        self.dist.all_gather_object(out, obj)
        return out

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


def partition(n, world, rank):
    """Sequences of an n-sequence job that rank `rank` of `world` serves: i mod world ==
    rank.  Every sequence is served by exactly one rank; there is no data-path exchange."""
    return [i for i in range(n) if i % world == rank]


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}",
                 "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return None
        sm, mx, reasons = [], 0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 6 or not parts[0].isdigit():
                continue
            sm.append(int(parts[0]))
            mx = max(mx, int(parts[1]))
            for n, v in zip(names, parts[2:]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def model_bytes(group):
    import numpy as np

    import mocha_q8
    if group.rank == 0:
        path = mocha_q8.model_path(MODEL_SEED)
    group.barrier()
    path = mocha_q8.model_path(MODEL_SEED)
    return path, np.fromfile(path, dtype=np.uint8)


def run_reference_engine(model_path, prompt, n, threads, sampling=("0", "42", "1.0", "1", "1.0"), metrics=False):
    """One run of the reference CPU engine (src/minimind.cpp built from the reference
    sources); sampling = (temperature, seed, repeat penalty, top-k, top-p)."""
    binary = os.path.join(ORACLE, "_ref", "minimind_cpu")
    temp, seed, pen, k, top_p = sampling
    with tempfile.NamedTemporaryFile("w", suffix=".txt", delete=False) as f:
        f.write(" ".join(map(str, prompt)))
    try:
        p = subprocess.run([binary, model_path, f.name, str(n), "cpu", temp, seed, "0", pen, k, top_p],
                           capture_output=True, text=True, env=dict(os.environ, OMP_NUM_THREADS=str(threads)))
    finally:
        os.unlink(f.name)
    if p.returncode != 0:
        raise RuntimeError(p.stderr)
    m = dict(re.findall(r"(\w+)=([^\s]+)", p.stderr))
    if metrics:
        return m
    gen = int(m["GENERATED"])
    tps = float(m["DECODE_TPS"])
    return gen, tps, (gen - 1) / tps if tps > 0 else 0.0


def reference_arm(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    import mocha_q8
    binary = os.path.join(ORACLE, "_ref", "minimind_cpu")
    if not os.path.exists(binary):
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/minimind_cpu not built"}))
        return 0
    path = mocha_q8.model_path(MODEL_SEED)
    prompt = mocha_q8.random_prompt(PROMPT_LEN, PROMPT_SEED)
    cores = os.cpu_count()
    for _ in range(args.warmup):
        run_reference_engine(path, prompt, NEW_TOKENS, cores)
    toks, secs = 0, 0.0
    for _ in range(args.steps):
        gen, tps, s = run_reference_engine(path, prompt, NEW_TOKENS, cores)
        toks += gen - 1
        secs += s
    value = toks / secs
    sample = (f"reference CPU engine (src/minimind.cpp -O3 -fopenmp, {cores} threads), the full workload per "
              f"step: {PROMPT_LEN}-token prompt + {NEW_TOKENS} greedy tokens, DECODE_TPS definition (tokens "
              f"after the first / decode wall time)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * secs / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": value / PUBLISHED_TOKS, "dtype": "f32",
        "data": "synthetic: random-init weights (seed 1), 34 random prompt ids",
        "config": {"workload": "Qwen2.5-0.5B grouped-Q8 b=1 greedy decode: 34-token prompt, 256 generated "
                               "(positions 33..288), one step = one 256-token decode",
                   "global_batch": 1, "seq_len": PROMPT_LEN + NEW_TOKENS, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))
    return 0


def peak_tflops():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def bench_batched(group, data, args, parts):
    """Prefill of one 1024-token prompt and the batched serving job on this rank's
    share of the 512 sequences (tcgen05 GEMM path)."""
    import numpy as np

    import mocha_native
    rank, world, local = group.rank, group.world, group.local
    h = mocha_native.Q8BatchHandle(local, data, max_rows=SERVE_BATCH * SERVE_PROMPT, slots=SERVE_BATCH)
    group.barrier()
    pre_ms = h.bench_prefill(PREFILL_LEN, 1234 + rank, args.warmup, args.steps) if "prefill" in parts else 0.0
    if "batched" not in parts:
        h.close()
        return {"prefill_ms": pre_ms, "decode_s": 0.0, "prefill_s": 0.0, "generated": 0, "nseq": 0, "wall": 0.0,
                "launches": 0}
    # batched serving: sequences i with i % world == rank
    mine = partition(args.serve_seqs, world, rank)
    prompts = np.random.default_rng(2024).integers(0, 151936, (args.serve_seqs, SERVE_PROMPT))[mine]
    h.generate(prompts[:SERVE_BATCH], 8, temperature=0.7, top_k=40, top_p=0.9, penalty=1.12, seed_base=7)
    group.barrier()
    t0 = time.perf_counter()
    toks, t = h.generate(prompts, args.serve_new, temperature=0.7, top_k=40, top_p=0.9, penalty=1.12, seed_base=7)
    wall = time.perf_counter() - t0
    launches = h.launches_per_step()
    h.close()
    return {"prefill_ms": pre_ms, "decode_s": t.decode_s, "prefill_s": t.prefill_s, "generated": t.generated,
            "nseq": len(mine), "wall": wall, "launches": launches}


def bench_gguf(group, args):
    """b=1 greedy decode of the two GGUF models (random-init, Q4_K_M mix) on this rank."""
    import numpy as np

    import mocha_gguf_model
    import mocha_native
    out = {}
    for arch, plen, nnew, wbytes, kvpos in GGUF_WORKLOADS:
        if args.gguf_arch and arch != args.gguf_arch:
            continue
        if args.gguf_tokens:
            plen, nnew = (int(v) for v in args.gguf_tokens.split(","))
        if group.rank == 0:
            mocha_gguf_model.model_path(arch)
        group.barrier()
        data = np.fromfile(mocha_gguf_model.model_path(arch), dtype=np.uint8)
        h = mocha_native.GgufHandle(group.local, data)
        prompt = np.random.default_rng(11 + group.rank).integers(0, h.info.vocab, plen).tolist()
        first, _ = h.generate(prompt, 1)
        tok = first[0] if first else prompt[-1]
        pos0, pos_end = plen - 1, plen - 1 + nnew
        ms = h.bench_decode(tok, pos0, pos_end, args.warmup * nnew, args.steps * nnew)
        t0 = time.perf_counter()
        h.generate(prompt, nnew)
        wall = time.perf_counter() - t0
        launches = mocha_native.load().mocha_gguf_launches_per_step(h.h)
        h.close()
        del data
        out[arch] = {"ms": ms, "wall": wall, "launches": launches}
    return out


def gguf_objects(gathered, args, world):
    hbm_peak, hbm_kind = peaks()
    res = {}
    for arch, plen, nnew, wbytes, kvpos in GGUF_WORKLOADS:
        if arch not in gathered[0]["gguf"]:
            continue
        if args.gguf_tokens:
            plen, nnew = (int(v) for v in args.gguf_tokens.split(","))
        ms = max(g["gguf"][arch]["ms"] for g in gathered)
        per_tok = ms / 1e3 / (args.steps * nnew)
        mean_pos1 = (plen + plen - 1 + nnew) / 2
        algo = wbytes + kvpos * mean_pos1
        achieved = algo / per_tok / 1e9
        wall = max(g["gguf"][arch]["wall"] for g in gathered)
        res[arch] = {
            "value": world / per_tok, "unit": "tok/s", "us_per_token": per_tok * 1e6,
            "config": {"workload": f"{arch} GGUF Q4_K_M-mix random-init, b=1 greedy, {plen}-token prompt + "
                                   f"{nnew} generated per GPU"},
            "e2e": {"value": world * nnew / wall, "unit": "tok/s",
                    "path": "mocha_gguf_generate (host prompt in, host tokens out), prompt pass included"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "peak_kind": hbm_kind, "algorithmic_bytes_per_token": algo},
            "gpu_launches_per_token": gathered[0]["gguf"][arch]["launches"]}
    return res


INT8_TOPS_DATASHEET = 4500.0   # B200 dense int8 tensor peak (datasheet; no measured int8 figure exists here)
PREFILL_GEMM_FLOP = 2 * 357_826_560 * 1024 + 2 * 136_134_656   # the GEMM part of PREFILL_FLOP


def prefill_object(gathered, args, world):
    tf_peak, tf_kind = peak_tflops()
    pre_ms = max(g["prefill_ms"] for g in gathered) / args.steps
    achieved_tf = PREFILL_FLOP / (pre_ms / 1e3) / 1e12
    issued_tops = (3 * PREFILL_GEMM_FLOP + (PREFILL_FLOP - PREFILL_GEMM_FLOP)) / (pre_ms / 1e3) / 1e12
    return {"value": PREFILL_LEN * world / (pre_ms / 1e3), "unit": "tok/s", "ms_per_prompt": pre_ms,
            "config": {"workload": "one 1024-token prompt of uniform random ids per GPU, head on the last position"},
            "roofline": {"bound": "tensor", "achieved": achieved_tf, "peak": INT8_TOPS_DATASHEET, "unit": "TFLOP/s",
                         "frac": achieved_tf / INT8_TOPS_DATASHEET, "peak_kind": "datasheet dense int8",
                         "algorithmic_flop_per_prompt": PREFILL_FLOP,
                         "issued_tops": issued_tops, "issued_frac": issued_tops / INT8_TOPS_DATASHEET,
                         "bf16_peak": tf_peak, "bf16_peak_kind": tf_kind, "bf16_frac": achieved_tf / tf_peak,
                         "note": "the GEMMs issue tcgen05.mma kind::i8 against three int8 limbs of each "
                                 "activation (3x the algorithmic MACs: issued_tops); the attention runs bf16 "
                                 "pairs. achieved counts the reference's int8 x fp32 MACs once"}}


def batched_object(gathered, args, world):
    hbm_peak, hbm_kind = peaks()
    decode_s = max(g["decode_s"] for g in gathered)
    wall = max(g["wall"] for g in gathered)
    gen = sum(g["generated"] for g in gathered)
    first = sum(g["nseq"] for g in gathered)
    # per GPU and decode step: weights once + the KV of 64 sequences at mean position
    steps_per_gpu = (args.serve_new - 1) * ((args.serve_seqs // world + SERVE_BATCH - 1) // SERVE_BATCH)
    mean_pos1 = (SERVE_PROMPT + 1 + SERVE_PROMPT + args.serve_new - 1) / 2
    step_bytes = WEIGHT_BYTES + SERVE_BATCH * KV_BYTES_PER_POS * mean_pos1
    achieved = step_bytes * steps_per_gpu / decode_s / 1e9
    return {"value": (gen - first) / decode_s, "unit": "tok/s", "decode_s": decode_s,
            "e2e": {"value": gen / wall, "unit": "tok/s", "path": "mocha_q8b_generate (prompt pass included)"},
            "config": {"workload": f"{args.serve_seqs} sequences x (128-token prompt + {args.serve_new} generated), "
                                   "T=0.7 top-k 40 top-p 0.9 penalty 1.12, 64 per GPU per wave",
                       "parallelism": f"replicas x{world}", "scaling": f"strong ({args.serve_seqs} sequences in total)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "peak_kind": hbm_kind,
                         "algorithmic_bytes_per_step": step_bytes,
                         "note": "weights counted in the reference format (int8 + fp32 scales), read as "
                                 "stored (q|k|v and gate|up from row-fused int8 copies)"},
            "gpu_launches_per_step": gathered[0]["launches"]}


def cpu_baseline(model_path, prompt):
    """The reference CPU engine on this host: the b=1 workload at all threads (its own
    DECODE_TPS) plus a bounded one-thread sample."""
    binary = os.path.join(ORACLE, "_ref", "minimind_cpu")
    cores = os.cpu_count()
    if os.path.exists(binary):
        gen, tps, _ = run_reference_engine(model_path, prompt, NEW_TOKENS, cores)
        _, tps1, _ = run_reference_engine(model_path, prompt, ONE_THREAD_TOKENS, 1)
        return {"value": tps, "unit": "tok/s", "cores": cores, "kind": "reference",
                "sample": f"reference CPU engine (src/minimind.cpp, -O3 -fopenmp), {PROMPT_LEN}-token prompt + "
                          f"{NEW_TOKENS} greedy tokens, DECODE_TPS",
                "one_thread": {"value": tps1, "unit": "tok/s", "cores": 1,
                               "sample": f"{PROMPT_LEN}-token prompt + {ONE_THREAD_TOKENS} greedy tokens, DECODE_TPS"}}
    sys.path.insert(0, ORACLE)
    import numpy as np
    import oracle_py
    o = oracle_py.Q8Oracle(np.fromfile(model_path, dtype=np.uint8))
    t0 = time.perf_counter()
    o.generate(prompt, 8)
    dt = time.perf_counter() - t0
    return {"value": 8 / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": "oracle restatement, 34-token prompt + 8 tokens, prompt included"}


def prefill_cpu_baseline(model_path):
    """The reference engine's own prefill of the longest prompt it accepts next to one
    generated token (prompt + n <= 1024, src/minimind.cpp:98): 1023 tokens, PREFILL_S."""
    binary = os.path.join(ORACLE, "_ref", "minimind_cpu")
    if not os.path.exists(binary):
        return None
    import mocha_q8
    prompt = mocha_q8.random_prompt(PREFILL_LEN - 1, 1234)
    cores = os.cpu_count()
    m = run_reference_engine(model_path, prompt, 1, cores, metrics=True)
    secs = float(m["PREFILL_S"])
    return {"value": (PREFILL_LEN - 1) / secs, "unit": "tok/s", "cores": cores, "kind": "reference",
            "prefill_s": secs,
            "sample": f"reference CPU engine, one {PREFILL_LEN - 1}-token prompt with 1 generated token (its cap), "
                      "prompt tokens / PREFILL_S"}


def batched_cpu_baseline(model_path):
    """The batched job on the reference engine: sequences run one after the other at all
    threads, tok/s = generated tokens / wall time (WALL_S), over a bounded sample."""
    binary = os.path.join(ORACLE, "_ref", "minimind_cpu")
    if not os.path.exists(binary):
        return None
    import numpy as np
    prompts = np.random.default_rng(2024).integers(0, 151936, (SERVE_SEQS, SERVE_PROMPT))
    cores = os.cpu_count()
    gen, wall = 0, 0.0
    for i in range(SERVE_REF_SEQS):
        m = run_reference_engine(model_path, prompts[i].tolist(), SERVE_NEW, cores,
                                 sampling=("0.7", str(7 + i), "1.12", "40", "0.9"), metrics=True)
        gen += int(m["GENERATED"])
        wall += float(m["WALL_S"])
    return {"value": gen / wall, "unit": "tok/s", "cores": cores, "kind": "reference",
            "sample": f"reference CPU engine, sequences 0..{SERVE_REF_SEQS - 1} of the job run one after the "
                      f"other ({SERVE_PROMPT}-token prompt + {SERVE_NEW} tokens, T 0.7, top-k 40, top-p 0.9, "
                      "penalty 1.12), generated tokens / WALL_S"}


# phase boundaries of the persistent step's trace stamps (offset within a layer, name),
# in the order a CTA reaches them; see mocha_q8_trace_step in include/mocha_b200.h
TRACE_PHASES = [(0, "x_in"), (12, "qkv input ready"), (11, "qkv chunk"), (13, "qkv products"), (1, "qkv stored"),
                (14, "att q/k/v in"), (15, "att past K/V"), (16, "att softmax+PV"), (3, "att merged+limbs"),
                (4, "att O products"), (23, "att split weight"), (2, "attention + O added"),
                (5, "x_mid"), (10, "ffn norm+limbs"), (9, "gate/up chunks"), (18, "gate/up products"),
                (7, "swiglu+limbs"), (20, "down chunk"), (21, "down products"), (6, "down added"),
                (8, "x_out")]


def trace_step(pos):
    """Phase timeline (%globaltimer stamps of every CTA) of one persistent b=1 decode step
    at position `pos` after a 34-token prompt: median and last CTA per phase boundary, in
    microseconds after the layer's input is complete, for layers 0, 12 and 23."""
    import numpy as np

    import mocha_native
    import mocha_q8
    data = np.fromfile(mocha_q8.model_path(MODEL_SEED), dtype=np.uint8)
    h = mocha_native.Q8Handle(0, data)
    toks, _ = h.generate(mocha_q8.random_prompt(PROMPT_LEN, PROMPT_SEED), 4)
    st = h.trace_step(toks[0], pos).astype(np.int64)
    rel = (st - st[:, 0].min()) / 1000.0
    rel[st == 0] = np.nan
    per = 24
    for layer in (0, 12, 23):
        base = np.nanmedian(rel[:, 2 + per * layer])
        print(f"layer {layer} (us after x_in; median / last CTA)")
        for k, name in TRACE_PHASES:
            col = rel[:, 2 + per * layer + k]
            if not np.all(np.isnan(col)):
                print(f"  {name:22s} {np.nanmedian(col) - base:6.2f} / {np.nanmax(col) - base:6.2f}  "
                      f"({int(np.sum(~np.isnan(col)))} CTAs)")
    head = 2 + per * 24
    xin = [np.nanmedian(rel[:, 2 + per * layer]) for layer in range(24)]
    print(f"layer average {(xin[23] - xin[1]) / 22:.2f} us; head {np.nanmedian(rel[:, head]):.1f} -> "
          f"{np.nanmax(rel[:, head + 1]):.1f} us; step {np.nanmax(rel[:, head + 2]):.1f} us")
    h.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the prefill and batched-serving objects")
    ap.add_argument("--serve-seqs", type=int, default=SERVE_SEQS, help="batched job size (smaller for profiling)")
    ap.add_argument("--serve-new", type=int, default=SERVE_NEW, help="tokens per sequence of the batched job")
    ap.add_argument("--gguf-arch", default="", help="run one GGUF model (llama1b or qwen15b) in the gguf part")
    ap.add_argument("--gguf-tokens", default="", help="PROMPT,NEW tokens of the gguf part (shorter for profiling)")
    ap.add_argument("--trace-step", type=int, default=0,
                    help="print the phase timeline of one persistent decode step at this position and exit")
    ap.add_argument("--parts", default="decode,prefill,batched,gguf",
                    help="comma list of workloads to run (profiling runs select one); the default runs all four")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    if args.trace_step:
        return trace_step(args.trace_step)
    if args.warmup < 3:
        args.warmup = 3

    import numpy as np

    import mocha_native
    import mocha_q8
    group = Group()
    rank, world, local = group.rank, group.world, group.local
    path, data = model_bytes(group)
    parts = set(args.parts.split(","))
    prompt = mocha_q8.random_prompt(PROMPT_LEN, PROMPT_SEED + rank)
    pos0, pos_end = PROMPT_LEN - 1, PROMPT_LEN - 1 + NEW_TOKENS
    ms, e2e_wall, clocks, launches = 0.0, 0.0, None, 0
    if "decode" in parts:
        h = mocha_native.Q8Handle(local, data)
        # fill the KV cache for the prompt and take its first token
        first, _ = h.generate(prompt, 1)
        tok = first[0] if first else prompt[-1]
        group.barrier()
        with Clocks(local) as clk:
            ms = h.bench_decode(tok, pos0, pos_end, args.warmup * NEW_TOKENS, args.steps * NEW_TOKENS)
        clocks = clk.summary()
        group.barrier()
        # end to end through the public C ABI with host buffers
        h.generate(prompt, NEW_TOKENS)
        for _ in range(args.steps):
            t0 = time.perf_counter()
            toks, t = h.generate(prompt, NEW_TOKENS)
            e2e_wall += time.perf_counter() - t0
        launches = mocha_native.load().mocha_q8_launches_per_step(h.h) * NEW_TOKENS * args.steps
        h.close()
    run_batched = not args.no_batched and bool(parts & {"prefill", "batched"})
    extra = bench_batched(group, data, args, parts) if run_batched else {}
    del data
    if "gguf" in parts:
        extra["gguf"] = bench_gguf(group, args)
    gathered = group.gather({"ms": ms, "e2e": e2e_wall, "clocks": clocks, **extra})
    if rank != 0:
        group.close()
        return 0
    out = {"metric": METRIC, "value": None, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "parts": sorted(parts)}
    if "decode" in parts:
        ms_max = max(g["ms"] for g in gathered)
        e2e_max = max(g["e2e"] for g in gathered)
        total_tokens = NEW_TOKENS * args.steps * world
        value = total_tokens / (ms_max / 1e3)
        e2e = NEW_TOKENS * args.steps * world / e2e_max
        per_token_s = ms_max / 1e3 / (NEW_TOKENS * args.steps)
        mean_pos1 = (pos0 + 1 + pos_end) / 2
        algo = WEIGHT_BYTES + KV_BYTES_PER_POS * mean_pos1
        peak, peak_kind = peaks()
        achieved = algo / per_token_s / 1e9
        out.update({
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": value / PUBLISHED_TOKS, "dtype": "f32",
            "data": "synthetic: random-init weights N(0,0.02) (seed 1), group-64 int8; 34 random prompt ids per rank",
            "config": {"workload": "Qwen2.5-0.5B grouped-Q8 b=1 greedy decode: 34-token prompt, 256 generated "
                                   "(positions 33..288), one step = one 256-token decode",
                       "global_batch": world, "seq_len": PROMPT_LEN + NEW_TOKENS,
                       "parallelism": f"replicas x{world}",
                       "l2": "weights (525 MB) exceed the 126 MB L2; no flush needed"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": TRAFFIC_PER_TOKEN,
                         "kernel": "k_step: one persistent cooperative launch per token",
                         "algorithmic_bytes_per_launch": algo, "peak_kind": peak_kind},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": PROMPT_LEN * 4 + 32,
                    "d2h_bytes_per_step": NEW_TOKENS * 4,
                    "path": "mocha_q8_generate (C ABI, host prompt in / host tokens out), prompt pass included"},
            "gpu_launches": launches * world,
            "clocks": gathered[0]["clocks"],
        })
    if run_batched and "prefill" in parts:
        out["prefill"] = prefill_object(gathered, args, world)
    if run_batched and "batched" in parts:
        out["batched"] = batched_object(gathered, args, world)
    if "gguf" in parts:
        out["gguf"] = gguf_objects(gathered, args, world)
    if not args.no_cpu_baseline and "decode" in parts:
        out["cpu_baseline"] = cpu_baseline(path, mocha_q8.random_prompt(PROMPT_LEN, PROMPT_SEED))
    if not args.no_cpu_baseline and "prefill" in out:
        out["prefill"]["cpu_baseline"] = prefill_cpu_baseline(path)
    if not args.no_cpu_baseline and "batched" in out:
        out["batched"]["cpu_baseline"] = batched_cpu_baseline(path)
    print(json.dumps(out))
    group.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
