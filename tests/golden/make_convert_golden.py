"""Golden output of the reference weight converter (tools/convert-qwen.py) on a tiny,
seeded BF16 checkpoint with the reference's tensor names.

The converter (tools/convert-qwen.py:15-61) checks only the source SHA-256 and the BF16
dtype, so a checkpoint with Qwen2.5's tensor names but small shapes (hidden 64, FFN 128,
K/V 64, vocabulary 256; 24 layers as the converter's loop requires) runs it in well under
a second.  This script writes that checkpoint, runs the reference converter on it with
SOURCE_SHA set to the checkpoint's own digest on the imported module, and records the
checkpoint and output digests in tests/golden/convert_golden.json.  The parity test
rebuilds the same checkpoint and requires this library's writer (mocha_q8.write_model)
to produce the same bytes.

Usage: python tests/golden/make_convert_golden.py   (needs the reference sources; the
directory comes from MOCHA_REFERENCE_DIR or the oracle recipe's default)
"""
import hashlib
import importlib.util
import json
import os
import struct
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
SEED = 5
DIM, HIDDEN, KV, VOCAB, LAYERS = 64, 128, 64, 256, 24
MATRICES = [("self_attn.q_proj", DIM, DIM), ("self_attn.k_proj", KV, DIM), ("self_attn.v_proj", KV, DIM),
            ("self_attn.o_proj", DIM, DIM), ("mlp.gate_proj", HIDDEN, DIM), ("mlp.up_proj", HIDDEN, DIM),
            ("mlp.down_proj", DIM, HIDDEN)]


def checkpoint_tensors():
    """(name, shape, kind) of the tiny checkpoint, in the order the converter reads them."""
    out = [("model.embed_tokens.weight", (VOCAB, DIM), "w")]
    for layer in range(LAYERS):
        b = f"model.layers.{layer}."
        out.append((b + "input_layernorm.weight", (DIM,), "norm"))
        out += [(b + n + ".weight", (r, c), "w") for n, r, c in MATRICES]
        out.append((b + "post_attention_layernorm.weight", (DIM,), "norm"))
        out += [(b + "self_attn.q_proj.bias", (DIM,), "bias"), (b + "self_attn.k_proj.bias", (KV,), "bias"),
                (b + "self_attn.v_proj.bias", (KV,), "bias")]
    out.append(("model.norm.weight", (DIM,), "norm"))
    return out


def to_bf16(x):
    """fp32 -> bf16 bits, rounded to nearest even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype("<u2")


def write_checkpoint(path):
    """The seeded BF16 safetensors file; returns its SHA-256."""
    rng = np.random.default_rng(SEED)
    header, blobs, off = {}, [], 0
    for name, shape, kind in checkpoint_tensors():
        v = rng.standard_normal(shape, dtype=np.float32)
        v = np.float32(1) + np.float32(0.01) * v if kind == "norm" else np.float32(0.02) * v
        if kind == "w" and name.endswith("down_proj.weight"):
            v[0, :64] = 0.0                         # an all-zero group: the 1e-12 scale floor
            v[1, 3] = np.float32(0.5)               # an outlier: every other weight of its group rounds small
        raw = to_bf16(v).tobytes()
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    return hashlib.sha256(open(path, "rb").read()).hexdigest()


def read_checkpoint(path):
    """{name: fp32 array} of a BF16 safetensors file (bf16 bits << 16)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    out = {}
    for name, info in header.items():
        a, b = info["data_offsets"]
        bits = np.frombuffer(data[a:b], dtype="<u2").astype("<u4") << 16
        out[name] = bits.view("<f4").reshape(info["shape"])
    return out


def reference_dir():
    p = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "refdir"], check=True,
                       capture_output=True, text=True)
    return p.stdout.strip()


def run_reference_converter(ckpt, out, ckpt_sha):
    """tools/convert-qwen.py's convert() with SOURCE_SHA overridden on the imported module."""
    src = os.path.join(reference_dir(), "tools", "convert-qwen.py")
    spec = importlib.util.spec_from_file_location("convert_qwen_reference", src)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.SOURCE_SHA = ckpt_sha
    import contextlib
    import io
    with contextlib.redirect_stdout(io.StringIO()):
        mod.convert(Path(ckpt), Path(out))


def main():
    with tempfile.TemporaryDirectory() as d:
        ckpt, out = os.path.join(d, "tiny.safetensors"), os.path.join(d, "tiny.q8")
        ckpt_sha = write_checkpoint(ckpt)
        run_reference_converter(ckpt, out, ckpt_sha)
        data = open(out, "rb").read()
    gold = {"seed": SEED, "shapes": {"dim": DIM, "hidden": HIDDEN, "kv": KV, "vocab": VOCAB, "layers": LAYERS},
            "checkpoint_sha256": ckpt_sha, "output_bytes": len(data),
            "output_sha256": hashlib.sha256(data).hexdigest(),
            "source": "tools/convert-qwen.py:15-61 run on the checkpoint above"}
    with open(os.path.join(HERE, "convert_golden.json"), "w") as f:
        json.dump(gold, f, indent=1)
    print(json.dumps(gold))


if __name__ == "__main__":
    sys.exit(main())
