"""Weight-converter parity: this library's grouped-Q8 writer (mocha_q8.write_model, the
quantisation rule of tools/convert-qwen.py:34-39 and the file layout of :46-61) writes the
same bytes as the reference converter for the same fp32 input.

The input is a tiny seeded BF16 checkpoint with the reference's tensor names
(tests/golden/make_convert_golden.py); the reference converter's output digest on it is
the committed golden.  When the reference sources are present the converter is also run
live and the two files are compared byte for byte."""
import hashlib
import json
import os
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_convert_golden as mk  # noqa: E402

import mocha_q8  # noqa: E402


def ours(ckpt, out):
    t = mk.read_checkpoint(ckpt)
    seq = [(t["model.embed_tokens.weight"], True)]
    for layer in range(mk.LAYERS):
        b = f"model.layers.{layer}."
        seq.append((t[b + "input_layernorm.weight"], False))
        seq += [(t[b + n + ".weight"], True) for n, _, _ in mk.MATRICES]
        seq.append((t[b + "post_attention_layernorm.weight"], False))
        seq += [(t[b + f"self_attn.{n}.bias"], False) for n in ("q_proj", "k_proj", "v_proj")]
    seq.append((t["model.norm.weight"], False))
    mocha_q8.write_model(out, iter(seq))
    return open(out, "rb").read()


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(HERE, "golden", "convert_golden.json")) as f:
        return json.load(f)


def test_writer_matches_reference_converter_digest(tmp_path, golden):
    ckpt = str(tmp_path / "tiny.safetensors")
    assert mk.write_checkpoint(ckpt) == golden["checkpoint_sha256"]   # the same input
    data = ours(ckpt, str(tmp_path / "ours.q8"))
    assert len(data) == golden["output_bytes"]
    assert hashlib.sha256(data).hexdigest() == golden["output_sha256"]


def test_writer_matches_reference_converter_live(tmp_path):
    if not os.path.isfile(os.path.join(mk.reference_dir(), "tools", "convert-qwen.py")):
        pytest.skip("reference sources not present")
    ckpt = str(tmp_path / "tiny.safetensors")
    sha = mk.write_checkpoint(ckpt)
    mk.run_reference_converter(ckpt, str(tmp_path / "ref.q8"), sha)
    ref = open(tmp_path / "ref.q8", "rb").read()
    data = ours(ckpt, str(tmp_path / "ours.q8"))
    assert data == ref
