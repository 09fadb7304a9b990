"""The GGUF-metadata BPE tokenizer (mocha-moze-llm_b200/gguf_tokenizer.py).

* Qwen2: the reference's Qwen2.5 tokenizer (models/qwen-tokenizer.json) written as GGUF
  tokenizer metadata reproduces the reference's own token-id fixtures
  (tests/qwen-tokenizer-reference.json) and the reference BPE (src/tokenizer.py) on the
  launcher's ChatML template (mocha-llm:41), special tokens included.  These need the
  reference sources and are skipped without them.
* Llama 3 (``llama-bpe``) on the synthetic vocabulary the random-init GGUF models carry:
  the launcher's Llama-3 template (mocha-llm:39-40) yields its header tokens in place,
  a doubled BOS as llama.cpp produces for a template that starts with one, digit runs of
  up to three, and text that decodes back to itself.
"""
import json
import os
import sys
import unicodedata

import pytest

import gguf_tokenizer as gt
import mocha_gguf_model

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_dir():
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
    import oracle_py
    return oracle_py.reference_dir()


@pytest.fixture(scope="module")
def qwen(tmp_path_factory):
    src = os.path.join(reference_dir(), "models", "qwen-tokenizer.json")
    if not os.path.isfile(src):
        pytest.skip("reference sources not present")
    with open(src, encoding="utf-8") as f:
        d = json.load(f)
    vocab = d["model"]["vocab"]
    n = 151936
    tokens = [f"[PAD{i}]" for i in range(n)]
    types = [5] * n
    for t, i in vocab.items():
        tokens[i], types[i] = t, 1
    for a in d["added_tokens"]:
        tokens[a["id"]], types[a["id"]] = a["content"], 3 if a["special"] else 4
    merges = [m if isinstance(m, str) else " ".join(m) for m in d["model"]["merges"]]
    path = str(tmp_path_factory.mktemp("tok") / "qwen-tokenizer.gguf")
    from gguf import GGUFWriter
    w = GGUFWriter(path, "qwen2")
    w.add_tokenizer_model("gpt2")
    w.add_tokenizer_pre("qwen2")
    w.add_token_list(tokens)
    w.add_token_types(types)
    w.add_token_merges(merges)
    w.add_bos_token_id(151643)
    w.add_eos_token_id(151645)
    w.add_add_bos_token(False)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.close()
    return gt.GgufTokenizer.from_gguf(path)


def test_qwen_reference_fixtures(qwen):
    with open(os.path.join(reference_dir(), "tests", "qwen-tokenizer-reference.json"), encoding="utf-8") as f:
        cases = json.load(f)
    for c in cases:
        text = unicodedata.normalize("NFC", c["text"])   # the HF tokenizer's normalizer
        ids = qwen.encode(text)
        assert ids == c["ids"], c["text"]
        assert qwen.decode(ids) == text


def test_qwen_chat_template_matches_reference_bpe(qwen):
    sys.path.insert(0, os.path.join(reference_dir(), "src"))
    from pathlib import Path

    import tokenizer as ref_tok
    ref = ref_tok.Tokenizer(Path(reference_dir()) / "models" / "qwen-tokenizer.json")
    for prompt in ("你好，请简单介绍一下自己。", "Please introduce yourself briefly. It's 2024!"):
        text = "<|im_start|>user\n" + prompt + "<|im_end|>\n<|im_start|>assistant\n"
        want = [151644] + ref.encode("user\n" + prompt) + [151645] + ref.encode("\n") + [151644] + \
            ref.encode("assistant\n")
        assert qwen.encode(text) == want
        # user text cannot inject delimiters when special parsing is off
        assert all(t < 151643 for t in qwen.encode(text, parse_special=False))


@pytest.fixture(scope="module")
def llama():
    arch = mocha_gguf_model.ARCHS["llama1b"]
    tokens, types, merges, meta = mocha_gguf_model.synthetic_tokenizer(arch)
    return gt.GgufTokenizer(tokens, types, merges, meta["pre"], meta["bos"], meta["eos"], meta["add_bos"])


def test_llama3_template(llama, capsys):
    prompt = "Please introduce yourself briefly."
    text = ("<|begin_of_text|><|start_header_id|>user<|end_header_id|>\n\n" + prompt +
            "<|eot_id|><|start_header_id|>assistant<|end_header_id|>\n\n")
    ids = llama.encode(text)
    sp = {t: llama.ids[t] for t in ("<|begin_of_text|>", "<|start_header_id|>", "<|end_header_id|>", "<|eot_id|>")}
    assert ids[:3] == [sp["<|begin_of_text|>"], sp["<|begin_of_text|>"], sp["<|start_header_id|>"]]
    assert "two BOS tokens" in capsys.readouterr().err
    assert ids.count(sp["<|start_header_id|>"]) == 2 and ids.count(sp["<|end_header_id|>"]) == 2
    assert ids.count(sp["<|eot_id|>"]) == 1
    body = ids[ids.index(sp["<|end_header_id|>"]) + 1:ids.index(sp["<|eot_id|>"])]
    assert llama.decode(body) == "\n\n" + prompt
    assert llama.decode(ids) == text.replace("<|begin_of_text|>", "").replace("<|start_header_id|>", "") \
        .replace("<|end_header_id|>", "").replace("<|eot_id|>", "")


def test_llama3_digits_and_round_trip(llama):
    pieces = llama.pattern.findall("year 1234567 and 89")
    assert pieces == ["year", " ", "123", "456", "7", " and", " ", "89"]
    for text in ("café 😂\r\n中文  x", "I'M testing. We've gone!", "  hello\n\nworld\t  ", ""):
        assert llama.decode(llama.encode(text, add_special=False)) == text
