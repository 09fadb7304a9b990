"""mocha-gguf-cli, the llama-cli-compatible GGUF host (mocha-llm:42-47).

CPU: its C++ tokenizer gives the same ids as gguf_tokenizer.py (--print-token-ids, no
GPU touched) on the Llama-3 launcher template and edge-case texts over the random
models' synthetic vocabulary, and -- when the reference sources are present -- on the
reference's Qwen2.5 tokenizer fixtures; its argument and backend errors.
GPU: the launcher's whole command line on the random-init Llama-1B and Qwen-1.5B models
prints exactly the text of the tokens the engine's handle API generates greedily for
the same prompt ids.
"""
import json
import os
import subprocess
import sys
import unicodedata

import numpy as np
import pytest

import gguf_tokenizer as gt
import mocha_gguf_model

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CLI = os.path.join(ROOT, "mocha-moze-llm_b200", "bin", "mocha-gguf-cli")
LLAMA3 = ("<|begin_of_text|><|start_header_id|>user<|end_header_id|>\n\n{}<|eot_id|>"
          "<|start_header_id|>assistant<|end_header_id|>\n\n")
CHATML = "<|im_start|>user\n{}<|im_end|>\n<|im_start|>assistant\n"
TEXTS = ["Please introduce yourself briefly.", "你好，请简单介绍一下自己。", "I'M testing. We've gone!",
         "  hello\n\nworld\t  ", "😂 café é\r\n中文123，测试", " \t a  b", "year 1234567 and 89", "x", "don't'll'VE",
         "a\n\n\nb  \n c", "tab\there,comma;semi:colon!?"]


@pytest.fixture(scope="session")
def cli():
    if not os.path.exists(CLI):
        subprocess.run(["make", "-C", os.path.dirname(os.path.dirname(CLI))], check=True, capture_output=True)
    return CLI


def write_tokenizer_gguf(path, tokens, types, merges, meta, arch):
    from gguf import GGUFWriter
    w = GGUFWriter(path, arch)
    w.add_tokenizer_model("gpt2")
    w.add_tokenizer_pre(meta["pre"])
    w.add_token_list(tokens)
    w.add_token_types(types)
    w.add_token_merges(merges)
    w.add_bos_token_id(meta["bos"])
    w.add_eos_token_id(meta["eos"])
    w.add_add_bos_token(meta["add_bos"])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.close()
    return path


def cli_ids(cli, path, text):
    p = subprocess.run([cli, "-m", path, "-p", text, "--print-token-ids"], capture_output=True, text=True)
    assert p.returncode == 0, p.stderr
    return [int(x) for x in p.stdout.split()]


@pytest.fixture(scope="module")
def llama_tok(tmp_path_factory):
    arch = mocha_gguf_model.ARCHS["llama1b"]
    tokens, types, merges, meta = mocha_gguf_model.synthetic_tokenizer(arch)
    path = write_tokenizer_gguf(str(tmp_path_factory.mktemp("t") / "llama-tok.gguf"), tokens, types, merges, meta,
                                "llama")
    return path, gt.GgufTokenizer(tokens, types, merges, meta["pre"], meta["bos"], meta["eos"], meta["add_bos"])


def test_cli_tokenizer_matches_python_llama3(cli, llama_tok):
    path, tok = llama_tok
    for text in [LLAMA3.format(TEXTS[0])] + TEXTS:
        assert cli_ids(cli, path, text) == tok.encode(text), text


def test_cli_tokenizer_matches_reference_qwen(cli, tmp_path):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_py
    ref = oracle_py.reference_dir()
    src = os.path.join(ref, "models", "qwen-tokenizer.json")
    if not os.path.isfile(src):
        pytest.skip("reference sources not present")
    with open(src, encoding="utf-8") as f:
        d = json.load(f)
    n = 151936
    tokens, types = [f"[PAD{i}]" for i in range(n)], [5] * n
    for t, i in d["model"]["vocab"].items():
        tokens[i], types[i] = t, 1
    for a in d["added_tokens"]:
        tokens[a["id"]], types[a["id"]] = a["content"], 3 if a["special"] else 4
    merges = [m if isinstance(m, str) else " ".join(m) for m in d["model"]["merges"]]
    meta = {"pre": "qwen2", "bos": 151643, "eos": 151645, "add_bos": False}
    path = write_tokenizer_gguf(str(tmp_path / "qwen-tok.gguf"), tokens, types, merges, meta, "qwen2")
    with open(os.path.join(ref, "tests", "qwen-tokenizer-reference.json"), encoding="utf-8") as f:
        cases = json.load(f)
    for c in cases:
        text = unicodedata.normalize("NFC", c["text"])
        assert cli_ids(cli, path, text) == c["ids"], c["text"]
    tok = gt.GgufTokenizer(tokens, types, merges, "qwen2", 151643, 151645, False)
    for text in [CHATML.format(TEXTS[1])] + TEXTS:
        assert cli_ids(cli, path, text) == tok.encode(text), text


def test_cli_errors(cli, llama_tok):
    path, _ = llama_tok
    p = subprocess.run([cli, "-m", path, "-p", "hi", "--bogus"], capture_output=True, text=True)
    assert p.returncode == 1 and "unknown argument" in p.stderr
    p = subprocess.run([cli, "-m", path, "-p", "hi", "-n", "4"], capture_output=True, text=True,
                       env=dict(os.environ, MOCHA_GGUF_CUDA="0"))
    assert p.returncode == 1 and "CPU backend" in p.stderr
    p = subprocess.run([cli, "-p", "hi"], capture_output=True, text=True)
    assert p.returncode == 1


def launcher_command(cli, path, text, n):
    """The argument list mocha-llm:42-45 builds (greedy: --temp 0)."""
    return [cli, "-m", path, "-p", text, "-n", str(n), "-c", "1024", "-b", "32", "-ub", "32", "-t", "4",
            "-ngl", "0", "-no-cnv", "--no-display-prompt", "--no-context-shift", "--temp", "0", "--seed", "42",
            "--repeat-penalty", "1.0", "--top-k", "40", "--top-p", "0.9"]


@pytest.mark.gpu
@pytest.mark.parametrize("arch,template,prompt", [("llama1b", LLAMA3, "Please introduce yourself briefly."),
                                                  ("qwen15b", CHATML, "你好，请简单介绍一下自己。")])
def test_cli_generates_the_engine_tokens(cli, native, arch, template, prompt):
    path = mocha_gguf_model.model_path(arch)
    text = template.format(prompt)
    n = 24
    p = subprocess.run(launcher_command(cli, path, text, n), capture_output=True,
                       env=dict(os.environ, MOCHA_GGUF_CUDA="1", MOCHA_GGUF_GPU_CACHE_MIB="512"))
    assert p.returncode == 0, p.stderr.decode(errors="replace")
    tok = gt.GgufTokenizer.from_gguf(path)
    ids = tok.encode(text)
    h = native.GgufHandle(0, np.fromfile(path, dtype=np.uint8))
    try:
        toks, _ = h.generate(ids, n)
    finally:
        h.close()
    want = b"".join(tok.token_bytes(t) for t in toks)
    assert p.stdout == want
    err = p.stderr.decode(errors="replace")
    assert f"PROMPT_TOKENS={len(ids)} GENERATED={len(toks)}" in err
