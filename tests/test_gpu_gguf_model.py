"""GGUF llama / qwen2 decoder on B200 against the C restatement of the forward
(oracle/gguf_model_oracle.c; llama.cpp itself is not available, so this parity is
unpinned).  Random-init Q4_K_M-mix models with the benchmark shapes."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=["llama1b", "qwen15b"])
def pair(request, native, oracle_lib):
    import mocha_gguf_model
    path = mocha_gguf_model.model_path(request.param)
    data = np.fromfile(path, dtype=np.uint8)
    h = native.GgufHandle(0, data)
    o = oracle_lib.GGUFOracle(path)
    yield request.param, h, o
    h.close()


def test_info(pair):
    name, h, _ = pair
    i = h.info
    if name == "llama1b":
        assert (i.arch, i.layers, i.dim, i.heads, i.kv_heads, i.head_dim, i.ffn, i.vocab) == (0, 16, 2048, 32, 8, 64, 8192, 128256)
        assert i.rope_neox == 0 and i.rope_factors == 1
    else:
        assert (i.arch, i.layers, i.dim, i.heads, i.kv_heads, i.head_dim, i.ffn, i.vocab) == (1, 28, 1536, 12, 2, 128, 8960, 151936)
        assert i.rope_neox == 1 and i.rope_factors == 0


def test_logits_match_oracle(pair):
    name, h, o = pair
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, h.info.vocab, 6).tolist()
    worst = 0.0
    for pos, tok in enumerate(prompt):
        got = h.forward(tok, pos, True)
        ref = o.forward(tok, pos, True)
        err = np.abs(got - ref)
        assert np.all(np.isfinite(got))
        assert np.all(err <= 0.003 * (1 + np.abs(ref))), (name, pos, float(err.max()))
        assert err.max() <= 2e-3 * float(ref.max() - ref.min())
        assert int(np.argmax(got)) == int(np.argmax(ref))
        worst = max(worst, float(err.max()))
    print(name, "max abs logit error", worst)


def test_greedy_tokens_match_oracle(pair, oracle_lib):
    name, h, _ = pair
    import mocha_gguf_model
    o = oracle_lib.GGUFOracle(mocha_gguf_model.model_path(name))  # fresh KV cache
    rng = np.random.default_rng(4)
    prompt = rng.integers(0, h.info.vocab, 8).tolist()
    toks, t = h.generate(prompt, 6)
    assert toks == o.greedy(prompt, 6)
