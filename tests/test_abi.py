"""The C-ABI library loads and exports every function include/*.h declares
(no GPU needed: nothing here calls into the device code)."""
import ctypes
import os
import re

REF_ENGINE_ABI = ["gpu_init", "gpu_forward", "gpu_finish", "gpu_head_init", "gpu_head_start", "gpu_head_finish",
                  "gpu_collect"]


def test_library_exports_declared_symbols(native):
    lib = ctypes.CDLL(native.LIB_PATH)
    names = native.declared_functions()
    assert set(REF_ENGINE_ABI) <= set(names)
    assert "mocha_gguf_matmul" in names
    for n in names:
        assert hasattr(lib, n), n


def test_reference_signatures_unchanged(native):
    """Same parameter lists as src/minimind.h:16-22 and src/gguf-cuda.cu:110."""
    text = open(os.path.join(native.INCLUDE_DIR, "mocha_minimind.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    sig = {m.group(1): re.sub(r"\s+", " ", m.group(2)).strip()
           for m in re.finditer(r"int (\w+)\((.*?)\);", text, flags=re.S)}
    assert sig["gpu_init"] == "const void *file, unsigned bytes"
    assert sig["gpu_forward"] == "float *logits, int token, int pos, int project, int readback"
    assert sig["gpu_finish"] == "void"
    assert sig["gpu_collect"] == "float *logits, const int *history, int count, float penalty, int k, int rows"
    g = open(os.path.join(native.INCLUDE_DIR, "mocha_gguf.h")).read()
    assert "int mocha_gguf_matmul(int type, const void *w, int cols, int rows, const float *x, int vectors," in g


def test_no_oracle_linkage(native):
    """The product library must not reference the oracle."""
    data = open(native.LIB_PATH, "rb").read()
    for sym in (b"q8o_forward", b"gguf_o_matmul", b"liboracle"):
        assert sym not in data
