"""ctypes access to the CPU oracle (liboracle.so) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
VOCAB = 151936
DIM = 896


def reference_dir() -> str:
    """The reference source directory the oracle recipe builds from (MOCHA_REFERENCE_DIR,
    else the recipe's default); it need not exist."""
    p = subprocess.run(["make", "-s", "-C", HERE, "refdir"], check=True, capture_output=True, text=True)
    return p.stdout.strip()


def build(ref: bool = True) -> None:
    """Build liboracle.so and, when the reference sources exist, oracle/_ref."""
    subprocess.run(["make", "-C", HERE, "all"], check=True, capture_output=True)
    if ref and os.path.isdir(os.path.join(reference_dir(), "src")):
        subprocess.run(["make", "-C", HERE, "ref"], check=True, capture_output=True)


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build(ref=False)
        L = C.CDLL(LIB)
        L.q8o_create.restype = C.c_void_p
        L.q8o_create.argtypes = [C.c_void_p, C.c_size_t]
        L.q8o_destroy.argtypes = [C.c_void_p]
        L.q8o_reset.argtypes = [C.c_void_p]
        L.q8o_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
        L.q8o_matvec.argtypes = [C.c_void_p, C.c_void_p, C.c_uint, C.c_uint, C.c_void_p, C.c_void_p, C.c_int,
                                 C.c_uint]
        L.q8o_rmsnorm.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_void_p]
        L.q8o_sample.restype = C.c_int
        L.q8o_sample.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_float, C.c_float, C.c_int,
                                 C.c_float, C.POINTER(C.c_uint32), C.c_int]
        L.q8o_collect.restype = C.c_int
        L.q8o_collect.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_int, C.c_int]
        L.gguf_o_half.restype = C.c_float
        L.gguf_o_half.argtypes = [C.c_uint16]
        L.gguf_o_row_bytes.restype = C.c_uint
        L.gguf_o_row_bytes.argtypes = [C.c_int, C.c_int]
        L.gguf_o_dequant_row.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_void_p]
        L.gguf_o_matmul.restype = C.c_int
        L.gguf_o_matmul.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_uint,
                                    C.c_void_p, C.c_uint]
        _lib = L
    return _lib


class Q8Oracle:
    """The reference CPU forward restated in C, with its own KV cache."""

    def __init__(self, file_bytes):
        self._arr = file_bytes if isinstance(file_bytes, np.ndarray) else np.frombuffer(file_bytes, dtype=np.uint8)
        self.m = lib().q8o_create(self._arr.ctypes.data, self._arr.nbytes)
        if not self.m:
            raise ValueError("oracle rejected the model file")

    def __del__(self):
        if getattr(self, "m", None):
            lib().q8o_destroy(self.m)
            self.m = None

    def reset(self):
        lib().q8o_reset(self.m)

    def forward(self, token: int, pos: int, project: bool = True, hidden_only: bool = False):
        out = np.zeros(DIM if hidden_only else VOCAB, dtype=np.float32)
        lib().q8o_forward(self.m, token, pos, int(project), int(hidden_only), out.ctypes.data)
        return out

    def generate(self, prompt, n, temperature=0.0, top_k=1, top_p=1.0, penalty=1.0, seed=42, logits_at=()):
        """Token loop of src/minimind.cpp:110-182 (cpu backend); returns tokens and
        the raw logits at the requested decode steps."""
        self.reset()
        history = list(prompt)
        token = prompt[0]
        s = C.c_uint32(seed)
        out, kept = [], {}
        for pos in range(len(prompt) + n - 1):
            project = pos + 1 >= len(prompt)
            logits = self.forward(token, pos, project)
            if pos + 1 < len(prompt):
                token = prompt[pos + 1]
                continue
            step = len(out)
            if step in logits_at:
                kept[step] = logits.copy()
            h = np.asarray(history, dtype=np.int32)
            token = lib().q8o_sample(logits.ctypes.data, VOCAB, h.ctypes.data, len(h), penalty, temperature,
                                     top_k, top_p, C.byref(s), 0)
            if token == 151645:
                break
            out.append(token)
            history.append(token)
        return out, kept


def sample(logits, history, temperature, top_k, top_p, penalty, seed, skip_penalty=False):
    arr = np.array(logits, dtype=np.float32)
    h = np.asarray(history, dtype=np.int32)
    s = C.c_uint32(seed)
    tok = lib().q8o_sample(arr.ctypes.data, len(arr), h.ctypes.data, len(h), penalty, temperature, top_k, top_p,
                           C.byref(s), int(skip_penalty))
    return tok, s.value, arr


def collect(logits, recent, penalty, k, rows):
    out = np.empty(rows, dtype=np.float32)
    r = np.asarray(recent, dtype=np.int32)
    rc = lib().q8o_collect(np.ascontiguousarray(logits, dtype=np.float32).ctypes.data, out.ctypes.data,
                           r.ctypes.data, len(r), penalty, k, rows)
    if rc:
        raise ValueError("bad k/count")
    return out


def gguf_dequant(type_id: int, raw: bytes, rows: int, cols: int):
    rb = lib().gguf_o_row_bytes(type_id, cols)
    a = np.frombuffer(raw, dtype=np.uint8)
    out = np.empty((rows, cols), dtype=np.float32)
    for r in range(rows):
        lib().gguf_o_dequant_row(type_id, a.ctypes.data + r * rb, cols, out[r].ctypes.data)
    return out


def gguf_matmul(type_id, raw, cols, rows, x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    v = x.shape[0]
    y = np.empty((v, rows), dtype=np.float32)
    a = np.frombuffer(raw, dtype=np.uint8)
    rc = lib().gguf_o_matmul(type_id, a.ctypes.data, cols, rows, x.ctypes.data, v, cols * 4, y.ctypes.data,
                             rows * 4)
    if rc:
        raise ValueError("gguf_o_matmul rejected the arguments")
    return y


# ---- GGUF model forward (llama / qwen2) ---------------------------------------------

class _GoTensor(C.Structure):
    _fields_ = [("type", C.c_int), ("rows", C.c_int), ("cols", C.c_int), ("data", C.c_void_p)]


class _GoModel(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("layers", "dim", "heads", "kv_heads", "head_dim", "ffn", "vocab", "context",
                                       "neox")] + \
               [("eps", C.c_float), ("rope_base", C.c_float), ("embd", _GoTensor), ("out_norm", _GoTensor),
                ("rope_freqs", _GoTensor)] + \
               [(n, C.POINTER(_GoTensor)) for n in ("attn_norm", "wq", "wk", "wv", "bq", "bk", "bv", "wo", "ffn_norm",
                                                    "wg", "wu", "wd")]


class GGUFOracle:
    """llama / qwen2 GGUF forward restated in C (unpinned: llama.cpp is not available)."""

    def __init__(self, path, context=1024):
        from gguf import GGUFReader
        L = lib()
        L.go_create.restype = C.c_void_p
        L.go_create.argtypes = [C.POINTER(_GoModel)]
        L.go_destroy.argtypes = [C.c_void_p]
        L.go_forward.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        self.reader = r = GGUFReader(path)
        arch = bytes(r.fields["general.architecture"].parts[-1]).decode()

        def num(key):
            f = r.fields[f"{arch}.{key}"]
            return f.parts[f.data[0]][0]

        self.tensors = {t.name: t for t in r.tensors}
        self._keep = []

        def gt(name):
            if name not in self.tensors:
                return _GoTensor(0, 0, 0, None)
            t = self.tensors[name]
            arr = np.ascontiguousarray(t.data)
            self._keep.append(arr)
            cols = int(t.shape[0])
            rows = int(t.shape[1]) if len(t.shape) > 1 else 1
            return _GoTensor(int(t.tensor_type), rows, cols, arr.ctypes.data)

        layers = int(num("block_count"))
        dim = int(num("embedding_length"))
        heads = int(num("attention.head_count"))
        m = _GoModel()
        m.layers, m.dim, m.heads = layers, dim, heads
        m.kv_heads = int(num("attention.head_count_kv"))
        m.head_dim = dim // heads
        m.ffn = int(num("feed_forward_length"))
        m.vocab = int(self.tensors["token_embd.weight"].shape[1])
        m.context = context
        m.neox = 1 if arch == "qwen2" else 0
        m.eps = float(num("attention.layer_norm_rms_epsilon"))
        m.rope_base = float(num("rope.freq_base"))
        m.embd = gt("token_embd.weight")
        m.out_norm = gt("output_norm.weight")
        m.rope_freqs = gt("rope_freqs.weight")
        arrays = {}
        for key, suffix in (("attn_norm", "attn_norm.weight"), ("wq", "attn_q.weight"), ("wk", "attn_k.weight"),
                            ("wv", "attn_v.weight"), ("bq", "attn_q.bias"), ("bk", "attn_k.bias"),
                            ("bv", "attn_v.bias"), ("wo", "attn_output.weight"), ("ffn_norm", "ffn_norm.weight"),
                            ("wg", "ffn_gate.weight"), ("wu", "ffn_up.weight"), ("wd", "ffn_down.weight")):
            arr = (_GoTensor * layers)(*[gt(f"blk.{l}.{suffix}") for l in range(layers)])
            arrays[key] = arr
            setattr(m, key, C.cast(arr, C.POINTER(_GoTensor)))
        self._arrays = arrays
        self.model = m
        self.vocab = m.vocab
        self.arch = arch
        self.s = L.go_create(C.byref(m))
        if not self.s:
            raise MemoryError("go_create failed")

    def __del__(self):
        if getattr(self, "s", None):
            lib().go_destroy(self.s)
            self.s = None

    def forward(self, token, pos, project=True):
        out = np.empty(self.vocab, np.float32) if project else None
        lib().go_forward(self.s, token, pos, out.ctypes.data if project else None)
        return out

    def greedy(self, prompt, n):
        out = []
        tok = prompt[0]
        for pos in range(len(prompt) + n - 1):
            project = pos + 1 >= len(prompt)
            logits = self.forward(tok, pos, project)
            if pos + 1 < len(prompt):
                tok = prompt[pos + 1]
                continue
            tok = int(np.argmax(logits))
            out.append(tok)
        return out
