"""ctypes view of libmocha_b200.so (the C ABI in include/*.h) and of the build.

The library is the product; this module only loads it and declares the argument
types, mirroring the reference's C entry points (src/minimind.h:16-22,
src/gguf-cuda.cu:110) and the handle API of include/mocha_b200.h.  It never falls
back to anything: when the shared object is missing, loading raises.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)
LIB_PATH = os.path.join(PKG_DIR, "libmocha_b200.so")
INCLUDE_DIR = os.path.join(ROOT, "include")


class MochaSampling(C.Structure):
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float),
                ("repeat_penalty", C.c_float), ("seed", C.c_uint)]


class MochaGgufInfo(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("arch", "layers", "dim", "ffn", "heads", "kv_heads", "head_dim", "vocab",
                                       "context")] + \
               [("eps", C.c_float), ("rope_base", C.c_float), ("rope_neox", C.c_int), ("rope_factors", C.c_int),
                ("eos", C.c_int)]


class MochaTiming(C.Structure):
    _fields_ = [("prefill_s", C.c_double), ("decode_s", C.c_double), ("generated", C.c_int)]


_SIGS = {
    # reference engine ABI
    "gpu_init": (C.c_int, [C.c_void_p, C.c_uint]),
    "gpu_forward": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]),
    "gpu_finish": (C.c_int, []),
    "gpu_head_init": (C.c_int, [C.c_void_p]),
    "gpu_head_start": (C.c_int, [C.c_void_p, C.c_int]),
    "gpu_head_finish": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "gpu_collect": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_float, C.c_int, C.c_int]),
    # reference GGUF bridge
    "mocha_gguf_matmul": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_uint,
                                    C.c_void_p, C.c_uint]),
    "mocha_gguf_dequant": (C.c_int, [C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    # handle API
    "mocha_b200_device_count": (C.c_int, []),
    "mocha_q8_open": (C.c_int, [C.c_int, C.c_void_p, C.c_ulonglong, C.POINTER(C.c_void_p)]),
    "mocha_q8_close": (C.c_int, [C.c_void_p]),
    "mocha_q8_forward": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "mocha_q8_generate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(MochaSampling),
                                    C.c_void_p, C.POINTER(C.c_int), C.POINTER(MochaTiming)]),
    "mocha_q8_bench_decode": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.POINTER(C.c_float)]),
    "mocha_q8_launches_per_step": (C.c_int, [C.c_void_p]),
    "mocha_q8_stream_begin": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(MochaSampling)]),
    "mocha_q8_stream_next": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "mocha_q8_stream_end": (C.c_int, [C.c_void_p]),
    "mocha_topk_static": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_float, C.c_int, C.c_void_p,
                                    C.c_void_p, C.c_void_p]),
    "mocha_q8_trace_step": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "mocha_gguf_open": (C.c_int, [C.c_int, C.c_void_p, C.c_ulonglong, C.POINTER(C.c_void_p)]),
    "mocha_gguf_close": (C.c_int, [C.c_void_p]),
    "mocha_gguf_get_info": (C.c_int, [C.c_void_p, C.c_void_p]),
    "mocha_gguf_forward": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "mocha_gguf_generate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.POINTER(MochaSampling),
                                      C.c_void_p, C.POINTER(C.c_int), C.POINTER(MochaTiming)]),
    "mocha_gguf_bench_decode": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                          C.POINTER(C.c_float)]),
    "mocha_gguf_launches_per_step": (C.c_int, [C.c_void_p]),
    "mocha_q8_counters": (C.c_int, [C.c_void_p, C.POINTER(C.c_ulonglong), C.POINTER(C.c_ulonglong)]),
    "mocha_q8b_open": (C.c_int, [C.c_int, C.c_void_p, C.c_ulonglong, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "mocha_q8b_close": (C.c_int, [C.c_void_p]),
    "mocha_q8b_forward": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                    C.c_void_p]),
    "mocha_q8b_prefill": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p]),
    "mocha_q8b_generate": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.POINTER(MochaSampling),
                                     C.c_uint, C.c_void_p, C.c_void_p, C.POINTER(MochaTiming)]),
    "mocha_q8b_generate_each": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                          C.POINTER(MochaSampling), C.c_uint, C.c_void_p, C.c_int, C.c_void_p,
                                          C.POINTER(MochaTiming)]),
    "mocha_q8b_launches_per_step": (C.c_int, [C.c_void_p]),
    "mocha_q8b_bench_prefill": (C.c_int, [C.c_void_p, C.c_int, C.c_uint, C.c_int, C.c_int, C.POINTER(C.c_float)]),
    "mocha_q8b_sample_check": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.POINTER(MochaSampling), C.c_void_p, C.c_void_p]),
    "mocha_tq_gemm_check": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_int]),
    "mocha_tc_gemm_check": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_int]),
}


def build(verbose: bool = False) -> str:
    """Compile libmocha_b200.so for sm_100a with the package Makefile."""
    out = subprocess.run(["make", "-C", PKG_DIR, "-j", str(min(8, os.cpu_count() or 1))],
                         capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("libmocha_b200 build failed:\n" + out.stdout[-4000:] + out.stderr[-4000:])
    if verbose:
        print(out.stdout)
    return LIB_PATH


_lib = None


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load the library (raises OSError when it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise OSError(f"{path} missing: build it with `make -C {PKG_DIR}` (no fallback exists)")
        lib = C.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def declared_functions() -> list[str]:
    """Every function name declared in include/*.h."""
    import re
    names = []
    for fn in sorted(os.listdir(INCLUDE_DIR)):
        if fn.endswith(".h"):
            text = open(os.path.join(INCLUDE_DIR, fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"^\s*(?:int|void|float|unsigned)\s+\**(\w+)\s*\(", text, flags=re.M)
    return names


class Q8Handle:
    """A grouped-Q8 model resident on one device (mocha_q8 handle)."""

    def __init__(self, device: int, file_bytes, lib: C.CDLL | None = None):
        self.lib = lib or load()
        self._buf = file_bytes  # keep the host buffer alive while opening
        ptr = C.c_void_p()
        addr, size = _addr(file_bytes)
        if self.lib.mocha_q8_open(device, addr, size, C.byref(ptr)) != 0:
            raise RuntimeError("mocha_q8_open failed")
        self.h = ptr

    def close(self):
        if self.h:
            self.lib.mocha_q8_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, token: int, pos: int, project: bool = True):
        import numpy as np
        out = np.empty(151936, dtype=np.float32)
        rc = self.lib.mocha_q8_forward(self.h, token, pos, int(project), out.ctypes.data)
        if rc != 0:
            raise RuntimeError("mocha_q8_forward failed")
        return out

    def generate(self, prompt, n_new, temperature=0.0, top_k=1, top_p=1.0, penalty=1.0, seed=42):
        import numpy as np
        p = np.asarray(prompt, dtype=np.int32)
        out = np.zeros(n_new, dtype=np.int32)
        n = C.c_int()
        t = MochaTiming()
        s = MochaSampling(temperature, top_k, top_p, penalty, seed)
        rc = self.lib.mocha_q8_generate(self.h, p.ctypes.data, len(p), n_new, C.byref(s), out.ctypes.data,
                                        C.byref(n), C.byref(t))
        if rc != 0:
            raise RuntimeError("mocha_q8_generate failed")
        return out[:n.value].tolist(), t

    def bench_decode(self, token, pos0, pos_end, warmup, steps) -> float:
        ms = C.c_float()
        rc = self.lib.mocha_q8_bench_decode(self.h, token, pos0, pos_end, warmup, steps, C.byref(ms))
        if rc != 0:
            raise RuntimeError("mocha_q8_bench_decode failed")
        return ms.value

    def trace_step(self, token: int, pos: int):
        """%globaltimer stamps [148 CTAs][640] of one persistent step (see mocha_q8_trace_step)."""
        import numpy as np
        st = np.zeros((148, 640), dtype=np.uint64)
        if self.lib.mocha_q8_trace_step(self.h, token, pos, st.ctypes.data) != 0:
            raise RuntimeError("mocha_q8_trace_step failed")
        return st


class GgufHandle:
    """A GGUF llama / qwen2 model resident on one device (mocha_gguf handle)."""

    def __init__(self, device: int, file_bytes, lib: C.CDLL | None = None):
        self.lib = lib or load()
        self._buf = file_bytes
        ptr = C.c_void_p()
        addr, size = _addr(file_bytes)
        if self.lib.mocha_gguf_open(device, addr, size, C.byref(ptr)) != 0:
            raise RuntimeError("mocha_gguf_open failed")
        self.h = ptr
        self.info = MochaGgufInfo()
        self.lib.mocha_gguf_get_info(self.h, C.byref(self.info))

    def close(self):
        if self.h:
            self.lib.mocha_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, token: int, pos: int, project: bool = True):
        import numpy as np
        out = np.empty(self.info.vocab, dtype=np.float32)
        if self.lib.mocha_gguf_forward(self.h, token, pos, int(project), out.ctypes.data) != 0:
            raise RuntimeError("mocha_gguf_forward failed")
        return out

    def generate(self, prompt, n_new, temperature=0.0, top_k=1, top_p=1.0, penalty=1.0, seed=42):
        import numpy as np
        p = np.asarray(prompt, dtype=np.int32)
        out = np.zeros(n_new, dtype=np.int32)
        n = C.c_int()
        t = MochaTiming()
        s = MochaSampling(temperature, top_k, top_p, penalty, seed)
        if self.lib.mocha_gguf_generate(self.h, p.ctypes.data, len(p), n_new, C.byref(s), out.ctypes.data,
                                        C.byref(n), C.byref(t)) != 0:
            raise RuntimeError("mocha_gguf_generate failed")
        return out[:n.value].tolist(), t

    def bench_decode(self, token, pos0, pos_end, warmup, steps) -> float:
        ms = C.c_float()
        if self.lib.mocha_gguf_bench_decode(self.h, token, pos0, pos_end, warmup, steps, C.byref(ms)) != 0:
            raise RuntimeError("mocha_gguf_bench_decode failed")
        return ms.value


def _addr(buf):
    """(address, size) of a bytes-like / numpy / mmap buffer without copying."""
    import numpy as np
    arr = np.frombuffer(buf, dtype=np.uint8) if not isinstance(buf, np.ndarray) else buf
    return arr.ctypes.data, arr.nbytes


class Q8BatchHandle:
    """The batched grouped-Q8 engine on one device (mocha_q8b handle): tcgen05 GEMMs
    over rows of (token, position, KV slot)."""

    VOCAB = 151936

    def __init__(self, device: int, file_bytes, max_rows: int = 1024, slots: int = 64, lib: C.CDLL | None = None):
        import numpy as np
        self.lib = lib or load()
        self._file = np.ascontiguousarray(file_bytes, dtype=np.uint8)
        h = C.c_void_p()
        if self.lib.mocha_q8b_open(device, self._file.ctypes.data, self._file.nbytes, max_rows, slots, C.byref(h)):
            raise RuntimeError("mocha_q8b_open failed")
        self.h = h
        self.slots = slots
        self.max_rows = max_rows

    def close(self):
        if getattr(self, "h", None):
            self.lib.mocha_q8b_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, tokens, pos, slots, project_rows=()):
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(pos, dtype=np.int32)
        s = np.ascontiguousarray(slots, dtype=np.int32)
        pr = np.ascontiguousarray(project_rows, dtype=np.int32)
        out = np.empty((len(pr), self.VOCAB), np.float32)
        rc = self.lib.mocha_q8b_forward(self.h, len(t), t.ctypes.data, p.ctypes.data, s.ctypes.data, len(pr),
                                        pr.ctypes.data if len(pr) else None, out.ctypes.data if len(pr) else None)
        if rc:
            raise RuntimeError("mocha_q8b_forward failed")
        return out

    def prefill(self, slot, tokens):
        import numpy as np
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.VOCAB, np.float32)
        if self.lib.mocha_q8b_prefill(self.h, slot, t.ctypes.data, len(t), out.ctypes.data):
            raise RuntimeError("mocha_q8b_prefill failed")
        return out

    def generate(self, prompts, n_new, temperature=0.0, top_k=1, top_p=1.0, penalty=1.0, seed_base=42):
        import numpy as np
        pr = np.ascontiguousarray(prompts, dtype=np.int32)
        nseq, plen = pr.shape
        out = np.zeros((nseq, n_new), np.int32)
        counts = np.zeros(nseq, np.int32)
        s = MochaSampling(temperature, top_k, top_p, penalty, 0)
        t = MochaTiming()
        if self.lib.mocha_q8b_generate(self.h, nseq, pr.ctypes.data, plen, n_new, C.byref(s), seed_base,
                                       out.ctypes.data, counts.ctypes.data, C.byref(t)):
            raise RuntimeError("mocha_q8b_generate failed")
        return [out[i, :counts[i]].tolist() for i in range(nseq)], t

    def generate_each(self, prompts, n_new, temperature=0.0, top_k=1, top_p=1.0, penalty=1.0, seed_base=42):
        """Per-sequence token budgets n_new[i] (continuous batching refills freed slots)."""
        import numpy as np
        pr = np.ascontiguousarray(prompts, dtype=np.int32)
        nseq, plen = pr.shape
        nn = np.ascontiguousarray(n_new, dtype=np.int32)
        stride = int(nn.max())
        out = np.zeros((nseq, stride), np.int32)
        counts = np.zeros(nseq, np.int32)
        s = MochaSampling(temperature, top_k, top_p, penalty, 0)
        t = MochaTiming()
        if self.lib.mocha_q8b_generate_each(self.h, nseq, pr.ctypes.data, plen, nn.ctypes.data, C.byref(s), seed_base,
                                            out.ctypes.data, stride, counts.ctypes.data, C.byref(t)):
            raise RuntimeError("mocha_q8b_generate_each failed")
        return [out[i, :counts[i]].tolist() for i in range(nseq)], t

    def bench_prefill(self, n, seed, warmup, steps) -> float:
        ms = C.c_float()
        if self.lib.mocha_q8b_bench_prefill(self.h, n, seed, warmup, steps, C.byref(ms)):
            raise RuntimeError("mocha_q8b_bench_prefill failed")
        return ms.value

    def launches_per_step(self) -> int:
        return self.lib.mocha_q8b_launches_per_step(self.h)

    def sample(self, logits, histories, temperature, top_k, top_p, penalty, seeds):
        import numpy as np
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        n = lg.shape[0]
        hist = np.zeros((n, 64), np.int32)
        counts = np.zeros(n, np.int32)
        for i, h in enumerate(histories):
            h = list(h)[-64:]
            hist[i, :len(h)] = h
            counts[i] = len(h)
        sd = np.ascontiguousarray(seeds, dtype=np.uint32)
        tok = np.zeros(n, np.int32)
        s = MochaSampling(temperature, top_k, top_p, penalty, 0)
        if self.lib.mocha_q8b_sample_check(self.h, n, lg.ctypes.data, hist.ctypes.data, counts.ctypes.data,
                                           C.byref(s), sd.ctypes.data, tok.ctypes.data):
            raise RuntimeError("mocha_q8b_sample_check failed")
        return tok.tolist()
