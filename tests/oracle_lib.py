"""ctypes wrapper of oracle/liboracle.so — the CPU checker. Test infrastructure:
only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use it."""
import ctypes
import os
import subprocess

import numpy as np

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_DIR = os.path.join(REPO, "oracle")
PATH = os.path.join(ORACLE_DIR, "liboracle.so")
VOCAB, HIDDEN, LAYERS = 131072, 3072, 26

F = ctypes.POINTER(ctypes.c_float)
P = ctypes.c_void_p
SZ = ctypes.c_size_t


class Oracle:
    def __init__(self, lib):
        self.lib = lib
        sig = {
            "oracle_fp8_decode": (ctypes.c_float, [ctypes.c_ubyte]),
            "oracle_yarn": (ctypes.c_int, [ctypes.c_uint32, P, P]),
            "oracle_project": (None, [P, P, P, SZ, SZ, SZ]),
            "oracle_project_fp8": (None, [P, ctypes.c_float, P, P, SZ, SZ, SZ]),
            "oracle_norm": (None, [P, P, P, SZ, SZ]),
            "oracle_element": (None, [P, P, P, SZ, ctypes.c_int]),
            "oracle_rope": (None, [P, P, P, P, P, SZ, SZ, ctypes.c_int]),
            "oracle_attention": (None, [P, P, P, P, SZ, SZ, P]),
            "oracle_set_threads": (None, [ctypes.c_int]),
            "oracle_set_rounding": (None, [ctypes.c_int, ctypes.c_int]),
            "oracle_set_accumulation": (None, [ctypes.c_int]),
            "oracle_threads": (ctypes.c_int, []),
            "oracle_open": (P, [ctypes.c_char_p, SZ, ctypes.c_char_p, SZ]),
            "oracle_close": (None, [P]),
            "oracle_reset": (None, [P]),
            "oracle_length": (SZ, [P]),
            "oracle_rewind": (ctypes.c_int, [P, SZ]),
            "oracle_forward": (ctypes.c_int, [P, P, SZ, P, P, P, ctypes.c_char_p, SZ]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args

    # ---- operator level; numpy float32 in/out
    def fp8_decode(self, code):
        return self.lib.oracle_fp8_decode(code)

    def yarn(self, position):
        c = np.zeros(128, np.float32)
        s = np.zeros(128, np.float32)
        rc = self.lib.oracle_yarn(position, c.ctypes.data, s.ctypes.data)
        return (c, s) if rc == 0 else None

    def project(self, w, x):
        w = np.ascontiguousarray(w, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        rows, cols = w.shape
        out = np.empty((x.shape[0], rows), np.float32)
        self.lib.oracle_project(w.ctypes.data, x.ctypes.data, out.ctypes.data, rows, cols, x.shape[0])
        return out

    def project_fp8(self, codes, scale, x):
        codes = np.ascontiguousarray(codes, np.uint8)
        x = np.ascontiguousarray(x, np.float32)
        rows, cols = codes.shape
        out = np.empty((x.shape[0], rows), np.float32)
        self.lib.oracle_project_fp8(codes.ctypes.data, float(scale), x.ctypes.data, out.ctypes.data,
                                    rows, cols, x.shape[0])
        return out

    def norm(self, gain, x):
        gain = np.ascontiguousarray(gain, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.lib.oracle_norm(gain.ctypes.data, x.ctypes.data, out.ctypes.data, x.shape[1], x.shape[0])
        return out

    def element(self, a, b, mode):
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        out = np.empty_like(a)
        self.lib.oracle_element(a.ctypes.data, b.ctypes.data, out.ctypes.data, a.size, mode)
        return out

    def rope(self, x, cos, sin, positions, query):
        x = np.ascontiguousarray(x, np.float32)
        cos = np.ascontiguousarray(cos, np.float32)
        sin = np.ascontiguousarray(sin, np.float32)
        pos = np.ascontiguousarray(positions, np.uint32)
        out = np.empty_like(x)
        self.lib.oracle_rope(x.ctypes.data, cos.ctypes.data, sin.ctypes.data, pos.ctypes.data,
                             out.ctypes.data, x.shape[1], x.shape[0], int(query))
        return out

    def attention(self, q, k, v, prefix):
        q = np.ascontiguousarray(q, np.float32)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        count = q.shape[0]
        out = np.empty((count, 4096), np.float32)
        self.lib.oracle_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, out.ctypes.data,
                                  count, prefix, None)
        return out

    def set_threads(self, n):
        self.lib.oracle_set_threads(n)

    def threads(self):
        return self.lib.oracle_threads()

    def open_model(self, path, context=256):
        return OracleModel(self, path, context)


class OracleModel:
    def __init__(self, oracle, path, context):
        self.o = oracle
        err = ctypes.create_string_buffer(512)
        self.handle = oracle.lib.oracle_open(os.fsencode(path), context, err, 512)
        if not self.handle:
            raise RuntimeError(err.value.decode())

    def close(self):
        if self.handle:
            self.o.lib.oracle_close(self.handle)
            self.handle = None

    def reset(self):
        self.o.lib.oracle_reset(self.handle)

    def length(self):
        return self.o.lib.oracle_length(self.handle)

    def rewind(self, n):
        if self.o.lib.oracle_rewind(self.handle, n):
            raise RuntimeError("rewind past length")

    def forward(self, ids, trace=False, final_norm=False):
        ids = np.ascontiguousarray(np.asarray(ids, np.int64))
        count = ids.size
        logits = np.empty(VOCAB, np.float32)
        tr = np.empty((LAYERS, count, HIDDEN), np.float32) if trace else None
        fn = np.empty((count, HIDDEN), np.float32) if final_norm else None
        err = ctypes.create_string_buffer(512)
        rc = self.o.lib.oracle_forward(self.handle, ids.ctypes.data, count, logits.ctypes.data,
                                       tr.ctypes.data if trace else None,
                                       fn.ctypes.data if final_norm else None, err, 512)
        if rc:
            raise RuntimeError(err.value.decode())
        return logits, tr, fn


def load():
    if not os.path.exists(PATH):
        subprocess.run(["make", "-C", ORACLE_DIR, "oracle"], check=True, capture_output=True)
    return Oracle(ctypes.CDLL(PATH))


SYNTH_PATH = os.path.join(ORACLE_DIR, "libsynth.so")


def synth_checkpoint(path, seed=0):
    """Write the seeded synthetic checkpoint with oracle/libsynth.so: the same
    writer as the product library's lunelette_cuda_synth_checkpoint, compiled on
    its own without CUDA, for callers that must not load the product library
    (the benchmark's CPU reference leg)."""
    if not os.path.exists(SYNTH_PATH):
        subprocess.run(["make", "-C", ORACLE_DIR, "synth"], check=True, capture_output=True)
    lib = ctypes.CDLL(SYNTH_PATH)
    fn = lib.lunelette_cuda_synth_checkpoint
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_char_p, ctypes.c_uint64, ctypes.c_char_p, SZ]
    err = ctypes.create_string_buffer(512)
    if fn(os.fsencode(path), seed, err, 512):
        raise RuntimeError(err.value.decode())
    return path


def greedy(logits):
    """argmax with strict '>' (lowest id wins ties), as src/generation.c:8-34."""
    return int(np.argmax(logits))
