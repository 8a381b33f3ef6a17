"""Python binding of the B200 Lunelette backend (ctypes over the C-ABI).

The product is the C library lunelette_b200/liblunelette_cuda.so, whose
drop-in contract is include/metal.h (the reference's include/metal.h:11-120)
and whose additive entry points are in include/lunelette_cuda.h. This module
mirrors the metal.h API one call per function for tests, benchmarks and Python
callers; it performs no computation of its own and never falls back to another
implementation: if the library is missing, every entry raises.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY_PATH = os.path.join(HERE, "liblunelette_cuda.so")
VOCAB = 131072
HIDDEN = 3072
LAYERS = 26

PREFILL_MPS, PREFILL_CUSTOM = 0, 1
RESIDENT_FP32, COMPACT_FP8_ARITHMETIC, COMPACT_FP8_LOOKUP = 0, 1, 2
STRATEGY_NAMES = {RESIDENT_FP32: "resident-fp32", COMPACT_FP8_ARITHMETIC: "compact-fp8-arithmetic",
                  COMPACT_FP8_LOOKUP: "compact-fp8-lookup"}


class LuneletteError(RuntimeError):
    """A call of the C-ABI returned failure; the message is its diagnostic."""


class Options(ctypes.Structure):
    _fields_ = [("prefill", ctypes.c_int), ("strategy", ctypes.c_int)]


class Limits(ctypes.Structure):
    _fields_ = [("context", ctypes.c_size_t), ("block", ctypes.c_size_t)]


class Memory(ctypes.Structure):
    _fields_ = [("strategy", ctypes.c_int), ("weight_bytes", ctypes.c_uint64),
                ("conversion_stage_bytes", ctypes.c_uint64), ("scratch_bytes", ctypes.c_uint64),
                ("kv_bytes", ctypes.c_uint64), ("total_bytes", ctypes.c_uint64)]


_lib = None
P = ctypes.c_void_p
SZ = ctypes.c_size_t
ERR = ctypes.c_char_p

# name -> (restype, argtypes); every symbol include/metal.h and include/lunelette_cuda.h declare
SIGNATURES = {
    "lunelette_metal_create": (P, [ctypes.c_char_p, ERR, SZ]),
    "lunelette_metal_create_with_options": (P, [ctypes.c_char_p, P, ERR, SZ]),
    "lunelette_metal_create_configured": (P, [ctypes.c_char_p, P, P, ERR, SZ]),
    "lunelette_metal_get_limits": (ctypes.c_int, [P, P]),
    "lunelette_metal_get_memory": (ctypes.c_int, [P, P]),
    "lunelette_metal_destroy": (None, [P]),
    "lunelette_metal_reset": (ctypes.c_int, [P, ERR, SZ]),
    "lunelette_metal_prefill": (ctypes.c_int, [P, P, SZ, P, ERR, SZ]),
    "lunelette_metal_decode": (ctypes.c_int, [P, ctypes.c_int64, P, ERR, SZ]),
    "lunelette_metal_append": (ctypes.c_int, [P, P, SZ, P, ERR, SZ]),
    "lunelette_metal_checkpoint_create": (ctypes.c_int, [P, P, ERR, SZ]),
    "lunelette_metal_checkpoint_restore": (ctypes.c_int, [P, P, P, ERR, SZ]),
    "lunelette_metal_checkpoint_destroy": (None, [P]),
    "lunelette_cuda_kernels_init": (ctypes.c_int, []),
    "lunelette_cuda_fp8_decode": (ctypes.c_int, [P, SZ, ctypes.c_float, P, P]),
    "lunelette_cuda_tile_fp8": (ctypes.c_int, [P, SZ, SZ, ctypes.c_int, P, P]),
    "lunelette_cuda_gemv_fp8": (ctypes.c_int, [P, SZ, SZ, ctypes.c_float, P, P, SZ, P, P]),
    "lunelette_cuda_qkv_rope": (ctypes.c_int, [P, P, P, P, SZ, SZ, P, P, P, P, P, SZ, SZ, P]),
    "lunelette_cuda_gateup_swiglu": (ctypes.c_int, [P, ctypes.c_float, ctypes.c_float, P, P, SZ, P, P]),
    "lunelette_cuda_gemm_fp8": (ctypes.c_int, [P, SZ, SZ, ctypes.c_float, P, P, SZ, P, P]),
    "lunelette_cuda_gemm_qkv_rope": (ctypes.c_int, [P, P, P, P, SZ, SZ, P, P, P, P, P, SZ, SZ, P]),
    "lunelette_cuda_gemm_gateup_swiglu": (ctypes.c_int, [P, ctypes.c_float, ctypes.c_float, P, P, SZ, P, P]),
    "lunelette_cuda_batch_create": (ctypes.c_void_p, [ctypes.c_char_p, SZ, SZ, SZ, SZ, ctypes.c_char_p, SZ]),
    "lunelette_cuda_batch_destroy": (None, [P]),
    "lunelette_cuda_batch_open": (ctypes.c_int, [P, P, ctypes.c_char_p, SZ]),
    "lunelette_cuda_batch_close": (ctypes.c_int, [P, ctypes.c_int]),
    "lunelette_cuda_batch_append": (ctypes.c_int, [P, ctypes.c_int, P, SZ, P, ctypes.c_char_p, SZ]),
    "lunelette_cuda_batch_decode": (ctypes.c_int, [P, P, P, SZ, P, P, ctypes.c_char_p, SZ]),
    "lunelette_cuda_batch_fork": (ctypes.c_int, [P, ctypes.c_int, SZ, P, ctypes.c_char_p, SZ]),
    "lunelette_cuda_batch_length": (SZ, [P, ctypes.c_int]),
    "lunelette_cuda_batch_free_positions": (SZ, [P]),
    "lunelette_cuda_kv_copy": (ctypes.c_int, [P, SZ, SZ, P, P, SZ, SZ, P]),
    "lunelette_cuda_gemm_fp8_timed": (ctypes.c_int, [P, SZ, SZ, SZ, ctypes.c_float, P, SZ, P, ctypes.c_int, P, P]),
    "lunelette_cuda_rmsnorm": (ctypes.c_int, [P, P, SZ, SZ, P, P]),
    "lunelette_cuda_head_bf16": (ctypes.c_int, [P, SZ, SZ, P, P, P, P, P]),
    "lunelette_cuda_attention": (ctypes.c_int, [P, P, P, SZ, SZ, SZ, SZ, P, P, P, SZ, P]),
    "lunelette_cuda_attention_noalloc": (ctypes.c_int, [P, P, P, SZ, SZ, SZ, SZ, P, P, ERR, SZ]),
    "lunelette_cuda_trace": (ctypes.c_int, [P, ctypes.c_int]),
    "lunelette_cuda_trace_copy": (ctypes.c_int, [P, ctypes.c_int, P, SZ]),
    "lunelette_cuda_snapshot": (P, [P, ctypes.c_int]),
    "lunelette_cuda_length": (SZ, [P]),
    "lunelette_cuda_decode_loop": (ctypes.c_int, [P, ctypes.c_int64, SZ, P, P, P, ERR, SZ]),
    "lunelette_cuda_yarn": (ctypes.c_int, [ctypes.c_uint32, P, P]),
    "lunelette_cuda_timeline": (ctypes.c_int, [P, ctypes.c_int]),
    "lunelette_cuda_timeline_copy": (ctypes.c_int, [P, P, SZ]),
    "lunelette_cuda_validate_checkpoint": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ERR, SZ]),
    "lunelette_cuda_synth_checkpoint": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_uint64, ERR, SZ]),
    "lunelette_cuda_e4m3_encode": (ctypes.c_ubyte, [ctypes.c_float]),
}


def library():
    """Load liblunelette_cuda.so (built by lunelette_b200.build); raise if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIBRARY_PATH):
            raise LuneletteError("liblunelette_cuda.so is not built: run python -m lunelette_b200.build")
        lib = ctypes.CDLL(LIBRARY_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def _error():
    return ctypes.create_string_buffer(512)


def _ids(ids):
    arr = np.ascontiguousarray(np.asarray(ids, dtype=np.int64))
    return arr, arr.ctypes.data


def synth_checkpoint(path, seed=0):
    """Write the seeded random-init checkpoint to path (3.8 GB)."""
    err = _error()
    if library().lunelette_cuda_synth_checkpoint(os.fsencode(path), seed, err, 512):
        raise LuneletteError(err.value.decode())
    return path


def validate_checkpoint(path, strategy=COMPACT_FP8_ARITHMETIC):
    err = _error()
    if library().lunelette_cuda_validate_checkpoint(os.fsencode(path), strategy, err, 512):
        raise LuneletteError(err.value.decode())


class Checkpoint:
    """Caller-owned handle of lunelette_metal_checkpoint_create."""

    def __init__(self, handle):
        self.handle = handle

    def destroy(self):
        if self.handle:
            library().lunelette_metal_checkpoint_destroy(self.handle)
            self.handle = None


class Runtime:
    """One lunelette_metal context (single caller, bound to the current device)."""

    def __init__(self, path, options=None, limits=None):
        lib = library()
        err = _error()
        opt = None
        if options is not None:
            opt = Options(*options) if isinstance(options, tuple) else options
        lim = None
        if limits is not None:
            lim = Limits(*limits) if isinstance(limits, tuple) else limits
        self.handle = lib.lunelette_metal_create_configured(
            os.fsencode(path) if path is not None else None,
            ctypes.byref(opt) if opt is not None else None,
            ctypes.byref(lim) if lim is not None else None, err, 512)
        if not self.handle:
            raise LuneletteError(err.value.decode())
        self._logits = ctypes.c_void_p()
        self._err = _error()
        self._view = None  # (address, array) of the last borrowed logits

    def close(self):
        if getattr(self, "handle", None):
            library().lunelette_metal_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _borrowed(self):
        # borrowed host logits: valid until the next mutating call; the context
        # reuses one host buffer, so the array over it is made once per address
        address = self._logits.value
        if self._view is None or self._view[0] != address:
            arr = np.ctypeslib.as_array(ctypes.cast(self._logits, ctypes.POINTER(ctypes.c_float)), shape=(VOCAB,))
            self._view = (address, arr)
        return self._view[1]

    def _call(self, fn, *args):
        err = self._err
        self._logits.value = None
        if fn(self.handle, *args, ctypes.byref(self._logits), err, 512):
            raise LuneletteError(err.value.decode())
        return self._borrowed()

    def prefill(self, ids):
        arr, ptr = _ids(ids)
        return self._call(library().lunelette_metal_prefill, ptr, arr.size)

    def append(self, ids):
        arr, ptr = _ids(ids)
        return self._call(library().lunelette_metal_append, ptr, arr.size)

    def decode(self, token):
        return self._call(library().lunelette_metal_decode, int(token))

    def reset(self):
        err = _error()
        if library().lunelette_metal_reset(self.handle, err, 512):
            raise LuneletteError(err.value.decode())

    def limits(self):
        lim = Limits()
        if library().lunelette_metal_get_limits(self.handle, ctypes.byref(lim)):
            raise LuneletteError("get_limits failed")
        return lim.context, lim.block

    def memory(self):
        mem = Memory()
        if library().lunelette_metal_get_memory(self.handle, ctypes.byref(mem)):
            raise LuneletteError("get_memory failed")
        return {name: getattr(mem, name) for name, _ in Memory._fields_}

    def checkpoint_create(self):
        err = _error()
        handle = ctypes.c_void_p()
        if library().lunelette_metal_checkpoint_create(self.handle, ctypes.byref(handle), err, 512):
            raise LuneletteError(err.value.decode())
        return Checkpoint(handle.value)

    def checkpoint_restore(self, checkpoint):
        return self._call(lambda h, lp, e, c: library().lunelette_metal_checkpoint_restore(
            h, checkpoint.handle, lp, e, c))

    def length(self):
        return library().lunelette_cuda_length(self.handle)

    def decode_loop(self, first_token, steps):
        """Device-resident greedy decode; returns (tokens, device milliseconds,
        kernel launches the call made)."""
        tokens = np.empty(steps, np.int64)
        ms = ctypes.c_float()
        launches = ctypes.c_int()
        err = _error()
        if library().lunelette_cuda_decode_loop(self.handle, int(first_token), steps, tokens.ctypes.data,
                                                ctypes.byref(ms), ctypes.byref(launches), err, 512):
            raise LuneletteError(err.value.decode())
        return tokens, ms.value, launches.value

    def timeline(self, enable=True):
        if library().lunelette_cuda_timeline(self.handle, 1 if enable else 0):
            raise LuneletteError("timeline enable failed")

    def timeline_copy(self, entries=80):
        out = np.zeros(entries, dtype=np.uint64)
        if library().lunelette_cuda_timeline_copy(self.handle, out.ctypes.data, entries):
            raise LuneletteError("timeline copy failed")
        return out

    def trace(self, enable=True):
        if library().lunelette_cuda_trace(self.handle, 1 if enable else 0):
            raise LuneletteError("trace enable failed")

    def trace_copy(self, which, count):
        out = np.empty((count, HIDDEN), dtype=np.float32)
        if library().lunelette_cuda_trace_copy(self.handle, which, out.ctypes.data, out.size):
            raise LuneletteError("trace copy failed")
        return out

    def snapshot(self, count, normalized=False):
        """The last call's layer-25 output rows (or its final-norm rows) while
        tracing is on: a copy of the `count` rows lunelette_cuda_snapshot
        borrows (the hook the reference's comparator reads)."""
        ptr = library().lunelette_cuda_snapshot(self.handle, 1 if normalized else 0)
        if not ptr:
            raise LuneletteError("no snapshot: tracing is off or the sequence holds no published result")
        view = np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctypes.c_float)), shape=(count, HIDDEN))
        return view.copy()


class Batch:
    """Many independent sessions over one weight replica and a paged KV pool
    (lunelette_cuda_batch_*): per-session appends, batched greedy decode steps."""

    def __init__(self, path, max_sessions, context=4352, pool_positions=None, block=256):
        lib = library()
        err = _error()
        pool = pool_positions if pool_positions is not None else max_sessions * context
        self.handle = lib.lunelette_cuda_batch_create(os.fsencode(path), max_sessions, context, pool, block, err, 512)
        if not self.handle:
            raise LuneletteError(err.value.decode())

    def close(self):
        if getattr(self, "handle", None):
            library().lunelette_cuda_batch_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def open(self):
        err = _error()
        s = ctypes.c_int()
        if library().lunelette_cuda_batch_open(self.handle, ctypes.byref(s), err, 512):
            raise LuneletteError(err.value.decode())
        return s.value

    def close_session(self, session):
        if library().lunelette_cuda_batch_close(self.handle, int(session)):
            raise LuneletteError("close of a session that is not open")

    def append(self, session, ids):
        arr, p = _ids(ids)
        err = _error()
        out = ctypes.c_void_p()
        if library().lunelette_cuda_batch_append(self.handle, int(session), p, arr.size, ctypes.byref(out), err, 512):
            raise LuneletteError(err.value.decode())
        return np.ctypeslib.as_array(ctypes.cast(out, ctypes.POINTER(ctypes.c_float)), shape=(VOCAB,))

    def decode(self, sessions, ids, logits=False):
        """One step: returns the greedy next ids (and the n x VOCAB logits)."""
        ss = np.ascontiguousarray(np.asarray(sessions, np.int32))
        arr, p = _ids(ids)
        nxt = np.empty(ss.size, np.int64)
        lg = np.empty((ss.size, VOCAB), np.float32) if logits else None
        err = _error()
        if library().lunelette_cuda_batch_decode(self.handle, ss.ctypes.data, p, ss.size,
                                                 lg.ctypes.data if logits else None, nxt.ctypes.data, err, 512):
            raise LuneletteError(err.value.decode())
        return (nxt, lg) if logits else nxt

    def fork(self, source, length):
        """A new session sharing the first `length` positions of `source`."""
        err = _error()
        s = ctypes.c_int()
        if library().lunelette_cuda_batch_fork(self.handle, int(source), int(length), ctypes.byref(s), err, 512):
            raise LuneletteError(err.value.decode())
        return s.value

    def length(self, session):
        return library().lunelette_cuda_batch_length(self.handle, int(session))

    def free_positions(self):
        return library().lunelette_cuda_batch_free_positions(self.handle)
