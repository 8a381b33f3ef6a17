"""The host runtime (csrc/runtime.c: the include/metal.h state machine and its
checkpoints), the batch manager (csrc/batch.c: page tables, forks, the pool)
and the upload path over a CPU stand-in for the CUDA layer
(tests/c_drivers/fake_device.c), built here twice: plain, and with the address
and undefined-behaviour sanitizers loaded into a child interpreter.

The stand-in's logits are a hash of the full token history read back through
the session's page table, so every check compares a call's logits with those
of a fresh sequence of the same ids (fake_device_reference_logits): a call
that mutated state it should not have, a checkpoint restored to the wrong
length, a fork given the wrong pages or a stale position read past the length
shows up as a mismatch. The contract is the reference's
(include/metal.h:79-123; src/metal_runtime.m:333-575): argument errors leave
the sequence as it was, execution and non-finite failures invalidate it until
reset, only the newest checkpoint restores, reset invalidates it."""
import ctypes
import json
import os
import struct
import subprocess
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(REPO, "lunelette_b200", "csrc")
SOURCES = ["runtime.c", "batch.c", "weights.c", "st.c"]
VOCAB = 131072
NAN_ID = 131071  # FAKE_NAN_ID: a block holding it gets non-finite logits
P = ctypes.c_void_p
SZ = ctypes.c_size_t
I64P = ctypes.POINTER(ctypes.c_int64)
F32P = ctypes.POINTER(ctypes.c_float)


def build(out, sanitize=False):
    """The host sources and the stand-in as one shared library. Under the
    thread sanitizer only the threaded code is instrumented (runtime.c: the
    reader's work split, error reporting and joins; batch.c): the byte loops
    of the admission scan (weights.c), the parser (st.c) and the stand-in's
    digests read memory that one thread owns and would only slow the run."""
    flags = {False: [], True: ["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined",
                               "-fno-omit-frame-pointer"],
             "thread": ["-fsanitize=thread"]}[sanitize]
    include = ["-I" + CSRC, "-I" + os.path.join(REPO, "include"), "-I/usr/local/cuda/include"]
    fake = os.path.join(REPO, "tests", "c_drivers", "fake_device.c")
    sources = [os.path.join(CSRC, s) for s in SOURCES] + [fake]
    objects = []
    if sanitize == "thread":
        plain = [os.path.join(CSRC, "weights.c"), os.path.join(CSRC, "st.c"), fake]
        for i, src in enumerate(plain):
            obj = "%s.%d.o" % (out, i)
            r = subprocess.run(["gcc", "-std=c11", "-O2", "-fPIC", "-c"] + include + [src, "-o", obj],
                               capture_output=True, text=True)
            assert r.returncode == 0, r.stderr
            objects.append(obj)
        sources = [src for src in sources if src not in plain]
    cmd = (["gcc", "-std=c11", "-O1", "-g", "-shared", "-fPIC"] + flags + include + sources + objects +
           ["-o", out, "-lm", "-lpthread", "-Wl,--no-undefined"])
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


class Limits(ctypes.Structure):
    _fields_ = [("context", SZ), ("block", SZ)]


class Memory(ctypes.Structure):
    _fields_ = [("strategy", ctypes.c_int), ("weight_bytes", ctypes.c_uint64),
                ("conversion_stage_bytes", ctypes.c_uint64), ("scratch_bytes", ctypes.c_uint64),
                ("kv_bytes", ctypes.c_uint64), ("total_bytes", ctypes.c_uint64)]


def bind(path):
    lib = ctypes.CDLL(path)
    sig = {
        "lunelette_metal_create_configured": (P, [ctypes.c_char_p, P, P, ctypes.c_char_p, SZ]),
        "lunelette_metal_destroy": (None, [P]),
        "lunelette_metal_get_limits": (ctypes.c_int, [P, P]),
        "lunelette_metal_get_memory": (ctypes.c_int, [P, P]),
        "lunelette_metal_reset": (ctypes.c_int, [P, ctypes.c_char_p, SZ]),
        "lunelette_metal_prefill": (ctypes.c_int, [P, I64P, SZ, P, ctypes.c_char_p, SZ]),
        "lunelette_metal_append": (ctypes.c_int, [P, I64P, SZ, P, ctypes.c_char_p, SZ]),
        "lunelette_metal_decode": (ctypes.c_int, [P, ctypes.c_int64, P, ctypes.c_char_p, SZ]),
        "lunelette_metal_checkpoint_create": (ctypes.c_int, [P, P, ctypes.c_char_p, SZ]),
        "lunelette_metal_checkpoint_restore": (ctypes.c_int, [P, P, P, ctypes.c_char_p, SZ]),
        "lunelette_metal_checkpoint_destroy": (None, [P]),
        "lunelette_cuda_length": (SZ, [P]),
        "lunelette_cuda_decode_loop": (ctypes.c_int, [P, ctypes.c_int64, SZ, I64P, F32P,
                                                      ctypes.POINTER(ctypes.c_int), ctypes.c_char_p, SZ]),
        "lunelette_cuda_trace": (ctypes.c_int, [P, ctypes.c_int]),
        "lunelette_cuda_trace_copy": (ctypes.c_int, [P, ctypes.c_int, F32P, SZ]),
        "lunelette_cuda_snapshot": (F32P, [P, ctypes.c_int]),
        "lunelette_cuda_batch_create": (P, [ctypes.c_char_p, SZ, SZ, SZ, SZ, ctypes.c_char_p, SZ]),
        "lunelette_cuda_batch_destroy": (None, [P]),
        "lunelette_cuda_batch_open": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int), ctypes.c_char_p, SZ]),
        "lunelette_cuda_batch_close": (ctypes.c_int, [P, ctypes.c_int]),
        "lunelette_cuda_batch_append": (ctypes.c_int, [P, ctypes.c_int, I64P, SZ, P, ctypes.c_char_p, SZ]),
        "lunelette_cuda_batch_decode": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int), I64P, SZ, F32P, I64P,
                                                       ctypes.c_char_p, SZ]),
        "lunelette_cuda_batch_fork": (ctypes.c_int, [P, ctypes.c_int, SZ, ctypes.POINTER(ctypes.c_int),
                                                     ctypes.c_char_p, SZ]),
        "lunelette_cuda_batch_length": (SZ, [P, ctypes.c_int]),
        "lunelette_cuda_batch_free_positions": (SZ, [P]),
        "fake_device_linear_digest": (ctypes.c_uint64, [ctypes.c_int, ctypes.c_int, F32P]),
        "fake_device_embedding_digest": (ctypes.c_uint64, [ctypes.POINTER(SZ)]),
        "fake_device_reference_logits": (None, [I64P, SZ, F32P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def ids_arg(ids):
    arr = np.ascontiguousarray(np.asarray(ids, np.int64))
    return arr, arr.ctypes.data_as(I64P)


def reference(lib, ids):
    """Logits of a fresh sequence of these ids at its last position."""
    arr, p = ids_arg(ids)
    out = np.empty(VOCAB, np.float32)
    lib.fake_device_reference_logits(p, arr.size, out.ctypes.data_as(F32P))
    return out


def greedy(logits):
    return int(np.argmax(logits))  # strict '>', lowest id on ties (src/generation.c:8-34)


class Context:
    """One lunelette_metal context of the fake build; every call returns
    (rc, copy of the borrowed logits or None) and checks that a failure
    leaves *logits NULL (include/metal.h:99-104)."""

    def __init__(self, lib, path, limits):
        self.lib, self.err, self.out = lib, ctypes.create_string_buffer(512), ctypes.c_void_p()
        lim = Limits(*limits)
        self.h = lib.lunelette_metal_create_configured(path.encode(), None, ctypes.byref(lim), self.err, 512)
        assert self.h, self.err.value

    def _call(self, fn, *args):
        self.out.value = 1  # must come back NULL on failure
        rc = fn(self.h, *args, ctypes.byref(self.out), self.err, 512)
        if rc:
            assert self.out.value is None, "a failed call left *logits set"
            return rc, None
        return rc, np.ctypeslib.as_array(ctypes.cast(self.out, F32P), (VOCAB,)).copy()

    def prefill(self, ids):
        arr, p = ids_arg(ids)
        return self._call(self.lib.lunelette_metal_prefill, p, arr.size)

    def append(self, ids):
        arr, p = ids_arg(ids)
        return self._call(self.lib.lunelette_metal_append, p, arr.size)

    def decode(self, token):
        return self._call(self.lib.lunelette_metal_decode, ctypes.c_int64(token))

    def reset(self):
        return self.lib.lunelette_metal_reset(self.h, self.err, 512)

    def length(self):
        return self.lib.lunelette_cuda_length(self.h)

    def checkpoint(self):
        cp = ctypes.c_void_p()
        assert self.lib.lunelette_metal_checkpoint_create(self.h, ctypes.byref(cp), self.err, 512) == 0, \
            self.err.value
        return cp

    def restore(self, cp):
        return self._call(self.lib.lunelette_metal_checkpoint_restore, cp)

    def close(self):
        self.lib.lunelette_metal_destroy(self.h)


def tensor_digest(path, header, base, name):
    """fake_device.c's digest_words of a tensor's bytes, in numpy."""
    start, end = header[name]["data_offsets"]
    data = np.memmap(path, np.uint8, "r", base + start, end - start)
    total = 0
    step = 1 << 26
    for first in range(0, end - start, step):
        words = np.frombuffer(data[first:first + step], np.uint64)
        weights = np.arange(first // 8, first // 8 + words.size, dtype=np.uint64) * np.uint64(2) + np.uint64(1)
        total = (total + int(np.sum(words * weights, dtype=np.uint64))) % (1 << 64)
    return total


def check_upload(lib, path):
    """Every tensor the runtime uploads lands in its (layer, slot) with its
    scale: digests of three layers' seven FP8 tensors and of the embedding."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    base = 8 + n
    prefix = "language_model.model."
    names = ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
             "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"]  # device.h slot order
    with open(path, "rb") as f:
        for layer in (0, 13, 25):
            for slot, name in enumerate(names):
                full = "%slayers.%d.%s." % (prefix, layer, name)
                scale = ctypes.c_float()
                got = lib.fake_device_linear_digest(layer, slot, ctypes.byref(scale))
                assert got == tensor_digest(path, header, base, full + "weight"), (layer, name)
                f.seek(base + header[full + "weight_scale_inv"]["data_offsets"][0])
                bits = struct.unpack("<H", f.read(2))[0]
                assert scale.value == struct.unpack("<f", struct.pack("<I", bits << 16))[0], (layer, name)
    nbytes = SZ()
    got = lib.fake_device_embedding_digest(ctypes.byref(nbytes))
    start, end = header[prefix + "embed_tokens.weight"]["data_offsets"]
    assert nbytes.value == end - start
    assert got == tensor_digest(path, header, base, prefix + "embed_tokens.weight")


def check_sequence(lib, path):
    rng = np.random.default_rng(9)
    ctx = Context(lib, path, (4352, 256))
    try:
        lim, mem = Limits(), Memory()
        assert lib.lunelette_metal_get_limits(ctx.h, ctypes.byref(lim)) == 0
        assert (lim.context, lim.block) == (4352, 256)
        assert lib.lunelette_metal_get_memory(ctx.h, ctypes.byref(mem)) == 0 and mem.strategy == 1
        check_upload(lib, path)
        # prefill, decode, append against fresh sequences of the same ids
        seq = list(rng.integers(0, 131071, 70))
        rc, lg = ctx.prefill(seq)
        assert rc == 0 and np.array_equal(lg, reference(lib, seq))
        seq.append(greedy(lg))
        rc, lg = ctx.decode(seq[-1])
        assert rc == 0 and np.array_equal(lg, reference(lib, seq))
        more = list(rng.integers(0, 131071, 100))
        rc, lg = ctx.append(more)
        seq += more
        assert rc == 0 and np.array_equal(lg, reference(lib, seq)) and ctx.length() == len(seq)
        # argument errors change nothing (the next call continues the same sequence)
        for rc, _ in (ctx.decode(-1), ctx.decode(VOCAB), ctx.append([]), ctx.append([1] * 257),
                      ctx.append([5, VOCAB]), ctx.prefill([3])):
            assert rc != 0
        assert ctx.length() == len(seq)
        seq.append(4242)
        rc, lg = ctx.decode(4242)
        assert rc == 0 and np.array_equal(lg, reference(lib, seq))
        # checkpoints: restore rewinds the length and republishes the saved logits;
        # positions written after it are not read again
        cp = ctx.checkpoint()
        saved = lg
        for t in (11, 12, 13):
            assert ctx.decode(t)[0] == 0
        rc, lg = ctx.restore(cp)
        assert rc == 0 and np.array_equal(lg, saved) and ctx.length() == len(seq)
        rc, lg = ctx.decode(77)
        assert rc == 0 and np.array_equal(lg, reference(lib, seq + [77]))
        seq.append(77)
        older, newer = cp, ctx.checkpoint()
        assert ctx.restore(older)[0] != 0  # only the newest handle restores
        assert ctx.restore(newer)[0] == 0 and ctx.length() == len(seq)
        # a non-finite step invalidates the sequence (and its checkpoint) until reset
        rc, _ = ctx.decode(NAN_ID)
        assert rc != 0 and b"reset" in ctx.err.value
        assert ctx.decode(5)[0] != 0 and ctx.append([5])[0] != 0 and ctx.restore(newer)[0] != 0
        for handle in (older, newer):
            lib.lunelette_metal_checkpoint_destroy(handle)
        assert ctx.reset() == 0 and ctx.length() == 0
        # the device greedy loop consumes first and then each step's argmax
        seq = list(rng.integers(0, 131071, 40))
        rc, lg = ctx.prefill(seq)
        first = greedy(lg)
        tokens = np.zeros(12, np.int64)
        ms, launches = ctypes.c_float(), ctypes.c_int()
        assert lib.lunelette_cuda_decode_loop(ctx.h, first, 12, tokens.ctypes.data_as(I64P), ctypes.byref(ms),
                                              ctypes.byref(launches), ctx.err, 512) == 0, ctx.err.value
        want, t = [], first
        for _ in range(12):
            seq.append(t)
            t = greedy(reference(lib, seq))
            want.append(t)
        assert tokens.tolist() == want and ctx.length() == len(seq)
        rc, lg = ctx.decode(int(tokens[-1]))
        assert rc == 0 and np.array_equal(lg, reference(lib, seq + [int(tokens[-1])]))
        # capacity: the context's last position takes a decode, one more does not
        assert ctx.reset() == 0
        rc, _ = ctx.prefill(list(range(256)))
        for start in range(256, 4352 - 1, 256):
            assert ctx.append(list(range(start, min(start + 256, 4351))))[0] == 0
        assert ctx.length() == 4351 and ctx.decode(1)[0] == 0
        assert ctx.decode(2)[0] != 0 and ctx.length() == 4352
    finally:
        ctx.close()


def check_trace(lib, path):
    """The snapshot hook hands out the traced call's layer-25 and final-norm rows."""
    os.environ["LUNELETTE_CUDA_TRACE"] = "1"
    try:
        ctx = Context(lib, path, (256, 256))
    finally:
        del os.environ["LUNELETTE_CUDA_TRACE"]
    try:
        assert lib.lunelette_cuda_trace(ctx.h, 1) == 0
        assert ctx.prefill([5, 6, 7, 8, 9])[0] == 0
        for which, normalized in ((25, 0), (26, 1)):
            rows = np.empty(5 * 3072, np.float32)
            assert lib.lunelette_cuda_trace_copy(ctx.h, which, rows.ctypes.data_as(F32P), rows.size) == 0
            snap = lib.lunelette_cuda_snapshot(ctx.h, normalized)
            assert snap and np.array_equal(np.ctypeslib.as_array(snap, (rows.size,)), rows)
        assert lib.lunelette_cuda_trace(ctx.h, 0) == 0
    finally:
        ctx.close()


def check_batch(lib, path):
    rng = np.random.default_rng(10)
    err = ctypes.create_string_buffer(512)
    b = lib.lunelette_cuda_batch_create(path.encode(), 6, 4352, 64 * 12, 256, err, 512)
    assert b, err.value
    out = ctypes.c_void_p()

    def open_session():
        s = ctypes.c_int()
        assert lib.lunelette_cuda_batch_open(b, ctypes.byref(s), err, 512) == 0, err.value
        return s.value

    def append(s, ids):
        arr, p = ids_arg(ids)
        rc = lib.lunelette_cuda_batch_append(b, s, p, arr.size, ctypes.byref(out), err, 512)
        return rc, (np.ctypeslib.as_array(ctypes.cast(out, F32P), (VOCAB,)).copy() if rc == 0 else None)

    def decode(sessions, ids):
        ss = (ctypes.c_int * len(sessions))(*sessions)
        arr, p = ids_arg(ids)
        logits = np.empty((len(sessions), VOCAB), np.float32)
        nxt = np.empty(len(sessions), np.int64)
        rc = lib.lunelette_cuda_batch_decode(b, ss, p, len(sessions), logits.ctypes.data_as(F32P),
                                             nxt.ctypes.data_as(I64P), err, 512)
        return rc, logits, nxt

    try:
        free0 = lib.lunelette_cuda_batch_free_positions(b)
        assert free0 == 64 * 12
        seqs = {}
        for n in (100, 64, 5):
            s = open_session()
            seqs[s] = list(rng.integers(0, 131071, n))
            rc, lg = append(s, seqs[s])
            assert rc == 0 and np.array_equal(lg, reference(lib, seqs[s]))
        order = list(seqs)
        toks = [greedy(reference(lib, seqs[s])) for s in order]
        rc, lg, nxt = decode(order, toks)
        assert rc == 0
        for i, s in enumerate(order):
            seqs[s].append(toks[i])
            assert np.array_equal(lg[i], reference(lib, seqs[s])) and nxt[i] == greedy(lg[i])
        # a session twice, an id out of range, an empty session: rejected, nothing written
        assert decode([order[0], order[0]], [1, 2])[0] != 0
        assert decode([order[0]], [VOCAB])[0] != 0
        empty = open_session()
        assert decode([empty], [1])[0] != 0
        # forks: 101 positions of the first session = one shared page plus a copied
        # partial page; 64 positions of the second = one shared page
        fork_a, fork_b = ctypes.c_int(), ctypes.c_int()
        src_a, src_b = order[0], order[1]
        assert lib.lunelette_cuda_batch_close(b, empty) == 0
        assert lib.lunelette_cuda_batch_fork(b, src_a, 101, ctypes.byref(fork_a), err, 512) == 0, err.value
        assert lib.lunelette_cuda_batch_fork(b, src_b, 64, ctypes.byref(fork_b), err, 512) == 0, err.value
        seqs[fork_a.value] = seqs[src_a][:101]
        seqs[fork_b.value] = seqs[src_b][:64]
        # the sources go on: their next positions must not reach the forks
        for s, t in ((src_a, 900), (src_b, 901)):
            rc, lg, _ = decode([s], [t])
            seqs[s].append(t)
            assert rc == 0 and np.array_equal(lg[0], reference(lib, seqs[s]))
        assert lib.lunelette_cuda_batch_close(b, src_a) == 0  # the fork keeps the shared page
        rc, lg, _ = decode([fork_a.value, fork_b.value], [902, 903])
        seqs[fork_a.value].append(902)
        seqs[fork_b.value].append(903)
        assert rc == 0
        assert np.array_equal(lg[0], reference(lib, seqs[fork_a.value]))
        assert np.array_equal(lg[1], reference(lib, seqs[fork_b.value]))
        # pool exhaustion is an error that leaves the session as it was
        s = order[2]
        before = lib.lunelette_cuda_batch_length(b, s)
        rc, _ = append(s, list(range(256)))
        rc2, _ = append(s, list(range(256)))
        assert rc != 0 or rc2 != 0
        assert b"exhausted" in err.value
        length = lib.lunelette_cuda_batch_length(b, s)
        assert length in (before, before + 256)
        # argument errors: forks of no positions, of more than the source holds, of
        # a closed session; calls on a closed session; too many tokens at once
        child = ctypes.c_int(-1)
        free_before = lib.lunelette_cuda_batch_free_positions(b)
        for source, length in ((order[1], 0), (order[1], len(seqs[order[1]]) + 1), (src_a, 10), (99, 10)):
            assert lib.lunelette_cuda_batch_fork(b, source, length, ctypes.byref(child), err, 512) != 0
        assert append(src_a, [1])[0] != 0 and decode([src_a], [1])[0] != 0
        assert lib.lunelette_cuda_batch_close(b, src_a) != 0  # already closed
        assert append(order[1], [1] * 257)[0] != 0
        assert decode(list(range(6)) * 43, [1] * 258)[0] != 0
        assert lib.lunelette_cuda_batch_free_positions(b) == free_before
        rc, lg, _ = decode([order[1]], [904])  # the rejected calls changed nothing
        seqs[order[1]].append(904)
        assert rc == 0 and np.array_equal(lg[0], reference(lib, seqs[order[1]]))
        # every page returns to the pool once every session is closed
        for s in (order[1], order[2], fork_a.value, fork_b.value):
            assert lib.lunelette_cuda_batch_close(b, s) == 0
        assert lib.lunelette_cuda_batch_free_positions(b) == free0
    finally:
        lib.lunelette_cuda_batch_destroy(b)


def contract_checks(lib_path, checkpoint):
    lib = bind(lib_path)
    check_sequence(lib, checkpoint)
    check_trace(lib, checkpoint)
    check_batch(lib, checkpoint)


def test_host_runtime_contract_over_fake_device(checkpoint_path, tmp_path):
    contract_checks(build(str(tmp_path / "libfake.so")), checkpoint_path)


def test_host_runtime_contract_under_sanitizers(checkpoint_path, tmp_path):
    """The same checks with the library built under the address and
    undefined-behaviour sanitizers, in a child interpreter that preloads the
    sanitizer runtime; any report ends it with a non-zero status."""
    asan = subprocess.run(["gcc", "-print-file-name=libasan.so"], capture_output=True, text=True).stdout.strip()
    if not os.path.isabs(asan) or not os.path.exists(asan):
        pytest.skip("no address-sanitizer runtime here")
    lib = build(str(tmp_path / "libfake_san.so"), sanitize=True)
    env = dict(os.environ, LD_PRELOAD=asan, ASAN_OPTIONS="detect_leaks=0", UBSAN_OPTIONS="print_stacktrace=1")
    code = "import sys; from tests.test_fake_device import contract_checks; contract_checks(sys.argv[1], sys.argv[2])"
    run = subprocess.run([sys.executable, "-c", code, lib, checkpoint_path], cwd=REPO, env=env,
                         capture_output=True, text=True, timeout=900)
    assert run.returncode == 0 and "runtime error" not in run.stderr, run.stderr[-3000:]


def parallel_reader_checks(lib_path, checkpoint):
    """A create (every tensor read by the parallel reader into the staging
    buffers, its FP8 codes admitted by the workers, then uploaded) and a
    prefill."""
    lib = bind(lib_path)
    ctx = Context(lib, checkpoint, (256, 256))
    try:
        assert ctx.prefill([1, 2, 3])[0] == 0
    finally:
        ctx.close()


def test_parallel_reader_under_thread_sanitizer(checkpoint_path, tmp_path):
    """The checkpoint reader's worker threads (runtime.c parallel_read) under
    the thread sanitizer: no data race reported over a create."""
    tsan = subprocess.run(["gcc", "-print-file-name=libtsan.so"], capture_output=True, text=True).stdout.strip()
    if not os.path.isabs(tsan) or not os.path.exists(tsan):
        pytest.skip("no thread-sanitizer runtime here")
    lib = build(str(tmp_path / "libfake_tsan.so"), sanitize="thread")
    env = dict(os.environ, LD_PRELOAD=tsan, TSAN_OPTIONS="halt_on_error=1")
    code = ("import sys; from tests.test_fake_device import parallel_reader_checks; "
            "parallel_reader_checks(sys.argv[1], sys.argv[2])")
    run = subprocess.run([sys.executable, "-c", code, lib, checkpoint_path], cwd=REPO, env=env,
                         capture_output=True, text=True, timeout=900)
    assert run.returncode == 0 and "ThreadSanitizer" not in run.stderr, run.stderr[-3000:]


REF_FAKE = os.path.join(REPO, "oracle", "_ref", "fake")


def fake_binary(name):
    path = os.path.join(REF_FAKE, name)
    if not os.path.exists(path):
        pytest.skip("%s not built (make -C oracle REF=<reference checkout>)" % name)
    return path


def test_reference_callers_over_fake_device(checkpoint_path, tmp_path):
    """The reference's own C callers of include/metal.h (compiled from its
    sources by oracle/Makefile into oracle/_ref/fake/, linked against the host
    runtime over the CPU stand-in): its generation loop (src/generation.c with
    the CLI's callback) generates the stand-in's greedy chain; its native
    regression harness (tests/compare_native.c) captures 8 teacher-forced steps
    after prompts of 6/24/150/248 ids and checks them bitwise over two reset
    cycles in a second process; its service generator (service/native.c) runs
    config 3's turn shape (512-id prefix, 2 turns of 200 + 64) with prefix reuse
    and a checkpointed replay of the last turn, every id the stand-in's chain."""
    from tests.test_gpu_c_callers import write_generated_fixture
    lib = bind(fake_binary("liblunelette_cuda.so"))
    rng = np.random.default_rng(4321)
    # the generation loop: greedy until id 2 or 32 tokens
    prompt = [int(i) for i in rng.integers(1000, 131072, 32)]
    proc = subprocess.run([fake_binary("generate_metal_next"), checkpoint_path, "32"] + [str(i) for i in prompt],
                          capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr
    lines = dict(line.split(":", 1) for line in proc.stdout.strip().splitlines())
    got = [int(t) for t in lines["tokens"].split()]
    seq, want = list(prompt), []
    while True:
        tok = greedy(reference(lib, seq))
        want.append(tok)
        if tok == 2 or len(want) == 32:
            break
        seq.append(tok)
    assert got == want and int(lines["calls"]) == len(got)
    # the native regression harness: capture, then check in another process
    pairs = []
    for count in (6, 24, 150, 248):
        ids_path = tmp_path / ("ids%d.txt" % count)
        ids_path.write_text(" ".join(str(int(i)) for i in rng.integers(1000, 131072, count)) + "\n")
        fixture = tmp_path / ("forced%d.safetensors" % count)
        write_generated_fixture(fixture, rng.integers(1000, 131072, 8))
        pairs += [str(ids_path), str(fixture)]
    out_dir = tmp_path / "capture"
    out_dir.mkdir()
    for mode in ("capture", "check"):
        proc = subprocess.run([fake_binary("compare_native"), mode, checkpoint_path, "mps", str(out_dir)] + pairs,
                              capture_output=True, text=True, timeout=600)
        assert proc.returncode == 0, (mode, proc.stdout[-2000:], proc.stderr[-2000:])
        assert ("PASS native %s" % mode) in proc.stdout
    assert "steps=64 cycles=2" in proc.stdout and "exact=0" not in proc.stdout
    # the service generator over config 3's turn shape
    prefix_len, turns, user_len, gen = 512, 2, 200, 64
    prefix = [int(i) for i in rng.integers(1000, 131072, prefix_len)]
    users = [[int(i) for i in rng.integers(1000, 131072, user_len)] for _ in range(turns)]
    ids_path = tmp_path / "turns.txt"
    ids_path.write_text(" ".join(str(i) for i in prefix + sum(users, [])) + "\n")
    proc = subprocess.run([fake_binary("service_native_turns"), checkpoint_path, str(ids_path), str(prefix_len),
                           str(turns), str(user_len), str(gen)],
                          capture_output=True, text=True, timeout=600, cwd=str(tmp_path))
    assert proc.returncode == 0, (proc.stdout[-2000:], proc.stderr[-2000:])
    lines = dict(line.split(":", 1) for line in proc.stdout.strip().splitlines())
    seq, pending = list(prefix), []
    for t in range(turns):
        seq += pending + users[t]
        want = [greedy(reference(lib, seq))]
        while len(want) < gen:
            seq.append(want[-1])
            want.append(greedy(reference(lib, seq)))
        assert [int(x) for x in lines["turn %d" % t].split()] == want, "turn %d" % t
        pending = [want[-1]]  # generated but not yet fed: opens the next turn
    assert [int(x) for x in lines["replay"].split()] == want


def history_hash(ids):
    """fake_device.c's hash of a token history (FNV-1a over id + 1, 64-bit)."""
    h = 1469598103934665603
    for i in ids:
        h = ((h ^ (int(i) + 1)) * 1099511628211) % (1 << 64)
    return h


def mix64(x):
    """fake_device.c's mix64 over a uint64 array."""
    with np.errstate(over="ignore"):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return x ^ (x >> np.uint64(31))


def trace_rows(h, which, rows):
    """fake_device.c's traced rows of a call whose history hash is h."""
    i = np.arange(rows * 3072, dtype=np.uint64)
    key = np.uint64(h) ^ (np.uint64(which) << np.uint64(40)) ^ i
    return ((mix64(key) >> np.uint64(40)).astype(np.float64) * 2.0 ** -24).astype(np.float32)


def test_reference_comparator_over_fake_device(checkpoint_path, tmp_path):
    """The reference's real-weight comparator (tests/compare_metal.c, with
    the snapshot hook over lunelette_cuda_snapshot) over the CPU stand-in, on
    fixtures that hold the stand-in's own logits, layer-25 rows and final-norm
    rows: its whole protocol (teacher-forced steps, two reset cycles, the
    256-position capacity check, destroy and recreate) passes and every
    tensor matches exactly."""
    from tests.test_gpu_c_callers import write_safetensors
    lib = bind(fake_binary("liblunelette_cuda.so"))
    rng = np.random.default_rng(2718)
    pairs = []
    for count, steps in ((6, 4), (248, 8)):
        ids = [int(i) for i in rng.integers(1000, 131072, count)]
        ids_path = tmp_path / ("ids%d.txt" % count)
        ids_path.write_text(" ".join(str(i) for i in ids) + "\n")
        history, feed, generated, tensors = [], ids, [], []
        for step in range(steps):
            history += feed
            logits = reference(lib, history)
            h = history_hash(history)
            tensors += [("logits_%d" % step, logits.reshape(1, -1)),
                        ("block_25_%d" % step, trace_rows(h, 25, len(feed)).reshape(1, len(feed), -1)),
                        ("final_norm_%d" % step, trace_rows(h, 26, len(feed)).reshape(1, len(feed), -1))]
            generated.append(greedy(logits))
            feed = [generated[-1]]
        fixture = tmp_path / ("fake%d.safetensors" % count)
        write_safetensors(fixture, [("generated", np.asarray(generated, np.int64))] + tensors)
        pairs += [str(ids_path), str(fixture)]
    env = dict(os.environ, LUNELETTE_CUDA_TRACE="1")
    proc = subprocess.run([fake_binary("compare_metal"), checkpoint_path] + pairs,
                          capture_output=True, text=True, timeout=600, env=env)
    assert proc.returncode == 0, (proc.stdout[-3000:], proc.stderr[-2000:])
    out = proc.stdout
    assert len([l for l in out.splitlines() if l.startswith("PASS /")]) == 24, out[-3000:]
    metrics = [l for l in out.splitlines() if l.startswith("metrics ")]
    assert len(metrics) == 72 and all(" mismatches0 " in l for l in metrics), out[-3000:]
    assert out.count("PASS capacity256 append then reject") == 2 and "PASS destroy/recreate" in out
