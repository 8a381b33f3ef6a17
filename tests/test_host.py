"""Host-side product tests that need no GPU: the C-ABI exports, argument
rejection before any I/O, the E4M3 encoder, the YaRN table, checkpoint
admission (including agreement with the reference's own loader and parser)."""
import ctypes
import json
import os
import re
import shutil
import struct
import tempfile

import numpy as np
import pytest

import lunelette_b200 as L

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for header in ("metal.h", "lunelette_cuda.h"):
        text = open(os.path.join(REPO, "include", header)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(lunelette_\w+)\s*\(", text))
    return names


def exported_functions():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIBRARY_PATH], capture_output=True,
                         text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_library_exports_exactly_the_declared_abi(lib):
    declared = declared_functions()
    exported = exported_functions()
    assert len([n for n in declared if n.startswith("lunelette_metal_")]) == 13
    assert declared <= exported, declared - exported
    assert exported <= declared, exported - declared
    for name in declared:
        assert name in L.SIGNATURES, name


def test_create_rejects_before_io(lib):
    err = ctypes.create_string_buffer(512)
    bad_limits = L.Limits(4352, 64)
    assert not lib.lunelette_metal_create_configured(b"/no-model", None, ctypes.byref(bad_limits), err, 512)
    assert b"unsupported context/block" in err.value
    bad = L.Options(7, 1)
    assert not lib.lunelette_metal_create_with_options(b"/no-model", ctypes.byref(bad), err, 512)
    assert b"invalid prefill option" in err.value
    bad = L.Options(0, 9)
    assert not lib.lunelette_metal_create_with_options(b"/no-model", ctypes.byref(bad), err, 512)
    assert b"invalid strategy" in err.value
    assert not lib.lunelette_metal_create(None, err, 512)
    assert b"explicit FP8 safetensors path" in err.value
    assert not lib.lunelette_metal_create(b"/no-model", None, 0)  # NULL error buffer allowed
    lim = L.Limits(1, 2)
    assert lib.lunelette_metal_get_limits(None, ctypes.byref(lim)) == -1
    assert (lim.context, lim.block) == (1, 2)
    assert lib.lunelette_metal_get_memory(None, None) == -1
    lib.lunelette_metal_destroy(None)
    assert lib.lunelette_metal_reset(None, err, 512) == -1
    logits = ctypes.c_void_p(1)
    ids = (ctypes.c_int64 * 1)(0)
    assert lib.lunelette_metal_prefill(None, ids, 1, ctypes.byref(logits), err, 512) == -1
    assert logits.value is None
    lib.lunelette_metal_checkpoint_destroy(None)


def test_e4m3_encoder_round_trips_and_matches_torch(lib, oracle):
    import torch
    for code in range(256):
        if code & 127 == 127:
            continue
        assert lib.lunelette_cuda_e4m3_encode(oracle.fp8_decode(code)) == code
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(20000) * s for s in (1e-3, 0.1, 3.0, 100.0)]).astype(np.float32)
    x = np.clip(x, -448, 448)
    # include exact ties between neighbouring codes
    decoded = np.array([oracle.fp8_decode(c) for c in range(126)], np.float32)
    mids = ((decoded[:-1].astype(np.float64) + decoded[1:]) / 2).astype(np.float32)
    x = np.concatenate([x, mids, -mids])
    ours = np.array([lib.lunelette_cuda_e4m3_encode(float(v)) for v in x], np.uint8)
    theirs = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, theirs)
    assert lib.lunelette_cuda_e4m3_encode(1000.0) == 0x7E
    assert lib.lunelette_cuda_e4m3_encode(-1000.0) == 0xFE


def test_product_yarn_bitwise_equals_reference(lib):
    g = json.load(open(os.path.join(REPO, "tests", "golden", "yarn_ref.json")))
    c = np.zeros(128, np.float32)
    s = np.zeros(128, np.float32)
    for pos in g["positions"]:
        assert lib.lunelette_cuda_yarn(pos, c.ctypes.data, s.ctypes.data) == 0
        assert [int(b) for b in c.view(np.uint32)] == g["tables"][str(pos)]["cos"]
        assert [int(b) for b in s.view(np.uint32)] == g["tables"][str(pos)]["sin"]
    assert lib.lunelette_cuda_yarn(262144, c.ctypes.data, s.ctypes.data) == -1


def test_calls_without_a_context_fail_before_any_work(lib):
    """The contract's argument rules on the host (include/metal.h:74-120): every
    mutating call and checkpoint call rejects a NULL context, clears the logits
    output and writes a diagnostic; NULL/0 error buffers are accepted."""
    err = ctypes.create_string_buffer(512)
    logits = ctypes.c_void_p(1)
    ids = (ctypes.c_int64 * 2)(1, 2)
    for call in (lambda: lib.lunelette_metal_append(None, ids, 2, ctypes.byref(logits), err, 512),
                 lambda: lib.lunelette_metal_decode(None, 5, ctypes.byref(logits), err, 512),
                 lambda: lib.lunelette_metal_prefill(None, ids, 2, ctypes.byref(logits), None, 0)):
        logits.value = 1
        assert call() == -1
        assert logits.value is None
    handle = ctypes.c_void_p(1)
    assert lib.lunelette_metal_checkpoint_create(None, ctypes.byref(handle), err, 512) == -1
    assert handle.value is None and err.value
    logits.value = 1
    assert lib.lunelette_metal_checkpoint_restore(None, None, ctypes.byref(logits), err, 512) == -1
    assert logits.value is None and err.value
    tokens = (ctypes.c_int64 * 4)()
    assert lib.lunelette_cuda_decode_loop(None, 1, 4, tokens, None, None, err, 512) == -1
    assert b"decode loop" in err.value
    assert not lib.lunelette_cuda_snapshot(None, 0) and not lib.lunelette_cuda_snapshot(None, 1)


def test_oracle_side_writer_matches_the_product_writer(checkpoint_path, tmp_path):
    """The benchmark's CPU reference leg writes its input with oracle/libsynth.so
    (no product library loaded): it must produce the product writer's file
    byte for byte, so both legs read the same weights."""
    import filecmp
    from tests import oracle_lib
    path = str(tmp_path / "synth.safetensors")
    oracle_lib.synth_checkpoint(path, 0)
    assert filecmp.cmp(path, checkpoint_path, shallow=False)
    os.remove(path)


def test_synthetic_checkpoint_admitted(checkpoint_path):
    for strategy in (L.RESIDENT_FP32, L.COMPACT_FP8_ARITHMETIC, L.COMPACT_FP8_LOOKUP):
        L.validate_checkpoint(checkpoint_path, strategy)


def test_reference_loader_accepts_synthetic_checkpoint(checkpoint_path, ref_lib):
    """The reference's own metadata validation and compact raw admission
    (src/metal_weights.c:51-231) accept the generated file."""
    ref_lib.lunelette_metal_weights_open.argtypes = [ctypes.c_void_p, ctypes.c_char_p,
                                                     ctypes.c_char_p, ctypes.c_size_t]
    ref_lib.lunelette_metal_weights_load_raw.argtypes = [ctypes.c_void_p, ctypes.c_size_t,
                                                         ctypes.c_void_p, ctypes.c_size_t,
                                                         ctypes.c_char_p, ctypes.c_size_t]
    ref_lib.lunelette_metal_weights_close.argtypes = [ctypes.c_void_p]
    state = ctypes.create_string_buffer(1 << 16)
    err = ctypes.create_string_buffer(512)
    assert ref_lib.lunelette_metal_weights_open(state, checkpoint_path.encode(), err, 512) == 0, err.value
    try:
        out = np.empty(9216 * 3072, np.uint8)
        sizes = [4096 * 3072, 1024 * 3072, 1024 * 3072, 3072 * 4096, 9216 * 3072, 9216 * 3072,
                 3072 * 9216]
        for layer in (0, 13, 25):
            for slot, size in zip((1, 2, 3, 4, 6, 7, 8), sizes):
                index = 2 + layer * 9 + slot
                rc = ref_lib.lunelette_metal_weights_load_raw(state, index, out.ctypes.data, size, err, 512)
                assert rc == 0, err.value
    finally:
        ref_lib.lunelette_metal_weights_close(state)


@pytest.fixture(scope="module")
def corrupt_copy(checkpoint_path):
    path = os.path.join(tempfile.gettempdir(), "lunelette_corrupt_%d.safetensors" % os.getpid())
    shutil.copyfile(checkpoint_path, path)
    yield path
    os.unlink(path)


def header_of(path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        return n, f.read(n).decode()


def patch(path, offset, data):
    with open(path, "r+b") as f:
        f.seek(offset)
        old = f.read(len(data))
        f.seek(offset)
        f.write(data)
    return old


def tensor_offset(path, name):
    n, header = header_of(path)
    meta = json.loads(header)[name]
    return 8 + n + meta["data_offsets"][0]


def test_admission_rejects_planted_faults(corrupt_copy):
    q = "language_model.model.layers.3.self_attn.q_proj.weight"
    base = tensor_offset(corrupt_copy, q)
    old = patch(corrupt_copy, base + 1000, b"\x7f")
    try:
        for strategy in (L.RESIDENT_FP32, L.COMPACT_FP8_ARITHMETIC):
            with pytest.raises(L.LuneletteError):
                L.validate_checkpoint(corrupt_copy, strategy)
        with pytest.raises(L.LuneletteError, match="byte 1000 code 0x7f"):
            L.validate_checkpoint(corrupt_copy, L.COMPACT_FP8_ARITHMETIC)
    finally:
        patch(corrupt_copy, base + 1000, old)
    scale = q[:-6] + "weight_scale_inv"
    at = tensor_offset(corrupt_copy, scale)
    old = patch(corrupt_copy, at, struct.pack("<H", 0x0001))  # subnormal BF16 scale
    try:
        with pytest.raises(L.LuneletteError, match="FP32-normal widened BF16"):
            L.validate_checkpoint(corrupt_copy, L.COMPACT_FP8_ARITHMETIC)
        L.validate_checkpoint(corrupt_copy, L.RESIDENT_FP32)  # resident admits it
    finally:
        patch(corrupt_copy, at, old)
    act = q[:-6] + "activation_scale"
    at = tensor_offset(corrupt_copy, act)
    old = patch(corrupt_copy, at, struct.pack("<H", 0xBF80))  # -1.0
    try:
        with pytest.raises(L.LuneletteError, match="positive finite BF16"):
            L.validate_checkpoint(corrupt_copy, L.RESIDENT_FP32)
    finally:
        patch(corrupt_copy, at, old)
    # a companion scalar under another name: the FP8 tensor lacks it (reported
    # before the stray name, in the contract's order)
    n, header = header_of(corrupt_copy)
    at = 8 + header.index(act) + len(act) - 1
    old = patch(corrupt_copy, at, b"f")
    try:
        with pytest.raises(L.LuneletteError, match="scalar " + act.replace(".", r"\.") + ": an FP8 tensor needs"):
            L.validate_checkpoint(corrupt_copy, L.COMPACT_FP8_ARITHMETIC)
    finally:
        patch(corrupt_copy, at, old)
    n, header = header_of(corrupt_copy)
    at = 8 + header.index("embed_tokens") + len("embed_token")
    old = patch(corrupt_copy, at, b"z")
    try:
        with pytest.raises(L.LuneletteError, match="embed_tokens.weight: not in the checkpoint"):
            L.validate_checkpoint(corrupt_copy, L.COMPACT_FP8_ARITHMETIC)
    finally:
        patch(corrupt_copy, at, old)
    L.validate_checkpoint(corrupt_copy, L.COMPACT_FP8_ARITHMETIC)


# ---- parser corpus: same accept/reject verdict as the reference's st_open ----

def small_file(header, data=b""):
    fd, path = tempfile.mkstemp(suffix=".safetensors")
    raw = header.encode() if isinstance(header, str) else header
    with os.fdopen(fd, "wb") as f:
        f.write(struct.pack("<Q", len(raw)) + raw + data)
    return path


PARSER_CASES = [
    ('{"w":{"dtype":"BF16","shape":[2,2],"data_offsets":[0,8]}}', b"\0" * 8, True),
    ('{"__metadata__":{"a":"b"},"w":{"dtype":"F32","shape":[],"data_offsets":[0,4]}}', b"\0" * 4, True),
    ('{}', b"", True),
    ('  {}', b"", False),  # first byte must be '{'
    ('{"w":{"dtype":"F16","shape":[1],"data_offsets":[0,2]}}', b"\0" * 2, False),
    ('{"w":{"dtype":"BF16","shape":[2],"data_offsets":[0,2]}}', b"\0" * 2, False),
    ('{"w":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]},"w":{"dtype":"BF16","shape":[1],"data_offsets":[2,4]}}', b"\0" * 4, False),
    ('{"a":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]},"b":{"dtype":"BF16","shape":[1],"data_offsets":[4,6]}}', b"\0" * 6, False),
    ('{"a":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]}}', b"\0" * 4, False),  # trailing bytes
    ('{"a":{"dtype":"I64","shape":[1,1,1,1,1,1,1,1,1],"data_offsets":[0,8]}}', b"\0" * 8, False),
    ('{"a":{"dtype":"I64","shape":[1],"shape":[1],"data_offsets":[0,8]}}', b"\0" * 8, False),
    ('{"a":{"dtype":"I64","shape":[01],"data_offsets":[0,8]}}', b"\0" * 8, False),
    ('{"__metadata__":{"a":1}}', b"", False),
    ('{"e":{"dtype":"BF16","shape":[0],"data_offsets":[0,0]},"a":{"dtype":"F8_E4M3","shape":[1],"data_offsets":[0,1]}}', b"\0", True),
    ('{"e":{"dtype":"BF16","shape":[0],"data_offsets":[1,1]},"a":{"dtype":"BF16","shape":[1],"data_offsets":[0,2]}}', b"\0\0", False),
    ('{"a\\u0041":{"dtype":"F8_E4M3","shape":[],"data_offsets":[0,1]}}', b"\0", True),
    ('{"a":{"dtype":"F8_E4M3","shape":[],"data_offsets":[0,1]}} ', b"\0", True),
    ('{"a":{"dtype":"F8_E4M3","shape":[],"data_offsets":[0,1]}}x', b"\0", False),
]


def st_open_verdicts(ref_lib, path):
    ref_lib.st_open.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]
    ref_lib.st_close.argtypes = [ctypes.c_void_p]
    state = ctypes.create_string_buffer(256)
    err = ctypes.create_string_buffer(512)
    ok = ref_lib.st_open(state, path.encode(), err, 512) == 0
    if ok:
        ref_lib.st_close(state)
    return ok


@pytest.mark.parametrize("case", range(len(PARSER_CASES)))
def test_parser_corpus(lib, case, request):
    header, data, accepted = PARSER_CASES[case]
    path = small_file(header, data)
    try:
        err = ctypes.create_string_buffer(512)
        lib.lunelette_cuda_validate_checkpoint(path.encode(), 1, err, 512)
        parsed = b"tensor language_model.model.embed_tokens.weight" in err.value
        assert parsed == accepted, err.value
        if os.path.exists(os.path.join(REPO, "oracle", "_ref", "libref.so")):
            ref = request.getfixturevalue("ref_lib")
            assert st_open_verdicts(ref, path) == accepted
    finally:
        os.unlink(path)


FUZZ_TOKENS = [b'{', b'}', b'[', b']', b',', b':', b'"', b'\\', b'0', b'-1', b'1e3', b'18446744073709551615',
               b'18446744073709551616', b'9223372036854775807', b'"dtype"', b'"shape"', b'"data_offsets"',
               b'"BF16"', b'"F8_E4M3"', b'"F32"', b'"I64"', b'"__metadata__"', b' ', b'\n', b'\x00', b'\xff',
               b'null', b'true', b'1.0', b'\\u0000', b'\\ud800', b'01', b'+1']


def fuzz_file(rng, directory):
    """One seeded mutation of a corpus case: up to three edits of its header
    (byte deleted, JSON token inserted, byte replaced, cut, span replaced), the
    data sometimes cut or padded, and the 8-byte header size sometimes wrong
    (too long, too short, or a huge value)."""
    header, data, _ = rng.choice(PARSER_CASES)
    h = bytearray(header.encode())
    for _ in range(rng.randint(1, 3)):
        if not h:
            h = bytearray(b'{')
        op, i = rng.randrange(5), rng.randrange(len(h) + 1)
        if op == 0 and len(h) > 1:
            del h[min(i, len(h) - 1)]
        elif op == 1:
            h[i:i] = rng.choice(FUZZ_TOKENS)
        elif op == 2 and i < len(h):
            h[i] = rng.randrange(256)
        elif op == 3:
            h = h[:i]
        elif op == 4:
            j = rng.randrange(len(h) + 1)
            h[min(i, j):max(i, j)] = rng.choice(FUZZ_TOKENS)
    if rng.random() < 0.2:
        data = data[:rng.randrange(len(data) + 1)] + b'\0' * rng.randrange(3)
    size, r = len(h), rng.random()
    if r < 0.05:
        size = len(h) + rng.randrange(1, 64)
    elif r < 0.10:
        size = max(0, len(h) - rng.randrange(1, 16))
    elif r < 0.12:
        size = rng.choice([0, 2 ** 63, 2 ** 64 - 1, 100_000_001, 2 ** 32])
    fd, path = tempfile.mkstemp(suffix=".safetensors", dir=directory)
    with os.fdopen(fd, "wb") as f:
        f.write(struct.pack("<Q", size) + bytes(h) + data)
    return path


FUZZ_DTYPES = {"BF16": 2, "F16": 2, "F32": 4, "F8_E4M3": 1, "I64": 8, "U8": 1, "BOOL": 1, "F64": 8,
               "bf16": 1, "F8_E5M2": 1}


def structured_file(rng, directory):
    """A well-formed header built at random: up to four tensors (names with
    escapes, empty or repeated names), dtypes the parser knows and some it does
    not, shapes of 0 to 9 dimensions, offsets that are contiguous or off by a
    byte, keys and fields in shuffled order, optional metadata (string and
    non-string values), whitespace between tokens, and data of the declared
    length or one byte off: about a fifth of these files are valid."""
    entries, off = [], 0
    for i in range(rng.randrange(0, 5)):
        name = rng.choice(["w", "a", "b", "x.y", "a\\u0041", "\\n", "", "w"]) + (str(i) if rng.random() < 0.7 else "")
        dtype = rng.choice(list(FUZZ_DTYPES))
        shape = [rng.choice([0, 1, 2, 3, 4]) for _ in range(rng.choice([0, 1, 1, 2, 2, 3, 8, 9]))]
        nbytes = int(np.prod(shape, dtype=np.int64)) * FUZZ_DTYPES[dtype]
        start = off if rng.random() < 0.85 else off + rng.choice([-1, 1, 2])
        end = start + nbytes if rng.random() < 0.85 else start + nbytes + rng.choice([-1, 1])
        entries.append((name, dtype, shape, max(0, start), max(0, end)))
        off = max(off, end)
    if rng.random() < 0.3:
        rng.shuffle(entries)
    ws = lambda: rng.choice(["", "", " ", "\n", "\t"])
    parts = []
    if rng.random() < 0.3:
        parts.append('"__metadata__":%s%s' % (ws(), rng.choice(['{"a":"b"}', '{}', '{"a":1}', '{"a":"b","c":"d"}'])))
    for name, dtype, shape, start, end in entries:
        fields = ['"dtype":%s"%s"' % (ws(), dtype), '"shape":[%s]' % ",".join(map(str, shape)),
                  '"data_offsets":[%d,%d]' % (start, end)]
        if rng.random() < 0.3:
            rng.shuffle(fields)
        parts.append('%s"%s"%s:%s{%s}' % (ws(), name, ws(), ws(), ",".join(fields)))
    header = ("{" + ",".join(parts) + "}" + rng.choice(["", "", " ", "  "])).encode()
    total = max([e[4] for e in entries] + [0])
    data = b"\0" * (total if rng.random() < 0.85 else max(0, total + rng.choice([-1, 1])))
    fd, path = tempfile.mkstemp(suffix=".safetensors", dir=directory)
    with os.fdopen(fd, "wb") as f:
        f.write(struct.pack("<Q", len(header)) + header + data)
    return path


def test_parser_agrees_with_reference_on_random_files(lib, tmp_path):
    """Differential fuzzing of the checkpoint parser against the reference's
    st_open (src/safetensors.c, compiled from its sources into oracle/_ref):
    800 seeded mutations of the corpus above (almost all malformed) and 800
    well-formed random headers (about a fifth valid) get the same
    accept/reject verdict from both, and neither crashes."""
    import random
    libref = os.path.join(REPO, "oracle", "_ref", "libref.so")
    if not os.path.exists(libref):
        pytest.skip("the reference's parser is not built here (oracle/Makefile with a reference checkout)")
    ref = ctypes.CDLL(libref)
    rng = random.Random(20261202)
    accepted = 0
    for case in range(1600):
        make = fuzz_file if case % 2 == 0 else structured_file
        path = make(rng, str(tmp_path))
        try:
            err = ctypes.create_string_buffer(512)
            lib.lunelette_cuda_validate_checkpoint(path.encode(), 1, err, 512)
            mine = b"tensor language_model.model.embed_tokens.weight" in err.value
            with open(path, "rb") as f:
                raw = f.read()
            assert mine == st_open_verdicts(ref, path), (case, raw[:200], err.value)
            accepted += mine
        finally:
            os.unlink(path)
    assert accepted > 100  # the structured half reaches the parser's semantic checks


def reference_admission(ref_lib, path, index):
    """The reference loader's verdicts on a checkpoint (src/metal_weights.c):
    open (names, shapes, dtypes, every scalar read and checked) and, for the
    weight at `index`, its compact raw admission and its resident FP32 load.
    Returns (compact admitted, resident admitted)."""
    ref_lib.lunelette_metal_weights_open.argtypes = [ctypes.c_void_p, ctypes.c_char_p,
                                                     ctypes.c_char_p, ctypes.c_size_t]
    ref_lib.lunelette_metal_weights_load_raw.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                                         ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t]
    ref_lib.lunelette_metal_weights_load.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                                     ctypes.c_size_t]
    ref_lib.lunelette_metal_weights_close.argtypes = [ctypes.c_void_p]
    state = ctypes.create_string_buffer(1 << 16)  # sizeof(lunelette_metal_weights) is 5704 bytes
    err = ctypes.create_string_buffer(512)
    if ref_lib.lunelette_metal_weights_open(state, path.encode(), err, 512) != 0:
        return False, False
    try:
        if index is None:
            return True, True
        rows, cols = {1: (4096, 3072), 8: (3072, 9216)}[(index - 2) % 9]
        raw = np.empty(rows * cols, np.uint8)
        compact = ref_lib.lunelette_metal_weights_load_raw(state, index, raw.ctypes.data, raw.size, err, 512) == 0
        wide = np.empty(rows * cols, np.float32)
        resident = ref_lib.lunelette_metal_weights_load(state, index, wide.ctypes.data, wide.size) == 0
        return compact, resident
    finally:
        ref_lib.lunelette_metal_weights_close(state)


def test_admission_verdicts_match_reference_loader(corrupt_copy, ref_lib):
    """The same planted faults through this library's admission and the
    reference's loader (compiled from its sources): for each, both strategies
    admit or reject alike. Faults: NaN codes in the first and the last FP8
    tensor of a layer, a subnormal, zero, infinite and negative weight scale, a
    NaN and a negative activation scale, a renamed companion scalar, a renamed
    embedding."""
    q = "language_model.model.layers.3.self_attn.q_proj.weight"
    down = "language_model.model.layers.25.mlp.down_proj.weight"
    q_index, down_index = 2 + 3 * 9 + 1, 2 + 25 * 9 + 8
    n, header = header_of(corrupt_copy)
    act = q[:-6] + "activation_scale"
    faults = [  # (offset, bytes, index of the affected weight or None)
        (tensor_offset(corrupt_copy, q) + 1000, b"\x7f", q_index),
        (tensor_offset(corrupt_copy, down) + 12345, b"\xff", down_index),
        (tensor_offset(corrupt_copy, q[:-6] + "weight_scale_inv"), struct.pack("<H", 0x0001), q_index),
        (tensor_offset(corrupt_copy, q[:-6] + "weight_scale_inv"), struct.pack("<H", 0x0000), q_index),
        (tensor_offset(corrupt_copy, down[:-6] + "weight_scale_inv"), struct.pack("<H", 0x7F80), down_index),
        (tensor_offset(corrupt_copy, down[:-6] + "weight_scale_inv"), struct.pack("<H", 0xBC00), down_index),
        (tensor_offset(corrupt_copy, act), struct.pack("<H", 0x7FC0), None),
        (tensor_offset(corrupt_copy, act), struct.pack("<H", 0xBF80), None),
        (8 + header.index(act) + len(act) - 1, b"f", None),
        (8 + header.index("embed_tokens") + len("embed_token"), b"z", None),
    ]
    for offset, data, index in faults:
        old = patch(corrupt_copy, offset, data)
        try:
            ours = []
            for strategy in (L.COMPACT_FP8_ARITHMETIC, L.RESIDENT_FP32):
                try:
                    L.validate_checkpoint(corrupt_copy, strategy)
                    ours.append(True)
                except L.LuneletteError:
                    ours.append(False)
            assert tuple(ours) == reference_admission(ref_lib, corrupt_copy, index), (offset, data)
        finally:
            patch(corrupt_copy, offset, old)
    assert reference_admission(ref_lib, corrupt_copy, q_index) == (True, True)


def test_parser_and_admission_memory_safe_under_sanitizers(checkpoint_path, tmp_path):
    """The checkpoint parser and admission catalogue (csrc/st.c, csrc/weights.c)
    built on their own with the address, undefined-behaviour and leak
    sanitizers (tests/c_drivers/open_checkpoints.c) and run over 2000 seeded
    random files of the two fuzz generators above, the synthetic checkpoint and
    three truncations of it: no sanitizer report, the checkpoint admitted, every
    truncation rejected."""
    import random
    import subprocess
    csrc = os.path.join(REPO, "lunelette_b200", "csrc")
    exe = str(tmp_path / "open_checkpoints")
    build = subprocess.run(["gcc", "-std=c11", "-g", "-O1", "-fsanitize=address,undefined",
                            "-fno-sanitize-recover=undefined", "-fno-omit-frame-pointer", "-I" + csrc,
                            "-I" + os.path.join(REPO, "include"), os.path.join(csrc, "st.c"),
                            os.path.join(csrc, "weights.c"),
                            os.path.join(REPO, "tests", "c_drivers", "open_checkpoints.c"),
                            "-o", exe, "-lm", "-lpthread"], capture_output=True, text=True)
    if build.returncode and "asan" in build.stderr.lower():
        pytest.skip("no sanitizer runtime here: " + build.stderr.strip()[:200])
    assert build.returncode == 0, build.stderr
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0", UBSAN_OPTIONS="print_stacktrace=1")
    files = tmp_path / "files"
    files.mkdir()
    rng = random.Random(7)
    for i in range(2000):
        (structured_file if i % 2 else fuzz_file)(rng, str(files))
    run = subprocess.run([exe, str(files)], capture_output=True, text=True, env=env, timeout=600)
    assert run.returncode == 0 and "runtime error" not in run.stderr and "Sanitizer" not in run.stderr, \
        run.stderr[-2000:]
    assert len(run.stdout.splitlines()) == 2000
    n, _ = header_of(checkpoint_path)
    with open(checkpoint_path, "rb") as f:
        head = f.read(8 + n + (1 << 20))
    cuts = []
    for name, size in (("header_only", 8 + n), ("header_1mb", len(head)), ("header_cut", 8 + n // 2)):
        path = tmp_path / (name + ".safetensors")
        path.write_bytes(head[:size])
        cuts.append(str(path))
    run = subprocess.run([exe, checkpoint_path] + cuts, capture_output=True, text=True, env=env, timeout=600)
    assert run.returncode == 0 and "runtime error" not in run.stderr and "Sanitizer" not in run.stderr, \
        run.stderr[-2000:]
    verdicts = [line.split(" ", 1)[0] for line in run.stdout.splitlines()]
    assert verdicts == ["0", "-1", "-1", "-1"], run.stdout


def test_admission_finds_nan_codes_at_every_word_position(corrupt_copy):
    """The admission scan tests eight bytes at a time when only the NaN codes
    are rejected: a NaN code (0x7F or 0xFF) at each position of an 8-byte word,
    at a tensor's first and last byte and in the bytes after its last whole
    word is still found and named by its byte offset."""
    q = "language_model.model.layers.7.mlp.down_proj.weight"
    base = tensor_offset(corrupt_copy, q)
    size = 3072 * 9216
    for offset, code in [(8 * 1000 + k, 0x7F if k % 2 else 0xFF) for k in range(8)] + \
                        [(0, 0xFF), (size - 1, 0x7F), (size - 3, 0xFF), (4 << 20, 0x7F), ((4 << 20) - 1, 0xFF)]:
        old = patch(corrupt_copy, base + offset, bytes([code]))
        try:
            with pytest.raises(L.LuneletteError, match="byte %d code 0x%02x" % (offset, code)):
                L.validate_checkpoint(corrupt_copy, L.COMPACT_FP8_ARITHMETIC)
        finally:
            patch(corrupt_copy, base + offset, old)
    L.validate_checkpoint(corrupt_copy, L.COMPACT_FP8_ARITHMETIC)
