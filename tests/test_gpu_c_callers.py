"""The drop-in boundary exercised from C: the reference's own callers of
include/metal.h, compiled from its sources with its headers (oracle/Makefile,
into oracle/_ref/) and linked against liblunelette_cuda.so unchanged.

  generate_metal_next   the reference's generation loop (src/generation.c)
                        with the CLI's logits callback (src/main.c:48-67):
                        its 32 greedy tokens after a 32-id prompt must equal
                        the oracle's greedy tokens.
  compare_native_cuda   the reference's native regression harness
                        (tests/compare_native.c:348-450): `capture` records 8
                        teacher-forced steps after prompts of 6/24/150/248 ids,
                        then `check` (a second process) replays them twice
                        over reset cycles and requires every logit to be
                        bitwise equal to the capture.

The binaries are built where the reference checkout exists and travel with the
repository; the GPU box needs no reference checkout."""
import os
import struct
import subprocess

import numpy as np
import pytest

from tests.oracle_lib import greedy

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BIN = os.path.join(REPO, "oracle", "_ref")


def binary(name):
    path = os.path.join(REF_BIN, name)
    if not os.path.exists(path):
        pytest.skip("%s not built (make -C oracle REF=<reference checkout> after building the library)" % name)
    return path


def test_reference_generation_loop_drives_the_runtime(lib, checkpoint_path, oracle):
    prompt = np.random.default_rng(4321).integers(1000, 131072, 32).astype(np.int64)
    proc = subprocess.run([binary("generate_metal_next"), checkpoint_path, "32"] + [str(int(i)) for i in prompt],
                          capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr
    lines = dict(line.split(":", 1) for line in proc.stdout.strip().splitlines())
    got = [int(t) for t in lines["tokens"].split()]
    assert int(lines["calls"]) == len(got)
    # the oracle with the same rule (strict '>', stop at EOS id 2 or the budget)
    m = oracle.open_model(checkpoint_path, 256)
    try:
        want = []
        logits, _, _ = m.forward(prompt)
        while True:
            tok = greedy(logits)
            want.append(tok)
            if tok == 2 or len(want) == 32:
                break
            logits, _, _ = m.forward([tok])
    finally:
        m.close()
    assert got == want
    assert int(lines["stop"]) == (1 if want[-1] == 2 else 0)


def write_generated_fixture(path, forced):
    """A safetensors file with the harness's teacher-forced ids: I64 [8]."""
    data = np.asarray(forced, np.int64).tobytes()
    header = ('{"generated":{"dtype":"I64","shape":[%d],"data_offsets":[0,%d]}}' % (len(forced), len(data))).encode()
    header += b" " * ((8 - len(header) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header)))
        f.write(header)
        f.write(data)


def test_reference_native_harness_capture_then_check(lib, checkpoint_path, tmp_path):
    rng = np.random.default_rng(606)
    pairs = []
    for count in (6, 24, 150, 248):
        ids_path = tmp_path / ("ids%d.txt" % count)
        ids_path.write_text(" ".join(str(int(i)) for i in rng.integers(1000, 131072, count)) + "\n")
        fixture = tmp_path / ("forced%d.safetensors" % count)
        write_generated_fixture(fixture, rng.integers(1000, 131072, 8))
        pairs += [str(ids_path), str(fixture)]
    out_dir = tmp_path / "capture"
    out_dir.mkdir()
    exe = binary("compare_native_cuda")
    for mode in ("capture", "check"):
        proc = subprocess.run([exe, mode, checkpoint_path, "mps", str(out_dir)] + pairs,
                              capture_output=True, text=True, timeout=900)
        assert proc.returncode == 0, (mode, proc.stdout[-2000:], proc.stderr[-2000:])
        assert ("PASS native %s" % mode) in proc.stdout
    # check compared 4 prompts x 8 steps x 2 reset cycles, every one bitwise
    # exact (its capture-file validation prints further exact=1 lines)
    assert "steps=64 cycles=2" in proc.stdout
    assert "exact=0" not in proc.stdout
    assert len([l for l in proc.stdout.splitlines() if l.startswith("check mode=mps cycle=")]) == 64
