"""Non-finite and out-of-range hidden values on both decode paths, against the
reference's contract (include/metal.h:79-86; src/metal_runtime.m:418-424 scans
every logit and fails the call with "reset required"): a NaN anywhere in the
step must fail it and leave the sequence unusable until reset, and a finite but
huge hidden state must give the reference's finite logits.

The persistent decode kernel sums each layer's output in 64-bit fixed point
(range +-2^31). It flags a term it cannot hold and the host reruns that step
on the FP32 kernels, so both paths must agree with the oracle here. The faults
are made in the input file on the host (two embedding rows of a copy of the
synthetic checkpoint are rewritten), never on the device:
  BIG_TOKEN  its row times 2^30 (|x| ~ 2e7 > the fixed point's per-term limit
             2^23): finite logits, compared with the oracle;
  NAN_TOKEN  its row all NaN: the step fails, later calls fail until reset.
"""
import json
import os
import shutil

import numpy as np
import pytest

import lunelette_b200 as L
from tests.oracle_lib import greedy

pytestmark = pytest.mark.gpu

BIG_TOKEN, NAN_TOKEN = 4242, 4343
MAX_ABS, REL_L2 = 2e-2, 1e-2


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def patched_checkpoint(checkpoint_path, tmp_path_factory):
    path = str(tmp_path_factory.mktemp("nonfinite") / "patched.safetensors")
    shutil.copyfile(checkpoint_path, path)
    with open(path, "r+b") as f:
        n = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(n))
        begin, _ = header["language_model.model.embed_tokens.weight"]["data_offsets"]
        row_bytes = 3072 * 2
        at = 8 + n + begin + BIG_TOKEN * row_bytes
        f.seek(at)
        row = np.frombuffer(f.read(row_bytes), np.uint16).copy()
        normal = (row & 0x7F80) != 0  # zero and subnormal values keep their bits
        row[normal] = row[normal] + np.uint16(30 << 7)  # exponent + 30: the value times 2^30, exactly
        f.seek(at)
        f.write(row.tobytes())
        f.seek(8 + n + begin + NAN_TOKEN * row_bytes)
        f.write(np.full(3072, 0x7FC0, np.uint16).tobytes())
    yield path
    os.remove(path)


@pytest.fixture(scope="module")
def patched_oracle(oracle, patched_checkpoint):
    m = oracle.open_model(patched_checkpoint, 256)
    yield m
    m.close()


@pytest.mark.parametrize("mega", ["1", "0"])
def test_huge_and_nan_hidden_values_follow_the_reference(patched_checkpoint, patched_oracle, monkeypatch,
                                                         mega):
    monkeypatch.setenv("LUNELETTE_MEGA", mega)
    ids = np.random.default_rng(55).integers(1000, 131072, 12).astype(np.int64)
    patched_oracle.reset()
    with L.Runtime(patched_checkpoint) as rt:
        got = rt.prefill(ids).copy()
        want, _, _ = patched_oracle.forward(ids)
        assert np.abs(got - want).max() <= MAX_ABS
        # a finite step whose hidden state leaves the fixed-point range
        for token in (BIG_TOKEN, int(greedy(want))):
            got = rt.decode(token).copy()
            want, _, _ = patched_oracle.forward([token])
            assert np.all(np.isfinite(got))
            err, rel = float(np.abs(got - want).max()), rel_l2(got, want)
            assert err <= MAX_ABS and rel <= REL_L2, (token, err, rel)
            assert greedy(got) == greedy(want)
        length = rt.length()
        # a NaN step fails and the sequence stays invalid until reset
        with pytest.raises(L.LuneletteError, match="reset required"):
            rt.decode(NAN_TOKEN)
        with pytest.raises(L.LuneletteError, match="reset required"):
            rt.decode(int(ids[0]))
        with pytest.raises(L.LuneletteError):
            rt.checkpoint_create()
        assert rt.length() == length
        rt.reset()
        again = rt.prefill(ids).copy()
        assert np.all(np.isfinite(again))
    # the oracle itself rejects the NaN step, as the reference does
    with pytest.raises(RuntimeError, match="nonfinite"):
        patched_oracle.forward([NAN_TOKEN])


def test_decode_loop_reports_a_flagged_step(patched_checkpoint, monkeypatch):
    """The device-greedy loop cannot rerun a step on the FP32 kernels, so a step
    whose hidden values leave the fixed-point range fails the call."""
    monkeypatch.setenv("LUNELETTE_MEGA", "1")
    ids = np.random.default_rng(56).integers(1000, 131072, 8).astype(np.int64)
    with L.Runtime(patched_checkpoint) as rt:
        rt.prefill(ids)
        with pytest.raises(L.LuneletteError, match="fixed-point range|non-finite"):
            rt.decode_loop(BIG_TOKEN, 4)
        with pytest.raises(L.LuneletteError):
            rt.decode(int(ids[0]))  # the failed loop left the sequence invalid
