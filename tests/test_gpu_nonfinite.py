"""Non-finite and out-of-range hidden values on both decode paths, against the
reference's contract (include/metal.h:79-86; src/metal_runtime.m:418-424 scans
every logit and fails the call with "reset required"): a NaN must fail the
call and leave the sequence unusable until reset, and a finite but huge hidden
state must give the reference's finite logits.

The persistent decode kernel sums each layer's output in 64-bit fixed point
(range +-2^31). It flags a term it cannot hold (non-finite, or not below 2^23)
and the host reruns that step on the FP32 kernels, so both paths must agree
with the oracle. The faults are made in the input file on the host, in copies
of the synthetic checkpoint, never on the device:
  huge  layer 0's post-attention norm gain set to 4096 (BF16 0x4580): the FFN
        output, and so every later hidden state, is ~1e7..1e9 (above the fixed
        point's per-term limit) but finite, at every position; logits stay
        finite and are compared with the oracle on both paths;
  nan   one embedding row set to NaN. The embedding is also the tied head, so
        that token's logit is NaN in every call: the first call (a prefill, on
        the FP32 kernels) must fail and leave the sequence invalid until reset.
The persistent kernel's flag test is `!(fabsf(v) < 2^23)`, true for NaN and
infinities as for huge values, so the huge case exercises the same check.
"""
import json
import os
import shutil

import numpy as np
import pytest

import lunelette_b200 as L
from tests.oracle_lib import greedy

pytestmark = pytest.mark.gpu

NAN_TOKEN = 4343
MAX_ABS, REL_L2 = 2e-2, 1e-2


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def patched_copy(src, dst, patch):
    """Copy the checkpoint and rewrite bytes of named tensors: patch(name) ->
    (byte offset within the tensor, bytes) or None."""
    shutil.copyfile(src, dst)
    with open(dst, "r+b") as f:
        n = int.from_bytes(f.read(8), "little")
        header = json.loads(f.read(n))
        for name, info in header.items():
            if name == "__metadata__":
                continue
            change = patch(name)
            if change is not None:
                offset, data = change
                f.seek(8 + n + info["data_offsets"][0] + offset)
                f.write(data)
    return dst


def test_nan_logit_fails_the_call_until_reset(checkpoint_path, tmp_path, oracle, monkeypatch):
    path = patched_copy(checkpoint_path, str(tmp_path / "nan.safetensors"), lambda name: (
        NAN_TOKEN * 3072 * 2, np.full(3072, 0x7FC0, np.uint16).tobytes())
        if name == "language_model.model.embed_tokens.weight" else None)
    try:
        ids = np.random.default_rng(57).integers(1000, 131072, 6).astype(np.int64)
        for mega in ("1", "0"):
            monkeypatch.setenv("LUNELETTE_MEGA", mega)
            with L.Runtime(path) as rt:
                with pytest.raises(L.LuneletteError, match="logit %d is not finite; reset required" % NAN_TOKEN):
                    rt.prefill(ids)
                with pytest.raises(L.LuneletteError, match="reset required"):
                    rt.prefill(ids)  # the failed call left the sequence invalid
                assert rt.length() == 0
                rt.reset()
                with pytest.raises(L.LuneletteError, match="not finite"):
                    rt.prefill(ids[:1])
        m = oracle.open_model(path, 256)
        try:
            with pytest.raises(RuntimeError, match="nonfinite logit %d" % NAN_TOKEN):
                m.forward(ids)  # the reference arithmetic fails the same call
        finally:
            m.close()
    finally:
        os.remove(path)


@pytest.fixture(scope="module")
def huge_checkpoint(checkpoint_path, tmp_path_factory):
    path = patched_copy(checkpoint_path, str(tmp_path_factory.mktemp("huge") / "huge.safetensors"),
                        lambda name: (0, np.full(3072, 0x4580, np.uint16).tobytes())
                        if name == "language_model.model.layers.0.post_attention_layernorm.weight" else None)
    yield path
    os.remove(path)


@pytest.fixture(scope="module")
def huge_oracle(oracle, huge_checkpoint):
    m = oracle.open_model(huge_checkpoint, 256)
    yield m
    m.close()


@pytest.mark.parametrize("mega", ["1", "0"])
def test_huge_hidden_values_match_the_oracle_on_both_paths(huge_checkpoint, huge_oracle, monkeypatch, mega):
    monkeypatch.setenv("LUNELETTE_MEGA", mega)
    ids = np.random.default_rng(55).integers(1000, 131072, 12).astype(np.int64)
    huge_oracle.reset()
    with L.Runtime(huge_checkpoint) as rt:
        rt.trace(True)
        got = rt.prefill(ids).copy()
        hidden = rt.trace_copy(0, len(ids))
        rt.trace(False)
        assert np.abs(hidden).max() > 2.0 ** 23  # the layer-0 output really is out of the fixed range
        want, _, _ = huge_oracle.forward(ids)
        assert np.abs(got - want).max() <= MAX_ABS
        tok = greedy(want)
        for step in range(4):
            got = rt.decode(tok).copy()
            want, _, _ = huge_oracle.forward([tok])
            assert np.all(np.isfinite(got))
            err, rel = float(np.abs(got - want).max()), rel_l2(got, want)
            assert err <= MAX_ABS and rel <= REL_L2, (step, err, rel)
            assert greedy(got) == greedy(want)
            tok = greedy(want)


def test_decode_loop_reports_a_flagged_step(huge_checkpoint, monkeypatch):
    """The device-greedy loop cannot rerun a step on the FP32 kernels, so a step
    whose hidden values leave the fixed-point range fails the call and leaves
    the sequence invalid."""
    monkeypatch.setenv("LUNELETTE_MEGA", "1")
    ids = np.random.default_rng(56).integers(1000, 131072, 8).astype(np.int64)
    with L.Runtime(huge_checkpoint) as rt:
        first = greedy(rt.prefill(ids))
        with pytest.raises(L.LuneletteError, match="fixed-point range"):
            rt.decode_loop(first, 4)
        with pytest.raises(L.LuneletteError, match="reset required"):
            rt.decode(first)
