"""Parity at the benchmark's own sizes: every configuration bench.py times is
also checked against the CPU oracle at the same size, on the same seeded ids.

The reference pins its runtime by full-prefix regression over several prompt
lengths and reset cycles (tests/compare_native.c:69-96, 348-450); these tests
do the same at the configurations' sizes:
  C0  lunelette_cuda_decode_loop (the bench's `value` path): 31 device-greedy
      tokens after the 32-token prompt equal the oracle's greedy tokens;
  C2  the 4096-token prompt in 16 chunks of 256 at context 4352 (tcgen05
      GEMMs, tiled prefill attention, YaRN positions to 4095), then greedy
      decode at ~4.1k positions on the persistent kernel (position ranges per
      KV head merged in order), both through lunelette_metal_decode (logits
      against the oracle) and through the device loop (tokens);
  C3  a 512-token prefix, then 2 of the bench's turns of 200 appended ids and
      64 greedy tokens, with the checkpoint saved before each turn and restored;
  C4  the bench's 64 ragged sessions (prompts U[256, 4096]) prefilled into one
      paged pool, then batched decode steps; 8 of the sessions (the 7 shortest
      and one of 2813 tokens) checked against the oracle for 3 steps.
Gates: logits within 2e-2 max-abs and 1e-2 relative L2, greedy tokens equal.
The ids are drawn exactly as bench.py's config_lines draws them (seed 1234 + 99).
"""
import numpy as np
import pytest

import lunelette_b200 as L
from tests.oracle_lib import greedy

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

MAX_ABS, REL_L2 = 2e-2, 1e-2
BENCH_SEED = 1234


def assert_close(got, want, what):
    err = float(np.abs(got - want).max())
    rel = float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))
    assert err <= MAX_ABS and rel <= REL_L2, "%s: max-abs %.3g rel-L2 %.3g" % (what, err, rel)


def bench_inputs():
    """The ids of bench.py's config_lines, in its draw order."""
    rng = np.random.default_rng(BENCH_SEED + 99)
    c2 = rng.integers(1000, 131072, 4096).astype(np.int64)
    prefix = rng.integers(1000, 131072, 512).astype(np.int64)
    users = [rng.integers(1000, 131072, 200).astype(np.int64) for _ in range(8)]
    lengths = rng.integers(256, 4097, 64)
    prompts = [rng.integers(1000, 131072, int(n)).astype(np.int64) for n in lengths]
    return c2, prefix, users, prompts


@pytest.fixture(scope="module")
def inputs():
    return bench_inputs()


@pytest.fixture(scope="module")
def long_oracle(oracle, checkpoint_path):
    m = oracle.open_model(checkpoint_path, 4352)
    yield m
    m.close()


def test_c0_decode_loop_tokens_match_the_oracle(lib, checkpoint_path, oracle):
    """The bench's timed path: one persistent launch generating 31 greedy tokens
    on the device after the C0 prompt (bench.py's prompt, seed 1234)."""
    prompt = np.random.default_rng(BENCH_SEED).integers(1000, 131072, 32).astype(np.int64)
    m = oracle.open_model(checkpoint_path, 256)
    try:
        want, _, _ = m.forward(prompt)
        first = greedy(want)
        expected = []
        tok = first
        for _ in range(31):
            logits, _, _ = m.forward([tok])
            tok = greedy(logits)
            expected.append(tok)
    finally:
        m.close()
    with L.Runtime(checkpoint_path) as rt:
        got = rt.prefill(prompt)
        assert greedy(got) == first
        cp = rt.checkpoint_create()
        for _ in range(2):  # the bench repeats the pass from the restored checkpoint
            tokens, ms, launches = rt.decode_loop(first, 31)
            assert launches == 1 and ms > 0
            assert [int(t) for t in tokens] == expected
            assert rt.length() == 32 + 31
            rt.checkpoint_restore(cp)
        cp.destroy()


def test_c2_full_prompt_then_decode_matches_the_oracle(lib, checkpoint_path, long_oracle, inputs):
    ids = inputs[0]
    long_oracle.reset()
    want, _, _ = long_oracle.forward(ids)
    with L.Runtime(checkpoint_path, limits=(4352, 256)) as rt:
        got = rt.prefill(ids[:256])
        for c in range(1, 16):
            got = rt.append(ids[256 * c:256 * (c + 1)])
        got = got.copy()
        assert_close(got, want, "C2 logits after 4096 chunked ids")
        first = greedy(got)
        assert first == greedy(want)
        cp = rt.checkpoint_create()
        tok_gpu = tok_cpu = first
        oracle_tokens = []
        for step in range(8):
            got = rt.decode(tok_gpu).copy()
            want, _, _ = long_oracle.forward([tok_cpu])
            assert_close(got, want, "C2 decode step %d at %d positions" % (step, 4096 + step))
            tok_gpu, tok_cpu = greedy(got), greedy(want)
            assert tok_gpu == tok_cpu, "greedy divergence at step %d" % step
            oracle_tokens.append(tok_cpu)
        # the device loop at the same context: same tokens
        rt.checkpoint_restore(cp)
        tokens, _, _ = rt.decode_loop(first, 8)
        assert [int(t) for t in tokens] == oracle_tokens
        cp.destroy()


def test_c3_bench_turns_with_checkpoint_restore_match_the_oracle(lib, checkpoint_path, long_oracle, inputs):
    _, prefix, users, _ = inputs
    long_oracle.reset()
    with L.Runtime(checkpoint_path, limits=(4352, 256)) as rt:
        rt.prefill(prefix[:256])
        got = rt.append(prefix[256:]).copy()
        want, _, _ = long_oracle.forward(prefix)
        assert_close(got, want, "C3 prefix")
        cp = None
        for turn in range(2):
            if cp is not None:
                cp.destroy()
            cp = rt.checkpoint_create()      # the service saves the session before a turn
            rt.checkpoint_restore(cp)        # and resumes from it
            got = rt.append(users[turn]).copy()
            want, _, _ = long_oracle.forward(users[turn])
            assert_close(got, want, "C3 turn %d user tokens" % turn)
            tok = greedy(got)
            assert tok == greedy(want)
            for step in range(63):
                got = rt.decode(tok).copy()
                want, _, _ = long_oracle.forward([tok])
                assert_close(got, want, "C3 turn %d decode %d" % (turn, step))
                tok = greedy(got)
                assert tok == greedy(want), "C3 turn %d: greedy divergence at step %d" % (turn, step)
        # back to the start of the last turn: the same user tokens give the same logits
        start = rt.length() - 200 - 63
        restored = rt.checkpoint_restore(cp).copy()
        assert rt.length() == start
        again = rt.append(users[1]).copy()
        long_oracle.rewind(start)
        want, _, _ = long_oracle.forward(users[1])
        assert_close(again, want, "C3 replay of the last turn")
        assert np.all(np.isfinite(restored))
        cp.destroy()


def test_c4_ragged_batch_sample_matches_the_oracle(lib, checkpoint_path, oracle, inputs):
    prompts = inputs[3]
    order = sorted(range(64), key=lambda i: prompts[i].size)
    checked = order[:7] + [order[40]]
    with L.Batch(checkpoint_path, max_sessions=64, context=4352, pool_positions=64 * 4352, block=256) as b:
        sessions = [b.open() for _ in range(64)]
        first = []
        for s, ids in zip(sessions, prompts):
            for c0 in range(0, ids.size, 256):
                logits = b.append(s, ids[c0:c0 + 256])
            first.append(greedy(logits))
        steps = []
        toks = first
        for _ in range(3):
            nxt, logits = b.decode(sessions, toks, logits=True)
            steps.append(logits[checked].copy())
            toks = [int(t) for t in nxt]
        for j, i in enumerate(checked):
            assert b.length(sessions[i]) == prompts[i].size + 3
    for j, i in enumerate(checked):
        m = oracle.open_model(checkpoint_path, 4352)
        try:
            want, _, _ = m.forward(prompts[i])
            assert greedy(want) == first[i], "session %d first token" % i
            tok = first[i]
            for step in range(3):
                want, _, _ = m.forward([tok])
                assert_close(steps[step][j], want, "C4 session %d (%d ids) step %d" % (i, prompts[i].size, step))
                assert greedy(steps[step][j]) == greedy(want)
                tok = greedy(want)
        finally:
            m.close()
