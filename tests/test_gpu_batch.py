"""Batched decode over independent sessions (lunelette_cuda_batch_*, survey
row f1, config 4 at reduced size) on the B200: every session's logits of a
batched step against the single-sequence runtime (itself pinned to the
oracle) on the same tokens and against the oracle directly; page recycling and
pool exhaustion."""
import numpy as np
import pytest

import lunelette_b200 as L
from tests.oracle_lib import greedy

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
REL_L2 = 1e-2


def assert_close(got, want, what):
    err = float(np.abs(got - want).max())
    rel = float(np.linalg.norm((got - want).ravel()) / max(np.linalg.norm(want.ravel()), 1e-30))
    assert err <= MAX_ABS and rel <= REL_L2, "%s: max-abs %.3g rel-L2 %.3g" % (what, err, rel)


def test_batched_decode_matches_single_sessions_and_oracle(lib, checkpoint_path, oracle):
    rng = np.random.default_rng(404)
    prompts = [rng.integers(1000, 131072, n) for n in (20, 45, 70)]
    with L.Batch(checkpoint_path, max_sessions=4, context=4352, pool_positions=1024, block=256) as b:
        sessions = [b.open() for _ in prompts]
        firsts = [greedy(b.append(s, p).copy()) for s, p in zip(sessions, prompts)]
        steps = 5
        toks = list(firsts)
        batched = []
        for _ in range(steps):
            nxt, lg = b.decode(sessions, toks, logits=True)
            batched.append(lg)
            assert [greedy(r) for r in lg] == nxt.tolist()
            toks = nxt.tolist()
        assert [b.length(s) for s in sessions] == [len(p) + steps for p in prompts]
    # the same sequences one at a time through the single-sequence runtime
    with L.Runtime(checkpoint_path, limits=(4352, 256)) as rt:
        for k, p in enumerate(prompts):
            rt.reset()
            tok = greedy(rt.prefill(p).copy())
            assert tok == firsts[k]
            for step in range(steps):
                want = rt.decode(tok).copy()
                assert_close(batched[step][k], want, "session %d step %d vs single" % (k, step))
                tok = greedy(want)
                assert tok == greedy(batched[step][k])
    # and session 1 against the oracle
    m = oracle.open_model(checkpoint_path, 4352)
    try:
        m.forward(prompts[1])
        tok = firsts[1]
        for step in range(steps):
            want, _, _ = m.forward([tok])
            assert_close(batched[step][1], want, "session 1 step %d vs oracle" % step)
            tok = greedy(want)
    finally:
        m.close()


def test_batch_pages_recycle_and_pool_exhaustion(lib, checkpoint_path):
    rng = np.random.default_rng(9)
    prompt = rng.integers(1000, 131072, 100)
    # 4 pages: one 100-token session takes 2, a second one 2, a third cannot start
    with L.Batch(checkpoint_path, max_sessions=3, context=256, pool_positions=256, block=128) as b:
        a = b.open()
        first = b.append(a, prompt).copy()
        c = b.open()
        b.append(c, prompt)
        assert b.free_positions() == 0
        d = b.open()
        with pytest.raises(L.LuneletteError):
            b.append(d, prompt[:10])
        with pytest.raises(L.LuneletteError):
            b.decode([a, a], [1, 2])  # a session twice
        b.close_session(c)
        assert b.free_positions() == 128
        # the freed pages serve a new session with the same results as before
        again = b.append(d, prompt).copy()
        assert np.array_equal(again.view(np.uint32), first.view(np.uint32))
        nxt = b.decode([a, d], [greedy(first), greedy(first)])
        assert nxt[0] == nxt[1]


def test_batch_decode_many_ragged_sessions(lib, checkpoint_path):
    """20 sessions with ragged lengths (some across page boundaries): two
    batched steps agree with per-session single decode for a sample."""
    rng = np.random.default_rng(77)
    lengths = rng.integers(5, 200, 20)
    prompts = [rng.integers(1000, 131072, n) for n in lengths]
    with L.Batch(checkpoint_path, max_sessions=20, context=4352, pool_positions=20 * 256, block=256) as b:
        sessions = [b.open() for _ in prompts]
        toks = [greedy(b.append(s, p).copy()) for s, p in zip(sessions, prompts)]
        first_toks = list(toks)
        step1, lg1 = b.decode(sessions, toks, logits=True)
        step2, lg2 = b.decode(sessions, step1.tolist(), logits=True)
    with L.Runtime(checkpoint_path, limits=(4352, 256)) as rt:
        for k in (0, 7, 13, 19):
            rt.reset()
            rt.prefill(prompts[k])
            w1 = rt.decode(first_toks[k]).copy()
            assert_close(lg1[k], w1, "session %d step 1" % k)
            w2 = rt.decode(int(step1[k])).copy()
            assert_close(lg2[k], w2, "session %d step 2" % k)


def test_forked_sessions_share_a_prefix_and_diverge(lib, checkpoint_path, oracle):
    """lunelette_cuda_batch_fork: sessions forked from a 300-position prefix (a
    partial last page: copied) and from its first 256 positions (whole pages:
    shared) continue independently; every logits vector against the oracle on
    the same full sequence, also after the source session is closed (its
    shared pages stay alive while a fork holds them), and every page returns to
    the pool at the end."""
    rng = np.random.default_rng(505)
    prefix = rng.integers(1000, 131072, 300)
    users = [rng.integers(1000, 131072, n) for n in (40, 17, 33)]
    with L.Batch(checkpoint_path, max_sessions=4, context=4352, pool_positions=2048, block=256) as b:
        free0 = b.free_positions()
        a = b.open()
        b.append(a, prefix[:256])
        b.append(a, prefix[256:])
        full = b.fork(a, 300)   # pages 0-3 shared, page 4 (44 positions) copied
        whole = b.fork(a, 256)  # pages 0-3 shared
        assert b.length(full) == 300 and b.length(whole) == 256
        # 5 pages for a, one more for the copied partial page
        assert b.free_positions() == free0 - 6 * 64
        got = {full: [b.append(full, users[0]).copy()], a: [b.append(a, users[1]).copy()],
               whole: [b.append(whole, users[2]).copy()]}
        toks = {s: greedy(v[0]) for s, v in got.items()}
        order = [full, a, whole]
        for _ in range(2):
            nxt, lg = b.decode(order, [toks[s] for s in order], logits=True)
            for i, s in enumerate(order):
                got[s].append(lg[i].copy())
                toks[s] = int(nxt[i])
        b.close_session(a)
        for _ in range(2):  # the forks keep decoding on the shared pages
            nxt, lg = b.decode([full, whole], [toks[full], toks[whole]], logits=True)
            for i, s in enumerate((full, whole)):
                got[s].append(lg[i].copy())
                toks[s] = int(nxt[i])
        b.close_session(full)
        b.close_session(whole)
        assert b.free_positions() == free0
    m = oracle.open_model(checkpoint_path, 4352)
    try:
        m.forward(prefix)
        for s, start, user in ((full, 300, users[0]), (a, 300, users[1]), (whole, 256, users[2])):
            m.rewind(start)
            want, _, _ = m.forward(user)
            seq = got[s]
            assert_close(seq[0], want, "fork %d: appended block" % s)
            for step, logits in enumerate(seq[1:]):
                want, _, _ = m.forward([greedy(seq[step])])
                assert_close(logits, want, "fork %d: decode step %d" % (s, step))
                assert greedy(logits) == greedy(want)
    finally:
        m.close()


def test_tcgen05_head_matches_mma_head_and_oracle(lib, checkpoint_path, oracle, monkeypatch):
    """The batched head on tcgen05 (head_tc.cuh, the default; LUNELETTE_HEAD_TC=1)
    against the mma.sync head (LUNELETTE_HEAD_TC=0) on the same tokens: 70 sessions, so the head runs as a
    pass of 64 tokens and a pass of 6; the logits agree to FP32 accumulation
    order, the greedy ids follow from them, and one session of the second pass
    against the oracle."""
    rng = np.random.default_rng(606)
    prompts = [rng.integers(1000, 131072, n) for n in rng.integers(5, 40, 70)]
    runs = {}
    feed = None
    for head in ("0", "1"):
        monkeypatch.setenv("LUNELETTE_HEAD_TC", head)
        with L.Batch(checkpoint_path, max_sessions=70, context=4352, pool_positions=70 * 128, block=256) as b:
            sessions = [b.open() for _ in prompts]
            firsts = [greedy(b.append(s, p).copy()) for s, p in zip(sessions, prompts)]
            toks = firsts if feed is None else feed[0]
            nxt1, lg1 = b.decode(sessions, toks, logits=True)
            assert [greedy(r) for r in lg1] == nxt1.tolist()
            toks2 = nxt1.tolist() if feed is None else feed[1]
            nxt2, lg2 = b.decode(sessions, toks2, logits=True)
            assert [greedy(r) for r in lg2] == nxt2.tolist()
            if feed is None:
                feed = (firsts, toks2)
            runs[head] = (lg1.copy(), lg2.copy())
    for step in range(2):
        got, want = runs["1"][step], runs["0"][step]
        assert np.all(np.isfinite(got))
        err = float(np.abs(got - want).max())
        rel = float(np.linalg.norm((got - want).ravel()) / np.linalg.norm(want.ravel()))
        assert err <= 1e-3 and rel <= 1e-5, "step %d: max-abs %.3g rel-L2 %.3g" % (step, err, rel)
    k = 66
    m = oracle.open_model(checkpoint_path, 4352)
    try:
        m.forward(prompts[k])
        want, _, _ = m.forward([feed[0][k]])
        assert_close(runs["1"][0][k], want, "session %d step 1 (tcgen05 head) vs oracle" % k)
    finally:
        m.close()
