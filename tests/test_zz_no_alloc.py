"""The allocation-free attention entry point, for callers that cannot call
cudaMalloc (an engine that has reserved the whole device for its own pool, or a
loop where an allocation would synchronise the device): it must give the same
output as lunelette_cuda_attention, which takes caller scratch, and as the FP32
oracle, on two calls in a row (the second call finds the first call's partial
results in the shared array).

Collected last on purpose (file name), and self-contained so it also passes
alone in a fresh process."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SLOTS = 4096  # the fixed scratch of the allocation-free entry point, in slots


def pool_from_rows(k_rows, v_rows, table, num_pages, layer, layers):
    pool = np.zeros((layers, num_pages, 2, 8, 64, 128), np.float32)
    for p in range(k_rows.shape[0]):
        page = table[p // 64]
        pool[layer, page, 0, :, p % 64, :] = k_rows[p].reshape(8, 128)
        pool[layer, page, 1, :, p % 64, :] = v_rows[p].reshape(8, 128)
    return pool.reshape(-1)


def test_noalloc_matches_scratch_entry_point_twice(lib, oracle):
    import torch
    torch.cuda.init()
    stream = torch.cuda.current_stream().cuda_stream
    err = ctypes.create_string_buffer(512)
    # (length, count, seed): one and five query rows split over positions (the
    # scratch is used); 40 rows on the block path at a long context, where the
    # split count is clamped to what the fixed scratch holds (3 splits x 40 x 32
    # = 3840 of its 4096 slots); 100 and 128 rows, where the clamp leaves one
    # split per key range
    cases = [(300, 1, 11), (1000, 5, 12), (3000, 40, 13), (2500, 100, 14), (1200, 128, 15)]
    for length, count, seed in cases:
        rng = np.random.default_rng(seed)
        total = length + count
        num_pages = (total + 63) // 64 + 1
        table = rng.permutation(num_pages).astype(np.int32)
        k = rng.standard_normal((total, 1024)).astype(np.float32)
        v = rng.standard_normal((total, 1024)).astype(np.float32)
        q = rng.standard_normal((count, 4096)).astype(np.float32)
        d_q = torch.from_numpy(q).cuda()
        d_pool = torch.from_numpy(pool_from_rows(k, v, table, num_pages, 1, 2)).cuda()
        d_table = torch.from_numpy(table).cuda()
        acc = torch.empty(SLOTS * 128, dtype=torch.float32, device="cuda")
        ml = torch.empty(SLOTS * 2, dtype=torch.float32, device="cuda")
        want = torch.empty((count, 4096), dtype=torch.float32, device="cuda")
        assert lib.lunelette_cuda_attention(d_q.data_ptr(), d_pool.data_ptr(), d_table.data_ptr(),
                                            num_pages, 1, length, count, want.data_ptr(),
                                            acc.data_ptr(), ml.data_ptr(), SLOTS, stream) == 0
        # the FP32 oracle on the same rows, so the fixed-scratch path is pinned to
        # the restatement directly and not only through the scratch-taking one
        exact = oracle.attention(q, k, v, length)
        for call in range(2):
            got = torch.full((count, 4096), float("nan"), dtype=torch.float32, device="cuda")
            rc = lib.lunelette_cuda_attention_noalloc(d_q.data_ptr(), d_pool.data_ptr(),
                                                      d_table.data_ptr(), num_pages, 1, length,
                                                      count, got.data_ptr(), stream, err, 512)
            assert rc == 0, err.value
            torch.cuda.synchronize()
            a, b = got.cpu().numpy(), want.cpu().numpy()
            assert np.all(np.isfinite(a))
            # the tolerance of the attention parity tests
            assert np.abs(a - b).max() < 1e-5 * max(1.0, np.abs(b).max()), (length, count, call)
            assert np.abs(a - exact).max() < 1e-5 * max(1.0, np.abs(exact).max()), \
                (length, count, call)


def test_noalloc_rejects_counts_beyond_its_scratch(lib):
    import torch
    err = ctypes.create_string_buffer(512)
    count, num_pages = 129, 4
    q = torch.zeros((count, 4096), dtype=torch.float32, device="cuda")
    pool = torch.zeros(2 * num_pages * 2 * 8 * 64 * 128, dtype=torch.float32, device="cuda")
    table = torch.arange(num_pages, dtype=torch.int32, device="cuda")
    out = torch.empty((count, 4096), dtype=torch.float32, device="cuda")
    rc = lib.lunelette_cuda_attention_noalloc(q.data_ptr(), pool.data_ptr(), table.data_ptr(),
                                              num_pages, 0, 0, count, out.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream, err, 512)
    assert rc == -1
    assert b"at most 128 query rows" in err.value
