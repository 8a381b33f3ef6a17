"""Kernel parity on the B200: each product kernel, called through the C-ABI on
device buffers, against the CPU oracle (or a float64 restatement of the
reference's own analytic expectations) on awkward and model shapes."""
import json
import os
import struct

import numpy as np
import pytest

from tests.tiling import ORDER_INTERLEAVE, ORDER_ROPE_PAIRS, ORDER_ROWS, tile_reference, tiled_bytes

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    torch.cuda.init()
    return torch


_KEEP = []  # device copies stay referenced until the test's kernels finished


@pytest.fixture(autouse=True)
def _release_device_copies():
    yield
    import torch
    torch.cuda.synchronize()
    _KEEP.clear()


def dev(torch, array):
    """Device copy that outlives the (asynchronous) launches of this test.
    A temporary would go back to torch's caching allocator at once and could be
    handed to the next copy before the kernel reads it."""
    t = torch.from_numpy(np.ascontiguousarray(array)).cuda()
    _KEEP.append(t)
    return t


def ptr(t):
    return t.data_ptr()


def tiled(lib, torch, codes, order=ORDER_ROWS):
    """Row-major codes -> the device's tiled layout, through the tile kernel."""
    rows, cols = codes.shape
    raw = dev(torch, codes)
    out = torch.full((tiled_bytes(rows, cols),), 0xAB, dtype=torch.uint8, device="cuda")
    _KEEP.append(out)
    assert lib.lunelette_cuda_tile_fp8(ptr(raw), rows, cols, order, ptr(out), stream(torch)) == 0
    return out


def stream(torch):
    return torch.cuda.current_stream().cuda_stream


def e4m3_table(oracle):
    return np.array([oracle.fp8_decode(c) for c in range(256)], np.float32)


def finite_codes(rng, shape):
    codes = rng.integers(0, 256, size=shape).astype(np.uint8)
    codes[(codes & 127) == 127] = 0x3A  # never NaN
    return codes


def bf16_round(x):
    b = np.array(x, np.float32).view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


def test_fp8_decode_bit_exact_all_codes(lib, torch_cuda):
    torch = torch_cuda
    golden = json.load(open(os.path.join(GOLDEN, "fp8_golden.json")))
    table = np.array(golden["bits"], np.uint32).view(np.float32)
    n = 1031  # odd: exercises the tail of the pair conversion
    codes = ((np.arange(n) * 37 + 11) % 256).astype(np.uint8)
    scales = [1.0, struct.unpack("<f", struct.pack("<I", 0x39FB << 16))[0], float.fromhex("0x1.f6p-12"),
              float.fromhex("0x1.02p+5"), 2.0 ** -110, 2.0 ** 100, 0.251953125, 3.140625]
    d_codes = dev(torch, codes)
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    for scale in scales:
        assert lib.lunelette_cuda_fp8_decode(ptr(d_codes), n, scale, ptr(out), stream(torch)) == 0
        got = out.cpu().numpy()
        want = table[codes] * np.float32(scale)
        nan = (codes & 127) == 127
        assert np.all(np.isnan(got[nan]))
        assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32)), scale


def gemv_check(lib, oracle, torch, rows, cols, count, seed, residual=False, entry="lunelette_cuda_gemv_fp8"):
    rng = np.random.default_rng(seed)
    codes = finite_codes(rng, (rows, cols))
    scale = float(bf16_round(np.float32(0.0003 + rng.random() * 0.01)))
    x = rng.standard_normal((count, cols)).astype(np.float32)
    res = rng.standard_normal((count, rows)).astype(np.float32) if residual else None
    d_w, d_x = tiled(lib, torch, codes), dev(torch, x)
    d_r = dev(torch, res) if residual else None
    y = torch.empty((count, rows), dtype=torch.float32, device="cuda")
    rc = getattr(lib, entry)(ptr(d_w), rows, cols, scale, ptr(d_x),
                             ptr(d_r) if residual else None, count, ptr(y), stream(torch))
    assert rc == 0
    got = y.cpu().numpy()
    w64 = e4m3_table(oracle)[codes].astype(np.float64) * scale
    exact = x.astype(np.float64) @ w64.T
    bound = np.abs(x.astype(np.float64)) @ np.abs(w64).T
    if residual:
        exact = exact + res
        bound = bound + np.abs(res)
    assert np.all(np.abs(got - exact) <= 1e-5 * bound + 1e-30)
    ref = oracle.project_fp8(codes, scale, x)
    if residual:
        ref = ref + res
    # same arithmetic within FP32 summation-order noise of the reference's lane loop
    assert np.all(np.abs(got - ref) <= 1e-5 * bound + 1e-30)


@pytest.mark.parametrize("rows,cols,count", [
    (7, 16, 1), (259, 48, 3), (65, 3072, 1), (1024, 3072, 2), (4096, 3072, 1),
    (3072, 4096, 4), (3072, 9216, 1), (3072, 9216, 5), (1, 9216, 4), (33, 112, 9)])
def test_gemv_fp8_matches_oracle(lib, oracle, torch_cuda, rows, cols, count):
    gemv_check(lib, oracle, torch_cuda, rows, cols, count, seed=rows * 7 + cols + count)


def test_gemv_fp8_residual(lib, oracle, torch_cuda):
    gemv_check(lib, oracle, torch_cuda, 3072, 4096, 3, seed=11, residual=True)


# The tcgen05 prefill GEMM: one and two 128-token tiles, partial row tiles
# (rows % 256 != 0), K ranges split across CTAs, K not a multiple of 64.
@pytest.mark.parametrize("rows,cols,count", [
    (256, 64, 1), (264, 3072, 5), (40, 112, 7), (3072, 4096, 130), (6144, 3072, 256),
    (3072, 9216, 37), (18432, 3072, 200), (1024, 3072, 128), (512, 9216, 129)])
def test_gemm_fp8_matches_oracle(lib, oracle, torch_cuda, rows, cols, count):
    gemv_check(lib, oracle, torch_cuda, rows, cols, count, seed=rows * 5 + cols + count,
               entry="lunelette_cuda_gemm_fp8")


# Blocks of up to 64 tokens run the GEMM with the weights as tensor-memory A
# (prefill_gemm_tmem.cuh): the model's shapes at the decode-batch sizes, a
# token count that is not a multiple of 16, and K ranges split across CTAs.
@pytest.mark.parametrize("rows,cols,count", [
    (6144, 3072, 64), (18432, 3072, 64), (3072, 4096, 33), (3072, 9216, 16), (128, 3072, 63), (136, 3072, 2)])
def test_small_block_gemm_matches_oracle(lib, oracle, torch_cuda, rows, cols, count):
    gemv_check(lib, oracle, torch_cuda, rows, cols, count, seed=rows * 3 + cols + count,
               entry="lunelette_cuda_gemm_fp8")


def test_gemm_fp8_residual(lib, oracle, torch_cuda):
    gemv_check(lib, oracle, torch_cuda, 3072, 4096, 77, seed=12, residual=True, entry="lunelette_cuda_gemm_fp8")


def test_gemm_rejects_unsupported_shapes(lib, torch_cuda):
    torch = torch_cuda
    w = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(1 << 16, dtype=torch.float32, device="cuda")
    y = torch.zeros(1 << 16, dtype=torch.float32, device="cuda")
    s = stream(torch)
    assert lib.lunelette_cuda_gemm_fp8(ptr(w), 12, 64, 1.0, ptr(x), None, 1, ptr(y), s) == -1  # rows % 8
    assert lib.lunelette_cuda_gemm_fp8(ptr(w), 16, 24, 1.0, ptr(x), None, 1, ptr(y), s) == -1  # cols % 16
    assert lib.lunelette_cuda_gemm_fp8(ptr(w), 16, 64, 1.0, ptr(x), None, 0, ptr(y), s) == -1  # no tokens


@pytest.mark.parametrize("k", [16, 32, 48, 64, 3072, 9216])
def test_gemv_exact_integer_dots(lib, torch_cuda, k):
    # all-ones weights (E4M3 0x38 = 1.0) and inputs give exactly K
    torch = torch_cuda
    rows, count = 5, 3
    d_w = tiled(lib, torch, np.full((rows, k), 0x38, np.uint8))
    d_x = dev(torch, np.ones((count, k), np.float32))
    y = torch.empty((count, rows), dtype=torch.float32, device="cuda")
    assert lib.lunelette_cuda_gemv_fp8(ptr(d_w), rows, k, 1.0, ptr(d_x), None, count, ptr(y),
                                       stream(torch)) == 0
    assert torch.all(y == float(k)).item()


@pytest.mark.parametrize("rows,cols,order", [(7, 16, ORDER_ROWS), (33, 112, ORDER_ROWS), (259, 48, ORDER_ROWS),
                                             (6144, 3072, ORDER_ROPE_PAIRS), (1024, 3072, ORDER_ROPE_PAIRS),
                                             (18432, 3072, ORDER_INTERLEAVE), (3072, 9216, ORDER_ROWS)])
def test_tile_kernel_matches_layout(lib, torch_cuda, rows, cols, order):
    torch = torch_cuda
    codes = np.random.default_rng(rows * 3 + cols + order).integers(0, 256, (rows, cols)).astype(np.uint8)
    got = tiled(lib, torch, codes, order).cpu().numpy()
    assert np.array_equal(got, tile_reference(codes, order))


def test_tile_rejects_bad_arguments(lib, torch_cuda):
    torch = torch_cuda
    d = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    assert lib.lunelette_cuda_tile_fp8(ptr(d), 16, 24, 0, ptr(d), stream(torch)) == -1   # cols % 16
    assert lib.lunelette_cuda_tile_fp8(ptr(d), 100, 64, 1, ptr(d), stream(torch)) == -1  # rows % 128
    assert lib.lunelette_cuda_tile_fp8(ptr(d), 15, 64, 2, ptr(d), stream(torch)) == -1   # odd rows
    assert lib.lunelette_cuda_tile_fp8(ptr(d), 16, 64, 3, ptr(d), stream(torch)) == -1   # order
    assert lib.lunelette_cuda_tile_fp8(None, 16, 64, 0, ptr(d), stream(torch)) == -1


def test_gemv_hi_lo_split_keeps_fp32_accuracy_over_wide_ranges(lib, oracle, torch_cuda):
    # activations spanning 2^-30..2^30 within one row: the power-of-two staging
    # scale follows the largest value, tiny ones ride in the lo half or vanish
    # below FP32 summation noise of the large ones
    torch = torch_cuda
    rng = np.random.default_rng(77)
    rows, cols, count = 48, 3072, 3
    codes = finite_codes(rng, (rows, cols))
    x = (rng.standard_normal((count, cols)) * np.exp2(rng.integers(-30, 31, (count, cols)))).astype(np.float32)
    x[1] *= np.float32(1e-20)
    x[2] = 0.0
    d_w, d_x = tiled(lib, torch, codes), dev(torch, x)
    y = torch.empty((count, rows), dtype=torch.float32, device="cuda")
    assert lib.lunelette_cuda_gemv_fp8(ptr(d_w), rows, cols, 0.001, ptr(d_x), None, count, ptr(y),
                                       stream(torch)) == 0
    got = y.cpu().numpy()
    w64 = e4m3_table(oracle)[codes].astype(np.float64) * 0.001
    exact = x.astype(np.float64) @ w64.T
    bound = np.abs(x.astype(np.float64)) @ np.abs(w64).T
    assert np.all(np.abs(got - exact) <= 1e-5 * bound + 1e-38)
    assert not got[2].any()


def test_gemv_rejects_unsupported_shapes(lib, torch_cuda):
    torch = torch_cuda
    d = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    f = torch.zeros(4096, dtype=torch.float32, device="cuda")
    assert lib.lunelette_cuda_gemv_fp8(ptr(d), 7, 67, 1.0, ptr(f), None, 3, ptr(f), stream(torch)) == -1
    assert lib.lunelette_cuda_gemv_fp8(ptr(d), 7, 0, 1.0, ptr(f), None, 3, ptr(f), stream(torch)) == -1
    assert lib.lunelette_cuda_gemv_fp8(None, 7, 16, 1.0, ptr(f), None, 3, ptr(f), stream(torch)) == -1


def test_rmsnorm_matches_oracle(lib, oracle, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(5)
    for width, count in [(67 * 16, 2), (3072, 7)]:
        x = (rng.standard_normal((count, width)) * 3).astype(np.float32)
        g = (0.5 + rng.random(width)).astype(np.float32)
        out = torch.empty((count, width), dtype=torch.float32, device="cuda")
        assert lib.lunelette_cuda_rmsnorm(ptr(dev(torch, g)), ptr(dev(torch, x)), width, count,
                                          ptr(out), stream(torch)) == 0
        assert np.abs(out.cpu().numpy() - oracle.norm(g, x)).max() < 2e-6 * 3 * 3


def pool_view(pool, num_pages):
    return pool.reshape(-1, num_pages, 2, 8, 64, 128)


def kv_rows(pool_np, page_table, num_pages, layer, kind, positions):
    v = pool_view(pool_np, num_pages)
    out = []
    for p in positions:
        page = page_table[p // 64]
        out.append(v[layer, page, kind, :, p % 64, :].reshape(1024))
    return np.stack(out)




@pytest.mark.parametrize("entry,count,length", [
    ("lunelette_cuda_qkv_rope", 6, 61),        # positions 61..66 cross a page boundary
    ("lunelette_cuda_gemm_qkv_rope", 6, 61),
    ("lunelette_cuda_gemm_qkv_rope", 150, 30),  # two token tiles over three pages
])
def test_qkv_rope_kv_store_matches_oracle(lib, oracle, torch_cuda, entry, count, length):
    torch = torch_cuda
    rng = np.random.default_rng(21 + count)
    layer = 1
    num_pages = 4
    page_table = np.array([2, 0, 3, 1], np.int32)
    codes = finite_codes(rng, (6144, 3072))
    scales = np.array([bf16_round(np.float32(s)) for s in (0.0007, 0.0011, 0.0005)], np.float32)
    gain = (0.5 + rng.random(3072)).astype(np.float32)
    x = rng.standard_normal((count, 3072)).astype(np.float32)
    positions = np.arange(length, length + count)
    cos = np.zeros((num_pages * 64, 128), np.float32)
    sin = np.zeros((num_pages * 64, 128), np.float32)
    for p in range(num_pages * 64):
        cos[p], sin[p] = oracle.yarn(p)
    pool = torch.zeros((layer + 1) * num_pages * 2 * 8 * 64 * 128, dtype=torch.float32, device="cuda")
    q_out = torch.empty((count, 4096), dtype=torch.float32, device="cuda")
    rc = getattr(lib, entry)(
        ptr(tiled(lib, torch, codes, ORDER_ROPE_PAIRS)), scales.ctypes.data, ptr(dev(torch, gain)),
        ptr(dev(torch, x)),
        count, length, ptr(dev(torch, cos)), ptr(dev(torch, sin)), ptr(q_out), ptr(pool),
        ptr(dev(torch, page_table)), num_pages, layer, stream(torch))
    assert rc == 0
    normed = oracle.norm(gain, x)
    q = oracle.project_fp8(codes[:4096], scales[0], normed)
    k = oracle.project_fp8(codes[4096:5120], scales[1], normed)
    v = oracle.project_fp8(codes[5120:], scales[2], normed)
    rq = oracle.rope(q, cos[positions], sin[positions], positions, 1)
    rk = oracle.rope(k, cos[positions], sin[positions], positions, 0)
    got_q = q_out.cpu().numpy()
    assert np.abs(got_q - rq).max() <= 1e-5 * np.abs(rq).max()
    pool_np = pool.cpu().numpy()
    got_k = kv_rows(pool_np, page_table, num_pages, layer, 0, positions)
    got_v = kv_rows(pool_np, page_table, num_pages, layer, 1, positions)
    # FP32 storage, as the reference's KV blit: only summation-order noise remains
    assert np.abs(got_k - rk).max() <= 1e-5 * np.abs(rk).max()
    assert np.abs(got_v - v).max() <= 1e-5 * np.abs(v).max()
    # layer 0 untouched
    assert not pool_view(pool_np, num_pages)[0].any()


@pytest.mark.parametrize("entry,count", [
    ("lunelette_cuda_gateup_swiglu", 3), ("lunelette_cuda_gemm_gateup_swiglu", 3),
    ("lunelette_cuda_gemm_gateup_swiglu", 131)])
def test_gateup_swiglu_matches_oracle(lib, oracle, torch_cuda, entry, count):
    torch = torch_cuda
    rng = np.random.default_rng(31 + count)
    gate = finite_codes(rng, (9216, 3072))
    up = finite_codes(rng, (9216, 3072))
    inter = tiled(lib, torch, np.concatenate([gate, up]), ORDER_INTERLEAVE)  # gate f at 2f, up f at 2f+1
    sg, su = float(bf16_round(np.float32(0.0004))), float(bf16_round(np.float32(0.0006)))
    gain = (0.5 + rng.random(3072)).astype(np.float32)
    x = rng.standard_normal((count, 3072)).astype(np.float32)
    act = torch.empty((count, 9216), dtype=torch.float32, device="cuda")
    assert getattr(lib, entry)(ptr(inter), sg, su, ptr(dev(torch, gain)),
                                            ptr(dev(torch, x)), count, ptr(act), stream(torch)) == 0
    normed = oracle.norm(gain, x)
    g = oracle.project_fp8(gate, sg, normed)
    u = oracle.project_fp8(up, su, normed)
    want = oracle.element(oracle.element(g, g, 1), u, 2)
    got = act.cpu().numpy()
    assert np.abs(got - want).max() <= 2e-5 * np.abs(want).max()


def test_head_bf16_matches_oracle_and_flags_nonfinite(lib, oracle, torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(41)
    rows, cols = 4099, 3072
    w = bf16_round((rng.standard_normal((rows, cols)) * 0.02).astype(np.float32))
    w16 = (w.view(np.uint32) >> 16).astype(np.uint16)
    x = (rng.standard_normal(cols) * 5).astype(np.float32)
    gain = (0.5 + rng.random(cols)).astype(np.float32)
    logits = torch.empty(rows, dtype=torch.float32, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    d_w = dev(torch, w16.view(np.int16))
    assert lib.lunelette_cuda_head_bf16(ptr(d_w), rows, cols, ptr(dev(torch, x)), ptr(dev(torch, gain)),
                                        ptr(logits), ptr(flag), stream(torch)) == 0
    normed = oracle.norm(gain, x[None])
    want = oracle.project(w, normed)[0]
    got = logits.cpu().numpy()
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()
    assert flag.item() == 0
    w16[1234, 17] = 0x7FC0  # NaN weight -> NaN logit
    d_w = dev(torch, w16.view(np.int16))
    assert lib.lunelette_cuda_head_bf16(ptr(d_w), rows, cols, ptr(dev(torch, x)), ptr(dev(torch, gain)),
                                        ptr(logits), ptr(flag), stream(torch)) == 0
    assert flag.item() == 1
    assert np.isnan(logits.cpu().numpy()[1234])


def write_pool(k_rows, v_rows, page_table, num_pages, layer, layers):
    """Lay FP32 K/V rows [positions][1024] into the paged FP32 pool layout."""
    pool = np.zeros((layers, num_pages, 2, 8, 64, 128), np.float32)
    for p in range(k_rows.shape[0]):
        page = page_table[p // 64]
        pool[layer, page, 0, :, p % 64, :] = k_rows[p].reshape(8, 128)
        pool[layer, page, 1, :, p % 64, :] = v_rows[p].reshape(8, 128)
    return pool.reshape(-1)


def run_attention(lib, torch, q, pool, page_table, num_pages, layer, length, count, slots=8192):
    out = torch.empty((count, 4096), dtype=torch.float32, device="cuda")
    acc = torch.empty(slots * 128, dtype=torch.float32, device="cuda")
    ml = torch.empty(slots * 2, dtype=torch.float32, device="cuda")
    rc = lib.lunelette_cuda_attention(ptr(dev(torch, q)), ptr(dev(torch, pool)),
                                      ptr(dev(torch, page_table)), num_pages, layer, length, count,
                                      ptr(out), ptr(acc), ptr(ml), slots, stream(torch))
    assert rc == 0
    return out.cpu().numpy()


def test_attention_prefix_matches_reference_expectation(lib, oracle, torch_cuda):
    # tests/test_metal.m:532-578 inputs
    torch = torch_cuda
    count, prefix = 2, 3
    total = count + prefix
    q = (((np.arange(count * 4096) % 11) - 5) * 0.03125).astype(np.float32).reshape(count, 4096)
    k = (((np.arange(total * 1024) % 17) - 8) * 0.03125).astype(np.float32).reshape(total, 1024)
    v = (((np.arange(total * 1024) % 23) - 11) * 0.0625).astype(np.float32).reshape(total, 1024)
    table = np.array([0], np.int32)
    pool = write_pool(k, v, table, 1, 0, 1)
    got = run_attention(lib, torch, q, pool, table, 1, 0, prefix, count)
    want = oracle.attention(q, k, v, prefix)
    assert np.abs(got - want).max() < 2e-6


def test_attention_long_causal_sentinel(lib, torch_cuda):
    # tests/test_metal.m:956-997 at C = 4352: row 0 masks the last value row, row 1 includes it
    torch = torch_cuda
    total, count = 4352, 2
    num_pages = total // 64
    table = np.arange(num_pages, dtype=np.int32)[::-1].copy()
    k = np.zeros((total, 1024), np.float32)
    v = np.ones((total, 1024), np.float32)
    v[total - 1] = 4352.0
    pool = write_pool(k, v, table, num_pages, 0, 1)
    got = run_attention(lib, torch, np.zeros((count, 4096), np.float32), pool, table, num_pages, 0,
                        total - count, count)
    assert np.abs(got[0] - 1.0).max() < 2e-4
    assert np.abs(got[1] - 8703.0 / 4352).max() < 2e-4


@pytest.mark.parametrize("length,count,slots", [(0, 1, 8192), (255, 1, 8192), (300, 1, 8192),
                                                (4351, 1, 8192), (100, 37, 8192), (0, 256, 8192),
                                                (1000, 5, 160), (2000, 3, 96), (4000, 64, 16384),
                                                (4096, 256, 65536), (63, 65, 8192)])
def test_attention_random_matches_oracle(lib, oracle, torch_cuda, length, count, slots):
    torch = torch_cuda
    rng = np.random.default_rng(length * 3 + count)
    total = length + count
    num_pages = (total + 63) // 64 + 1
    table = rng.permutation(num_pages).astype(np.int32)
    k = rng.standard_normal((total, 1024)).astype(np.float32)
    v = rng.standard_normal((total, 1024)).astype(np.float32)
    q = rng.standard_normal((count, 4096)).astype(np.float32)
    layer = 2
    pool = write_pool(k, v, table, num_pages, layer, 3)
    got = run_attention(lib, torch, q, pool, table, num_pages, layer, length, count, slots)
    want = oracle.attention(q, k, v, length)
    assert np.abs(got - want).max() < 1e-5 * max(1.0, np.abs(want).max())


def test_attention_block_ignores_stale_pool_rows(lib, oracle, torch_cuda):
    """Blocks of tokens (the tensor-core kernel) copy whole pages of the pool:
    slots past the sequence's last position and every other page hold NaN here
    (stale or never-written rows) and must not reach the output, whose key
    ranges end inside a page and are split across CTAs."""
    torch = torch_cuda
    rng = np.random.default_rng(77)
    for length, count in ((150, 40), (1200, 90)):
        total = length + count
        num_pages = (total + 63) // 64 + 2
        table = rng.permutation(num_pages).astype(np.int32)
        k = rng.standard_normal((total, 1024)).astype(np.float32)
        v = rng.standard_normal((total, 1024)).astype(np.float32)
        q = rng.standard_normal((count, 4096)).astype(np.float32)
        pool = np.full((2, num_pages, 2, 8, 64, 128), np.nan, np.float32)
        for pos in range(total):
            page = table[pos // 64]
            pool[1, page, 0, :, pos % 64, :] = k[pos].reshape(8, 128)
            pool[1, page, 1, :, pos % 64, :] = v[pos].reshape(8, 128)
        got = run_attention(lib, torch, q, pool.reshape(-1), table, num_pages, 1, length, count)
        want = oracle.attention(q, k, v, length)
        assert np.all(np.isfinite(got)), (length, count)
        assert np.abs(got - want).max() < 1e-5 * max(1.0, np.abs(want).max()), (length, count)


def test_kv_copy_fork_pages_bit_exact(lib, torch_cuda):
    """KV prefix reuse: a forked sequence copies pages of the pool. Full pages
    move whole; the last pair moves only its first last_slots positions; every
    other page and layer is untouched."""
    torch = torch_cuda
    layers, num_pages = 26, 9
    rng = np.random.default_rng(41)
    pool = rng.standard_normal(layers * num_pages * 2 * 8 * 64 * 128).astype(np.float32)
    src = np.array([4, 7, 2], np.int32)   # the source sequence's pages (positions 0..63, 64..127, 128..)
    dst = np.array([1, 8, 5], np.int32)   # the forked sequence's own pages
    last = 23                              # the prefix ends at position 128 + 23
    d_pool = dev(torch, pool)
    assert lib.lunelette_cuda_kv_copy(ptr(d_pool), num_pages, layers, ptr(dev(torch, src)), ptr(dev(torch, dst)),
                                      3, last, stream(torch)) == 0
    got = d_pool.cpu().numpy().reshape(layers, num_pages, 2, 8, 64, 128)
    want = pool.reshape(layers, num_pages, 2, 8, 64, 128).copy()
    for i, (a, b) in enumerate(zip(src, dst)):
        n = last if i == 2 else 64
        want[:, b, :, :, :n] = want[:, a, :, :, :n]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # argument checks
    assert lib.lunelette_cuda_kv_copy(ptr(d_pool), num_pages, layers, ptr(dev(torch, src)), ptr(dev(torch, dst)),
                                      3, 65, stream(torch)) == -1
    assert lib.lunelette_cuda_kv_copy(ptr(d_pool), num_pages, layers, ptr(dev(torch, src)), ptr(dev(torch, dst)),
                                      0, 5, stream(torch)) == -1
