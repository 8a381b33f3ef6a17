"""CPU restatements of the index arithmetic of three kernels, checked against
the dense operation they implement (no GPU): the persistent decode kernel's
down slices (one 4-D tensor copy gathers 24 tile pieces of a 64-column slice,
paired into m16n8k16 A tiles), the batched head's column order (A fragments
read straight from row-major BF16 rows, B rows staged in the same order), and
the split attention's warp reduce-scatter (lane l ends with the sum of index l).
"""
import numpy as np

from tests.tiling import tile_reference

HIDDEN, INNER, TILE_ROWS = 3072, 9216, 8
SLICES, ITEM_TILES = INNER // 64, 24


def fragment_columns():
    """Column (within a 64-column half block) of byte lane * 16 + j * 4 + e of a
    512-byte piece, and its row: the tiled layout of gemv.cuh."""
    lane = np.arange(32)[:, None, None]
    j = np.arange(4)[None, :, None]
    e = np.arange(4)[None, None, :]
    col = 16 * j + 2 * (lane & 3) + (e & 1) + 8 * (e >> 1)
    row = np.broadcast_to(lane >> 2, col.shape)
    return row.reshape(-1), col.reshape(-1)


def down_item(tiled, s, i):
    """The box {256 x u16, 1, 24, 1} at {0, s, 24 i, layer 0} of the down tensor
    map: dims {256, 144, 384, layers}, byte strides {512, 72 * 1024, ...}."""
    tile_stride = (INNER // 128) * 1024
    return np.concatenate([tiled[(ITEM_TILES * i + k) * tile_stride + s * 512:
                                 (ITEM_TILES * i + k) * tile_stride + s * 512 + 512]
                           for k in range(ITEM_TILES)])


def test_down_slice_items_hold_the_slice_columns_of_consecutive_rows():
    rng = np.random.default_rng(5)
    codes = rng.integers(0, 256, (HIDDEN, INNER), dtype=np.uint8)
    tiled = tile_reference(codes)
    row_of, col_of = fragment_columns()
    for s in (0, 1, 77, SLICES - 1):
        for i in (0, 9, HIDDEN // TILE_ROWS // ITEM_TILES - 1):
            item = down_item(tiled, s, i).reshape(ITEM_TILES, 512)
            for k in range(ITEM_TILES):
                got = np.zeros((TILE_ROWS, 64), np.uint8)
                got[row_of, col_of] = item[k]
                r0 = TILE_ROWS * (ITEM_TILES * i + k)
                assert np.array_equal(got, codes[r0:r0 + TILE_ROWS, 64 * s:64 * s + 64])


def test_down_pair_mma_is_the_row_dot_over_the_slice():
    """Pieces 2q and 2q + 1 are the A rows g and g + 8 of one m16n8k16 tile;
    k step j of lane (g, t4) takes columns 16 j + 2 t4 + {0, 1} (a0, a1) and
    + {8, 9} (a2, a3); B column 0 holds the same columns of the act slice."""
    rng = np.random.default_rng(6)
    w = rng.standard_normal((16, 64))
    act = rng.standard_normal(64)
    # the piece bytes of rows 0-7 and 8-15 in fragment order
    row_of, col_of = fragment_columns()
    wa, wb = w[:8][row_of, col_of].reshape(32, 4, 4), w[8:][row_of, col_of].reshape(32, 4, 4)
    d = np.zeros(16)
    for lane in range(32):
        g, t4 = lane >> 2, lane & 3
        for j in range(4):
            cols = [16 * j + 2 * t4, 16 * j + 2 * t4 + 1, 16 * j + 2 * t4 + 8, 16 * j + 2 * t4 + 9]
            d[g] += np.dot(wa[lane, j], act[cols])
            d[g + 8] += np.dot(wb[lane, j], act[cols])
    assert np.allclose(d, w @ act)


def test_head_fragment_column_order_pairs_the_same_columns():
    """Lane (g, t4) holds columns 16 t4 .. 16 t4 + 15 of rows g and g + 8; k step
    s uses its pairs 2 s (logical k = 2 t4, +1) and 2 s + 1 (2 t4 + 8, +9); the
    staged B row of column n is read with the same pairs."""
    rng = np.random.default_rng(7)
    a = rng.standard_normal((16, 64))   # 16 vocabulary rows, one 64-column chunk
    b = rng.standard_normal((8, 64))    # 8 B columns (token, part)
    d = np.zeros((16, 8))
    for s in range(4):
        for lane in range(32):
            g, t4 = lane >> 2, lane & 3
            base = 16 * t4
            a_lo, a_hi = [base + 4 * s, base + 4 * s + 1], [base + 4 * s + 2, base + 4 * s + 3]
            for n in range(8):
                # lane (n, t4) supplies B column n: b0 = pair 2 s, b1 = pair 2 s + 1 of its row
                for r in (g, g + 8):
                    d[r, n] += np.dot(a[r, a_lo], b[n, a_lo]) + np.dot(a[r, a_hi], b[n, a_hi])
    assert np.allclose(d, a @ b.T)


def test_reduce_scatter_leaves_lane_l_with_index_l():
    """attention_split_kernel: 32 partial values per lane; rounds of width
    16, 8, 4, 2, 1 keep the half selected by the lane's bit and add the
    partner's other half."""
    rng = np.random.default_rng(8)
    vals = rng.standard_normal((32, 32))   # [lane][index]
    d = [list(vals[lane]) for lane in range(32)]
    width = 16
    while width >= 1:
        new = []
        for lane in range(32):
            partner = lane ^ width
            upper = (lane & width) != 0
            row = []
            for i in range(width):
                # the partner sends the half it does not keep: the half this lane keeps
                mine = d[lane][i + width] if upper else d[lane][i]
                received = d[partner][i + width] if upper else d[partner][i]
                row.append(mine + received)
            new.append(row)
        d = new
        width //= 2
    assert np.allclose([d[lane][0] for lane in range(32)], vals.sum(axis=0))
