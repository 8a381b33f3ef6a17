"""The numpy restatement of the tiled weight layout (tests/tiling.py) against an
element-by-element reading of its definition, on CPU."""
import numpy as np
import pytest

from tests.tiling import ORDER_INTERLEAVE, ORDER_ROPE_PAIRS, ORDER_ROWS, storage_rows, tile_reference, tiled_bytes


def element_reference(codes, order):
    rows, cols = codes.shape
    out = np.zeros(tiled_bytes(rows, cols), np.uint8)
    nb = -(-cols // 128)
    srow = storage_rows(rows, order)
    for r in range(rows):
        s = int(srow[r])
        for c in range(cols):
            tile, g = s // 8, s % 8
            kb, h, w = c // 128, (c // 64) % 2, c % 64
            j, ww = w // 16, w % 16
            t4 = (ww % 8) // 2
            i = (ww & 1) | ((ww >> 3) << 1)
            out[(tile * nb + kb) * 1024 + h * 512 + (g * 4 + t4) * 16 + j * 4 + i] = codes[r, c]
    return out


@pytest.mark.parametrize("rows,cols,order", [(16, 64, ORDER_ROWS), (7, 16, ORDER_ROWS), (33, 112, ORDER_ROWS),
                                             (256, 64, ORDER_ROPE_PAIRS), (32, 128, ORDER_INTERLEAVE)])
def test_tile_reference_matches_definition(rows, cols, order):
    codes = np.random.default_rng(rows + cols).integers(0, 256, (rows, cols)).astype(np.uint8)
    assert np.array_equal(tile_reference(codes, order), element_reference(codes, order))


def test_storage_orders_are_permutations():
    assert sorted(storage_rows(6144, ORDER_ROPE_PAIRS)) == list(range(6144))
    assert sorted(storage_rows(18432, ORDER_INTERLEAVE)) == list(range(18432))
    s = storage_rows(256, ORDER_ROPE_PAIRS)
    assert s[0] == 0 and s[64] == 1 and s[1] == 2 and s[127] == 127 and s[128] == 128
    s = storage_rows(8, ORDER_INTERLEAVE)
    assert list(s) == [0, 2, 4, 6, 1, 3, 5, 7]
