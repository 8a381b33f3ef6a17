"""Numpy restatement of the device's tiled FP8 weight layout (gemv.cuh) and of
the row orders the upload applies, used to prepare kernel inputs and to check
the tile kernel byte for byte.

Byte ((T * NB + kb) * 1024 + h * 512 + (g * 4 + t4) * 16 + j * 4 + i) of the
tiled matrix holds storage row 8T + g and column
128kb + 64h + 16j + 2t4 + (i & 1) + 8(i >> 1); rows pad to 8 and columns to 128
with zeros.
"""
import numpy as np

ORDER_ROWS, ORDER_ROPE_PAIRS, ORDER_INTERLEAVE = 0, 1, 2


def storage_rows(rows, order):
    """Storage row of every source row under `order` (whole-matrix form)."""
    r = np.arange(rows)
    if order == ORDER_ROPE_PAIRS:
        j = r % 128
        return (r - j) + np.where(j < 64, 2 * j, 2 * (j - 64) + 1)
    if order == ORDER_INTERLEAVE:
        half = rows // 2
        return np.where(r < half, 2 * r, 2 * (r - half) + 1)
    return r


def tiled_bytes(rows, cols):
    return -(-rows // 8) * 8 * (-(-cols // 128) * 128)


def tile_reference(codes, order=ORDER_ROWS):
    """Row-major uint8 [rows][cols] -> flat uint8 tiled buffer."""
    rows, cols = codes.shape
    R, C = -(-rows // 8) * 8, -(-cols // 128) * 128
    S = np.zeros((R, C), np.uint8)
    S[storage_rows(rows, order), :cols] = codes
    T, NB = R // 8, C // 128
    A = S.reshape(T, 8, NB, 2, 4, 16)  # tile, g, kb, h, j, w
    w_of = np.array([[2 * t4 + (i & 1) + 8 * (i >> 1) for i in range(4)] for t4 in range(4)])
    B = A[..., w_of]  # tile, g, kb, h, j, t4, i
    return np.ascontiguousarray(B.transpose(0, 2, 3, 1, 5, 4, 6)).reshape(-1)
