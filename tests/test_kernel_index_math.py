"""CPU restatements of the index arithmetic of the kernels, checked against
the dense operation they implement (no GPU): the persistent decode kernel's
down slices (one 4-D tensor copy gathers 24 tile pieces of a 64-column slice,
paired into m16n8k16 A tiles), the batched head's column order (A fragments
read straight from row-major BF16 rows, B rows staged in the same order), the
split attention's warp reduce-scatter (lane l ends with the sum of index l),
the small-block tcgen05 GEMM's converter reads and joint hi|lo operand, and
the tcgen05 block attention's swizzled K and V^T operand tiles.
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


def sw128_offset(r, k):
    """Byte offset of FP16 element (row r, k < 64) in a K-major 128-byte-swizzle
    tile (8-row atoms of 1024 bytes): the operand layout of the tcgen05 kernels."""
    return (r >> 3) * 1024 + (r & 7) * 128 + ((((k >> 3) ^ (r & 7)) & 7) << 4) + (k & 7) * 2


def test_small_block_gemm_converters_rebuild_each_weight_row():
    """prefill_gemm_tmem.cuh: a stage is one 512-byte piece (8 rows x 64
    columns) of each of 16 tiles; thread r reads its row's four 16-byte chunks
    starting at chunk (lane >> 1) & 3, undoes the rotation and stores words
    a[8 j + c] (columns 16 j + 2 c + {0, 1}) and a[8 j + c + 4] (+ {8, 9}) into
    tensor-memory columns 0..31, column m holding K elements 2 m and 2 m + 1."""
    rng = np.random.default_rng(8)
    rows, cols = 128, 3072
    codes = rng.integers(0, 256, (rows, cols), dtype=np.uint8)
    tiled = tile_reference(codes)
    nb = cols // 128
    for chunk in (0, 5, 47):
        stage = np.concatenate([tiled[t * nb * 1024 + chunk * 512: t * nb * 1024 + chunk * 512 + 512]
                                for t in range(16)])
        for r in range(rows):
            lane = r & 31
            rot = (lane >> 1) & 3
            base = (r >> 3) * 512 + (r & 7) * 64
            reads = [stage[base + 16 * ((k + rot) & 3): base + 16 * ((k + rot) & 3) + 16] for k in range(4)]
            cols_of_word = np.zeros(32 * 2, np.uint8)  # TMEM column m -> K elements 2m, 2m+1
            for c in range(4):
                chunk_bytes = reads[(c - rot) & 3]
                for j in range(4):
                    word = chunk_bytes[4 * j: 4 * j + 4]
                    for half, m in ((0, 8 * j + c), (1, 8 * j + c + 4)):
                        cols_of_word[2 * m: 2 * m + 2] = word[2 * half: 2 * half + 2]
            assert np.array_equal(cols_of_word, codes[r, 64 * chunk: 64 * chunk + 64]), (chunk, r)


def test_small_block_gemm_hi_and_lo_tiles_form_one_operand():
    """One MMA per k-step reads B rows 0..n-1 from the hi tile and n..2n-1 from
    the lo tile copied right after it (n a multiple of 16): row n + r of the
    joint operand is row r of the lo part."""
    for n in (16, 32, 48, 64):
        nbytes = n // 8 * 1024
        for r in range(n):
            for k in (0, 7, 8, 33, 63):
                assert sw128_offset(n + r, k) == nbytes + sw128_offset(r, k)


def test_tc_attention_operand_tiles_cover_their_buffers_once():
    """attention_tc.cuh converters: K unit g = (key g >> 4, dims 8 (g & 15) ..)
    goes to chunk (g & 15) >> 3 (8 KB each) at sw128_offset(key, 8 (g & 7));
    V^T unit (dim d, keys 8 kg ..) to sw128_offset(d, 8 kg). Every FP16 element
    of the 16 KB parts is written exactly once, where the K-major swizzled
    layout puts element (row, k)."""
    k_seen = np.zeros(16384, np.int32)
    for ct in range(64):
        for it in range(16):
            g = ct + 64 * it
            key, grp = g >> 4, g & 15
            off = (grp >> 3) * 8192 + sw128_offset(key, (grp & 7) * 8)
            for e in range(8):
                dim = 8 * grp + e
                assert off + 2 * e == (dim // 64) * 8192 + sw128_offset(key, dim % 64)
                k_seen[off + 2 * e: off + 2 * e + 2] += 1
    assert np.all(k_seen == 1)
    v_seen = np.zeros(16384, np.int32)
    for ct in range(64):
        for it in range(16):
            d, kg = ct + 64 * (it & 1), it >> 1
            off = sw128_offset(d, 8 * kg)
            for e in range(8):
                assert off + 2 * e == sw128_offset(d, 8 * kg + e)
                v_seen[off + 2 * e: off + 2 * e + 2] += 1
    assert np.all(v_seen == 1)


def bf16_bits(v):
    """Round-to-nearest-even FP32 -> BF16 bit patterns (finite inputs)."""
    u = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_value(bits):
    return (np.asarray(bits, np.uint32) << 16).view(np.float32)


def test_tcgen05_head_operands_and_epilogue_give_the_tied_head():
    """head_tc.cuh on two CTAs of 128 vocabulary rows: the split kernel's B rows
    2 t (hi) and 2 t + 1 (lo) at head_tc_b_offset, one 16 KB tile per 64-column
    chunk; the embedding tile as the 2-D tensor copy lands it with the 128-byte
    swizzle (box row r at 128 r bytes, 16-byte chunk j moved to j ^ (r % 8));
    the MMA's K-major swizzled reads (four K = 16 steps per chunk at start
    offsets 32 k); and the epilogue's column 32 cb + 2 j (+ 1) = token
    16 cb + j, hi (lo). The result is E times (hi + lo) for every token below
    count, whatever the stale B rows of the other tokens hold."""
    rng = np.random.default_rng(21)
    rows, hidden, n_rows, chunk = 256, 3072, 128, 64
    count = 37
    emb = bf16_bits(rng.standard_normal((rows, hidden)).astype(np.float32) * 0.02)
    v = rng.standard_normal((64, hidden)).astype(np.float32)
    hi = bf16_bits(v)
    lo = bf16_bits(v - bf16_value(hi))
    # B operand: rows 2 t and 2 t + 1, tokens >= count zeroed by the split kernel
    b_rows = np.zeros((n_rows, hidden), np.uint16)
    b_rows[0:2 * count:2] = hi[:count]
    b_rows[1:2 * count:2] = lo[:count]
    xb = np.zeros(hidden // chunk * 16384 // 2, np.uint16)
    cols = np.arange(hidden)
    for n in range(n_rows):
        off = (cols // chunk) * 16384 + sw128_offset(n, cols % chunk)
        xb[off // 2] = b_rows[n]
    k = np.arange(chunk)
    r = np.arange(n_rows)[:, None]
    read_idx = sw128_offset(r, k[None, :]) // 2  # the MMA's K-major swizzled reads
    logits = np.zeros((count, rows))
    for cta in range(rows // n_rows):
        row0 = cta * n_rows
        acc = np.zeros((n_rows, n_rows))
        for c in range(hidden // chunk):
            box = emb[row0:row0 + n_rows, c * chunk:(c + 1) * chunk]
            tile_a = np.zeros(8192, np.uint16)
            for rr in range(n_rows):
                for j in range(8):
                    dst = rr * 64 + ((j ^ (rr % 8)) * 8)
                    tile_a[dst:dst + 8] = box[rr, 8 * j:8 * j + 8]
            tile_b = xb[c * 8192:(c + 1) * 8192]
            for ks in range(chunk // 16):
                a = bf16_value(tile_a[read_idx[:, 16 * ks:16 * ks + 16]]).astype(np.float64)
                b = bf16_value(tile_b[read_idx[:, 16 * ks:16 * ks + 16]]).astype(np.float64)
                acc += a @ b.T
        for q in range(4):
            for lane in range(32):
                m = 32 * q + lane
                for cb in range(4):
                    if 16 * cb >= count:
                        break
                    for j in range(16):
                        tok = 16 * cb + j
                        if tok < count:
                            logits[tok, row0 + m] = acc[m, 32 * cb + 2 * j] + acc[m, 32 * cb + 2 * j + 1]
    want = (bf16_value(hi[:count]).astype(np.float64) + bf16_value(lo[:count]).astype(np.float64)) @ \
        bf16_value(emb).astype(np.float64).T
    assert np.allclose(logits, want, rtol=1e-12, atol=1e-12)
