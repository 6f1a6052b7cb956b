"""The packed tile layout of the tensor-core GEMM (b2_q4_gemm_pack), on the CPU: a
byte permutation of each q4nx tile whose dequantised values equal the oracle's."""

import numpy as np

from oracle import q4nx_oracle as orc
from tests import gemm_pack_layout as gpl


def test_pack_is_a_permutation_with_the_oracle_values():
    rng = np.random.default_rng(11)
    tiles = orc.synth_q4_tiles(rng, 6)
    packed = gpl.pack_tiles(tiles)
    assert packed.shape == tiles.shape
    # every byte of the scales survives; the code nibbles are the same multiset per tile
    assert np.array_equal(np.sort(packed[:, :1024].view(np.uint16), axis=1), np.sort(tiles[:, :1024].view(np.uint16), axis=1))
    assert np.array_equal(np.sort(orc.q4_codes(packed[:, 1024:]), axis=1), np.sort(orc.q4_codes(tiles[:, 1024:]), axis=1))
    # dequantised through the packed layout = the oracle's dequantisation of the q4nx tile
    # oracle weights in weight-index order rb*4096 + k*16 + r -> [row rb*16 + r][k]
    ref = orc.q4_tiles_f32(tiles).reshape(6, 2, 256, 16).transpose(0, 1, 3, 2).reshape(6, 32, 256)
    assert np.array_equal(gpl.dequant_packed(packed), ref)


def test_pack_places_known_codes():
    """One hand-placed code: row 19 (row-block 1, r 3), k 77 (block 2, word 1, slot 6)."""
    t = np.zeros((1, orc.Q4_TILE_BYTES), np.uint8)
    i = 1 * 4096 + 77 * 16 + 3          # weight index of (row 19, k 77)
    t[0, 1024 + i // 2] = 0x9 << (4 * (i & 1))
    p = gpl.pack_tiles(t)
    w = p[0, 1024:].view(np.uint32).reshape(8, 32, 4)
    # k 77 = 32*2 + 8*1 + 5: odd offset 5 = 2*(i-4)+1 -> i = 6
    assert w[2, 19, 1] == 0x9 << 24
    assert np.count_nonzero(w) == 1


def test_pack_orders_tiles_pair_major():
    """Tile (tr, kt) of a 5 x 3 weight lands at (tr//2)*6 + kt*np + tr%2 (np 1 for tile-row 4)."""
    n_t, k_t = 5, 3
    t = np.zeros((n_t * k_t, orc.Q4_TILE_BYTES), np.uint8)
    t[:, 0] = np.arange(n_t * k_t)  # d entry 0 (row 0, block 0) tags the tile
    p = gpl.pack(t, n_t, k_t)
    tags = p[:, 0]  # the tag moves to scale entry (0, 0) of the packed tile: byte 0
    want = {gpl.packed_position(tr, kt, n_t, k_t): tr * k_t + kt for tr in range(n_t) for kt in range(k_t)}
    assert sorted(want) == list(range(n_t * k_t))
    assert all(tags[pos] == src for pos, src in want.items())
    assert want[12] == 12 and want[13] == 13 and want[14] == 14  # the odd last tile-row keeps its K order


def test_pack8_is_a_permutation_with_the_oracle_values():
    rng = np.random.default_rng(12)
    tiles = orc.synth_q8_tiles(rng, 5)
    packed = gpl.pack8_tiles(tiles)
    assert np.array_equal(np.sort(packed, axis=1), np.sort(tiles, axis=1))
    ref = orc.q8_tiles_f32(tiles).reshape(5, 2, 256, 16).transpose(0, 1, 3, 2).reshape(5, 32, 256)
    assert np.array_equal(gpl.dequant_packed8(packed), ref)
    # one hand-placed code: row 21 (row-block 1, r 5), k 70 (block 2, byte 6)
    t = np.zeros((1, orc.Q8_TILE_BYTES), np.uint8)
    t[0, 512 + 1 * 4096 + 70 * 16 + 5] = 0x7B
    p = gpl.pack8_tiles(t)
    assert p[0, 512 + (2 * 32 + 21) * 32 + 6] == 0x7B and np.count_nonzero(p) == 1
