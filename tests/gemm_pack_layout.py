"""numpy statement of the packed tile layout of b2_q4_gemm_pack (a test helper).

The packed layout is this library's own (the reference reads the q4nx tiles as
stored, tools/q4nx.py:80-111): the same 5120 bytes per tile, reordered so that row l's
codes for the 32-k block s sit in 16 contiguous bytes; and the tiles of a weight
[n_tile_rows][k_tiles] reordered tile-row-pair-major: tile (tr, kt) at position
(tr//2)*2*k_tiles + kt*np + tr%2, np = 2 (1 for a last odd tile-row).
  bytes    0..1023  entry s*32 + l: bf16 d | bf16 m << 16 (row l, block s)
  bytes 1024..5119  at 1024 + (s*32 + l)*16: four little-endian words w; nibble i of
                    word w is the code of k = 32s + 8w + 2i (i < 4) or 32s + 8w + 2(i-4) + 1
"""

import numpy as np

from oracle import q4nx_oracle as orc


def _k_of_slot() -> np.ndarray:
    """[32] k (within the 32-k block) held by nibble slot 8w + i."""
    k = np.empty(32, np.int64)
    for w in range(4):
        for i in range(8):
            k[8 * w + i] = 8 * w + (2 * i if i < 4 else 2 * (i - 4) + 1)
    return k


def packed_position(tr: int, kt: int, n_tile_rows: int, k_tiles: int) -> int:
    pr = tr // 2
    np_ = 2 if n_tile_rows - 2 * pr >= 2 else 1
    return pr * 2 * k_tiles + kt * np_ + tr % 2


def pack(weight: np.ndarray, n_tile_rows: int, k_tiles: int) -> np.ndarray:
    """q4nx weight [n_tile_rows * k_tiles, 5120] (or flat) -> the packed weight."""
    t = pack_tiles(weight).reshape(-1, orc.Q4_TILE_BYTES)
    out = np.empty_like(t)
    for tr in range(n_tile_rows):
        for kt in range(k_tiles):
            out[packed_position(tr, kt, n_tile_rows, k_tiles)] = t[tr * k_tiles + kt]
    return out.reshape(np.asarray(weight).shape)


def pack_tiles(tiles: np.ndarray) -> np.ndarray:
    """Each q4nx tile [n, 5120] (or flat) -> its packed tile, in the same order."""
    t = np.ascontiguousarray(tiles, dtype=np.uint8).reshape(-1, orc.Q4_TILE_BYTES)
    n = t.shape[0]
    d = t[:, 0:512].view(np.uint16).reshape(n, 8, 32)       # [tile][block s][row l]
    m = t[:, 512:1024].view(np.uint16).reshape(n, 8, 32)
    codes = orc.q4_codes(t[:, 1024:])                        # [tile][8192] by weight index
    # weight index rb*4096 + k*16 + r  ->  [row = rb*16 + r][k]
    c = codes.reshape(n, 2, 256, 16).transpose(0, 1, 3, 2).reshape(n, 32, 256)
    out = np.empty_like(t)
    sc = (d.astype(np.uint32) | (m.astype(np.uint32) << 16))  # [n][s][l]
    out[:, 0:1024] = sc.reshape(n, 256).view(np.uint8).reshape(n, 1024)
    ks = _k_of_slot()
    blk = c.reshape(n, 32, 8, 32).transpose(0, 2, 1, 3)      # [n][s][l][k in block]
    slots = blk[..., ks].astype(np.uint32).reshape(n, 8, 32, 4, 8)  # [n][s][l][w][i]
    words = np.zeros((n, 8, 32, 4), np.uint32)
    for i in range(8):
        words |= slots[..., i] << np.uint32(4 * i)
    out[:, 1024:] = words.reshape(n, 8 * 32 * 4).view(np.uint8).reshape(n, 4096)
    return out.reshape(tiles.shape)


def dequant_packed(packed: np.ndarray) -> np.ndarray:
    """Packed tiles -> float32 [n, 32 rows, 256 k], code*d + m (tools/q4nx.py:97-111)."""
    p = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1, orc.Q4_TILE_BYTES)
    n = p.shape[0]
    sc = p[:, 0:1024].view(np.uint32).reshape(n, 8, 32)
    d = (sc & 0xFFFF).astype(np.uint16).view(orc.bfloat16).astype(np.float32)
    m = (sc >> 16).astype(np.uint16).view(orc.bfloat16).astype(np.float32)
    words = p[:, 1024:].view(np.uint32).reshape(n, 8, 32, 4)
    ks = _k_of_slot()
    out = np.empty((n, 32, 256), np.float32)
    for s in range(8):
        for w in range(4):
            for i in range(8):
                code = ((words[:, s, :, w] >> np.uint32(4 * i)) & 0xF).astype(np.float32)  # [n][l]
                out[:, :, 32 * s + ks[8 * w + i]] = code * d[:, s, :] + m[:, s, :]
    return out


def pack8_tiles(tiles: np.ndarray) -> np.ndarray:
    """Each q8 tile [n, 8704] -> its packed tile: scales (s*32 + l)*2, then row l's 32 codes
    of block s at 512 + (s*32 + l)*32 in k order."""
    t = np.ascontiguousarray(tiles, dtype=np.uint8).reshape(-1, orc.Q8_TILE_BYTES)
    n = t.shape[0]
    out = np.empty_like(t)
    out[:, :512] = t[:, :512]  # entry (k/32)*32 + row is already [s][l]
    codes = t[:, 512:].reshape(n, 2, 256, 16).transpose(0, 1, 3, 2).reshape(n, 32, 256)  # [row][k]
    out[:, 512:] = codes.reshape(n, 32, 8, 32).transpose(0, 2, 1, 3).reshape(n, 8192)  # [s][l][j]
    return out.reshape(np.asarray(tiles).shape)


def pack8(weight: np.ndarray, n_tile_rows: int, k_tiles: int) -> np.ndarray:
    """q8 weight [n_tile_rows * k_tiles, 8704] -> the packed q8 weight (pair-major tiles)."""
    t = pack8_tiles(weight).reshape(-1, orc.Q8_TILE_BYTES)
    out = np.empty_like(t)
    for tr in range(n_tile_rows):
        for kt in range(k_tiles):
            out[packed_position(tr, kt, n_tile_rows, k_tiles)] = t[tr * k_tiles + kt]
    return out.reshape(np.asarray(weight).shape)


def dequant_packed8(packed: np.ndarray) -> np.ndarray:
    """Packed q8 tiles -> float32 [n, 32 rows, 256 k], code*scale (tools/q4nx.py:140-143)."""
    p = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1, orc.Q8_TILE_BYTES)
    n = p.shape[0]
    sc = p[:, :512].view(np.uint16).view(orc.bfloat16).astype(np.float32).reshape(n, 8, 32)  # [s][l]
    codes = p[:, 512:].view(np.int8).astype(np.float32).reshape(n, 8, 32, 32)  # [s][l][j]
    w = codes * sc[..., None]
    return w.transpose(0, 2, 1, 3).reshape(n, 32, 256)
