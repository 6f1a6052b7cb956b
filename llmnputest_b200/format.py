"""The q4nx container: constants, header parsing and the reader.

Drop-in for the reference's tools/q4nx.py (same names and return types), with
the decode work on the GPU: `Q4NX.tensor()` and `dequant_q4`/`dequant_q8` run
the bit-exact device decode kernels (b2_*_dequant_*), and `device_tiles()`
uploads a tensor's raw tiles once so the GEMV kernels can stream them as
stored.

File layout (tools/q4nx.py:1-33): a safetensors file -- u64 little-endian
header length, JSON header {name: {dtype, shape, data_offsets}}, data.  Tiled
weights are dtype "I8" with shape [n_t, k_t, tile_bytes] (Qwen3.5 files) or
[n_t*k_t, tile_bytes] (granite files); in the second form (N, K) must come from
the model config, since e.g. gate_proj and down_proj share a stored shape
(designs/granite_gemv/granite_gemv.py:11-16, 282-289).
"""

from __future__ import annotations

import json
import struct
from pathlib import Path
from typing import BinaryIO

import numpy as np
from ml_dtypes import bfloat16

GROUP = 32
TILE_ROWS = 32
TILE_K = 256
ROW_BLOCK = 16
N_META = TILE_ROWS * (TILE_K // GROUP)  # 256
N_WEIGHTS = TILE_ROWS * TILE_K  # 8192
Q4_TILE_BYTES = 2 * 2 * N_META + N_WEIGHTS // 2  # 5120
Q8_TILE_BYTES = 2 * N_META + N_WEIGHTS  # 8704
LOW_NIBBLE_IS_EVEN = True  # tools/q4nx.py:56 (settled against the upstream checkpoint)


def read_header(f: BinaryIO) -> dict:
    """The safetensors JSON header; reads nothing past it."""
    raw = f.read(8)
    if len(raw) != 8:
        raise ValueError("truncated q4nx header")
    (n,) = struct.unpack("<Q", raw)
    return json.loads(f.read(n))


def meta_index() -> np.ndarray:
    """Scale-plane entry of each weight-index position: (k//32)*32 + rb*16 + r."""
    i = np.arange(N_WEIGHTS)
    return ((i >> 4) & 255) // GROUP * TILE_ROWS + (i >> 12) * ROW_BLOCK + (i & 15)


def unpack_nibbles(nib: np.ndarray) -> np.ndarray:
    """uint8[4096] -> codes uint8[8192] in weight-index order (low nibble = even index)."""
    nib = np.asarray(nib, np.uint8)
    out = np.empty(nib.size * 2, np.uint8)
    out[0::2] = nib & 0x0F
    out[1::2] = nib >> 4
    return out


def split_q4_tile(raw: bytes) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """5120-byte q4 tile -> (nibbles uint8[4096], d bf16[256], m bf16[256])."""
    if len(raw) != Q4_TILE_BYTES:
        raise ValueError(f"{len(raw)} bytes, expected a {Q4_TILE_BYTES} B q4 tile")
    b = np.frombuffer(raw, np.uint8)
    return b[1024:].copy(), b[:512].copy().view(bfloat16), b[512:1024].copy().view(bfloat16)


def pack_meta(d: np.ndarray, m: np.ndarray) -> np.ndarray:
    return np.concatenate([np.asarray(d), np.asarray(m)]).astype(bfloat16)


def to_matrix(flat: np.ndarray) -> np.ndarray:
    """Weight-index order -> [32 rows][256 k]."""
    return np.asarray(flat).reshape(2, TILE_K, ROW_BLOCK).swapaxes(1, 2).reshape(TILE_ROWS, TILE_K)


def _device():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("q4nx decode runs on the GPU; no CUDA device is available (no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


def _decode_tiles_bf16(tile_bytes: bytes, q8: bool) -> np.ndarray:
    import torch
    from . import ops
    t = torch.frombuffer(bytearray(tile_bytes), dtype=torch.uint8).to(_device())
    out = ops.dequant_tiles(t, q8=q8)
    return out.view(torch.int16).cpu().numpy().view(np.uint16).view(bfloat16).reshape(-1)


def dequant_q4(nib: np.ndarray, d: np.ndarray, m: np.ndarray) -> np.ndarray:
    """One q4 tile's weights as bf16[8192], RNE(code*d + m), decoded on the GPU."""
    raw = (np.asarray(d).astype(bfloat16).view(np.uint8).tobytes()
           + np.asarray(m).astype(bfloat16).view(np.uint8).tobytes()
           + np.asarray(nib, np.uint8).tobytes())
    return _decode_tiles_bf16(raw, q8=False)


def dequant_q8(raw: bytes) -> np.ndarray:
    """One 8704-byte q8 tile as bf16[8192], decoded on the GPU."""
    if len(raw) != Q8_TILE_BYTES:
        raise ValueError(f"{len(raw)} bytes, expected a {Q8_TILE_BYTES} B q8 tile")
    return _decode_tiles_bf16(bytes(raw), q8=True)


def upload_segments(segs: list[np.ndarray], device=None, chunk_bytes: int = 32 << 20):
    """Concatenate uint8 host arrays into one device tensor through pinned staging.

    Two pinned buffers alternate: while the DMA of chunk i runs on a side stream the
    host fills the other buffer with chunk i + 1 (from page cache or disk when the
    segments are views of a mapped file).  The call returns once the copies are done
    (the staging buffers are released with it).
    """
    import torch
    dev = torch.device(device) if device is not None else _device()
    total = sum(int(s.size) for s in segs)
    out = torch.empty(total, dtype=torch.uint8, device=dev)
    if dev.type != "cuda":
        o = out.numpy()
        off = 0
        for s in segs:
            o[off:off + s.size] = s
            off += s.size
        return out
    if total == 0:
        return out
    chunk = max(1, min(int(chunk_bytes), total))
    stage = [torch.empty(chunk, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
    done = [torch.cuda.Event(), torch.cuda.Event()]
    used = [False, False]
    cs = torch.cuda.Stream(dev)
    cs.wait_stream(torch.cuda.current_stream(dev))  # `out` was allocated on the current stream
    i = 0
    dst = 0
    pieces = iter(segs)
    cur, pos = next(pieces), 0
    while dst < total:
        b = i & 1
        if used[b]:
            done[b].synchronize()  # the DMA that last read this buffer has finished
        buf = stage[b].numpy()
        fill = 0
        while fill < chunk and dst + fill < total:  # gather the next chunk from the segments
            if pos == cur.size:
                cur, pos = next(pieces), 0
                continue
            m = min(chunk - fill, cur.size - pos)
            buf[fill:fill + m] = cur[pos:pos + m]
            fill += m
            pos += m
        with torch.cuda.stream(cs):
            out[dst:dst + fill].copy_(stage[b][:fill], non_blocking=True)
            done[b].record(cs)
        used[b] = True
        dst += fill
        i += 1
    cs.synchronize()
    out.record_stream(cs)
    return out


class Q4NX:
    """A .q4nx model file (tools/q4nx.py:152-197 interface)."""

    _DT = {"BF16": bfloat16, "F32": np.float32, "F16": np.float16, "I8": np.int8}

    def __init__(self, path):
        self.path = Path(path)
        with self.path.open("rb") as f:
            self.header = read_header(f)
            self._data_start = f.tell()
        self.header.pop("__metadata__", None)
        self._mm = None

    def __contains__(self, name: str) -> bool:
        return name in self.header

    def names(self) -> list[str]:
        return sorted(self.header)

    def raw(self, name: str) -> bytes:
        first, last = self.header[name]["data_offsets"]
        with self.path.open("rb") as f:
            f.seek(self._data_start + first)
            return f.read(last - first)

    def tiled_shape(self, name: str, n: int | None = None, k: int | None = None) -> tuple[int, int, int]:
        """(n_tile_rows, k_tiles, tile_bytes) of a tiled weight.

        A 2-D stored shape [n_t*k_t, bytes] does not determine the factoring, so
        the logical N (or K) must be given; it is then checked against the file.
        """
        e = self.header[name]
        if e["dtype"] != "I8":
            raise ValueError(f"{name} is {e['dtype']}, not a tiled weight")
        shape = e["shape"]
        if len(shape) == 3:
            n_t, k_t, tb = shape
        elif len(shape) == 2:
            tiles, tb = shape
            if n is None and k is None:
                raise ValueError(f"{name}: stored as {shape}; pass the logical N or K")
            n_t = -(-n // TILE_ROWS) if n is not None else tiles // -(-k // TILE_K)
            k_t = tiles // n_t
            if n_t * k_t != tiles:
                raise ValueError(f"{name}: N={n} K={k} does not factor the stored {shape}")
        else:
            raise ValueError(f"{name}: unexpected tiled shape {shape}")
        if tb not in (Q4_TILE_BYTES, Q8_TILE_BYTES):
            raise ValueError(f"{name}: {tb} B/tile is neither q4 nor q8")
        if k is not None and k_t != -(-k // TILE_K):
            raise ValueError(f"{name}: K={k} but the file holds {k_t} K-tiles")
        return int(n_t), int(k_t), int(tb)

    def raw_view(self, name: str) -> np.ndarray:
        """The tensor's bytes as a read-only uint8 view of the file (mmap, no copy)."""
        if self._mm is None:
            self._mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        first, last = self.header[name]["data_offsets"]
        return self._mm[self._data_start + first:self._data_start + last]

    def tile_segments(self, name: str, tile_rows=None, k_tiles=None, n: int | None = None,
                      k: int | None = None) -> list[np.ndarray]:
        """Contiguous pieces of a tiled weight's bytes, as stored, for a slice of it.

        tile_rows: the tile-rows to keep, in the order given (a TP shard's rows, e.g.
        `ShardPlan.qkv_tile_rows()`), default all; k_tiles: (k0, k1), the K-tiles to
        keep of each row (a K shard, whole 256-wide tiles), default all.  The slice of
        a [n_t][k_t][tile] weight is itself [rows][k1 - k0][tile].  n / k: the logical
        shape, needed when the stored shape is 2-D (see `tiled_shape`).
        """
        n_t, k_t, tb = self.tiled_shape(name, n, k)
        view = self.raw_view(name)
        rows = list(range(n_t)) if tile_rows is None else [int(r) for r in tile_rows]
        k0, k1 = (0, k_t) if k_tiles is None else (int(k_tiles[0]), int(k_tiles[1]))
        if not 0 <= k0 < k1 <= k_t:
            raise ValueError(f"{name}: K-tiles {k0}..{k1} outside 0..{k_t}")
        if not rows or min(rows) < 0 or max(rows) >= n_t:
            raise ValueError(f"{name}: tile-rows must lie in 0..{n_t - 1}")
        segs: list[np.ndarray] = []
        start = prev = None
        for r in rows + [None]:  # whole rows: merge consecutive ones into one piece
            if r is not None and prev is not None and r == prev + 1 and (k0, k1) == (0, k_t):
                prev = r
                continue
            if start is not None:
                segs.append(view[(start * k_t + k0) * tb:(prev * k_t + k1) * tb])
            start = prev = r
        return segs

    def device_tiles(self, name: str, device=None, *, tile_rows=None, k_tiles=None, n: int | None = None,
                     k: int | None = None, chunk_bytes: int = 32 << 20):
        """The tensor's raw tile bytes (or a slice of them, see `tile_segments`) as a
        resident uint8 tensor, uploaded once.

        The bytes go from the mmap of the file through two pinned staging buffers of
        `chunk_bytes`: the host copy of one chunk overlaps the DMA of the previous one
        on a side stream.  Returns once the data is on the device.
        """
        if tile_rows is None and k_tiles is None:
            segs = [self.raw_view(name)]
        else:
            segs = self.tile_segments(name, tile_rows, k_tiles, n, k)
        return upload_segments(segs, device, chunk_bytes)

    def device_tensor(self, name: str, shape: tuple[int, int] | None = None, device=None):
        """Dequantised, untiled float32 [N, K] CUDA tensor (decoded on the GPU)."""
        from . import ops
        n = shape[0] if shape is not None else None
        k = shape[1] if shape is not None else None
        n_t, k_t, tb = self.tiled_shape(name, n, k)
        w = ops.dequant_matrix(self.device_tiles(name, device), n_t, k_t, q8=(tb == Q8_TILE_BYTES))
        return w if shape is None else w[: shape[0], : shape[1]]

    def tensor(self, name: str, shape: tuple[int, int] | None = None) -> np.ndarray:
        """Dequantised and untiled (numpy float32 for tiled weights, as stored otherwise).

        `shape` trims the tile padding, as in tools/q4nx.py:175-197.
        """
        e = self.header[name]
        if e["dtype"] != "I8":
            return np.frombuffer(self.raw(name), dtype=self._DT[e["dtype"]]).reshape(e["shape"])
        return self.device_tensor(name, shape).cpu().numpy()
