"""torch-facing wrappers of the C ABI: device tensors in, device tensors out.

Every function here checks dtype/device/contiguity and raises on anything the
kernels do not support -- there is no eager or CPU fallback.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native
from .format import Q4_TILE_BYTES, Q8_TILE_BYTES, TILE_K, TILE_ROWS

GEMV_ACCUMULATE = 1
GEMV_PREFETCH = 2
GEMM_PACKED = 4


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _need(t: torch.Tensor, name: str, dtype: torch.dtype) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU fallback)")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")


def _tiles(tiles: torch.Tensor, n_tile_rows: int, k_tiles: int, tile_bytes: int, name: str) -> None:
    _need(tiles, name, torch.uint8)
    if not tiles.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    want = n_tile_rows * k_tiles * tile_bytes
    if tiles.numel() != want:
        raise ValueError(f"{name}: {tiles.numel()} bytes, expected {n_tile_rows}x{k_tiles}x{tile_bytes} = {want}")


def _x2d(x: torch.Tensor, k: int) -> torch.Tensor:
    _need(x, "x", torch.bfloat16)
    x2 = x.reshape(1, -1) if x.dim() == 1 else x
    if x2.dim() != 2 or x2.shape[1] != k:
        raise ValueError(f"x must be [K] or [B, K] with K={k}, got {tuple(x.shape)}")
    if x2.stride(1) != 1 or x2.stride(0) % 8 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
        if k % 8:
            raise ValueError("K must be a multiple of 8")
    return x2


def _gemv(name: str, tiles, n_tile_rows, k_tiles, tile_bytes, x, out, accumulate, prefetch):
    _tiles(tiles, n_tile_rows, k_tiles, tile_bytes, "tiles")
    k, n = k_tiles * TILE_K, n_tile_rows * TILE_ROWS
    x2 = _x2d(x, k)
    b = x2.shape[0]
    if out is None:
        if accumulate:
            raise ValueError("accumulate=True needs out")
        out = torch.empty((b, n), dtype=torch.float32, device=x2.device)
    _need(out, "out", torch.float32)
    if out.dim() != 2 or out.shape[0] != b or out.shape[1] < n or out.stride(1) != 1:
        raise ValueError(f"out must be [B, >=N] row-major, got {tuple(out.shape)}")
    flags = (GEMV_ACCUMULATE if accumulate else 0) | (GEMV_PREFETCH if prefetch else 0)
    for b0 in range(0, b, 16):  # the kernel takes 16 tokens per weight pass
        bb = min(16, b - b0)
        _native.call(name, _ptr(tiles), n_tile_rows, k_tiles, ctypes.c_void_p(x2[b0].data_ptr()), bb,
                     x2.stride(0), ctypes.c_void_p(out[b0].data_ptr()), out.stride(0), flags, _stream())
    return out if x.dim() == 2 else out[0, :n]


def q4_gemv(tiles: torch.Tensor, n_tile_rows: int, k_tiles: int, x: torch.Tensor,
            out: torch.Tensor | None = None, accumulate: bool = False, prefetch: bool = False) -> torch.Tensor:
    """fp32 y = W x for a q4nx q4 weight (raw tiles as stored); x bf16 [K] or [B, K]."""
    return _gemv("b2_q4_gemv", tiles, n_tile_rows, k_tiles, Q4_TILE_BYTES, x, out, accumulate, prefetch)


def q8_gemv(tiles: torch.Tensor, n_tile_rows: int, k_tiles: int, x: torch.Tensor,
            out: torch.Tensor | None = None, accumulate: bool = False, prefetch: bool = False) -> torch.Tensor:
    """fp32 y = W x for a q4nx q8 weight."""
    return _gemv("b2_q8_gemv", tiles, n_tile_rows, k_tiles, Q8_TILE_BYTES, x, out, accumulate, prefetch)


def q4_swiglu_gemv(gate: torch.Tensor, up: torch.Tensor, n_tile_rows: int, k_tiles: int, x: torch.Tensor,
                   out: torch.Tensor | None = None, prefetch: bool = False) -> torch.Tensor:
    """bf16 h = silu(bf16(G x)) * bf16(U x), one fused kernel."""
    _tiles(gate, n_tile_rows, k_tiles, Q4_TILE_BYTES, "gate")
    _tiles(up, n_tile_rows, k_tiles, Q4_TILE_BYTES, "up")
    k, n = k_tiles * TILE_K, n_tile_rows * TILE_ROWS
    x2 = _x2d(x, k)
    b = x2.shape[0]
    if out is None:
        out = torch.empty((b, n), dtype=torch.bfloat16, device=x2.device)
    _need(out, "out", torch.bfloat16)
    if out.dim() != 2 or out.shape[0] != b or out.shape[1] < n or out.stride(1) != 1:
        raise ValueError(f"out must be [B, >=N] row-major, got {tuple(out.shape)}")
    for b0 in range(0, b, 16):
        bb = min(16, b - b0)
        _native.call("b2_q4_swiglu_gemv", _ptr(gate), _ptr(up), n_tile_rows, k_tiles,
                     ctypes.c_void_p(x2[b0].data_ptr()), bb, x2.stride(0),
                     ctypes.c_void_p(out[b0].data_ptr()), out.stride(0), GEMV_PREFETCH if prefetch else 0,
                     _stream())
    return out if x.dim() == 2 else out[0, :n]


def gemm_workspace_bytes(batch: int, k_tiles: int) -> int:
    """Workspace of the tensor-core GEMM (staged fp16 x + exponents)."""
    nb = ctypes.c_size_t(0)
    _native.call("b2_q4_gemm_workspace_size", batch, k_tiles, ctypes.byref(nb))
    return nb.value


def _gemm_ws(workspace, batch: int, k_tiles: int, device) -> torch.Tensor:
    need = gemm_workspace_bytes(batch, k_tiles)
    if workspace is None:
        return torch.empty(need + 256, dtype=torch.uint8, device=device)
    if workspace.numel() < need or workspace.data_ptr() % 256:
        raise ValueError(f"workspace must hold {need} bytes, 256-byte aligned")
    return workspace


def _aligned_ws(ws: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p((ws.data_ptr() + 255) // 256 * 256)


def q4_gemm_pack(tiles: torch.Tensor, n_tile_rows: int, k_tiles: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """The packed layout of a q4nx weight [n_tile_rows][k_tiles] for the tensor-core GEMM
    (b2_q4_gemm_pack): same size, every code and scale kept, reordered lane-per-row and
    tile-row-pair-major.  A load-time step."""
    _tiles(tiles, n_tile_rows, k_tiles, Q4_TILE_BYTES, "tiles")
    if out is None:
        out = torch.empty_like(tiles)
    if out.shape != tiles.shape or out.dtype != torch.uint8:
        raise ValueError("out must match tiles")
    _native.call("b2_q4_gemm_pack", _ptr(tiles), n_tile_rows, k_tiles, _ptr(out), _stream())
    return out


def q8_gemm_pack(tiles: torch.Tensor, n_tile_rows: int, k_tiles: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """The packed layout of a q8 weight [n_tile_rows][k_tiles] for the tensor-core GEMM
    (b2_q8_gemm_pack).  A load-time step."""
    _tiles(tiles, n_tile_rows, k_tiles, Q8_TILE_BYTES, "tiles")
    if out is None:
        out = torch.empty_like(tiles)
    if out.shape != tiles.shape or out.dtype != torch.uint8:
        raise ValueError("out must match tiles")
    _native.call("b2_q8_gemm_pack", _ptr(tiles), n_tile_rows, k_tiles, _ptr(out), _stream())
    return out


def q8_gemm(packed: torch.Tensor, n_tile_rows: int, k_tiles: int, x: torch.Tensor, out: torch.Tensor | None = None,
            accumulate: bool = False, workspace: torch.Tensor | None = None, prefetch: bool = False,
            norm_w: torch.Tensor | None = None, eps: float = 0.0, peer_sum: PeerSum | None = None) -> torch.Tensor:
    """fp32 y [B, N] = W x for a packed q8 weight (q8_gemm_pack) on the tensor cores; with
    norm_w, x is the fp32 residual and its RMSNorm is fused (b2_q8_gemm_rmsnorm); peer_sum
    (with norm_w): x += the seam's sum over ranks first, in place (b2_gemm_rmsnorm_seam)."""
    if peer_sum is not None and norm_w is None:
        raise ValueError("peer_sum needs norm_w (the _rmsnorm form)")
    _tiles(packed, n_tile_rows, k_tiles, Q8_TILE_BYTES, "packed")
    k, n = k_tiles * TILE_K, n_tile_rows * TILE_ROWS
    x2 = _norm_in(x, norm_w, k) if norm_w is not None else _x2d(x, k)
    b = x2.shape[0]
    if out is None:
        out = torch.zeros((b, n), dtype=torch.float32, device=x2.device)
    _need(out, "out", torch.float32)
    ws = _gemm_ws(workspace, b, k_tiles, x2.device)
    flags = GEMM_PACKED | (GEMV_ACCUMULATE if accumulate else 0) | (GEMV_PREFETCH if prefetch else 0)
    wsp = _aligned_ws(ws) if workspace is None else _ptr(ws)
    wsn = ws.numel() - (256 if workspace is None else 0)
    if peer_sum is not None:
        if x2.data_ptr() != x.data_ptr():
            raise ValueError("peer_sum updates x in place: x must be fp32 row-major and 16-byte aligned")
        _seam_call(SEAM_Q8_F32, packed, None, n_tile_rows, k_tiles, x2, norm_w, eps, out, flags, wsp, wsn, peer_sum)
    elif norm_w is not None:
        _native.call("b2_q8_gemm_rmsnorm", _ptr(packed), n_tile_rows, k_tiles, _ptr(x2), b, x2.stride(0),
                     _ptr(norm_w), float(eps), _ptr(out), out.stride(0), flags, wsp, wsn, _stream())
    else:
        _native.call("b2_q8_gemm", _ptr(packed), n_tile_rows, k_tiles, _ptr(x2), b, x2.stride(0), _ptr(out),
                     out.stride(0), flags, wsp, wsn, _stream())
    return out


SEAM_Q4_F32, SEAM_Q4_SWIGLU, SEAM_Q8_F32 = 0, 1, 2  # B2_SEAM_* forms


class PeerSum:
    """A pulled seam (b2_gemm_rmsnorm_seam) for an _rmsnorm GEMM: before the norm, the fp32
    residual x gains, in place, the sum over ranks of the partials in `buffer` of the peer
    region `region` (a peer.PeerRegion), with counters `seam`."""

    def __init__(self, region, buffer: str, seam: int):
        off, shape, dtype = region.offsets[buffer]
        if dtype != torch.float32 or len(shape) != 2:
            raise ValueError(f"seam buffer {buffer} must be fp32 [rows, cols]")
        self.region, self.offset, self.ld, self.rows, self.seam = region, off, shape[1], shape[0], seam


def _seam_call(form: int, w0, w1, n_tile_rows: int, k_tiles: int, x2: torch.Tensor, norm_w, eps: float,
               out: torch.Tensor, flags: int, wsp, wsn: int, ps: PeerSum) -> None:
    if x2.shape[0] > ps.rows:
        raise ValueError("more rows than the seam buffer holds")
    r = ps.region
    _native.call("b2_gemm_rmsnorm_seam", form, _ptr(w0), _ptr(w1) if w1 is not None else None, n_tile_rows, k_tiles,
                 _ptr(x2), x2.shape[0], x2.stride(0), _ptr(norm_w), float(eps), _ptr(out), out.stride(0), flags, wsp,
                 wsn, ctypes.c_void_p(r.peers_dev.data_ptr()), r.world, r.rank, ps.offset, ps.ld, ps.seam, _stream())


def q4_gemm(tiles: torch.Tensor, n_tile_rows: int, k_tiles: int, x: torch.Tensor, out: torch.Tensor | None = None,
            accumulate: bool = False, workspace: torch.Tensor | None = None, prefetch: bool = False,
            norm_w: torch.Tensor | None = None, eps: float = 0.0, packed: bool = False,
            swiglu_in: bool = False, peer_sum: PeerSum | None = None) -> torch.Tensor:
    """fp32 y [B, N] = W x on the tcgen05 tensor cores (batches up to 256).

    With norm_w, x is the fp32 residual [B, K] and the GEMM multiplies
    bf16(rmsnorm(x) * norm_w), the norm done in its x pre-pass (b2_q4_gemm_rmsnorm).
    With swiglu_in, x is the fp32 output [B, 2K] of a gate+up GEMM (gate columns first)
    and the GEMM multiplies bf16(silu(bf16 g) * bf16 u), formed in its x pre-pass
    (b2_q4_gemm_swiglu_in).
    packed: the tiles come from q4_gemm_pack (A is dequantised into tensor memory).
    peer_sum (with norm_w): x += the seam's sum over ranks first, in place (b2_gemm_rmsnorm_seam)."""
    _tiles(tiles, n_tile_rows, k_tiles, Q4_TILE_BYTES, "tiles")
    k, n = k_tiles * TILE_K, n_tile_rows * TILE_ROWS
    if peer_sum is not None and norm_w is None:
        raise ValueError("peer_sum needs norm_w (the _rmsnorm form)")
    if swiglu_in:
        if norm_w is not None:
            raise ValueError("swiglu_in and norm_w are exclusive")
        _need(x, "x", torch.float32)
        x2 = x.reshape(1, -1) if x.dim() == 1 else x
        if x2.dim() != 2 or x2.shape[1] != 2 * k:
            raise ValueError(f"swiglu_in wants x [B, {2 * k}] fp32 (gate columns, then up)")
        if x2.stride(1) != 1 or x2.stride(0) % 4 or x2.data_ptr() % 16:
            x2 = x2.contiguous()
    else:
        x2 = _norm_in(x, norm_w, k) if norm_w is not None else _x2d(x, k)
    b = x2.shape[0]
    if out is None:
        out = torch.zeros((b, n), dtype=torch.float32, device=x2.device)
    _need(out, "out", torch.float32)
    ws = _gemm_ws(workspace, b, k_tiles, x2.device)
    flags = (GEMV_ACCUMULATE if accumulate else 0) | (GEMV_PREFETCH if prefetch else 0) | (GEMM_PACKED if packed else 0)
    wsp = _aligned_ws(ws) if workspace is None else _ptr(ws)
    wsn = ws.numel() - (256 if workspace is None else 0)
    if peer_sum is not None:
        if x2.data_ptr() != x.data_ptr():
            raise ValueError("peer_sum updates x in place: x must be fp32 row-major and 16-byte aligned")
        _seam_call(SEAM_Q4_F32, tiles, None, n_tile_rows, k_tiles, x2, norm_w, eps, out, flags, wsp, wsn, peer_sum)
    elif swiglu_in:
        _native.call("b2_q4_gemm_swiglu_in", _ptr(tiles), n_tile_rows, k_tiles, _ptr(x2), b, x2.stride(0),
                     _ptr(out), out.stride(0), flags, wsp, wsn, _stream())
    elif norm_w is not None:
        _native.call("b2_q4_gemm_rmsnorm", _ptr(tiles), n_tile_rows, k_tiles, _ptr(x2), b, x2.stride(0),
                     _ptr(norm_w), float(eps), _ptr(out), out.stride(0), flags, wsp, wsn, _stream())
    else:
        _native.call("b2_q4_gemm", _ptr(tiles), n_tile_rows, k_tiles, _ptr(x2), b, x2.stride(0), _ptr(out),
                     out.stride(0), flags, wsp, wsn, _stream())
    return out


def q4_swiglu_gemm(gate: torch.Tensor, up: torch.Tensor, n_tile_rows: int, k_tiles: int, x: torch.Tensor,
                   out: torch.Tensor | None = None, workspace: torch.Tensor | None = None, prefetch: bool = False,
                   norm_w: torch.Tensor | None = None, eps: float = 0.0, packed: bool = False,
                   peer_sum: PeerSum | None = None) -> torch.Tensor:
    """bf16 h = silu(bf16(G x)) * bf16(U x) on the tensor cores (batches up to 256); with
    norm_w, x is the fp32 residual and its RMSNorm is fused (b2_q4_swiglu_gemm_rmsnorm);
    peer_sum (with norm_w): x += the seam's sum over ranks first, in place.
    packed: gate and up come from q4_gemm_pack."""
    _tiles(gate, n_tile_rows, k_tiles, Q4_TILE_BYTES, "gate")
    _tiles(up, n_tile_rows, k_tiles, Q4_TILE_BYTES, "up")
    k, n = k_tiles * TILE_K, n_tile_rows * TILE_ROWS
    x2 = _norm_in(x, norm_w, k) if norm_w is not None else _x2d(x, k)
    b = x2.shape[0]
    if out is None:
        out = torch.empty((b, n), dtype=torch.bfloat16, device=x2.device)
    _need(out, "out", torch.bfloat16)
    ws = _gemm_ws(workspace, b, k_tiles, x2.device)
    flags = (GEMV_PREFETCH if prefetch else 0) | (GEMM_PACKED if packed else 0)
    wsp = _aligned_ws(ws) if workspace is None else _ptr(ws)
    wsn = ws.numel() - (256 if workspace is None else 0)
    if peer_sum is not None:
        if norm_w is None or x2.data_ptr() != x.data_ptr():
            raise ValueError("peer_sum needs norm_w and an fp32 row-major, 16-byte aligned x (updated in place)")
        _seam_call(SEAM_Q4_SWIGLU, gate, up, n_tile_rows, k_tiles, x2, norm_w, eps, out, flags, wsp, wsn, peer_sum)
    elif norm_w is not None:
        _native.call("b2_q4_swiglu_gemm_rmsnorm", _ptr(gate), _ptr(up), n_tile_rows, k_tiles, _ptr(x2), b,
                     x2.stride(0), _ptr(norm_w), float(eps), _ptr(out), out.stride(0), flags, wsp, wsn, _stream())
    else:
        _native.call("b2_q4_swiglu_gemm", _ptr(gate), _ptr(up), n_tile_rows, k_tiles, _ptr(x2), b, x2.stride(0),
                     _ptr(out), out.stride(0), flags, wsp, wsn, _stream())
    return out


def _norm_in(x: torch.Tensor, w: torch.Tensor, k: int) -> torch.Tensor:
    _need(x, "x", torch.float32)
    _need(w, "norm_w", torch.bfloat16)
    x2 = x.reshape(1, -1) if x.dim() == 1 else x
    if x2.dim() != 2 or x2.shape[1] != k or w.numel() != k:
        raise ValueError(f"x must be [B, {k}] fp32 and norm_w [{k}]")
    if x2.stride(1) != 1 or x2.stride(0) % 4 or x2.data_ptr() % 16:
        x2 = x2.contiguous()
    if not w.is_contiguous() or w.data_ptr() % 16:
        raise ValueError("norm_w must be contiguous and 16-byte aligned")
    return x2


def gemv_rmsnorm(tiles: torch.Tensor, n_tile_rows: int, k_tiles: int, x: torch.Tensor, norm_w: torch.Tensor,
                 eps: float, out: torch.Tensor | None = None, accumulate: bool = False, prefetch: bool = False,
                 q8: bool = False) -> torch.Tensor:
    """fp32 y = W bf16(rmsnorm(x) * norm_w) in one kernel; x fp32 [B, K] (e.g. the residual stream)."""
    tb = Q8_TILE_BYTES if q8 else Q4_TILE_BYTES
    _tiles(tiles, n_tile_rows, k_tiles, tb, "tiles")
    k, n = k_tiles * TILE_K, n_tile_rows * TILE_ROWS
    x2 = _norm_in(x, norm_w, k)
    b = x2.shape[0]
    if out is None:
        out = torch.empty((b, n), dtype=torch.float32, device=x2.device)
    _need(out, "out", torch.float32)
    flags = (GEMV_ACCUMULATE if accumulate else 0) | (GEMV_PREFETCH if prefetch else 0)
    name = "b2_q8_gemv_rmsnorm" if q8 else "b2_q4_gemv_rmsnorm"
    for b0 in range(0, b, 16):
        bb = min(16, b - b0)
        _native.call(name, _ptr(tiles), n_tile_rows, k_tiles, ctypes.c_void_p(x2[b0].data_ptr()), bb, x2.stride(0),
                     _ptr(norm_w), float(eps), ctypes.c_void_p(out[b0].data_ptr()), out.stride(0), flags, _stream())
    return out if x.dim() == 2 else out[0, :n]


def swiglu_gemv_rmsnorm(gate: torch.Tensor, up: torch.Tensor, n_tile_rows: int, k_tiles: int, x: torch.Tensor,
                        norm_w: torch.Tensor, eps: float, out: torch.Tensor | None = None,
                        prefetch: bool = False) -> torch.Tensor:
    """bf16 h = silu(G xn) * (U xn) with xn = bf16(rmsnorm(x) * norm_w), one kernel."""
    _tiles(gate, n_tile_rows, k_tiles, Q4_TILE_BYTES, "gate")
    _tiles(up, n_tile_rows, k_tiles, Q4_TILE_BYTES, "up")
    k, n = k_tiles * TILE_K, n_tile_rows * TILE_ROWS
    x2 = _norm_in(x, norm_w, k)
    b = x2.shape[0]
    if out is None:
        out = torch.empty((b, n), dtype=torch.bfloat16, device=x2.device)
    _need(out, "out", torch.bfloat16)
    for b0 in range(0, b, 16):
        bb = min(16, b - b0)
        _native.call("b2_q4_swiglu_gemv_rmsnorm", _ptr(gate), _ptr(up), n_tile_rows, k_tiles,
                     ctypes.c_void_p(x2[b0].data_ptr()), bb, x2.stride(0), _ptr(norm_w), float(eps),
                     ctypes.c_void_p(out[b0].data_ptr()), out.stride(0), GEMV_PREFETCH if prefetch else 0, _stream())
    return out if x.dim() == 2 else out[0, :n]


def dequant_tiles(tiles: torch.Tensor, q8: bool = False) -> torch.Tensor:
    """[T, tile] uint8 -> [T, 8192] bf16 in weight-index order (bit-exact decode)."""
    tb = Q8_TILE_BYTES if q8 else Q4_TILE_BYTES
    _need(tiles, "tiles", torch.uint8)
    if not tiles.is_contiguous() or tiles.numel() % tb:
        raise ValueError(f"tiles must be contiguous whole {tb}-byte tiles")
    n = tiles.numel() // tb
    out = torch.empty((n, 8192), dtype=torch.bfloat16, device=tiles.device)
    _native.call("b2_q8_dequant_tiles" if q8 else "b2_q4_dequant_tiles", _ptr(tiles), n, _ptr(out), _stream())
    return out


def dequant_matrix(tiles: torch.Tensor, n_tile_rows: int, k_tiles: int, q8: bool = False) -> torch.Tensor:
    """Whole tiled tensor -> float32 [N, K], untiled (the GPU form of Q4NX.tensor)."""
    tb = Q8_TILE_BYTES if q8 else Q4_TILE_BYTES
    _tiles(tiles, n_tile_rows, k_tiles, tb, "tiles")
    out = torch.empty((n_tile_rows * TILE_ROWS, k_tiles * TILE_K), dtype=torch.float32, device=tiles.device)
    _native.call("b2_q8_dequant_matrix" if q8 else "b2_q4_dequant_matrix", _ptr(tiles), n_tile_rows, k_tiles,
                 _ptr(out), out.stride(0), _stream())
    return out


def set_launch_options(pdl: bool = True) -> None:
    _native.call("b2_set_launch_options", 1 if pdl else 0)


def device_error() -> int:
    """Read and clear the device error word (synchronises the current stream)."""
    return _native.read_device_error(torch.cuda.current_stream().cuda_stream)


ATTN_NO_APPEND = 1
ATTN_NO_ROPE = 2
ATTN_OUT_F32 = 4
ATTN_PREFETCH_KV = 8


def gqa_decode_workspace_bytes(batch: int, n_q_heads: int, n_kv_heads: int, head_dim: int, max_len: int) -> int:
    n = ctypes.c_size_t(0)
    _native.check(_native.lib().b2_gqa_decode_workspace_size(batch, n_q_heads, n_kv_heads, head_dim, max_len,
                                                              ctypes.byref(n)), "b2_gqa_decode_workspace_size")
    return n.value


def gqa_decode(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, k_cache: torch.Tensor,
               v_cache: torch.Tensor, pos: torch.Tensor, *, n_q_heads: int, n_kv_heads: int,
               theta: float = 10000.0, scale: float | None = None, max_len: int | None = None,
               out: torch.Tensor | None = None, append: bool = True, rope: bool = True,
               out_f32: bool = False, workspace: torch.Tensor | None = None,
               prefetch_kv: bool = False) -> torch.Tensor:
    """GQA flash-decode for one new token per sequence (see b2_gqa_decode).

    prefetch_kv (B2_ATTN_PREFETCH_KV): pos and the cache rows before pos are final
    when the call is made (no kernel still in flight writes them), so the kernel
    reads its first K/V chunks before waiting on the preceding kernel.

    q [B, >=Hq*D], k_new/v_new [B, >=Hkv*D] fp32 with a common row stride (e.g.
    slices of the QKV GEMV output); caches bf16 [B, Hkv, ctx_max, D]; pos int32 [B].
    Returns out [B, Hq*D] (bf16, or fp32 with out_f32).
    """
    for name, t in (("q", q), ("k_new", k_new), ("v_new", v_new)):
        _need(t, name, torch.float32)
        if t.dim() != 2 or t.stride(1) != 1:
            raise ValueError(f"{name} must be a 2-D row-major view")
    ld_new = q.stride(0)
    if q.shape[0] == 1:  # one sequence: the row stride is never used
        ld_new = max(q.shape[1], n_q_heads * k_cache.shape[-1])
    elif not (q.stride(0) == k_new.stride(0) == v_new.stride(0)):
        raise ValueError("q, k_new, v_new must share a row stride")
    _need(k_cache, "k_cache", torch.bfloat16)
    _need(v_cache, "v_cache", torch.bfloat16)
    _need(pos, "pos", torch.int32)
    if not (k_cache.is_contiguous() and v_cache.is_contiguous() and pos.is_contiguous()):
        raise ValueError("caches and pos must be contiguous")
    b, hkv, ctx_max, d = k_cache.shape
    if v_cache.shape != k_cache.shape or hkv != n_kv_heads or pos.numel() != b or q.shape[0] != b:
        raise ValueError("inconsistent attention shapes")
    max_len = ctx_max if max_len is None else max_len
    scale = d ** -0.5 if scale is None else scale
    odt = torch.float32 if out_f32 else torch.bfloat16
    if out is None:
        out = torch.empty((b, n_q_heads * d), dtype=odt, device=q.device)
    _need(out, "out", odt)
    ws_n = gqa_decode_workspace_bytes(b, n_q_heads, n_kv_heads, d, max_len)
    if workspace is None or workspace.numel() < ws_n:
        workspace = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=q.device)
    flags = (0 if append else ATTN_NO_APPEND) | (0 if rope else ATTN_NO_ROPE) | (ATTN_OUT_F32 if out_f32 else 0)
    flags |= ATTN_PREFETCH_KV if prefetch_kv else 0
    _native.call("b2_gqa_decode", _ptr(q), _ptr(k_new), _ptr(v_new), ld_new, _ptr(k_cache), _ptr(v_cache),
                 _ptr(pos), b, n_q_heads, n_kv_heads, d, ctx_max, max_len, float(theta), float(scale), _ptr(out),
                 out.stride(0), _ptr(workspace), workspace.numel(), flags, _stream())
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 y = x * rsqrt(mean(x^2) + eps) * w over the last dim; x bf16 or fp32 [B, n] or [n]."""
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError("x must be bf16 or fp32")
    _need(x, "x", x.dtype)
    _need(w, "w", torch.bfloat16)
    x2 = x.reshape(1, -1) if x.dim() == 1 else x
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    b, n = x2.shape
    if w.numel() != n:
        raise ValueError("weight length mismatch")
    if out is None:
        out = torch.empty((b, n), dtype=torch.bfloat16, device=x.device)
    _need(out, "out", torch.bfloat16)
    _native.call("b2_rmsnorm", _ptr(x2), 1 if x2.dtype == torch.float32 else 0, x2.stride(0), _ptr(w),
                 float(eps), b, n, _ptr(out), out.stride(0), _stream())
    return out if x.dim() == 2 else out[0]


DELTA_OUT_F32 = 1
DELTA_PREFETCH_STATE = 2
DELTA_HEAD_DIM = 128


def _rows(t: torch.Tensor, name: str, width: int) -> torch.Tensor:
    """fp32 [B, >= width] with unit column stride (a slice of a wider projection output is fine)."""
    _need(t, name, torch.float32)
    if t.dim() != 2 or t.shape[1] < width or t.stride(1) != 1:
        raise ValueError(f"{name} must be fp32 [B, >= {width}] with unit column stride, got {tuple(t.shape)}")
    return t


def _dense(t: torch.Tensor, name: str, shape: tuple) -> None:
    _need(t, name, torch.float32)
    if tuple(t.shape) != shape or not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous fp32 {shape}, got {tuple(t.shape)}")


def gated_delta_step(qkv: torch.Tensor, z: torch.Tensor, b: torch.Tensor, a: torch.Tensor,
                     conv_state: torch.Tensor, conv_w: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor,
                     norm_w: torch.Tensor, state: torch.Tensor, n_k_heads: int, n_v_heads: int,
                     eps: float = 1e-6, out: torch.Tensor | None = None, out_f32: bool = False,
                     prefetch_state: bool = False) -> torch.Tensor:
    """One gated DeltaNet decode step (see b2_gated_delta_step); conv_state and state update in place.

    qkv [B, >= conv_dim], z [B, >= nv*128], b and a [B, >= nv] fp32 (slices of one
    projection output are accepted); conv_state [B, conv_dim, 4], conv_w [conv_dim, 4],
    state [B, nv, 128, 128], A_log / dt_bias [nv], norm_w [128], all fp32.
    Mirrors the decode branch of transformers' Qwen3_5GatedDeltaNet.forward between
    its in_proj_* and out_proj calls."""
    d = DELTA_HEAD_DIM
    bsz = qkv.shape[0]
    conv_dim = 2 * n_k_heads * d + n_v_heads * d
    _rows(qkv, "qkv", conv_dim)
    _rows(z, "z", n_v_heads * d)
    _rows(b, "b", n_v_heads)
    _rows(a, "a", n_v_heads)
    if b.stride(0) != a.stride(0):
        raise ValueError("b and a must share one row stride")
    for t, name in ((z, "z"), (b, "b"), (a, "a")):
        if t.shape[0] != bsz:
            raise ValueError(f"{name} batch {t.shape[0]} != {bsz}")
    _dense(conv_state, "conv_state", (bsz, conv_dim, 4))
    _dense(conv_w, "conv_w", (conv_dim, 4))
    _dense(A_log, "A_log", (n_v_heads,))
    _dense(dt_bias, "dt_bias", (n_v_heads,))
    _dense(norm_w, "norm_w", (d,))
    _dense(state, "state", (bsz, n_v_heads, d, d))
    odt = torch.float32 if out_f32 else torch.bfloat16
    if out is None:
        out = torch.empty((bsz, n_v_heads * d), dtype=odt, device=qkv.device)
    _need(out, "out", odt)
    if out.dim() != 2 or out.stride(1) != 1 or out.shape[0] != bsz:
        raise ValueError("out must be [B, >= nv*128] with unit column stride")
    flags = (DELTA_OUT_F32 if out_f32 else 0) | (DELTA_PREFETCH_STATE if prefetch_state else 0)
    _native.call("b2_gated_delta_step", _ptr(qkv), qkv.stride(0), _ptr(z), z.stride(0), _ptr(b), _ptr(a),
                 b.stride(0), _ptr(conv_state), _ptr(conv_w), _ptr(A_log), _ptr(dt_bias), _ptr(norm_w),
                 _ptr(state), bsz, n_k_heads, n_v_heads, d, float(eps), _ptr(out), out.stride(0), flags,
                 _stream())
    return out


GATED_OUT_F32 = 1
GATED_HEAD_DIM = 256


def gated_attn_workspace_bytes(batch: int, n_q_heads: int, n_kv_heads: int, max_len: int) -> int:
    n = ctypes.c_size_t()
    _native.check(_native.lib().b2_gated_attn_decode_workspace_size(batch, n_q_heads, n_kv_heads, GATED_HEAD_DIM,
                                                                     max_len, ctypes.byref(n)),
                  "b2_gated_attn_decode_workspace_size")
    return n.value


def gated_attn_decode(qg: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, q_norm_w: torch.Tensor,
                      k_norm_w: torch.Tensor, inv_freq: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      pos: torch.Tensor, n_q_heads: int, n_kv_heads: int, max_len: int | None = None,
                      eps: float = 1e-6, out: torch.Tensor | None = None, out_f32: bool = False,
                      workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Qwen3.5 gated full-attention decode step (see b2_gated_attn_decode); appends k/v at pos.

    qg [B, >= nq*512] (q | gate per head), k_new / v_new [B, >= nkv*256] fp32 (slices of
    one projection output are accepted, unit column stride); q_norm_w / k_norm_w [256]
    and inv_freq [rot_dim/2] fp32; k_cache / v_cache bf16 [B, nkv, ctx_max, 256]; pos
    int32 [B].  max_len (default ctx_max) bounds pos + 1 and sets the split plan."""
    d = GATED_HEAD_DIM
    bsz = qg.shape[0]
    _rows(qg, "qg", n_q_heads * 2 * d)
    _rows(k_new, "k_new", n_kv_heads * d)
    _rows(v_new, "v_new", n_kv_heads * d)
    if k_new.stride(0) != v_new.stride(0):
        raise ValueError("k_new and v_new must share one row stride")
    _dense(q_norm_w, "q_norm_w", (d,))
    _dense(k_norm_w, "k_norm_w", (d,))
    _need(inv_freq, "inv_freq", torch.float32)
    if inv_freq.dim() != 1 or not inv_freq.is_contiguous():
        raise ValueError("inv_freq must be contiguous fp32 [rot_dim/2]")
    for c, name in ((k_cache, "k_cache"), (v_cache, "v_cache")):
        _need(c, name, torch.bfloat16)
        if c.dim() != 4 or c.shape[0] != bsz or c.shape[1] != n_kv_heads or c.shape[3] != d or not c.is_contiguous():
            raise ValueError(f"{name} must be contiguous bf16 [B, nkv, ctx_max, 256], got {tuple(c.shape)}")
    if k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache shapes differ")
    _need(pos, "pos", torch.int32)
    if pos.numel() != bsz or not pos.is_contiguous():
        raise ValueError("pos must be contiguous int32 [B]")
    ctx_max = k_cache.shape[2]
    max_len = ctx_max if max_len is None else max_len
    odt = torch.float32 if out_f32 else torch.bfloat16
    if out is None:
        out = torch.empty((bsz, n_q_heads * d), dtype=odt, device=qg.device)
    _need(out, "out", odt)
    if out.dim() != 2 or out.stride(1) != 1 or out.shape[0] != bsz:
        raise ValueError("out must be [B, >= nq*256] with unit column stride")
    ws_n = gated_attn_workspace_bytes(bsz, n_q_heads, n_kv_heads, max_len)
    if workspace is None and ws_n:
        workspace = torch.empty(ws_n, dtype=torch.uint8, device=qg.device)
    wp = _ptr(workspace) if workspace is not None else ctypes.c_void_p(0)
    wn = workspace.numel() * workspace.element_size() if workspace is not None else 0
    _native.call("b2_gated_attn_decode", _ptr(qg), qg.stride(0), _ptr(k_new), _ptr(v_new), k_new.stride(0),
                 _ptr(q_norm_w), _ptr(k_norm_w), _ptr(inv_freq), 2 * inv_freq.numel(), _ptr(k_cache), _ptr(v_cache),
                 _ptr(pos), bsz, n_q_heads, n_kv_heads, d, ctx_max, max_len, float(eps), _ptr(out), out.stride(0),
                 GATED_OUT_F32 if out_f32 else 0, wp, wn, _stream())
    return out
