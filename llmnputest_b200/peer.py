"""Peer regions and the tensor-parallel exchanges of include/b2q4nx.h (b2_peer_*, b2_tp_*).

One process per GPU.  Every rank allocates one region (b2_peer_alloc), the ranks swap
their CUDA IPC handles over the process group (all_gather_object: the host channel
torch.distributed already has), and each maps the others' (b2_peer_open).  Buffers
that other ranks read or write -- the residual stream, the all-reduce slots or the
partials a pulled seam reads, the gathered logits -- are carved out of the region at
the same offsets on every rank and wrapped as torch tensors without a copy.

The exchanges replace the NCCL calls of a tensor-parallel decode step (all-reduce of
the K-sharded O and down projections, all-gather of the vocab-sharded logits); each is
one small kernel that stores straight into the peers' memory and waits, bounded, for
theirs.  On the GEMM path the all-reduces need no kernel: ops.PeerSum hands a region
buffer to the next GEMM's x pre-pass, which sums every rank's partial itself.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native

CTL_BYTES = 65536  # B2_PEER_CTL_BYTES: the control words at the start of every region
ALIGN = 256
IPC_HANDLE_BYTES = 64

_TYPESTR = {torch.float32: "<f4", torch.bfloat16: "<V2", torch.int32: "<i4", torch.uint8: "|u1"}


class _CudaArray:
    """Minimal __cuda_array_interface__ provider so torch can wrap a raw device pointer."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


def wrap(ptr: int, shape: tuple, dtype: torch.dtype, device) -> torch.Tensor:
    """A torch tensor over `ptr` (contiguous, `shape`, `dtype`) on `device`, sharing the memory."""
    if dtype == torch.bfloat16:  # no bf16 typestr: wrap as int16 and reinterpret
        t = torch.as_tensor(_CudaArray(ptr, tuple(shape), "<i2"), device=device)
        return t.view(torch.bfloat16)
    return torch.as_tensor(_CudaArray(ptr, tuple(shape), _TYPESTR[dtype]), device=device)


class PeerRegion:
    """This rank's region plus mappings of every other rank's, and a bump allocator for
    buffers at identical offsets on all ranks (call `buffer` in the same order everywhere).

    `layout` lists (name, shape, dtype); the region is sized for them.  Collective: every
    rank of `group` must construct it together."""

    def __init__(self, layout: list[tuple[str, tuple, torch.dtype]], group=None, device=None):
        import torch.distributed as dist
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        offs, off = {}, CTL_BYTES
        for name, shape, dtype in layout:
            n = 1
            for d in shape:
                n *= int(d)
            offs[name] = (off, tuple(shape), dtype)
            off += (n * torch.empty((), dtype=dtype).element_size() + ALIGN - 1) // ALIGN * ALIGN
        self.nbytes = off
        self.offsets = offs
        L = _native.lib()
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        _native.check(L.b2_peer_alloc(ctypes.c_size_t(self.nbytes), ctypes.byref(ptr), handle), "b2_peer_alloc")
        self.base = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        self.ptrs, self._opened = [], []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.base)
                continue
            p = ctypes.c_void_p()
            _native.check(L.b2_peer_open(ctypes.create_string_buffer(h, IPC_HANDLE_BYTES), ctypes.byref(p)),
                          "b2_peer_open")
            self.ptrs.append(p.value)
            self._opened.append(p.value)
        self.peers_dev = torch.tensor(self.ptrs, dtype=torch.int64, device=self.device)
        self.buffers = {name: wrap(self.base + o, shape, dtype, self.device) for name, (o, shape, dtype) in offs.items()}
        for t in self.buffers.values():
            t.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)  # every mapping in place before any rank's first exchange

    def offset(self, name: str) -> int:
        return self.offsets[name][0]

    def close(self) -> None:
        """Unmap the peers' regions and free this rank's (after every rank stopped exchanging)."""
        L = _native.lib()
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            L.b2_peer_close(ctypes.c_void_p(p))
        self._opened = []
        self.buffers = {}
        if self.base:
            L.b2_peer_free(ctypes.c_void_p(self.base))
            self.base = 0


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def gather(region: PeerRegion, src: torch.Tensor, dst: str, add_base: torch.Tensor | None = None) -> None:
    """Every rank's src [rows, cols] into every rank's region buffer `dst` [rows, cols*world]
    at column rank*cols (b2_tp_gather); with add_base (this rank's copy of a replicated
    fp32 `dst`) the block is added into all copies."""
    if src.dim() != 2 or src.stride(1) != 1:
        raise ValueError("src must be 2-D row-major")
    off, shape, dtype = region.offsets[dst]
    if src.dtype != dtype or shape[0] != src.shape[0] or shape[1] < src.shape[1] * region.world:
        raise ValueError(f"src {tuple(src.shape)} {src.dtype} does not fit {dst} {shape} {dtype}")
    _native.call("b2_tp_gather", ctypes.c_void_p(region.peers_dev.data_ptr()), region.world, region.rank,
                 ctypes.c_void_p(src.data_ptr()), src.shape[0], src.shape[1], src.stride(0), src.element_size(),
                 off, shape[1], ctypes.c_void_p(add_base.data_ptr()) if add_base is not None else None, _stream())


def allreduce_add(region: PeerRegion, src: torch.Tensor, slots: str, y: torch.Tensor) -> None:
    """y += sum over ranks of src (fp32 [rows, cols]), in rank order on every rank (b2_tp_allreduce)."""
    if src.dtype != torch.float32 or y.dtype != torch.float32 or src.dim() != 2 or src.stride(1) != 1:
        raise ValueError("src and y must be fp32 2-D row-major")
    off, shape, _ = region.offsets[slots]
    if shape[0] != region.world or shape[1] != src.shape[0] or shape[2] != src.shape[1]:
        raise ValueError(f"slots {shape} do not match world {region.world} x {tuple(src.shape)}")
    _native.call("b2_tp_allreduce", ctypes.c_void_p(region.peers_dev.data_ptr()), region.world, region.rank,
                 ctypes.c_void_p(src.data_ptr()), src.shape[0], src.shape[1], src.stride(0), off,
                 ctypes.c_void_p(y.data_ptr()), y.stride(0), _stream())


class PeerExchange:
    """The exchange object TPDecoder uses with comm="peer": a PeerRegion laid out as
    `layout` (the buffers other ranks write into) and its gather / allreduce_add."""

    def __init__(self, layout, group=None, device=None):
        self.region = PeerRegion(layout, group=group, device=device)
        self.buffers = self.region.buffers

    def gather(self, src: torch.Tensor, name: str, add_base: torch.Tensor | None = None) -> None:
        gather(self.region, src, name, add_base)

    def allreduce_add(self, src: torch.Tensor, name: str, y: torch.Tensor) -> None:
        allreduce_add(self.region, src, name, y)

    def close(self) -> None:
        self.region.close()
