"""Decode program: a chain of q4 GEMVs and GQA attention as ONE persistent launch.

Host side of b2_program_* (include/b2q4nx.h).  A program is a list of phases
(`Phase`, the ctypes mirror of `b2_phase`) validated and uploaded once; every
launch then runs the whole list on one CTA per SM with grid barriers between
dependent phases, while each SM's producer warp streams the weights of the
phases ahead.

It replaces the per-op token loop (chat.py:74-78 -> one call per projection,
designs/granite_gemv/granite_layer.py:54-59): the reference measured that issue
cost dominates small matmuls (README.md:117-137), and on B200 the same holds for
kernel launches of 4-6 MB GEMVs.

Phases hold raw device pointers: the tensors they point into must outlive the
Program (the builders in decode.py keep them on the decoder object).
"""

from __future__ import annotations

import ctypes

import torch

from . import _native

PHASE_GEMV_Q4, PHASE_ATTENTION, PHASE_PREP = 0, 1, 2
X_BF16, X_RMSNORM, X_ATTENTION, X_SWIGLU = 0, 1, 2, 3

_INT_FIELDS = ("kind", "x_source", "barrier_after", "n_tile_rows", "k_tiles", "ldx", "half", "ldy", "n_q_heads",
               "n_kv_heads", "n_splits", "split_len", "ld_qkv", "ctx_max", "zero0_n", "zero1_n", "copy_n")
_PTR_FIELDS = ("w", "x", "norm_w", "y", "part", "qkv", "k_cache", "v_cache", "zero0", "zero1", "copy_src",
               "copy_dst")


class Phase(ctypes.Structure):
    """ctypes mirror of `b2_phase`; b2_phase_struct_bytes() checks the size."""

    _fields_ = ([(n, ctypes.c_int32) for n in _INT_FIELDS]
                + [("eps", ctypes.c_float), ("scale", ctypes.c_float), ("reserved", ctypes.c_int32)]
                + [(n, ctypes.c_void_p) for n in _PTR_FIELDS])


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t if isinstance(t, int) else t.data_ptr()


def attention_plan(batch: int, n_q_heads: int, n_kv_heads: int, max_len: int, head_dim: int = 64):
    """(n_splits, split_len, part_bytes) of an attention phase."""
    s, ln, nb = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_size_t(0)
    _native.call("b2_program_attention_plan", batch, n_q_heads, n_kv_heads, head_dim, max_len, ctypes.byref(s),
                 ctypes.byref(ln), ctypes.byref(nb))
    return s.value, ln.value, nb.value


def prep_phase(*, copy_src=None, copy_dst=None, copy_n: int = 0, zero0=None, zero0_n: int = 0, zero1=None,
               zero1_n: int = 0) -> Phase:
    """Copy / zero side tasks and the RoPE cos/sin table of this launch's positions; barrier after."""
    return Phase(kind=PHASE_PREP, barrier_after=1, copy_src=_ptr(copy_src), copy_dst=_ptr(copy_dst), copy_n=copy_n,
                 zero0=_ptr(zero0), zero0_n=zero0_n, zero1=_ptr(zero1), zero1_n=zero1_n)


def gemv_phase(w, n_tile_rows: int, k_tiles: int, x_source: int, x, ldx: int, y, ldy: int, *, norm_w=None,
               eps: float = 0.0, half: int = 0, attn: Phase | None = None, barrier: bool = True,
               zero0=None, zero0_n: int = 0) -> Phase:
    """y[b][:n] += W x'[b]; x' from `x_source` (attn: the attention phase whose partials are merged)."""
    ph = Phase(kind=PHASE_GEMV_Q4, x_source=x_source, barrier_after=int(barrier), n_tile_rows=n_tile_rows,
               k_tiles=k_tiles, ldx=ldx, half=half, ldy=ldy, eps=eps, w=_ptr(w), x=_ptr(x), norm_w=_ptr(norm_w),
               y=_ptr(y), zero0=_ptr(zero0), zero0_n=zero0_n)
    if attn is not None:
        ph.n_q_heads, ph.n_kv_heads, ph.n_splits, ph.part = attn.n_q_heads, attn.n_kv_heads, attn.n_splits, attn.part
    return ph


def attention_phase(qkv, ld_qkv: int, k_cache, v_cache, n_q_heads: int, n_kv_heads: int, ctx_max: int,
                    n_splits: int, split_len: int, part, scale: float, *, zero0=None, zero0_n: int = 0,
                    zero1=None, zero1_n: int = 0) -> Phase:
    """GQA decode attention of the new token (RoPE, cache append, split partials); barrier after."""
    return Phase(kind=PHASE_ATTENTION, barrier_after=1, n_q_heads=n_q_heads, n_kv_heads=n_kv_heads,
                 n_splits=n_splits, split_len=split_len, ld_qkv=ld_qkv, ctx_max=ctx_max, scale=scale,
                 qkv=_ptr(qkv), k_cache=_ptr(k_cache), v_cache=_ptr(v_cache), part=_ptr(part), zero0=_ptr(zero0),
                 zero0_n=zero0_n, zero1=_ptr(zero1), zero1_n=zero1_n)


class Program:
    """An uploaded phase list plus its launch scratch, on one device."""

    def __init__(self, phases: list[Phase], batch: int, device):
        if ctypes.sizeof(Phase) != _native.lib().b2_phase_struct_bytes():
            raise RuntimeError("b2_phase layout differs between the library and its binding")
        self.device = torch.device(device)
        self.batch = batch
        self.n = len(phases)
        self.phases = (Phase * self.n)(*phases)
        nbytes = self.n * ctypes.sizeof(Phase)
        self.dev_phases = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        sz = ctypes.c_size_t(0)
        _native.call("b2_program_scratch_size", batch, ctypes.byref(sz))
        self.scratch = torch.empty(sz.value, dtype=torch.uint8, device=self.device)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _native.call("b2_program_upload", ctypes.cast(self.phases, ctypes.c_void_p), self.n, batch,
                     ctypes.c_void_p(self.dev_phases.data_ptr()), nbytes, ctypes.c_void_p(stream))

    def launch(self, pos: torch.Tensor, theta: float = 10000.0) -> None:
        """Run the program on the current stream; pos: int32 [batch] on the device."""
        if pos.dtype != torch.int32 or pos.numel() < self.batch or not pos.is_cuda:
            raise ValueError("pos must be an int32 CUDA tensor of >= batch entries")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _native.call("b2_program_launch", ctypes.c_void_p(self.dev_phases.data_ptr()), self.n, self.batch,
                     ctypes.c_void_p(pos.data_ptr()), theta, ctypes.c_void_p(self.scratch.data_ptr()),
                     self.scratch.numel(), ctypes.c_void_p(stream))
