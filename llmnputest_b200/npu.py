"""Drop-in for the reference's op entry points (reference/npu.py), on B200.

Same names, arguments and error behaviour as reference/npu.py:41-163:

  NpuDesign(name)        one design, resident on the device; .meta, .upload(i, arr),
                         .run(), .download(i, dtype, count), .close(), .calls, .seconds
  NpuLmHead(fallback)    the lm_head module: .load_weights(raw), .forward(h),
                         .n_rows, .k, .npu_calls, .cpu_calls, .design
  attach_lm_head(model, f)

A "design" here is a CUDA kernel of libb2q4nx.so with its device buffers instead
of an xclbin + instruction stream.  Buffers are uploaded once and stay resident
(reference/npu.py:44-48); run() launches on the current CUDA stream and, like
the reference's blocking `h.wait()` (npu.py:93-97), waits for completion and
raises RuntimeError on any failure.

Differences that are deliberate:
  * there is no CPU fallback: NpuLmHead.forward runs multi-position inputs
    (prefill) on the GPU too, 16 positions per weight pass; `fallback` is kept
    for the constructor signature and never called, so `cpu_calls` stays 0;
  * the design table is built in rather than read from artifacts/<name>/design.json;
    pass meta=... to describe another shape.
"""

from __future__ import annotations

import time

import numpy as np
import torch
from ml_dtypes import bfloat16

from . import _native, ops
from .format import Q4_TILE_BYTES, Q8_TILE_BYTES, TILE_K, TILE_ROWS

# name -> meta.  "buffers" are byte sizes in argument order, as in design.json.
DESIGNS: dict[str, dict] = {
    # Qwen3.5-0.8B tied lm_head, q8, 248320 x 1024 (designs/lm_head/lm_head.py:150-155)
    "lm_head": {"kind": "q8_gemv", "n_rows": 248320, "k": 1024},
    # granite-4.2-3B lm_head, q4, 100352 x 2560 (designs/granite_gemv/granite_gemv.py:6-9)
    "granite_lm_head": {"kind": "q4_gemv", "n_rows": 100352, "k": 2560},
}


def _with_buffers(meta: dict) -> dict:
    m = dict(meta)
    n_t, k_t = m["n_rows"] // TILE_ROWS, m["k"] // TILE_K
    if n_t * TILE_ROWS != m["n_rows"] or k_t * TILE_K != m["k"]:
        raise ValueError(f"n_rows {m['n_rows']} / k {m['k']} are not whole tiles")
    tile = Q8_TILE_BYTES if m["kind"] == "q8_gemv" else Q4_TILE_BYTES
    batch = int(m.get("batch", 1))
    m.setdefault("buffers", [n_t * k_t * tile, batch * m["k"] * 2, batch * m["n_rows"] * 4])
    m["batch"] = batch
    return m


class NpuDesign:
    """One design resident on the GPU (reference/npu.py:41-114)."""

    def __init__(self, name: str, device=None, meta: dict | None = None):
        if meta is None:
            if name not in DESIGNS:
                raise SystemExit(f"no design named {name!r}; known: {sorted(DESIGNS)} (or pass meta=...)")
            meta = DESIGNS[name]
        if not torch.cuda.is_available():
            raise SystemExit("no CUDA device: this design runs on the GPU only (no CPU fallback)")
        _native.lib()  # fail here, loudly, if the library is not built
        self.name = name
        self.meta = _with_buffers(meta)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.bos = [torch.zeros(n, dtype=torch.uint8, device=self.device) for n in self.meta["buffers"]]
        self.calls = 0
        self.seconds = 0.0

    def upload(self, i: int, data) -> None:
        """Copy host data into buffer i (reference/npu.py:89-91)."""
        if isinstance(data, torch.Tensor):
            src = data.detach().contiguous().reshape(-1).view(torch.uint8)
        else:
            src = torch.from_numpy(np.ascontiguousarray(data).reshape(-1).view(np.uint8))
        if src.numel() > self.bos[i].numel():
            raise ValueError(f"buffer {i}: {src.numel()} bytes > {self.bos[i].numel()}")
        self.bos[i][: src.numel()].copy_(src, non_blocking=False)

    def launch(self, batch: int | None = None) -> None:
        """Enqueue the design on the current stream without waiting."""
        m = self.meta
        b = m["batch"] if batch is None else batch
        n_t, k_t = m["n_rows"] // TILE_ROWS, m["k"] // TILE_K
        x = self.bos[1].view(torch.bfloat16)[: b * m["k"]].view(b, m["k"])
        y = self.bos[2].view(torch.float32)[: b * m["n_rows"]].view(b, m["n_rows"])
        fn = ops.q8_gemv if m["kind"] == "q8_gemv" else ops.q4_gemv
        fn(self.bos[0], n_t, k_t, x, out=y)

    def run(self, batch: int | None = None) -> None:
        """Launch and wait, raising on failure (reference/npu.py:93-97)."""
        self.launch(batch)
        torch.cuda.current_stream(self.device).synchronize()
        code = ops.device_error()
        if code:
            raise RuntimeError(f"GPU design {self.name} recorded device error {code}")

    def download(self, i: int, dtype, count: int) -> np.ndarray:
        """Read `count` values of `dtype` from buffer i (reference/npu.py:111-114)."""
        nbytes = count * np.dtype(dtype).itemsize
        return self.bos[i][:nbytes].cpu().numpy().view(dtype)

    def close(self) -> None:
        """Release the device buffers (reference/npu.py:99-109)."""
        for attr in ("bos",):
            if hasattr(self, attr):
                delattr(self, attr)


class NpuLmHead(torch.nn.Module):
    """The lm_head, computed on the GPU from the q4nx tiles as stored (reference/npu.py:117-150)."""

    def __init__(self, fallback: torch.nn.Module | None = None, design: str = "lm_head", meta: dict | None = None):
        super().__init__()
        self.design = NpuDesign(design, meta=meta)
        self.fallback = fallback  # kept for the reference's signature; never called
        self.n_rows = self.design.meta["n_rows"]
        self.k = self.design.meta["k"]
        self.npu_calls = 0
        self.cpu_calls = 0

    def load_weights(self, raw: bytes) -> None:
        self.design.upload(0, np.frombuffer(raw, dtype=np.uint8))

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        t = time.perf_counter()
        lead = h.shape[:-1]
        x = h.detach().reshape(-1, self.k).to(device=self.design.device, dtype=torch.bfloat16)
        m = self.design.meta
        n_t, k_t = self.n_rows // TILE_ROWS, self.k // TILE_K
        fn = ops.q8_gemv if m["kind"] == "q8_gemv" else ops.q4_gemv
        y = fn(self.design.bos[0], n_t, k_t, x)  # [positions, n_rows] fp32, 16 positions per pass
        torch.cuda.current_stream(self.design.device).synchronize()
        out = y.reshape(*lead, self.n_rows).to(device=h.device, dtype=h.dtype)
        self.design.seconds += time.perf_counter() - t
        self.design.calls += 1
        self.npu_calls += 1
        return out


def attach_lm_head(model, f) -> NpuLmHead:
    """Swap the model's lm_head for the GPU one and upload its weights (reference/npu.py:153-163)."""
    e = f.header["lm_head.weight"]
    first, last = e["data_offsets"]
    with f.path.open("rb") as fh:
        fh.seek(f._data_start + first)
        raw = fh.read(last - first)
    mod = NpuLmHead(model.lm_head)
    mod.load_weights(raw)
    model.lm_head = mod
    return mod


def bf16_host(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 RNE on the host, the conversion reference/npu.py:143 applies."""
    return np.asarray(x, np.float32).astype(bfloat16)
