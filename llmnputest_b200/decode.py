"""One decode step of a dense GQA decoder on q4nx weights.

Per layer, in the order of designs/granite_gemv/granite_layer.py:54-59 (one GEMV
per group of projections that share an input):

    qkv  = W_qkv bf16(rmsnorm(resid, attn_norm))         b2_q4_gemv_rmsnorm (q|k|v rows concatenated,
                                                         the norm fused into the GEMV prologue)
    attn = attention(rope(q), rope(k) -> cache, v -> cache)   b2_gqa_decode
    resid += W_o attn                                    b2_q4_gemv, accumulate
    h    = silu(W_gate xn) * (W_up xn),
           xn = bf16(rmsnorm(resid, mlp_norm))           b2_q4_swiglu_gemv_rmsnorm (norm + gate/up + SiLU*up)
    resid += W_down h                                    b2_q4_gemv, accumulate

then the final norm fused into the q8 lm_head (b2_q8_gemv_rmsnorm): five
launches per layer.  The residual stream is
fp32; GEMV inputs are bf16 as in the reference.  Weights are the raw q4nx tiles,
resident on the device; the step is captured in one CUDA graph.  Batches of 9
and more run the projections on the tcgen05 GEMM (b2_q4_gemm / _swiglu_gemm, the
norms fused into their x pre-pass: b2_q4_gemm_rmsnorm / _swiglu_gemm_rmsnorm).

The reference never ran a granite token loop (README.md:299-301); this module
is the composition its layer design estimates (granite_layer.py:158-164).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import ops
from .format import Q4_TILE_BYTES, Q8_TILE_BYTES, TILE_K, TILE_ROWS


@dataclass(frozen=True)
class DecoderConfig:
    n_layers: int = 40
    hidden: int = 2560
    n_heads: int = 40
    n_kv_heads: int = 8
    head_dim: int = 64
    intermediate: int = 8192
    vocab: int = 100352
    rms_eps: float = 1e-6
    rope_theta: float = 10000.0

    @property
    def qkv_rows(self) -> int:
        return (self.n_heads + 2 * self.n_kv_heads) * self.head_dim

    def weight_bytes(self) -> dict:
        kt_h, kt_i = self.hidden // TILE_K, self.intermediate // TILE_K
        per_layer = (self.qkv_rows // TILE_ROWS * kt_h + self.hidden // TILE_ROWS * (self.n_heads * self.head_dim // TILE_K)
                     + 2 * self.intermediate // TILE_ROWS * kt_h + self.hidden // TILE_ROWS * kt_i) * Q4_TILE_BYTES
        return {"per_layer": per_layer, "layers": per_layer * self.n_layers,
                "lm_head": self.vocab // TILE_ROWS * kt_h * Q8_TILE_BYTES}


GRANITE_3B = DecoderConfig()


def synth_q4(n_tiles: int, gen: torch.Generator, device) -> torch.Tensor:
    """Seeded q4 tiles on the device: codes uniform 0..15, d = |N(0,.02)|, m = -|N(0,.02)| (bf16)."""
    w = torch.randint(0, 256, (n_tiles, Q4_TILE_BYTES), dtype=torch.uint8, device=device, generator=gen)
    w[:, 0:512] = (torch.randn(n_tiles, 256, device=device, generator=gen) * 0.02).abs().to(torch.bfloat16).view(torch.uint8)
    w[:, 512:1024] = (-(torch.randn(n_tiles, 256, device=device, generator=gen) * 0.02).abs()).to(torch.bfloat16).view(torch.uint8)
    return w.reshape(-1)


def synth_q8(n_tiles: int, gen: torch.Generator, device) -> torch.Tensor:
    """Seeded q8 tiles on the device: codes uniform int8 [-127, 127], scales |N(0,.02)| (bf16)."""
    w = torch.randint(-127, 128, (n_tiles, Q8_TILE_BYTES), dtype=torch.int16, device=device, generator=gen)
    w = w.to(torch.int8).view(torch.uint8)
    w[:, 0:512] = (torch.randn(n_tiles, 256, device=device, generator=gen) * 0.02).abs().to(torch.bfloat16).view(torch.uint8)
    return w.reshape(-1)


def pack_projections(layer: dict, shapes: dict) -> dict:
    """One layer's q4 projections in the tensor-core GEMM's packed layout (a load-time
    step); shapes maps each projection to its (n_tile_rows, k_tiles)."""
    return {k: ops.q4_gemm_pack(layer[k], *shape) for k, shape in shapes.items()}


class Q4Decoder:
    """Resident weights, KV cache and buffers for batched decode; `step()` is graph-capturable."""

    def __init__(self, cfg: DecoderConfig, batch: int, ctx_max: int, device=None, seed: int = 0,
                 weights: dict | None = None, gemm_min_batch: int = 9, pack_gemm: bool = True):
        self.cfg = cfg
        self.batch = batch
        self.ctx_max = ctx_max
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        c = cfg
        self.kt_h = c.hidden // TILE_K
        self.kt_q = c.n_heads * c.head_dim // TILE_K
        self.kt_i = c.intermediate // TILE_K
        self.nt_qkv = c.qkv_rows // TILE_ROWS
        self.nt_h = c.hidden // TILE_ROWS
        self.nt_i = c.intermediate // TILE_ROWS
        self.nt_v = c.vocab // TILE_ROWS
        if weights is None:
            weights = self._synthetic(seed)
        self.w = weights
        # KV cache per layer: [B][Hkv][ctx_max][D] bf16
        kv_shape = (batch, c.n_kv_heads, ctx_max, c.head_dim)
        self.k_cache = [torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev) for _ in range(c.n_layers)]
        self.v_cache = [torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev) for _ in range(c.n_layers)]
        # activations
        self.x_in = torch.zeros(batch, c.hidden, dtype=torch.float32, device=dev)
        self.resid = torch.zeros(batch, c.hidden, dtype=torch.float32, device=dev)
        self.xn = torch.zeros(batch, c.hidden, dtype=torch.bfloat16, device=dev)
        self.qkv = torch.zeros(batch, c.qkv_rows, dtype=torch.float32, device=dev)
        self.attn = torch.zeros(batch, c.n_heads * c.head_dim, dtype=torch.bfloat16, device=dev)
        self.h = torch.zeros(batch, c.intermediate, dtype=torch.bfloat16, device=dev)
        self.logits = torch.zeros(batch, c.vocab, dtype=torch.float32, device=dev)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        ws = ops.gqa_decode_workspace_bytes(batch, c.n_heads, c.n_kv_heads, c.head_dim, ctx_max)
        self.attn_ws = torch.empty(max(ws, 1), dtype=torch.uint8, device=dev)
        # batches of gemm_min_batch and more run the projections on the tcgen05 GEMM
        self.use_gemm = batch >= gemm_min_batch
        if self.use_gemm:
            nbytes = ops.gemm_workspace_bytes(batch, max(self.kt_h, self.kt_q, self.kt_i))
            self.gemm_ws_raw = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
            off = (256 - self.gemm_ws_raw.data_ptr() % 256) % 256
            self.gemm_ws = self.gemm_ws_raw[off:off + nbytes]
        # the GEMM's projections repacked once (b2_q4_gemm_pack): A is dequantised into TMEM
        self.packed = self.use_gemm and pack_gemm
        shapes = {"qkv": (self.nt_qkv, self.kt_h), "o": (self.nt_h, self.kt_q), "gate": (self.nt_i, self.kt_h),
                  "up": (self.nt_i, self.kt_h), "down": (self.nt_h, self.kt_i)}
        self.wg = ([pack_projections(L, shapes) if self.packed else L for L in self.w["layers"]]
                   if self.use_gemm else None)
        # the q8 lm_head on the tensor cores too (one pass for the whole batch)
        self.lm_packed = ops.q8_gemm_pack(self.w["lm_head"], self.nt_v, self.kt_h) if self.packed else None

    def _synthetic(self, seed: int) -> dict:
        c, dev = self.cfg, self.device
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        layers = []
        for _ in range(c.n_layers):
            layers.append({
                "qkv": synth_q4(self.nt_qkv * self.kt_h, g, dev),
                "o": synth_q4(self.nt_h * self.kt_q, g, dev),
                "gate": synth_q4(self.nt_i * self.kt_h, g, dev),
                "up": synth_q4(self.nt_i * self.kt_h, g, dev),
                "down": synth_q4(self.nt_h * self.kt_i, g, dev),
                # RMSNorm weights N(1, 0.1), non-uniform (granite_rmsnorm.py:130-133)
                "attn_norm": (1.0 + 0.1 * torch.randn(c.hidden, device=dev, generator=g)).to(torch.bfloat16),
                "mlp_norm": (1.0 + 0.1 * torch.randn(c.hidden, device=dev, generator=g)).to(torch.bfloat16),
            })
        return {"layers": layers,
                "final_norm": (1.0 + 0.1 * torch.randn(c.hidden, device=dev, generator=g)).to(torch.bfloat16),
                "lm_head": synth_q8(self.nt_v * self.kt_h, g, dev)}

    def step(self, prefetch: bool = True) -> torch.Tensor:
        """One decode step: x_in (fp32 [B, hidden]) at positions `pos` -> logits (fp32 [B, vocab]).

        Appends each layer's k/v at `pos`; the caller advances `pos` between steps
        (with an ordinary stream operation, so that pos and the cache rows before it
        are final when the step's kernels launch: attention reads them before its
        wait on the preceding kernel).
        """
        c = self.cfg
        d = c.head_dim
        qd = c.n_heads * d
        kd = c.n_kv_heads * d
        self.resid.copy_(self.x_in)
        if self.use_gemm:
            return self._step_gemm()
        for li, L in enumerate(self.w["layers"]):
            ops.gemv_rmsnorm(L["qkv"], self.nt_qkv, self.kt_h, self.resid, L["attn_norm"], c.rms_eps, out=self.qkv,
                             prefetch=prefetch)
            ops.gqa_decode(self.qkv[:, :qd], self.qkv[:, qd:qd + kd], self.qkv[:, qd + kd:],
                           self.k_cache[li], self.v_cache[li], self.pos, n_q_heads=c.n_heads,
                           n_kv_heads=c.n_kv_heads, theta=c.rope_theta, scale=d ** -0.5, max_len=self.ctx_max,
                           out=self.attn, workspace=self.attn_ws, prefetch_kv=prefetch)
            ops.q4_gemv(L["o"], self.nt_h, self.kt_q, self.attn, out=self.resid, accumulate=True, prefetch=prefetch)
            ops.swiglu_gemv_rmsnorm(L["gate"], L["up"], self.nt_i, self.kt_h, self.resid, L["mlp_norm"], c.rms_eps,
                                    out=self.h, prefetch=prefetch)
            ops.q4_gemv(L["down"], self.nt_h, self.kt_i, self.h, out=self.resid, accumulate=True, prefetch=prefetch)
        ops.gemv_rmsnorm(self.w["lm_head"], self.nt_v, self.kt_h, self.resid, self.w["final_norm"], c.rms_eps,
                         out=self.logits, prefetch=prefetch, q8=True)
        return self.logits

    def _step_gemm(self) -> torch.Tensor:
        """Large-batch step: tcgen05 GEMMs for every projection (packed weights, A in TMEM),
        RMSNorm fused into their x pre-pass."""
        c = self.cfg
        d = c.head_dim
        qd, kd = c.n_heads * d, c.n_kv_heads * d
        ws = self.gemm_ws
        pk = self.packed
        for li, L in enumerate(self.w["layers"]):
            G = self.wg[li]
            # RMSNorm fused into the GEMMs' x pre-pass; weights stream before each PDL wait
            ops.q4_gemm(G["qkv"], self.nt_qkv, self.kt_h, self.resid, out=self.qkv, workspace=ws, prefetch=True,
                        norm_w=L["attn_norm"], eps=c.rms_eps, packed=pk)
            ops.gqa_decode(self.qkv[:, :qd], self.qkv[:, qd:qd + kd], self.qkv[:, qd + kd:],
                           self.k_cache[li], self.v_cache[li], self.pos, n_q_heads=c.n_heads,
                           n_kv_heads=c.n_kv_heads, theta=c.rope_theta, scale=d ** -0.5, max_len=self.ctx_max,
                           out=self.attn, workspace=self.attn_ws, prefetch_kv=True)
            ops.q4_gemm(G["o"], self.nt_h, self.kt_q, self.attn, out=self.resid, accumulate=True, workspace=ws,
                        prefetch=True, packed=pk)
            ops.q4_swiglu_gemm(G["gate"], G["up"], self.nt_i, self.kt_h, self.resid, out=self.h, workspace=ws,
                               prefetch=True, norm_w=L["mlp_norm"], eps=c.rms_eps, packed=pk)
            ops.q4_gemm(G["down"], self.nt_h, self.kt_i, self.h, out=self.resid, accumulate=True, workspace=ws,
                        prefetch=True, packed=pk)
        self.lm_head()
        return self.logits

    def lm_head(self) -> torch.Tensor:
        """logits = lm_head(rmsnorm(resid)): the q8 tensor-core GEMM on the packed head at
        GEMM batches, else the q8 GEMV (RMSNorm fused either way)."""
        c = self.cfg
        if self.lm_packed is not None:
            return ops.q8_gemm(self.lm_packed, self.nt_v, self.kt_h, self.resid, out=self.logits,
                               workspace=self.gemm_ws, prefetch=True, norm_w=self.w["final_norm"], eps=c.rms_eps)
        return ops.gemv_rmsnorm(self.w["lm_head"], self.nt_v, self.kt_h, self.resid, self.w["final_norm"],
                                c.rms_eps, out=self.logits, q8=True)

    def capture(self) -> torch.cuda.CUDAGraph:
        """The step as one CUDA graph (warm once outside the capture first)."""
        fn = self.step
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g

    def bytes_per_step(self, lengths) -> int:
        """Algorithmic HBM bytes of one step: weights + KV read (+ new token written)."""
        wb = self.cfg.weight_bytes()
        kv = sum(int(n) for n in lengths) * self.cfg.n_kv_heads * self.cfg.head_dim * 2 * 2 * self.cfg.n_layers
        return wb["layers"] + wb["lm_head"] + kv


def tokens_per_second(ms_per_step: float, batch: int) -> float:
    return batch / (ms_per_step * 1e-3) if ms_per_step > 0 else math.nan
