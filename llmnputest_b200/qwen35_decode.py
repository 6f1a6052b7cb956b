"""Batched decode step of a Qwen3.5 (config 5) stack on resident q4nx weights.

Per layer, `Qwen3_5DecoderLayer.forward` (transformers 5.5.0,
models/qwen3_5/modeling_qwen3_5.py:744-785; the reference runs it in float32,
reference/from_q4nx.py:140-171):

    resid += token_mixer(input_layernorm(resid))        DeltaNetLayer | GatedAttentionLayer
    resid += down(silu(gate(x)) * up(x)),  x = post_attention_layernorm(resid)

then the final norm and the q8 lm_head.  The layer types follow the config
(three linear-attention layers, then one full-attention layer,
six times).  Batches below `gemm_min_batch` run the GEMVs with the norms fused into
their inputs; larger batches run RMSNorm and the tcgen05 GEMMs.  The lm_head is the
q8 GEMV in passes of 16 tokens.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import ops
from .decode import synth_q4, synth_q8
from .deltanet import DeltaNetLayer
from .format import TILE_K, TILE_ROWS
from .gated_attention import GatedAttentionLayer


def _pattern(n_layers: int) -> list[str]:
    return ["full_attention" if i % 4 == 3 else "linear_attention" for i in range(n_layers)]


@dataclass(frozen=True)
class Qwen35Config:
    """Config 5's shapes: 24 layers of hidden 1024, 18 gated DeltaNet + 6 gated attention
    (8 q / 2 kv heads of 256, rotary over 64 dims), intermediate 3584, q8 lm_head 248320."""

    hidden: int = 1024
    n_layers: int = 24
    layer_types: tuple = field(default_factory=lambda: tuple(_pattern(24)))
    n_k_heads: int = 16   # linear attention (the model's config.json is not available: stated dims)
    n_v_heads: int = 16
    n_q_heads: int = 8    # gated full attention
    n_kv_heads: int = 2
    rot_dim: int = 64
    rope_theta: float = 10000000.0
    intermediate: int = 3584
    vocab: int = 248320
    eps: float = 1e-6


class Qwen35Decoder:
    """Resident weights, caches and buffers of a Qwen3.5 stack; `step()` is graph-capturable."""

    def __init__(self, cfg: Qwen35Config, batch: int, ctx_max: int, device=None, seed: int = 0,
                 weights: dict | None = None, gemm_min_batch: int = 9, ops_impl=None):
        self.ops = ops_impl if ops_impl is not None else ops
        self.cfg, self.batch, self.ctx_max = cfg, batch, ctx_max
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        c, dev = cfg, self.device
        self.kt_h, self.kt_i = c.hidden // TILE_K, c.intermediate // TILE_K
        self.nt_h, self.nt_i, self.nt_v = c.hidden // TILE_ROWS, c.intermediate // TILE_ROWS, c.vocab // TILE_ROWS
        w = weights if weights is not None else self._synthetic(seed)
        self.w = w
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.mixers = []
        for i, kind in enumerate(c.layer_types):
            lw = w["layers"][i]["mixer"]
            if kind == "linear_attention":
                m = DeltaNetLayer(c.hidden, c.n_k_heads, c.n_v_heads, batch, device=dev, weights=lw, eps=c.eps,
                                  gemm_min_batch=gemm_min_batch, ops_impl=self.ops)
            else:
                m = GatedAttentionLayer(c.hidden, c.n_q_heads, c.n_kv_heads, batch, ctx_max, device=dev,
                                        weights=lw, eps=c.eps, rot_dim=c.rot_dim, theta=c.rope_theta,
                                        gemm_min_batch=gemm_min_batch, ops_impl=self.ops)
                m.pos = self.pos  # one position per sequence for every attention layer
            self.mixers.append(m)
        self.x_in = torch.zeros(batch, c.hidden, dtype=torch.float32, device=dev)
        self.resid = torch.zeros(batch, c.hidden, dtype=torch.float32, device=dev)
        self.xn = torch.zeros(batch, c.hidden, dtype=torch.bfloat16, device=dev)
        self.h = torch.zeros(batch, c.intermediate, dtype=torch.bfloat16, device=dev)
        self.logits = torch.zeros(batch, c.vocab, dtype=torch.float32, device=dev)
        self.use_gemm = batch >= gemm_min_batch
        if self.use_gemm:
            nbytes = self.ops.gemm_workspace_bytes(batch, max(self.kt_h, self.kt_i))
            self._ws_raw = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
            off = (256 - self._ws_raw.data_ptr() % 256) % 256
            self.gemm_ws = self._ws_raw[off:off + nbytes]
            # the MLP projections repacked once for the tensor-core GEMM (A dequantised into TMEM)
            pk = self.ops.q4_gemm_pack
            self.wg = [{"gate": pk(L["gate"], self.nt_i, self.kt_h), "up": pk(L["up"], self.nt_i, self.kt_h),
                        "down": pk(L["down"], self.nt_h, self.kt_i)} for L in self.w["layers"]]
            self.lm_packed = self.ops.q8_gemm_pack(self.w["lm_head"], self.nt_v, self.kt_h)

    def _synthetic(self, seed: int) -> dict:
        c, dev = self.cfg, self.device
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        norm = lambda: (1.0 + 0.1 * torch.randn(c.hidden, device=dev, generator=g)).to(torch.bfloat16)
        layers = []
        for i, kind in enumerate(c.layer_types):
            if kind == "linear_attention":
                mixer = DeltaNetLayer(c.hidden, c.n_k_heads, c.n_v_heads, 1, device=dev, seed=seed * 131 + i,
                                      ops_impl=self.ops).w
            else:
                mixer = GatedAttentionLayer(c.hidden, c.n_q_heads, c.n_kv_heads, 1, 1, device=dev,
                                            seed=seed * 131 + i, rot_dim=c.rot_dim, theta=c.rope_theta,
                                            ops_impl=self.ops).w
            layers.append({"mixer": mixer,
                           "gate": synth_q4(self.nt_i * self.kt_h, g, dev),
                           "up": synth_q4(self.nt_i * self.kt_h, g, dev),
                           "down": synth_q4(self.nt_h * self.kt_i, g, dev),
                           "post_norm": norm()})
        return {"layers": layers, "final_norm": norm(), "lm_head": synth_q8(self.nt_v * self.kt_h, g, dev)}

    def step(self) -> torch.Tensor:
        """One decode step: x_in (fp32 [B, hidden]) at positions `pos` -> logits (fp32 [B, vocab]).
        The attention layers append their k/v at `pos`; the caller advances `pos` between
        steps with an ordinary stream operation."""
        ops, c = self.ops, self.cfg
        self.resid.copy_(self.x_in)
        for li, (m, L) in enumerate(zip(self.mixers, self.w["layers"])):
            m.step(self.resid)
            if self.use_gemm:  # RMSNorm fused into the SwiGLU GEMM's x pre-pass
                G = self.wg[li]
                ops.q4_swiglu_gemm(G["gate"], G["up"], self.nt_i, self.kt_h, self.resid, out=self.h,
                                   workspace=self.gemm_ws, prefetch=True, norm_w=L["post_norm"], eps=c.eps,
                                   packed=True)
                ops.q4_gemm(G["down"], self.nt_h, self.kt_i, self.h, out=self.resid, accumulate=True,
                            workspace=self.gemm_ws, prefetch=True, packed=True)
            else:
                ops.swiglu_gemv_rmsnorm(L["gate"], L["up"], self.nt_i, self.kt_h, self.resid, L["post_norm"],
                                        c.eps, out=self.h, prefetch=True)
                ops.q4_gemv(L["down"], self.nt_h, self.kt_i, self.h, out=self.resid, accumulate=True,
                            prefetch=True)
        if self.use_gemm:  # the q8 lm_head on the tensor cores, the whole batch in one pass
            ops.q8_gemm(self.lm_packed, self.nt_v, self.kt_h, self.resid, out=self.logits, workspace=self.gemm_ws,
                        prefetch=True, norm_w=self.w["final_norm"], eps=c.eps)
        else:
            ops.gemv_rmsnorm(self.w["lm_head"], self.nt_v, self.kt_h, self.resid, self.w["final_norm"], c.eps,
                             out=self.logits, prefetch=True, q8=True)
        return self.logits
