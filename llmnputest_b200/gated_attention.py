"""One Qwen3.5 gated full-attention layer half for batched decode.

The token mixer of Qwen3.5's full-attention layers (transformers 5.5.0
`Qwen3_5Attention.forward`, models/qwen3_5/modeling_qwen3_5.py:647-692, run by the
reference in float32: reference/from_q4nx.py:140-171) with its input RMSNorm and
residual add (`Qwen3_5DecoderLayer.forward`, :744-785):

    resid += o_proj(gated_attn_decode(in_proj(rmsnorm(resid))))

as three launches on resident q4nx weights.  in_proj is ONE q4nx weight whose output
rows are q_proj's (per q head: 256 q rows then 256 gate rows, transformers' layout),
then k_proj's and v_proj's (256 rows per kv head): every head is whole tile-rows.
Batches below `gemm_min_batch` use the GEMV with the RMSNorm fused into its input;
larger batches run RMSNorm and the tcgen05 GEMM.
"""

from __future__ import annotations

import torch

from . import ops
from .decode import synth_q4
from .format import TILE_K, TILE_ROWS

HEAD_DIM = ops.GATED_HEAD_DIM


def rope_inv_freq(rot_dim: int, theta: float, device=None) -> torch.Tensor:
    """Qwen3_5TextRotaryEmbedding's default frequencies (modeling_qwen3_5.py:106-137) in fp32."""
    e = torch.arange(0, rot_dim, 2, dtype=torch.int64, device=device).to(torch.float32) / rot_dim
    return (1.0 / (theta ** e)).contiguous()


class GatedAttentionLayer:
    """Resident weights and KV cache of one gated full-attention layer; `step()` is graph-capturable."""

    def __init__(self, hidden: int, n_q_heads: int, n_kv_heads: int, batch: int, ctx_max: int, device=None,
                 seed: int = 0, weights: dict | None = None, eps: float = 1e-6, rot_dim: int = 64,
                 theta: float = 10000000.0, gemm_min_batch: int = 9, *, ops_impl=None):
        if hidden % TILE_K:
            raise ValueError("hidden must be a multiple of 256 (whole K-tiles)")
        self.ops = ops_impl if ops_impl is not None else ops
        self.hidden, self.nq, self.nkv, self.batch, self.ctx_max, self.eps = (hidden, n_q_heads, n_kv_heads, batch,
                                                                             ctx_max, eps)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        d = HEAD_DIM
        self.c_k = n_q_heads * 2 * d            # first k column of the in_proj output
        self.c_v = self.c_k + n_kv_heads * d
        self.nt_in = (self.c_v + n_kv_heads * d) // TILE_ROWS
        self.kt_h = hidden // TILE_K
        self.nt_h = hidden // TILE_ROWS
        self.kt_o = n_q_heads * d // TILE_K
        self.rot_dim, self.theta = rot_dim, theta
        self.w = weights if weights is not None else self._synthetic(seed)
        dev = self.device
        self.k_cache = torch.zeros(batch, n_kv_heads, ctx_max, d, dtype=torch.bfloat16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.proj = torch.zeros(batch, self.nt_in * TILE_ROWS, dtype=torch.float32, device=dev)
        self.xn = torch.zeros(batch, hidden, dtype=torch.bfloat16, device=dev)
        self.attn = torch.zeros(batch, n_q_heads * d, dtype=torch.bfloat16, device=dev)
        ws = self.ops.gated_attn_workspace_bytes(batch, n_q_heads, n_kv_heads, ctx_max)
        self.attn_ws = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
        self.use_gemm = batch >= gemm_min_batch
        if self.use_gemm:
            nbytes = self.ops.gemm_workspace_bytes(batch, max(self.kt_h, self.kt_o))
            self._ws_raw = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
            off = (256 - self._ws_raw.data_ptr() % 256) % 256
            self.gemm_ws = self._ws_raw[off:off + nbytes]
            # the projections repacked once for the tensor-core GEMM (A dequantised into TMEM)
            self.wg = {"in_proj": self.ops.q4_gemm_pack(self.w["in_proj"], self.nt_in, self.kt_h),
                       "o_proj": self.ops.q4_gemm_pack(self.w["o_proj"], self.nt_h, self.kt_o)}

    def _synthetic(self, seed: int) -> dict:
        dev, d = self.device, HEAD_DIM
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        return {
            "in_proj": synth_q4(self.nt_in * self.kt_h, g, dev),
            "o_proj": synth_q4(self.nt_h * self.kt_o, g, dev),
            "q_norm_w": 0.1 * torch.randn(d, device=dev, generator=g),
            "k_norm_w": 0.1 * torch.randn(d, device=dev, generator=g),
            "inv_freq": rope_inv_freq(self.rot_dim, self.theta, dev),
            "input_norm": (1.0 + 0.1 * torch.randn(self.hidden, device=dev, generator=g)).to(torch.bfloat16),
        }

    def step(self, resid: torch.Tensor) -> torch.Tensor:
        """resid (fp32 [B, hidden]) += the layer's token mixer at positions `pos` (the new
        k/v rows are appended there; the caller advances `pos` between steps)."""
        self.mix(resid)
        self.o_proj(self.attn, resid, accumulate=True)
        return resid

    def o_proj(self, a: torch.Tensor, out: torch.Tensor, accumulate: bool) -> torch.Tensor:
        ops, w = self.ops, self.w
        if self.use_gemm:
            return ops.q4_gemm(self.wg["o_proj"], self.nt_h, self.kt_o, a, out=out, accumulate=accumulate,
                               workspace=self.gemm_ws, prefetch=True, packed=True)
        return ops.q4_gemv(w["o_proj"], self.nt_h, self.kt_o, a, out=out, accumulate=accumulate, prefetch=True)

    def mix(self, resid: torch.Tensor) -> torch.Tensor:
        """Input RMSNorm, in_proj and the gated attention; returns the bf16 [B, nq*256] output."""
        ops, w = self.ops, self.w
        if self.use_gemm:  # RMSNorm fused into the GEMM's x pre-pass
            ops.q4_gemm(self.wg["in_proj"], self.nt_in, self.kt_h, resid, out=self.proj, workspace=self.gemm_ws,
                        prefetch=True, norm_w=w["input_norm"], eps=self.eps, packed=True)
        else:
            ops.gemv_rmsnorm(w["in_proj"], self.nt_in, self.kt_h, resid, w["input_norm"], self.eps, out=self.proj,
                             prefetch=True)
        p = self.proj
        ops.gated_attn_decode(p[:, :self.c_k], p[:, self.c_k:self.c_v], p[:, self.c_v:], w["q_norm_w"],
                              w["k_norm_w"], w["inv_freq"], self.k_cache, self.v_cache, self.pos, self.nq, self.nkv,
                              eps=self.eps, out=self.attn, workspace=self.attn_ws)
        return self.attn
