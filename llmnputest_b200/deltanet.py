"""One gated DeltaNet (linear-attention) layer half for batched decode.

The token mixer of Qwen3.5's linear-attention layers (transformers 5.5.0
`Qwen3_5GatedDeltaNet.forward`, models/qwen3_5/modeling_qwen3_5.py:422-533, run
by the reference in float32: reference/from_q4nx.py:140-171) with its input
RMSNorm and residual add (`Qwen3_5DecoderLayer.forward`, :744-785):

    resid += out_proj(gated_delta_step(in_proj(rmsnorm(resid))))

as three launches on resident q4nx weights.  in_proj is ONE q4nx weight whose
output rows are q | k | v | z | b | a (transformers' in_proj_qkv, in_proj_z,
in_proj_b and in_proj_a stacked, padded to whole 32-row tiles), so the step
kernel reads its four inputs as column slices of one fp32 projection output.
Batches below `gemm_min_batch` use the GEMV with the RMSNorm fused into its input;
larger batches run RMSNorm and the tcgen05 GEMM.
"""

from __future__ import annotations

import torch

from . import ops
from .decode import synth_q4
from .format import TILE_K, TILE_ROWS

HEAD_DIM = ops.DELTA_HEAD_DIM


class DeltaNetLayer:
    """Resident weights and states of one linear-attention layer; `step()` is graph-capturable."""

    def __init__(self, hidden: int, n_k_heads: int, n_v_heads: int, batch: int, device=None, seed: int = 0,
                 weights: dict | None = None, eps: float = 1e-6, gemm_min_batch: int = 9, *, ops_impl=None,
                 cols: tuple[int, int] | None = None, n_in_tile_rows: int | None = None):
        """cols / n_in_tile_rows: the columns of b and a in the in_proj output and its tile-row
        count, when the in_proj is not the plain q|k|v|z|b|a stack of these heads (a
        tensor-parallel shard, llmnputest_b200.tp).  ops_impl: the op implementation (default
        the GPU path; host-logic tests pass another)."""
        if hidden % TILE_K or (n_v_heads * HEAD_DIM) % TILE_K:
            raise ValueError("hidden and n_v_heads*128 must be multiples of 256 (whole K-tiles)")
        self.ops = ops_impl if ops_impl is not None else ops
        self.hidden, self.nk, self.nv, self.batch, self.eps = hidden, n_k_heads, n_v_heads, batch, eps
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        d = HEAD_DIM
        self.conv_dim = (2 * n_k_heads + n_v_heads) * d
        # column offsets of q|k|v, z, b, a in the in_proj output
        self.c_z = self.conv_dim
        self.c_b = self.c_z + n_v_heads * d
        self.c_a = self.c_b + n_v_heads
        n_rows = self.c_a + n_v_heads
        self.nt_in = -(-n_rows // TILE_ROWS)
        # in_proj_b / in_proj_a as a dense fp32 matrix [2*nv][hidden] (a q4nx file stores them
        # as plain bf16, not tiles): the q4 in_proj is then q|k|v|z only, and b|a follow it
        self.ba_dense = weights is not None and "ba_dense" in weights
        if self.ba_dense:
            if cols is not None:
                raise ValueError("a tensor-parallel shard keeps b|a as tile-rows, not ba_dense")
            self.nt_in = (self.c_z + n_v_heads * d) // TILE_ROWS
            self.c_b = self.nt_in * TILE_ROWS
            self.c_a = self.c_b + n_v_heads
        if cols is not None:
            self.c_b, self.c_a = cols
            self.nt_in = n_in_tile_rows
        self.kt_h = hidden // TILE_K
        self.nt_h = hidden // TILE_ROWS
        self.kt_v = n_v_heads * d // TILE_K
        self.w = weights if weights is not None else self._synthetic(seed)
        dev = self.device
        self.conv_state = torch.zeros(batch, self.conv_dim, 4, dtype=torch.float32, device=dev)
        self.state = torch.zeros(batch, n_v_heads, d, d, dtype=torch.float32, device=dev)
        self.xn = torch.zeros(batch, hidden, dtype=torch.bfloat16, device=dev)
        self.proj = torch.zeros(batch, max(self.nt_in * TILE_ROWS, self.c_a + n_v_heads), dtype=torch.float32,
                                device=dev)
        if self.ba_dense:
            self.w_ba_t = self.w["ba_dense"].t().contiguous()  # [hidden][2*nv]
            self.xn_f = torch.zeros(batch, hidden, dtype=torch.float32, device=dev)
            self.ba_out = torch.zeros(batch, 2 * n_v_heads, dtype=torch.float32, device=dev)
        self.h = torch.zeros(batch, n_v_heads * d, dtype=torch.bfloat16, device=dev)
        self.use_gemm = batch >= gemm_min_batch
        if self.use_gemm:
            nbytes = self.ops.gemm_workspace_bytes(batch, max(self.kt_h, self.kt_v))
            self._ws_raw = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
            off = (256 - self._ws_raw.data_ptr() % 256) % 256
            self.gemm_ws = self._ws_raw[off:off + nbytes]
            # the projections repacked once for the tensor-core GEMM (A dequantised into TMEM)
            self.wg = {"in_proj": self.ops.q4_gemm_pack(self.w["in_proj"], self.nt_in, self.kt_h),
                       "out_proj": self.ops.q4_gemm_pack(self.w["out_proj"], self.nt_h, self.kt_v)}

    def _synthetic(self, seed: int) -> dict:
        dev, d = self.device, HEAD_DIM
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        return {
            "in_proj": synth_q4(self.nt_in * self.kt_h, g, dev),
            "out_proj": synth_q4(self.nt_h * self.kt_v, g, dev),
            "conv_w": 0.5 * torch.randn(self.conv_dim, 4, device=dev, generator=g),
            "A_log": torch.log(1.0 + 15.0 * torch.rand(self.nv, device=dev, generator=g)),
            "dt_bias": torch.randn(self.nv, device=dev, generator=g),
            "norm_w": 1.0 + 0.1 * torch.randn(d, device=dev, generator=g),
            # input RMSNorm weight N(1, 0.1), as the decoders' norms
            "input_norm": (1.0 + 0.1 * torch.randn(self.hidden, device=dev, generator=g)).to(torch.bfloat16),
        }

    def bytes_per_step(self) -> int:
        """Algorithmic HBM bytes of one step: both weights' tiles, the states read and
        written, the projection output written and read, the residual read and written."""
        d, b = HEAD_DIM, self.batch
        w = self.w["in_proj"].numel() + self.w["out_proj"].numel()
        if self.ba_dense:
            w += self.w["ba_dense"].numel() * 4
        states = 2 * 4 * b * (self.nv * d * d + self.conv_dim * 4)
        proj = 2 * 4 * b * self.nt_in * TILE_ROWS
        return w + states + proj + 2 * b * self.nv * d + 2 * 4 * b * self.hidden

    def step(self, resid: torch.Tensor, prefetch_state: bool = False) -> torch.Tensor:
        """resid (fp32 [B, hidden]) += the layer's token mixer; returns resid.

        prefetch_state=True lets the step kernel read its states before its wait on the
        preceding kernel.  The projections launch their dependents early, so this is only
        correct when a non-PDL stream operation or a graph boundary separates this
        layer's consecutive steps (the state's previous write is that earlier step)."""
        self.mix(resid, prefetch_state)
        self.out_proj(self.h, resid, accumulate=True)
        return resid

    def out_proj(self, h: torch.Tensor, out: torch.Tensor, accumulate: bool) -> torch.Tensor:
        """out (fp32 [B, hidden]) = (or +=) out_proj h."""
        ops, w = self.ops, self.w
        if self.use_gemm:
            return ops.q4_gemm(self.wg["out_proj"], self.nt_h, self.kt_v, h, out=out, accumulate=accumulate,
                               workspace=self.gemm_ws, prefetch=True, packed=True)
        return ops.q4_gemv(w["out_proj"], self.nt_h, self.kt_v, h, out=out, accumulate=accumulate, prefetch=True)

    def mix(self, resid: torch.Tensor, prefetch_state: bool = False) -> torch.Tensor:
        """Input RMSNorm, in_proj and the gated delta step; returns the bf16 [B, nv*128] step output."""
        ops, w, nv = self.ops, self.w, self.nv
        q4_out = self.proj[:, :self.nt_in * TILE_ROWS]  # the whole buffer unless b|a follow the q4 rows
        if self.use_gemm:  # RMSNorm fused into the GEMM's x pre-pass
            ops.q4_gemm(self.wg["in_proj"], self.nt_in, self.kt_h, resid, out=q4_out, workspace=self.gemm_ws,
                        prefetch=True, norm_w=w["input_norm"], eps=self.eps, packed=True)
        else:
            ops.gemv_rmsnorm(w["in_proj"], self.nt_in, self.kt_h, resid, w["input_norm"], self.eps, out=q4_out,
                             prefetch=True)
        if self.ba_dense:  # b|a = bf16(rmsnorm(x)) W_ba^T in fp32 (a plain library GEMM of 2*nv columns)
            ops.rmsnorm(resid, w["input_norm"], self.eps, out=self.xn)
            self.xn_f.copy_(self.xn)
            torch.mm(self.xn_f, self.w_ba_t, out=self.ba_out)
            self.proj[:, self.c_b:self.c_a + nv].copy_(self.ba_out)
        p = self.proj
        ops.gated_delta_step(p[:, :self.c_z], p[:, self.c_z:self.c_b], p[:, self.c_b:self.c_a],
                             p[:, self.c_a:self.c_a + nv], self.conv_state, w["conv_w"], w["A_log"], w["dt_bias"],
                             w["norm_w"], self.state, self.nk, nv, eps=self.eps, out=self.h,
                             prefetch_state=prefetch_state)
        return self.h
