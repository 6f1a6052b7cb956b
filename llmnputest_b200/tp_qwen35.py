"""Tensor-parallel decode of a Qwen3.5 (config 5) stack, one process per GPU.

Per layer, whole tiles everywhere:
  gated DeltaNet   by k head (`tp.DeltaNetShardPlan`): local states, one all-reduce
                   of the out_proj partials;
  gated attention  by kv head (`tp.GatedAttnShardPlan`) while the kv heads divide
                   over the ranks (config 5: 2 kv heads, W <= 2); beyond that the layer
                   runs replicated on every rank (full heads, no collective);
  SwiGLU MLP       gate/up by the intermediate rows of whole 256-wide K-tiles of down,
                   down by those K-tiles, one all-reduce.  Config 5's 3584 = 14 K-tiles
                   split unevenly over 4 or 8 ranks (e.g. 4, 4, 3, 3): partial sums make
                   an uneven split exact;
  q8 lm_head       by vocab tile-rows, the fp32 logits all-gathered (
                   248320 rows = 7760 tile-rows, even over 1/2/4/8 ranks).
The residual stream is replicated (fp32 [B, hidden] on every rank).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .format import Q4_TILE_BYTES, Q8_TILE_BYTES, TILE_K, TILE_ROWS
from .qwen35_decode import Qwen35Config
from .tp import (DeltaNetShardPlan, GatedAttnShardPlan, TPDeltaNetLayer, TPGatedAttentionLayer, shard_deltanet,
                 shard_gated_attention, take_k_tiles, take_tile_rows)


def split_even(n: int, world: int, rank: int) -> range:
    """Rank `rank`'s share of n units, the first n % world ranks taking one more."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


@dataclass(frozen=True)
class Qwen35ShardPlan:
    cfg: Qwen35Config
    world: int
    rank: int

    def __post_init__(self):
        if (self.cfg.vocab // TILE_ROWS) % self.world:
            raise ValueError("vocab tile-rows do not split evenly (the logits all-gather needs equal shares)")
        if self.cfg.intermediate // TILE_K < self.world:
            raise ValueError("fewer intermediate K-tiles than ranks")

    def delta(self) -> DeltaNetShardPlan:
        c = self.cfg
        return DeltaNetShardPlan(c.hidden, c.n_k_heads, c.n_v_heads, self.world, self.rank)

    def attn(self) -> GatedAttnShardPlan | None:
        """The kv-head plan, or None where the layer runs replicated (kv heads < ranks)."""
        c = self.cfg
        if c.n_kv_heads % self.world:
            return None
        return GatedAttnShardPlan(c.hidden, c.n_q_heads, c.n_kv_heads, self.world, self.rank)

    def ffn_k_tiles(self) -> range:
        return split_even(self.cfg.intermediate // TILE_K, self.world, self.rank)

    def ffn_tile_rows(self) -> list[int]:
        per = TILE_K // TILE_ROWS  # gate/up tile-rows per down K-tile
        return [r for kt in self.ffn_k_tiles() for r in range(kt * per, (kt + 1) * per)]

    def vocab_tile_rows(self) -> range:
        return split_even(self.cfg.vocab // TILE_ROWS, self.world, self.rank)


def shard_qwen35(full: dict, plan: Qwen35ShardPlan) -> dict:
    """One rank's slice of a full Qwen35Decoder weight dict."""
    c = plan.cfg
    kt_h, kt_i, nt_h = c.hidden // TILE_K, c.intermediate // TILE_K, c.hidden // TILE_ROWS
    ks = plan.ffn_k_tiles()
    layers = []
    for kind, L in zip(c.layer_types, full["layers"]):
        if kind == "linear_attention":
            mixer = shard_deltanet(L["mixer"], plan.delta())
        else:
            ap = plan.attn()
            mixer = L["mixer"] if ap is None else shard_gated_attention(L["mixer"], ap)
        layers.append({"mixer": mixer,
                       "gate": take_tile_rows(L["gate"], kt_h, Q4_TILE_BYTES, plan.ffn_tile_rows()),
                       "up": take_tile_rows(L["up"], kt_h, Q4_TILE_BYTES, plan.ffn_tile_rows()),
                       "down": take_k_tiles(L["down"], nt_h, kt_i, Q4_TILE_BYTES, ks),
                       "post_norm": L["post_norm"]})
    return {"layers": layers, "final_norm": full["final_norm"],
            "lm_head": take_tile_rows(full["lm_head"], kt_h, Q8_TILE_BYTES, plan.vocab_tile_rows())}


class TPQwen35Decoder:
    """This rank's part of the Qwen3.5 step; collectives on the default process group."""

    def __init__(self, cfg: Qwen35Config, batch: int, ctx_max: int, shard: dict, plan: Qwen35ShardPlan, device=None,
                 ops=None, gemm_min_batch: int = 9):
        if ops is None:
            from . import ops  # the GPU path; host-logic tests pass another implementation
        from .gated_attention import GatedAttentionLayer
        self.ops, self.cfg, self.plan, self.batch = ops, cfg, plan, batch
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        c, dev, W = cfg, self.device, plan.world
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.mixers = []
        for kind, L in zip(c.layer_types, shard["layers"]):
            if kind == "linear_attention":
                m = TPDeltaNetLayer(plan.delta(), batch, L["mixer"], device=dev, eps=c.eps, ops=ops,
                                    gemm_min_batch=gemm_min_batch)
            elif plan.attn() is not None:
                m = TPGatedAttentionLayer(plan.attn(), batch, ctx_max, L["mixer"], device=dev, eps=c.eps, ops=ops,
                                          gemm_min_batch=gemm_min_batch)
                m.layer.pos = self.pos
            else:
                m = GatedAttentionLayer(c.hidden, c.n_q_heads, c.n_kv_heads, batch, ctx_max, device=dev,
                                        weights=L["mixer"], eps=c.eps, rot_dim=c.rot_dim, theta=c.rope_theta,
                                        gemm_min_batch=gemm_min_batch, ops_impl=ops)
                m.pos = self.pos
            self.mixers.append(m)
        self.w = shard
        self.kt_h, self.nt_h = c.hidden // TILE_K, c.hidden // TILE_ROWS
        self.kt_i_local = len(plan.ffn_k_tiles())
        self.nt_i_local = len(plan.ffn_tile_rows())
        self.nt_v_local = len(plan.vocab_tile_rows())
        self.x_in = torch.zeros(batch, c.hidden, dtype=torch.float32, device=dev)
        self.resid = torch.zeros(batch, c.hidden, dtype=torch.float32, device=dev)
        self.h = torch.zeros(batch, self.nt_i_local * TILE_ROWS, dtype=torch.bfloat16, device=dev)
        self.xn = torch.zeros(batch, c.hidden, dtype=torch.bfloat16, device=dev)
        self.use_gemm = batch >= gemm_min_batch
        if self.use_gemm:
            nbytes = ops.gemm_workspace_bytes(batch, max(self.kt_h, self.kt_i_local))
            self._ws_raw = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
            off = (256 - self._ws_raw.data_ptr() % 256) % 256
            self.gemm_ws = self._ws_raw[off:off + nbytes]
            # this rank's MLP shards repacked once for the tensor-core GEMM (A dequantised into TMEM)
            self.wg = [{"gate": ops.q4_gemm_pack(L["gate"], self.nt_i_local, self.kt_h),
                        "up": ops.q4_gemm_pack(L["up"], self.nt_i_local, self.kt_h),
                        "down": ops.q4_gemm_pack(L["down"], self.nt_h, self.kt_i_local)} for L in self.w["layers"]]
            self.lm_packed = ops.q8_gemm_pack(self.w["lm_head"], self.nt_v_local, self.kt_h)
        self.down = torch.zeros(batch, c.hidden, dtype=torch.float32, device=dev)
        self.logits_local = torch.zeros(batch, self.nt_v_local * TILE_ROWS, dtype=torch.float32, device=dev)
        self.logits_all = torch.zeros(W * batch, self.nt_v_local * TILE_ROWS, dtype=torch.float32, device=dev)
        self.logits = torch.zeros(batch, c.vocab, dtype=torch.float32, device=dev)

    def step(self) -> torch.Tensor:
        """One decode step: x_in at positions `pos` -> logits [B, vocab] on every rank (GEMVs
        below gemm_min_batch, tcgen05 GEMMs from it, the lm_head included)."""
        ops, c, W = self.ops, self.cfg, self.plan.world
        self.resid.copy_(self.x_in)
        for li, (m, L) in enumerate(zip(self.mixers, self.w["layers"])):
            m.step(self.resid)
            if self.use_gemm:  # RMSNorm fused into the SwiGLU GEMM's x pre-pass
                G = self.wg[li]
                ops.q4_swiglu_gemm(G["gate"], G["up"], self.nt_i_local, self.kt_h, self.resid, out=self.h,
                                   workspace=self.gemm_ws, prefetch=True, norm_w=L["post_norm"], eps=c.eps,
                                   packed=True)
                ops.q4_gemm(G["down"], self.nt_h, self.kt_i_local, self.h, out=self.down, workspace=self.gemm_ws,
                            prefetch=True, packed=True)
            else:
                ops.swiglu_gemv_rmsnorm(L["gate"], L["up"], self.nt_i_local, self.kt_h, self.resid, L["post_norm"],
                                        c.eps, out=self.h, prefetch=True)
                ops.q4_gemv(L["down"], self.nt_h, self.kt_i_local, self.h, out=self.down, prefetch=True)
            if W > 1:
                dist.all_reduce(self.down)
            self.resid.add_(self.down)
        if self.use_gemm:  # the q8 lm_head shard on the tensor cores
            ops.q8_gemm(self.lm_packed, self.nt_v_local, self.kt_h, self.resid, out=self.logits_local,
                        workspace=self.gemm_ws, prefetch=True, norm_w=self.w["final_norm"], eps=c.eps)
        else:
            ops.gemv_rmsnorm(self.w["lm_head"], self.nt_v_local, self.kt_h, self.resid, self.w["final_norm"], c.eps,
                             out=self.logits_local, prefetch=True, q8=True)
        if W > 1:
            dist.all_gather_into_tensor(self.logits_all, self.logits_local)
            self.logits.view(self.batch, W, -1).copy_(self.logits_all.view(W, self.batch, -1).permute(1, 0, 2))
        else:
            self.logits.copy_(self.logits_local)
        return self.logits
