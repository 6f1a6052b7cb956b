"""Tensor-parallel decode over one node (NCCL over NVLink), one process per GPU.

Sharding follows the natural seams of the q4nx tiles (all cuts are whole tiles;
tile bytes are never modified):

  QKV + attention  by kv head: rank r owns kv heads [r*Hkv/W, (r+1)*Hkv/W) and
                   their q heads; its QKV weight is those heads' whole tile-rows
                   (q: grp*D rows per kv head, k and v: D rows each), and its KV
                   cache holds only its heads.  No collective.
  O                by input columns: rank r owns the columns of its own q heads, so
                   its attention output is its O input with no exchange.  Those
                   columns (640 or 320 at W = 4 or 8) cut 256-wide K-tiles, so the
                   shard is re-tiled by whole 32-column quantisation blocks (every
                   code and scale kept, the last K-tile zero-padded) and the input
                   row padded with zeros to match; the fp32 partial outputs are
                   all-reduced (sum) into the residual.
  FFN              gate/up by intermediate rows (I/W rows each), SwiGLU local;
                   down by whole K-tiles of the intermediate axis (I/W/256 per
                   rank), its fp32 partials all-reduced (sum) into the residual.
  lm_head          by vocab tile-rows; fp32 logits all-gathered.

ShardPlan and shard_weights are plain host logic (they run on CPU tensors too);
TPDecoder runs the step on the GPU.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .format import Q4_TILE_BYTES, Q8_TILE_BYTES, TILE_K, TILE_ROWS


@dataclass(frozen=True)
class ShardPlan:
    """Which rows / K-tiles / heads rank `rank` of `world` owns."""

    n_heads: int
    n_kv_heads: int
    head_dim: int
    hidden: int
    intermediate: int
    vocab: int
    world: int
    rank: int

    def __post_init__(self):
        w = self.world
        if self.n_kv_heads % w:
            raise ValueError(f"{self.n_kv_heads} kv heads do not split over {w} ranks")
        if self.hidden % (TILE_ROWS * w) or self.intermediate % (TILE_K * w):
            raise ValueError("hidden / intermediate do not split into whole tiles")
        if (self.vocab // TILE_ROWS) % w:
            raise ValueError("vocab tile-rows do not split evenly")

    @property
    def grp(self) -> int:
        return self.n_heads // self.n_kv_heads

    @property
    def kv_local(self) -> int:
        return self.n_kv_heads // self.world

    @property
    def q_local(self) -> int:
        return self.kv_local * self.grp

    def qkv_tile_rows(self) -> list[int]:
        """Tile-rows of the full [q | k | v] QKV weight that this rank owns, in its order q|k|v."""
        d, tpr = self.head_dim, self.head_dim // TILE_ROWS  # tile-rows per head
        kv0 = self.rank * self.kv_local
        q_rows = range(kv0 * self.grp * tpr, (kv0 + self.kv_local) * self.grp * tpr)
        k_base = self.n_heads * d // TILE_ROWS
        v_base = k_base + self.n_kv_heads * d // TILE_ROWS
        k_rows = range(k_base + kv0 * tpr, k_base + (kv0 + self.kv_local) * tpr)
        v_rows = range(v_base + kv0 * tpr, v_base + (kv0 + self.kv_local) * tpr)
        return list(q_rows) + list(k_rows) + list(v_rows)

    def row_range(self, n_rows: int) -> tuple[int, int]:
        per = n_rows // self.world
        return self.rank * per, (self.rank + 1) * per

    def o_k_range(self) -> tuple[int, int]:
        """Input columns of O this rank owns: its q heads' attention outputs."""
        w = self.q_local * self.head_dim
        return self.rank * w, (self.rank + 1) * w

    @property
    def o_k_tiles(self) -> int:
        """K-tiles of this rank's O shard (its columns re-tiled from column 0, zero-padded)."""
        return -(-self.q_local * self.head_dim // TILE_K)

    def ffn_tile_rows(self) -> range:
        return range(*self.row_range(self.intermediate // TILE_ROWS))

    def down_k_tiles(self) -> range:
        return range(*self.row_range(self.intermediate // TILE_K))

    def vocab_tile_rows(self) -> range:
        return range(*self.row_range(self.vocab // TILE_ROWS))


def take_tile_rows(tiles: torch.Tensor, k_tiles: int, tile_bytes: int, rows) -> torch.Tensor:
    """Gather whole tile-rows (each k_tiles*tile_bytes contiguous bytes) into a new contiguous buffer."""
    t = tiles.view(-1, k_tiles * tile_bytes)
    idx = torch.as_tensor(list(rows), dtype=torch.long, device=tiles.device)
    return t.index_select(0, idx).reshape(-1).contiguous()


def take_k_tiles(tiles: torch.Tensor, n_tile_rows: int, k_tiles: int, tile_bytes: int, ks) -> torch.Tensor:
    """Keep K-tiles `ks` of every tile-row: [n_t][k_t][tile] -> [n_t][len(ks)][tile]."""
    t = tiles.view(n_tile_rows, k_tiles, tile_bytes)
    idx = torch.as_tensor(list(ks), dtype=torch.long, device=tiles.device)
    return t.index_select(1, idx).reshape(-1).contiguous()


def take_k_blocks(tiles: torch.Tensor, n_tile_rows: int, k_tiles: int, k0: int, k1: int) -> torch.Tensor:
    """q4 columns [k0, k1) of every tile-row, re-tiled from column 0: [n_t][ceil((k1-k0)/256)][tile].

    k0 and k1 are multiples of the 32-wide quantisation block, so every block moves whole
    (its 32 d and 32 m entries and, per row block, its 256 nibble bytes) and every
    weight keeps its exact codes and scales; blocks past k1 in the last K-tile are zero
    (d = m = 0, codes 0: weight 0).  In a q4 tile (tools/q4nx.py:89-94) block kb owns scale
    entries [32kb, 32kb+32) of each plane and nibble bytes rb*2048 + [256kb, 256kb+256).
    """
    blk = 32
    if k0 % blk or k1 % blk or not 0 <= k0 < k1 <= k_tiles * TILE_K:
        raise ValueError(f"columns [{k0}, {k1}) are not whole 32-blocks inside K = {k_tiles * TILE_K}")
    t = tiles.view(n_tile_rows, k_tiles, Q4_TILE_BYTES)
    per_tile = TILE_K // blk  # 8 blocks
    # the four byte runs of every block: d, m, nibbles of row block 0, of row block 1
    runs = [t[:, :, 0:512].reshape(n_tile_rows, k_tiles * per_tile, 64),
            t[:, :, 512:1024].reshape(n_tile_rows, k_tiles * per_tile, 64),
            t[:, :, 1024:3072].reshape(n_tile_rows, k_tiles * per_tile, 256),
            t[:, :, 3072:5120].reshape(n_tile_rows, k_tiles * per_tile, 256)]
    nb = (k1 - k0) // blk
    kt_out = -(-nb // per_tile)
    out = torch.zeros(n_tile_rows, kt_out, Q4_TILE_BYTES, dtype=torch.uint8, device=tiles.device)
    offs = (0, 512, 1024, 3072)
    for run, off in zip(runs, offs):
        w = run.shape[2]
        sel = torch.zeros(n_tile_rows, kt_out * per_tile, w, dtype=torch.uint8, device=tiles.device)
        sel[:, :nb] = run[:, k0 // blk:k1 // blk]
        out[:, :, off:off + per_tile * w] = sel.view(n_tile_rows, kt_out, per_tile * w)
    return out.reshape(-1)


def shard_weights(full: dict, plan: ShardPlan) -> dict:
    """One rank's slice of a full (unsharded) weight dict in the layout of decode.Q4Decoder."""
    kt_h = plan.hidden // TILE_K
    kt_q = plan.n_heads * plan.head_dim // TILE_K
    kt_i = plan.intermediate // TILE_K
    nt_h = plan.hidden // TILE_ROWS
    out = {"layers": []}
    for L in full["layers"]:
        out["layers"].append({
            "qkv": take_tile_rows(L["qkv"], kt_h, Q4_TILE_BYTES, plan.qkv_tile_rows()),
            "o": take_k_blocks(L["o"], nt_h, kt_q, *plan.o_k_range()),
            "gate": take_tile_rows(L["gate"], kt_h, Q4_TILE_BYTES, plan.ffn_tile_rows()),
            "up": take_tile_rows(L["up"], kt_h, Q4_TILE_BYTES, plan.ffn_tile_rows()),
            "down": take_k_tiles(L["down"], nt_h, kt_i, Q4_TILE_BYTES, plan.down_k_tiles()),
            "attn_norm": L["attn_norm"],
            "mlp_norm": L["mlp_norm"],
        })
    out["final_norm"] = full["final_norm"]
    out["lm_head"] = take_tile_rows(full["lm_head"], kt_h, Q8_TILE_BYTES, plan.vocab_tile_rows())
    return out


def tp_exchange_layout(cfg, batch: int, world: int, pulled: bool = False) -> list:
    """The peer buffers of TPDecoder: the replicated residual, the gathered logits, and per
    all-reduce seam either a slot array for its exchange kernel or (pulled) the partial
    itself, which the consuming GEMM's pre-pass reads from every rank.  The O and down
    seams alternate, each with its own buffer, so a rank never rewrites one that another
    rank may still be reading: between two uses of a buffer every rank has entered the
    other seam."""
    seams = ([("o_part", (batch, cfg.hidden), torch.float32), ("down_part", (batch, cfg.hidden), torch.float32)]
             if pulled else
             [("slots_o", (world, batch, cfg.hidden), torch.float32),
              ("slots", (world, batch, cfg.hidden), torch.float32)])
    return [("resid", (batch, cfg.hidden), torch.float32)] + seams + [("logits", (batch, cfg.vocab), torch.float32)]


class TPDecoder:
    """Tensor-parallel decode step on this rank's shard.

    comm selects how the ranks meet at the seams of a layer:
      "peer"        (GPU default) the exchanges of peer.py: the O and down projections'
                    fp32 partials are all-reduced into every rank's copy of the residual
                    stream (summed in rank order, so every copy is bit-identical): two
                    small kernels per layer that store straight into the other GPUs'
                    memory, captured in the step's CUDA graph; the logits are gathered
                    once per step.  On the GEMM path with pulled seams (the GPU default
                    there) the all-reduces have no kernel of their own: each projection
                    leaves its partial in the peer region and the next GEMM's x pre-pass
                    signals it, waits for every rank's and adds them, in rank order, into
                    the residual before its RMSNorm (b2_gemm_rmsnorm_seam).
      "collective"  torch.distributed all_gather / all_reduce (NCCL on GPUs, gloo on CPU).
    `xchg` (comm="peer"): an exchange object with .buffers, .gather(src, name, add_base)
    and .allreduce_add(src, name, y); built from peer.PeerRegion when not given.
    Batches of gemm_min_batch and more run the projections on the tcgen05 GEMM, as
    decode.Q4Decoder does.  swiglu_split (GEMM batches): gate and up as one plain GEMM
    over their stacked tile-rows, which splits K over CTAs, with the SwiGLU formed in the
    down GEMM's x pre-pass -- instead of the fused SwiGLU GEMM, whose one CTA per 64
    gate + 64 up rows leaves most SMs idle on a shard; None: split when those row tiles
    would fill at most half the SMs."""

    def __init__(self, cfg, batch: int, ctx_max: int, shard: dict, plan: ShardPlan, device=None, ops=None,
                 comm: str | None = None, xchg=None, gemm_min_batch: int = 9, swiglu_split: bool | None = None,
                 pulled: bool | None = None):
        if ops is None:
            from . import ops  # the GPU path; tests of the host logic may pass another implementation
        self.ops = ops
        self.cfg, self.plan, self.batch, self.ctx_max = cfg, plan, batch, ctx_max
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        dev, c, p, W = self.device, cfg, plan, plan.world
        if comm is None:
            comm = "peer" if (dev.type == "cuda" and W > 1) else "collective"
        if comm not in ("peer", "collective"):
            raise ValueError(f"unknown comm {comm!r}")
        self.comm = comm
        self.w = shard
        self.kt_h, self.kt_q, self.kt_i = c.hidden // TILE_K, c.n_heads * c.head_dim // TILE_K, c.intermediate // TILE_K
        self.kt_i_local = self.kt_i // W
        self.nt_qkv_local = len(p.qkv_tile_rows())
        self.kt_o_local = p.o_k_tiles
        self.nt_i_local = c.intermediate // TILE_ROWS // W
        self.nt_v_local = c.vocab // TILE_ROWS // W
        d = c.head_dim
        kv_shape = (batch, p.kv_local, ctx_max, d)
        self.k_cache = [torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev) for _ in range(c.n_layers)]
        self.v_cache = [torch.zeros(kv_shape, dtype=torch.bfloat16, device=dev) for _ in range(c.n_layers)]
        self.x_in = torch.zeros(batch, c.hidden, dtype=torch.float32, device=dev)
        self.xn = torch.zeros(batch, c.hidden, dtype=torch.bfloat16, device=dev)
        self.qkv = torch.zeros(batch, self.nt_qkv_local * TILE_ROWS, dtype=torch.float32, device=dev)
        # this rank's heads' attention output = its O input, zero past q_local*d (the padding
        # columns of the re-tiled O shard; the attention writes only the first q_local*d)
        self.attn_local = torch.zeros(batch, self.kt_o_local * TILE_K, dtype=torch.bfloat16, device=dev)
        self.o_part = torch.zeros(batch, c.hidden, dtype=torch.float32, device=dev)
        self.h = torch.zeros(batch, c.intermediate // W, dtype=torch.bfloat16, device=dev)
        self.down = torch.zeros(batch, c.hidden, dtype=torch.float32, device=dev)
        self.logits_local = torch.zeros(batch, c.vocab // W, dtype=torch.float32, device=dev)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.use_gemm = batch >= gemm_min_batch
        # pulled seams: the O and down all-reduces inside the next GEMM's x pre-pass
        if pulled is None:
            pulled = comm == "peer" and self.use_gemm and xchg is None and dev.type == "cuda" and W > 1
        if pulled and not (comm == "peer" and self.use_gemm):
            raise ValueError("pulled seams need comm='peer' and the GEMM path")
        self.pulled = bool(pulled)
        if comm == "peer":
            if xchg is None:
                from .peer import PeerExchange
                xchg = PeerExchange(tp_exchange_layout(cfg, batch, W, self.pulled), device=dev)
            self.xchg = xchg
            self.resid = xchg.buffers["resid"]
            self.logits = xchg.buffers["logits"]
            if self.pulled:
                self.o_part = xchg.buffers["o_part"]
                self.down = xchg.buffers["down_part"]
                self.ps_o = ops.PeerSum(xchg.region, "o_part", 0)
                self.ps_down = ops.PeerSum(xchg.region, "down_part", 1)
        else:
            self.xchg = None
            # gathered buffers are [W*B, n] (rank-major), viewed as [W, B, n] when merged
            self.logits_all = torch.zeros(W * batch, c.vocab // W, dtype=torch.float32, device=dev)
            self.resid = torch.zeros(batch, c.hidden, dtype=torch.float32, device=dev)
            self.logits = torch.zeros(batch, c.vocab, dtype=torch.float32, device=dev)
        ws = ops.gqa_decode_workspace_bytes(batch, p.q_local, p.kv_local, d, ctx_max)
        self.attn_ws = torch.empty(max(ws, 1), dtype=torch.uint8, device=dev)
        self.swiglu_split = False
        if self.use_gemm:
            nbytes = ops.gemm_workspace_bytes(batch, max(self.kt_h, self.kt_o_local, self.kt_i_local))
            self.gemm_ws_raw = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
            off = (256 - self.gemm_ws_raw.data_ptr() % 256) % 256
            self.gemm_ws = self.gemm_ws_raw[off:off + nbytes]
            # this rank's projection shards repacked once for the GEMM (A dequantised into TMEM)
            if swiglu_split is None:
                sms = torch.cuda.get_device_properties(dev).multi_processor_count if dev.type == "cuda" else 148
                swiglu_split = self.nt_i_local // 2 <= sms // 2
            self.swiglu_split = bool(swiglu_split)
            shapes = {"qkv": (self.nt_qkv_local, self.kt_h), "o": (c.hidden // TILE_ROWS, self.kt_o_local),
                      "down": (cfg.hidden // TILE_ROWS, self.kt_i_local)}
            if not swiglu_split:
                shapes.update(gate=(self.nt_i_local, self.kt_h), up=(self.nt_i_local, self.kt_h))
            self.wg = [{k: self.ops.q4_gemm_pack(L[k], *shp) for k, shp in shapes.items()} for L in self.w["layers"]]
            if swiglu_split:
                for G, L in zip(self.wg, self.w["layers"]):
                    G["gu"] = self.ops.q4_gemm_pack(torch.cat([L["gate"], L["up"]]), 2 * self.nt_i_local, self.kt_h)
                # gate outputs in columns [0, I/W), up outputs in [I/W, 2I/W)
                self.gu = torch.zeros(batch, 2 * c.intermediate // W, dtype=torch.float32, device=dev)
            self.lm_packed = self.ops.q8_gemm_pack(self.w["lm_head"], self.nt_v_local, self.kt_h)

    def close(self) -> None:
        """Release the peer mappings (every rank, after its last step)."""
        if self.xchg is not None and hasattr(self.xchg, "close"):
            self.xchg.close()
        self.xchg = None

    # ---------------------------------------------------------------- seams
    def _reduce_o(self) -> None:
        if self.comm == "peer":
            self.xchg.allreduce_add(self.o_part, "slots_o", self.resid)
        else:
            if self.plan.world > 1:
                dist.all_reduce(self.o_part)
            self.resid.add_(self.o_part)

    def _reduce_down(self) -> None:
        if self.comm == "peer":
            self.xchg.allreduce_add(self.down, "slots", self.resid)
        else:
            if self.plan.world > 1:
                dist.all_reduce(self.down)
            self.resid.add_(self.down)

    def _gather_logits(self) -> None:
        W, B = self.plan.world, self.batch
        if self.comm == "peer":
            self.xchg.gather(self.logits_local, "logits")
        elif W > 1:
            dist.all_gather_into_tensor(self.logits_all, self.logits_local)
            self.logits.view(B, W, -1).copy_(self.logits_all.view(W, B, -1).permute(1, 0, 2))
        else:
            self.logits.copy_(self.logits_local)

    # ---------------------------------------------------------------- step
    def step(self) -> torch.Tensor:
        ops, c, p = self.ops, self.cfg, self.plan
        d = c.head_dim
        qd, kd = p.q_local * d, p.kv_local * d
        ws = self.gemm_ws if self.use_gemm else None
        self.resid.copy_(self.x_in)
        pulled = self.pulled
        for li, L in enumerate(self.w["layers"]):
            G = self.wg[li] if self.use_gemm else None
            if self.use_gemm:
                # pulled: the previous layer's down seam summed into the residual here
                ops.q4_gemm(G["qkv"], self.nt_qkv_local, self.kt_h, self.resid, out=self.qkv, workspace=ws,
                            prefetch=True, norm_w=L["attn_norm"], eps=c.rms_eps, packed=True,
                            peer_sum=self.ps_down if pulled and li > 0 else None)
            else:
                ops.gemv_rmsnorm(L["qkv"], self.nt_qkv_local, self.kt_h, self.resid, L["attn_norm"], c.rms_eps,
                                 out=self.qkv, prefetch=True)
            ops.gqa_decode(self.qkv[:, :qd], self.qkv[:, qd:qd + kd], self.qkv[:, qd + kd:], self.k_cache[li],
                           self.v_cache[li], self.pos, n_q_heads=p.q_local, n_kv_heads=p.kv_local,
                           theta=c.rope_theta, scale=d ** -0.5, max_len=self.ctx_max, out=self.attn_local[:, :qd],
                           workspace=self.attn_ws, prefetch_kv=True)
            if self.use_gemm:
                ops.q4_gemm(G["o"], c.hidden // TILE_ROWS, self.kt_o_local, self.attn_local, out=self.o_part,
                            workspace=ws, prefetch=True, packed=True)
            else:
                ops.q4_gemv(L["o"], c.hidden // TILE_ROWS, self.kt_o_local, self.attn_local, out=self.o_part,
                            prefetch=True)
            if not pulled:
                self._reduce_o()
            ps_o = self.ps_o if pulled else None  # pulled: the O seam summed in the next pre-pass
            if self.swiglu_split:
                ops.q4_gemm(G["gu"], 2 * self.nt_i_local, self.kt_h, self.resid, out=self.gu, workspace=ws,
                            prefetch=True, norm_w=L["mlp_norm"], eps=c.rms_eps, packed=True, peer_sum=ps_o)
                ops.q4_gemm(G["down"], c.hidden // TILE_ROWS, self.kt_i_local, self.gu, out=self.down, workspace=ws,
                            prefetch=True, packed=True, swiglu_in=True)
            elif self.use_gemm:
                ops.q4_swiglu_gemm(G["gate"], G["up"], self.nt_i_local, self.kt_h, self.resid, out=self.h,
                                   workspace=ws, prefetch=True, norm_w=L["mlp_norm"], eps=c.rms_eps, packed=True,
                                   peer_sum=ps_o)
                ops.q4_gemm(G["down"], c.hidden // TILE_ROWS, self.kt_i_local, self.h, out=self.down, workspace=ws,
                            prefetch=True, packed=True)
            else:
                ops.swiglu_gemv_rmsnorm(L["gate"], L["up"], self.nt_i_local, self.kt_h, self.resid, L["mlp_norm"],
                                        c.rms_eps, out=self.h, prefetch=True)
                ops.q4_gemv(L["down"], c.hidden // TILE_ROWS, self.kt_i_local, self.h, out=self.down, prefetch=True)
            if not pulled:
                self._reduce_down()
        if self.use_gemm:
            ops.q8_gemm(self.lm_packed, self.nt_v_local, self.kt_h, self.resid, out=self.logits_local, workspace=ws,
                        prefetch=True, norm_w=self.w["final_norm"], eps=c.rms_eps,
                        peer_sum=self.ps_down if pulled and self.w["layers"] else None)
        else:
            ops.gemv_rmsnorm(self.w["lm_head"], self.nt_v_local, self.kt_h, self.resid, self.w["final_norm"],
                             c.rms_eps, out=self.logits_local, prefetch=True, q8=True)
        self._gather_logits()
        return self.logits

    def capture(self) -> torch.cuda.CUDAGraph:
        """The step as one CUDA graph (warm once outside the capture first)."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step()
        return g


# ------------------------------------------------------------------ Qwen3.5 linear attention
DELTA_D = 128  # linear-attention head dim


@dataclass(frozen=True)
class DeltaNetShardPlan:
    """Tensor-parallel gated DeltaNet layer: rank `rank` of `world` owns k heads
    [r*nk/W, (r+1)*nk/W) and the v heads that read them, so its recurrent and conv
    states, and its step kernel, hold only its heads and need no collective.  Its in_proj
    is those heads' whole tile-rows of the stacked q|k|v|z|b|a weight plus the b|a
    tile-rows (one per 32 of the 2*nv b/a rows), which every rank keeps whole; out_proj is
    split by its heads' whole 256-wide K-tiles and the fp32 partial outputs are
    all-reduced (sum) into the replicated residual."""

    hidden: int
    n_k_heads: int
    n_v_heads: int
    world: int
    rank: int

    def __post_init__(self):
        if self.n_k_heads % self.world or self.n_v_heads % self.n_k_heads:
            raise ValueError(f"{self.n_k_heads} k heads do not split over {self.world} ranks")
        if (self.nv_local * DELTA_D) % TILE_K:
            raise ValueError("each rank's v heads must fill whole 256-wide out_proj K-tiles")

    @property
    def ratio(self) -> int:
        return self.n_v_heads // self.n_k_heads

    @property
    def nk_local(self) -> int:
        return self.n_k_heads // self.world

    @property
    def nv_local(self) -> int:
        return self.nk_local * self.ratio

    @property
    def k0(self) -> int:
        return self.rank * self.nk_local

    @property
    def v0(self) -> int:
        return self.rank * self.nv_local

    @property
    def c_b_full(self) -> int:
        """First b column of the full stacked in_proj output (a multiple of 32)."""
        return (2 * self.n_k_heads + 2 * self.n_v_heads) * DELTA_D

    def in_proj_tile_rows(self) -> list[int]:
        """Tile-rows of the full stacked in_proj this rank owns, in its order q|k|v|z|b+a."""
        tph = DELTA_D // TILE_ROWS  # tile-rows per head
        nk, nv = self.n_k_heads, self.n_v_heads
        q = range(self.k0 * tph, (self.k0 + self.nk_local) * tph)
        k = range((nk + self.k0) * tph, (nk + self.k0 + self.nk_local) * tph)
        v = range((2 * nk + self.v0) * tph, (2 * nk + self.v0 + self.nv_local) * tph)
        z = range((2 * nk + nv + self.v0) * tph, (2 * nk + nv + self.v0 + self.nv_local) * tph)
        ba = range(self.c_b_full // TILE_ROWS, -(-(self.c_b_full + 2 * nv) // TILE_ROWS))
        return [*q, *k, *v, *z, *ba]

    @property
    def n_ba_tile_rows(self) -> int:
        """Tile-rows of the b|a rows at the end of the stacked in_proj."""
        return -(-(self.c_b_full + 2 * self.n_v_heads) // TILE_ROWS) - self.c_b_full // TILE_ROWS

    def local_cols(self) -> tuple[int, int]:
        """(b, a) columns of this rank's first v head in its in_proj output."""
        c_ba = (2 * self.nk_local + 2 * self.nv_local) * DELTA_D
        return c_ba + self.v0, c_ba + self.n_v_heads + self.v0

    def conv_channels(self) -> list[int]:
        """Channels of the full conv (q|k|v, conv_dim wide) this rank owns, in its order q|k|v."""
        d, nk = DELTA_D, self.n_k_heads
        return [*range(self.k0 * d, (self.k0 + self.nk_local) * d),
                *range((nk + self.k0) * d, (nk + self.k0 + self.nk_local) * d),
                *range((2 * nk + self.v0) * d, (2 * nk + self.v0 + self.nv_local) * d)]

    def out_proj_k_tiles(self) -> range:
        per = self.nv_local * DELTA_D // TILE_K
        return range(self.rank * per, (self.rank + 1) * per)


def shard_deltanet(full: dict, plan: DeltaNetShardPlan) -> dict:
    """One rank's slice of a full DeltaNetLayer weight dict (llmnputest_b200.deltanet).

    With b|a as q4 tile-rows the rank keeps those rows whole (`local_cols` locates its
    heads); with b|a dense ("ba_dense", as read from a q4nx file) it keeps its heads'
    rows of b and of a, and its in_proj is q|k|v|z only: the layer's own dense layout."""
    kt_h = plan.hidden // TILE_K
    kt_v = plan.n_v_heads * DELTA_D // TILE_K
    ch = torch.as_tensor(plan.conv_channels(), dtype=torch.long, device=full["conv_w"].device)
    vh = slice(plan.v0, plan.v0 + plan.nv_local)
    rows = plan.in_proj_tile_rows()
    extra = {}
    if "ba_dense" in full:
        rows = rows[:len(rows) - plan.n_ba_tile_rows]
        nv = plan.n_v_heads
        extra["ba_dense"] = torch.cat([full["ba_dense"][vh], full["ba_dense"][nv + plan.v0:nv + plan.v0 + plan.nv_local]])
    return {
        **extra,
        "in_proj": take_tile_rows(full["in_proj"], kt_h, Q4_TILE_BYTES, rows),
        "out_proj": take_k_tiles(full["out_proj"], plan.hidden // TILE_ROWS, kt_v, Q4_TILE_BYTES,
                                 plan.out_proj_k_tiles()),
        "conv_w": full["conv_w"].index_select(0, ch).contiguous(),
        "A_log": full["A_log"][vh].contiguous(),
        "dt_bias": full["dt_bias"][vh].contiguous(),
        "norm_w": full["norm_w"],
        "input_norm": full["input_norm"],
    }


class TPDeltaNetLayer:
    """This rank's part of a gated DeltaNet layer: the local heads' mixer, the out_proj
    K-slice, and an all-reduce of its fp32 partial into the residual."""

    def __init__(self, plan: DeltaNetShardPlan, batch: int, shard: dict, device=None, eps: float = 1e-6,
                 ops=None, gemm_min_batch: int = 9):
        from .deltanet import DeltaNetLayer
        self.plan = plan
        dense = "ba_dense" in shard  # b|a dense: the layer's own layout for its heads
        self.layer = DeltaNetLayer(plan.hidden, plan.nk_local, plan.nv_local, batch, device=device, weights=shard,
                                   eps=eps, gemm_min_batch=gemm_min_batch, ops_impl=ops,
                                   cols=None if dense else plan.local_cols(),
                                   n_in_tile_rows=None if dense else len(plan.in_proj_tile_rows()))
        self.partial = torch.zeros(batch, plan.hidden, dtype=torch.float32, device=self.layer.device)

    def step(self, resid: torch.Tensor) -> torch.Tensor:
        """resid (fp32 [B, hidden], the same on every rank) += the layer's token mixer."""
        h = self.layer.mix(resid)
        if self.plan.world == 1:
            return self.layer.out_proj(h, resid, accumulate=True)
        self.layer.out_proj(h, self.partial, accumulate=False)
        dist.all_reduce(self.partial)
        resid.add_(self.partial)
        return resid


# ------------------------------------------------------------------ Qwen3.5 gated full attention
GATED_D = 256  # gated-attention head dim


@dataclass(frozen=True)
class GatedAttnShardPlan:
    """Tensor-parallel gated full-attention layer: rank `rank` of `world` owns kv heads
    [r*nkv/W, (r+1)*nkv/W) and their q heads, so its KV cache and attention kernel hold
    only its heads; its in_proj is those heads' whole tile-rows of the stacked
    q_proj (q|gate per head) | k_proj | v_proj weight, its o_proj the heads' whole
    256-wide K-tiles, and the fp32 partial outputs are all-reduced into the residual."""

    hidden: int
    n_q_heads: int
    n_kv_heads: int
    world: int
    rank: int

    def __post_init__(self):
        if self.n_kv_heads % self.world or self.n_q_heads % self.n_kv_heads:
            raise ValueError(f"{self.n_kv_heads} kv heads do not split over {self.world} ranks")

    @property
    def kv_local(self) -> int:
        return self.n_kv_heads // self.world

    @property
    def q_local(self) -> int:
        return self.kv_local * (self.n_q_heads // self.n_kv_heads)

    @property
    def kv0(self) -> int:
        return self.rank * self.kv_local

    @property
    def q0(self) -> int:
        return self.rank * self.q_local

    def in_proj_tile_rows(self) -> list[int]:
        """Tile-rows of the full stacked in_proj this rank owns, in its order q|k|v."""
        tq, tkv = 2 * GATED_D // TILE_ROWS, GATED_D // TILE_ROWS  # tile-rows per q head (q|gate), per k/v head
        k_base = self.n_q_heads * tq
        v_base = k_base + self.n_kv_heads * tkv
        return [*range(self.q0 * tq, (self.q0 + self.q_local) * tq),
                *range(k_base + self.kv0 * tkv, k_base + (self.kv0 + self.kv_local) * tkv),
                *range(v_base + self.kv0 * tkv, v_base + (self.kv0 + self.kv_local) * tkv)]

    def o_proj_k_tiles(self) -> range:
        per = GATED_D // TILE_K
        return range(self.q0 * per, (self.q0 + self.q_local) * per)


def shard_gated_attention(full: dict, plan: GatedAttnShardPlan) -> dict:
    """One rank's slice of a full GatedAttentionLayer weight dict (llmnputest_b200.gated_attention)."""
    kt_h = plan.hidden // TILE_K
    kt_o = plan.n_q_heads * GATED_D // TILE_K
    return {
        "in_proj": take_tile_rows(full["in_proj"], kt_h, Q4_TILE_BYTES, plan.in_proj_tile_rows()),
        "o_proj": take_k_tiles(full["o_proj"], plan.hidden // TILE_ROWS, kt_o, Q4_TILE_BYTES, plan.o_proj_k_tiles()),
        "q_norm_w": full["q_norm_w"],
        "k_norm_w": full["k_norm_w"],
        "inv_freq": full["inv_freq"],
        "input_norm": full["input_norm"],
    }


class TPGatedAttentionLayer:
    """This rank's part of a gated full-attention layer: its heads' attention, the o_proj
    K-slice, and an all-reduce of its fp32 partial into the residual."""

    def __init__(self, plan: GatedAttnShardPlan, batch: int, ctx_max: int, shard: dict, device=None,
                 eps: float = 1e-6, ops=None, gemm_min_batch: int = 9):
        from .gated_attention import GatedAttentionLayer
        self.plan = plan
        self.layer = GatedAttentionLayer(plan.hidden, plan.q_local, plan.kv_local, batch, ctx_max, device=device,
                                         weights=shard, eps=eps, gemm_min_batch=gemm_min_batch, ops_impl=ops)
        self.partial = torch.zeros(batch, plan.hidden, dtype=torch.float32, device=self.layer.device)

    @property
    def pos(self) -> torch.Tensor:
        return self.layer.pos

    def step(self, resid: torch.Tensor) -> torch.Tensor:
        """resid (fp32 [B, hidden], the same on every rank) += the layer's token mixer at `pos`."""
        a = self.layer.mix(resid)
        if self.plan.world == 1:
            return self.layer.o_proj(a, resid, accumulate=True)
        self.layer.o_proj(a, self.partial, accumulate=False)
        dist.all_reduce(self.partial)
        resid.add_(self.partial)
        return resid
