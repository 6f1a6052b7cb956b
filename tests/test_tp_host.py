"""Tensor-parallel host logic on CPU: shard plans reassemble the full projections,
and a 2-rank gloo run of TPDecoder.step (collectives and reshapes) equals the
unsharded step.  The GPU ops are replaced by an oracle-backed shim here -- this
file tests the sharding and collective plumbing, not the kernels."""

import os
import socket
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from ml_dtypes import bfloat16

from oracle import q4nx_oracle as orc
from llmnputest_b200.decode import DecoderConfig
from llmnputest_b200.tp import ShardPlan, TPDecoder, shard_weights, take_k_blocks, tp_exchange_layout

CFG = DecoderConfig(n_layers=2, hidden=512, n_heads=8, n_kv_heads=2, head_dim=64, intermediate=1024, vocab=512)


def _bf(t):
    return torch.from_numpy(np.asarray(t, np.float32)).to(torch.bfloat16)


def full_weights(cfg, seed=0):
    rng = np.random.default_rng(seed)
    kt_h, kt_q, kt_i = cfg.hidden // 256, cfg.n_heads * cfg.head_dim // 256, cfg.intermediate // 256
    u8 = lambda a: torch.from_numpy(np.ascontiguousarray(a).reshape(-1))
    norm = lambda: _bf(rng.standard_normal(cfg.hidden) * 0.1 + 1)
    layers = [{"qkv": u8(orc.synth_q4_tiles(rng, cfg.qkv_rows // 32 * kt_h)),
               "o": u8(orc.synth_q4_tiles(rng, cfg.hidden // 32 * kt_q)),
               "gate": u8(orc.synth_q4_tiles(rng, cfg.intermediate // 32 * kt_h)),
               "up": u8(orc.synth_q4_tiles(rng, cfg.intermediate // 32 * kt_h)),
               "down": u8(orc.synth_q4_tiles(rng, cfg.hidden // 32 * kt_i)),
               "attn_norm": norm(), "mlp_norm": norm()} for _ in range(cfg.n_layers)]
    return {"layers": layers, "final_norm": norm(), "lm_head": u8(orc.synth_q8_tiles(rng, cfg.vocab // 32 * kt_h))}


class OracleOps:
    """The ops signatures of llmnputest_b200.ops, computed by the CPU oracle (test infrastructure)."""

    @staticmethod
    def _x(x):
        return x.float().numpy()

    def q4_gemv(self, tiles, n_t, k_t, x, out=None, accumulate=False, prefetch=False):
        y = torch.from_numpy(orc.gemv_q4(tiles.numpy(), self._x(x).astype(bfloat16), n_t, k_t))
        out.add_(y) if accumulate else out.copy_(y)
        return out

    def q8_gemv(self, tiles, n_t, k_t, x, out=None, accumulate=False, prefetch=False):
        out.copy_(torch.from_numpy(orc.gemv_q8(tiles.numpy(), self._x(x).astype(bfloat16), n_t, k_t)))
        return out

    def q4_swiglu_gemv(self, gate, up, n_t, k_t, x, out=None, prefetch=False):
        xb = self._x(x).astype(bfloat16)
        h = orc.swiglu_from_accumulators(orc.gemv_q4(gate.numpy(), xb, n_t, k_t), orc.gemv_q4(up.numpy(), xb, n_t, k_t))
        out.copy_(_bf(h))
        return out

    def gemv_rmsnorm(self, tiles, n_t, k_t, x, norm_w, eps, out=None, accumulate=False, prefetch=False, q8=False):
        xn = _bf(orc.rmsnorm(self._x(x), norm_w.float().numpy(), eps))
        return (self.q8_gemv if q8 else self.q4_gemv)(tiles, n_t, k_t, xn, out=out, accumulate=accumulate)

    def swiglu_gemv_rmsnorm(self, gate, up, n_t, k_t, x, norm_w, eps, out=None, prefetch=False):
        xn = _bf(orc.rmsnorm(self._x(x), norm_w.float().numpy(), eps))
        return self.q4_swiglu_gemv(gate, up, n_t, k_t, xn, out=out)

    def rmsnorm(self, x, w, eps, out=None):
        out.copy_(_bf(orc.rmsnorm(self._x(x), w.float().numpy(), eps)))
        return out

    def gqa_decode(self, q, k_new, v_new, k_cache, v_cache, pos, *, n_q_heads, n_kv_heads, theta, scale,
                   max_len, out, workspace=None, **_):
        d = k_cache.shape[-1]
        bsz = q.shape[0]
        qr = np.zeros((bsz, n_q_heads, d), np.float32)
        for b in range(bsz):
            p = int(pos[b])
            qr[b] = orc.rope_half_split(q[b].numpy().reshape(n_q_heads, d), p, theta).astype(np.float32).astype(bfloat16)
            k_cache[b, :, p] = _bf(orc.rope_half_split(k_new[b].numpy().reshape(n_kv_heads, d), p, theta))
            v_cache[b, :, p] = _bf(v_new[b].numpy().reshape(n_kv_heads, d))
        o = orc.gqa_decode(qr, k_cache.float().numpy(), v_cache.float().numpy(), pos.numpy() + 1, scale)
        out.copy_(_bf(o.reshape(bsz, -1)))
        return out

    def gqa_decode_workspace_bytes(self, *a):
        return 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shards_reassemble_full_projections(world):
    cfg = DecoderConfig(n_layers=1, hidden=2048, n_heads=16, n_kv_heads=8, head_dim=64, intermediate=4096, vocab=2048)
    W = full_weights(cfg, seed=world)
    L = W["layers"][0]
    rng = np.random.default_rng(0)
    x = orc.synth_bf16(rng, cfg.hidden)
    kt_h, kt_i = cfg.hidden // 256, cfg.intermediate // 256
    full_qkv = orc.gemv_q4(L["qkv"].numpy(), x, cfg.qkv_rows // 32, kt_h)
    h = orc.synth_bf16(rng, cfg.intermediate)
    full_down = orc.gemv_q4(L["down"].numpy(), h, cfg.hidden // 32, kt_i)
    down_sum = np.zeros(cfg.hidden)
    a = orc.synth_bf16(rng, cfg.n_heads * 64)  # attention output, all heads
    full_o = orc.gemv_q4(L["o"].numpy(), a, cfg.hidden // 32, cfg.n_heads * 64 // 256)
    o_sum = np.zeros(cfg.hidden)
    heads = []
    for r in range(world):
        plan = ShardPlan(cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.hidden, cfg.intermediate, cfg.vocab, world, r)
        S = shard_weights(W, plan)["layers"][0]
        qkv = orc.gemv_q4(S["qkv"].numpy(), x, len(plan.qkv_tile_rows()), kt_h)
        rows = np.concatenate([np.arange(t * 32, t * 32 + 32) for t in plan.qkv_tile_rows()])
        assert np.array_equal(qkv, full_qkv[rows])  # same tiles, same arithmetic: bit-identical
        heads.append(qkv[:plan.q_local * 64])
        ks = list(plan.down_k_tiles())
        down_sum += orc.gemv_q4(S["down"].numpy(), h[ks[0] * 256:(ks[-1] + 1) * 256], cfg.hidden // 32, len(ks))
        k0, k1 = plan.o_k_range()
        a_loc = np.zeros(plan.o_k_tiles * 256, dtype=a.dtype)  # the rank's heads, zero-padded
        a_loc[:k1 - k0] = a[k0:k1]
        o_sum += orc.gemv_q4(S["o"].numpy(), a_loc, cfg.hidden // 32, plan.o_k_tiles)
    assert np.array_equal(np.concatenate(heads), full_qkv[:cfg.n_heads * 64])  # q heads in rank order
    np.testing.assert_allclose(down_sum, full_down, rtol=1e-4, atol=1e-3 * np.abs(full_down).max())
    np.testing.assert_allclose(o_sum, full_o, rtol=1e-4, atol=1e-3 * np.abs(full_o).max())


@pytest.mark.parametrize("k0,k1", [(0, 256), (64, 320), (640, 1280), (320, 640), (2048 - 32, 2048), (96, 1056)])
def test_take_k_blocks_moves_whole_blocks(k0, k1):
    """Re-tiling by 32-column blocks keeps every dequantised weight bit-identical and pads
    the last K-tile with exact zeros."""
    rng = np.random.default_rng(k0 + 7 * k1)
    n_t, k_t = 3, 8
    tiles = orc.synth_q4_tiles(rng, n_t * k_t)
    out = take_k_blocks(torch.from_numpy(tiles.reshape(-1)), n_t, k_t, k0, k1).numpy()
    kt_out = -(-(k1 - k0) // 256)
    assert out.size == n_t * kt_out * 5120
    full = orc.q4_matrix(tiles.reshape(-1), n_t, k_t)
    got = orc.q4_matrix(out, n_t, kt_out)
    assert np.array_equal(got[:, :k1 - k0], full[:, k0:k1])
    assert not got[:, k1 - k0:].any()


@pytest.mark.parametrize("k0,k1", [(16, 256), (0, 300), (256, 256), (0, 2304)])
def test_take_k_blocks_rejects_partial_blocks(k0, k1):
    tiles = torch.zeros(2 * 8 * 5120, dtype=torch.uint8)
    with pytest.raises(ValueError):
        take_k_blocks(tiles, 2, 8, k0, k1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class GlooExchange:
    """The peer exchanges' semantics (llmnputest_b200.peer) over gloo, for the host logic of
    TPDecoder(comm="peer"): gather places every rank's block at column rank*cols of every
    rank's buffer (adding it when add_base is given), allreduce_add sums the partials in
    rank order into y."""

    def __init__(self, layout):
        self.buffers = {name: torch.zeros(shape, dtype=dtype) for name, shape, dtype in layout}

    def gather(self, src, name, add_base=None):
        w = dist.get_world_size()
        parts = [torch.empty(src.shape, dtype=torch.float32) for _ in range(w)]
        dist.all_gather(parts, src.float().contiguous())
        dst, cols = self.buffers[name], src.shape[1]
        for r, part in enumerate(parts):
            blk = dst[:, r * cols:(r + 1) * cols]
            if add_base is not None:
                assert add_base.data_ptr() == dst.data_ptr()  # the replicated copy itself
                blk.add_(part.to(dst.dtype))
            else:
                blk.copy_(part.to(dst.dtype))

    def allreduce_add(self, src, name, y):
        w = dist.get_world_size()
        parts = [torch.empty_like(src) for _ in range(w)]
        dist.all_gather(parts, src.contiguous())
        total = parts[0].clone()
        for part in parts[1:]:
            total += part
        y += total


def _run_rank(rank, world, port, x, pos, ctx, result_path, comm="collective"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W = full_weights(CFG)
        plan = ShardPlan(CFG.n_heads, CFG.n_kv_heads, CFG.head_dim, CFG.hidden, CFG.intermediate, CFG.vocab,
                         world, rank)
        xchg = None
        if comm == "peer":
            b, d = x.shape[1], CFG.head_dim
            xchg = GlooExchange(tp_exchange_layout(CFG, b, world))
        dec = TPDecoder(CFG, x.shape[1], ctx, shard_weights(W, plan), plan, device="cpu", ops=OracleOps(), comm=comm,
                        xchg=xchg)
        for step in range(2):
            dec.x_in.copy_(x[step])
            dec.pos.copy_(pos + step)
            logits = dec.step().clone()
        if rank == 0:
            torch.save(logits, result_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("comm", ["collective", "peer"])
def test_tp_step_gloo_matches_single_rank(tmp_path, comm):
    rng = np.random.default_rng(5)
    bsz, ctx = 2, 16
    x = torch.from_numpy(rng.standard_normal((2, bsz, CFG.hidden)).astype(np.float32))
    pos = torch.tensor([3, 9], dtype=torch.int32)
    out1 = tmp_path / "w1.pt"
    out2 = tmp_path / "w2.pt"
    ctx_mp = mp.get_context("spawn")
    for world, path in ((1, out1), (2, out2)):
        port = _free_port()
        procs = [ctx_mp.Process(target=_run_rank, args=(r, world, port, x, pos, ctx, str(path), comm))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=240)
            assert p.exitcode == 0
    a, b = torch.load(out1), torch.load(out2)
    cos, rel = orc.compare(b.numpy(), a.numpy())
    assert cos >= 0.99999 and rel <= 1e-3, (cos, rel)


def test_pulled_seam_layout_and_peer_sum_checks():
    """The peer region of the pulled-seam decoder holds each seam's partial (not a slot
    array), and ops.PeerSum takes only fp32 [rows, cols] region buffers."""
    from llmnputest_b200.ops import PeerSum
    layout = tp_exchange_layout(CFG, 4, 2, pulled=True)
    names = [n for n, _, _ in layout]
    assert names == ["resid", "o_part", "down_part", "logits"]
    assert dict((n, s) for n, s, _ in layout)["o_part"] == (4, CFG.hidden)
    assert [n for n, _, _ in tp_exchange_layout(CFG, 4, 2)] == ["resid", "slots_o", "slots", "logits"]
    region = SimpleNamespace(offsets={"o_part": (65536, (4, CFG.hidden), torch.float32),
                                      "slots": (131072, (2, 4, CFG.hidden), torch.float32),
                                      "attn": (196608, (4, 512), torch.bfloat16)})
    ps = PeerSum(region, "o_part", 1)
    assert (ps.offset, ps.ld, ps.rows, ps.seam) == (65536, CFG.hidden, 4, 1)
    for bad in ("slots", "attn"):
        with pytest.raises(ValueError):
            PeerSum(region, bad, 0)
