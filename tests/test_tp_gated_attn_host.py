"""Tensor-parallel gated full-attention host logic on CPU: the kv-head shard plan
reassembles the full layer (in_proj rows bit-identical, o_proj K-slices), and a
2-rank gloo run of TPGatedAttentionLayer (two steps at advancing positions, each
reading the rows the earlier one appended) equals the single-rank layer.  The GPU
ops are replaced by the oracle-backed shim of tests/test_tp_host.py, extended with
the gated attention step: this file tests the sharding and collective plumbing,
not the kernels."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from ml_dtypes import bfloat16

from llmnputest_b200.tp import GatedAttnShardPlan, TPGatedAttentionLayer, shard_gated_attention
from oracle import gated_attention_oracle as ga
from oracle import q4nx_oracle as orc
from tests.test_tp_host import OracleOps, _bf, _free_port

HIDDEN, D = 256, 256


def _to_bf16(x):
    return np.asarray(x, np.float32).astype(bfloat16).astype(np.float32)


class GatedOracleOps(OracleOps):
    def gated_attn_workspace_bytes(self, *a):
        return 0

    def gated_attn_decode(self, qg, k_new, v_new, q_norm_w, k_norm_w, inv_freq, k_cache, v_cache, pos, n_q_heads,
                          n_kv_heads, max_len=None, eps=1e-6, out=None, out_f32=False, workspace=None):
        o, k_row, v_row = ga.gated_attention_step(
            qg.numpy(), k_new.numpy(), v_new.numpy(), q_norm_w.numpy(), k_norm_w.numpy(), inv_freq.numpy(),
            k_cache.float().numpy(), v_cache.float().numpy(), pos.numpy(), n_q_heads, n_kv_heads, eps,
            stored=_to_bf16)
        for b, p in enumerate(pos.tolist()):  # the kernel appends the rows it attends to
            k_cache[b, :, p] = _bf(k_row[b])
            v_cache[b, :, p] = _bf(v_row[b])
        out.copy_(_bf(o))
        return out


def full_layer(nq, nkv, seed=0):
    rng = np.random.default_rng(seed)
    n_in = (nq * 2 * D + 2 * nkv * D) // 32
    u8 = lambda t: torch.from_numpy(np.ascontiguousarray(t).reshape(-1))
    f32 = lambda t: torch.from_numpy(np.asarray(t, np.float32))
    return {
        "in_proj": u8(orc.synth_q4_tiles(rng, n_in * (HIDDEN // 256))),
        "o_proj": u8(orc.synth_q4_tiles(rng, HIDDEN // 32 * nq)),
        "q_norm_w": f32(0.1 * rng.standard_normal(D)),
        "k_norm_w": f32(0.1 * rng.standard_normal(D)),
        "inv_freq": f32(1.0 / (1e7 ** (np.arange(0, 64, 2) / 64.0))),
        "input_norm": _bf(1 + 0.1 * rng.standard_normal(HIDDEN)),
    }, n_in


@pytest.mark.parametrize("nq,nkv,world", [(8, 2, 2), (16, 4, 4), (4, 4, 4)])
def test_gated_attn_shards_reassemble_full_layer(nq, nkv, world):
    W, n_in = full_layer(nq, nkv, seed=world)
    rng = np.random.default_rng(2)
    x = orc.synth_bf16(rng, HIDDEN)
    full = orc.gemv_q4(W["in_proj"].numpy(), x, n_in, 1)
    a = orc.synth_bf16(rng, nq * D)
    full_o = orc.gemv_q4(W["o_proj"].numpy(), a, HIDDEN // 32, nq)
    o_sum = np.zeros(HIDDEN)
    for r in range(world):
        plan = GatedAttnShardPlan(HIDDEN, nq, nkv, world, r)
        S = shard_gated_attention(W, plan)
        rows = plan.in_proj_tile_rows()
        loc = orc.gemv_q4(S["in_proj"].numpy(), x, len(rows), 1)
        assert np.array_equal(loc, np.concatenate([full[t * 32:(t + 1) * 32] for t in rows]))
        # its q|gate heads come first, in head order
        assert np.array_equal(loc[:plan.q_local * 2 * D], full[plan.q0 * 2 * D:(plan.q0 + plan.q_local) * 2 * D])
        ks = list(plan.o_proj_k_tiles())
        o_sum += orc.gemv_q4(S["o_proj"].numpy(), a[ks[0] * 256:(ks[-1] + 1) * 256], HIDDEN // 32, len(ks))
    np.testing.assert_allclose(o_sum, full_o, rtol=1e-4, atol=1e-3 * np.abs(full_o).max())


NQ, NKV, CTX = 4, 2, 12


def _run_rank(rank, world, port, xs, pos0, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full, _ = full_layer(NQ, NKV, seed=5)
        plan = GatedAttnShardPlan(HIDDEN, NQ, NKV, world, rank)
        bsz = xs.shape[1]
        layer = TPGatedAttentionLayer(plan, bsz, CTX, shard_gated_attention(full, plan), device="cpu",
                                      ops=GatedOracleOps())
        rng = np.random.default_rng(9)  # one seeded full cache; each rank holds its kv heads
        kc = _to_bf16(rng.standard_normal((bsz, NKV, CTX, D)))
        vc = _to_bf16(rng.standard_normal((bsz, NKV, CTX, D)))
        heads = slice(plan.kv0, plan.kv0 + plan.kv_local)
        layer.layer.k_cache.copy_(_bf(kc[:, heads]))
        layer.layer.v_cache.copy_(_bf(vc[:, heads]))
        outs = []
        for t in range(xs.shape[0]):
            layer.pos.copy_(pos0 + t)
            resid = xs[t].clone()
            outs.append(layer.step(resid).clone())
        if rank == 0:
            torch.save(torch.stack(outs), result_path)
    finally:
        dist.destroy_process_group()


def test_tp_gated_attn_gloo_matches_single_rank(tmp_path):
    rng = np.random.default_rng(13)
    xs = torch.from_numpy(rng.standard_normal((2, 2, HIDDEN)).astype(np.float32))
    pos0 = torch.tensor([4, 9], dtype=torch.int32)
    ctx_mp = mp.get_context("spawn")
    paths = {}
    for world in (1, 2):
        paths[world] = tmp_path / f"w{world}.pt"
        port = _free_port()
        procs = [ctx_mp.Process(target=_run_rank, args=(r, world, port, xs, pos0, str(paths[world])))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=240)
            assert p.exitcode == 0
    a, b = torch.load(paths[1]), torch.load(paths[2])
    for t in range(2):
        cos, rel = orc.compare(b[t].numpy(), a[t].numpy())
        assert cos >= 0.99999 and rel <= 1e-3, (t, cos, rel)
