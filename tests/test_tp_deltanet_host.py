"""Tensor-parallel gated DeltaNet host logic on CPU: the shard plan reassembles the
full layer (in_proj rows bit-identical, b/a columns, conv channels, out_proj
K-slices), and a 2-rank gloo run of TPDeltaNetLayer (two chained steps) equals the
single-rank layer.  The GPU ops are replaced by the oracle-backed shim of
tests/test_tp_host.py, extended with the DeltaNet step: this file tests the
sharding and collective plumbing, not the kernels."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llmnputest_b200.tp import DeltaNetShardPlan, TPDeltaNetLayer, shard_deltanet
from oracle import deltanet_oracle as dn
from oracle import q4nx_oracle as orc
from tests.test_tp_host import OracleOps, _bf, _free_port

HIDDEN = 256


class DeltaOracleOps(OracleOps):
    def gated_delta_step(self, qkv, z, b, a, conv_state, conv_w, A_log, dt_bias, norm_w, state, n_k_heads,
                         n_v_heads, eps=1e-6, out=None, out_f32=False, prefetch_state=False):
        d = 128
        conv_dim = (2 * n_k_heads + n_v_heads) * d
        o, conv_new, s_new = dn.gated_delta_step(
            qkv.numpy()[:, :conv_dim], z.numpy()[:, :n_v_heads * d], b.numpy()[:, :n_v_heads],
            a.numpy()[:, :n_v_heads], conv_state.numpy(), conv_w.numpy(), A_log.numpy(), dt_bias.numpy(),
            norm_w.numpy(), state.numpy(), n_k_heads, n_v_heads, d, d, eps)
        conv_state.copy_(torch.from_numpy(conv_new.astype(np.float32)))
        state.copy_(torch.from_numpy(s_new.astype(np.float32)))
        out.copy_(_bf(o))
        return out


def full_layer(nk, nv, seed=0, dense=False):
    """Seeded full layer weights; dense=True keeps b|a as a dense fp32 matrix (as a q4nx
    file's bf16 in_proj_b / in_proj_a are loaded) instead of q4 tile-rows."""
    rng = np.random.default_rng(seed)
    d = 128
    n_in = -(-((2 * nk + 2 * nv) * d + (0 if dense else 2 * nv)) // 32)
    u8 = lambda t: torch.from_numpy(np.ascontiguousarray(t).reshape(-1))
    f32 = lambda t: torch.from_numpy(np.asarray(t, np.float32))
    return {
        "in_proj": u8(orc.synth_q4_tiles(rng, n_in * (HIDDEN // 256))),
        "out_proj": u8(orc.synth_q4_tiles(rng, HIDDEN // 32 * (nv * d // 256))),
        "conv_w": f32(0.5 * rng.standard_normal(((2 * nk + nv) * d, 4))),
        "A_log": f32(np.log(rng.uniform(1, 16, nv))),
        "dt_bias": f32(rng.standard_normal(nv)),
        "norm_w": f32(1 + 0.1 * rng.standard_normal(d)),
        "input_norm": _bf(1 + 0.1 * rng.standard_normal(HIDDEN)),
        **({"ba_dense": f32(0.05 * rng.standard_normal((2 * nv, HIDDEN)))} if dense else {}),
    }, n_in


@pytest.mark.parametrize("world", [2, 4, 8])
def test_deltanet_shards_reassemble_full_layer(world):
    nk, nv = 8, 16
    W, n_in = full_layer(nk, nv, seed=world)
    rng = np.random.default_rng(1)
    x = orc.synth_bf16(rng, HIDDEN)
    full = orc.gemv_q4(W["in_proj"].numpy(), x, n_in, 1)
    c_b = (2 * nk + 2 * nv) * 128
    h = orc.synth_bf16(rng, nv * 128)
    full_out = orc.gemv_q4(W["out_proj"].numpy(), h, HIDDEN // 32, nv * 128 // 256)
    out_sum = np.zeros(HIDDEN)
    for r in range(world):
        plan = DeltaNetShardPlan(HIDDEN, nk, nv, world, r)
        S = shard_deltanet(W, plan)
        rows = plan.in_proj_tile_rows()
        loc = orc.gemv_q4(S["in_proj"].numpy(), x, len(rows), 1)
        want = np.concatenate([full[t * 32:(t + 1) * 32] for t in rows])
        assert np.array_equal(loc, want)  # the same tiles and arithmetic: bit-identical
        cb, ca = plan.local_cols()
        vh = slice(plan.v0, plan.v0 + plan.nv_local)
        assert np.array_equal(loc[cb:cb + plan.nv_local], full[c_b:c_b + nv][vh])
        assert np.array_equal(loc[ca:ca + plan.nv_local], full[c_b + nv:c_b + 2 * nv][vh])
        # the local q|k|v|z columns are the rank's heads of the full output
        d = 128
        kq = slice(plan.k0 * d, (plan.k0 + plan.nk_local) * d)
        assert np.array_equal(loc[:plan.nk_local * d], full[kq])
        assert np.array_equal(S["conv_w"].numpy(), W["conv_w"].numpy()[plan.conv_channels()])
        ks = list(plan.out_proj_k_tiles())
        out_sum += orc.gemv_q4(S["out_proj"].numpy(), h[ks[0] * 256:(ks[-1] + 1) * 256], HIDDEN // 32, len(ks))
    np.testing.assert_allclose(out_sum, full_out, rtol=1e-4, atol=1e-3 * np.abs(full_out).max())


def test_plan_refuses_cuts_inside_tiles():
    with pytest.raises(ValueError):
        DeltaNetShardPlan(HIDDEN, 4, 4, 8, 0)   # 4 k heads over 8 ranks
    with pytest.raises(ValueError):
        DeltaNetShardPlan(HIDDEN, 4, 4, 4, 0)   # one 128-wide v head per rank: half an out_proj K-tile


NK, NV = 2, 4


def _run_rank(rank, world, port, xs, result_path, dense=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full, _ = full_layer(NK, NV, seed=3, dense=dense)
        plan = DeltaNetShardPlan(HIDDEN, NK, NV, world, rank)
        layer = TPDeltaNetLayer(plan, xs.shape[1], shard_deltanet(full, plan), device="cpu", ops=DeltaOracleOps())
        # the same nonzero starting states on every world size: rank's heads of one seeded full state
        rng = np.random.default_rng(7)
        conv0 = rng.standard_normal((xs.shape[1], (2 * NK + NV) * 128, 4)).astype(np.float32)
        st0 = (0.5 * rng.standard_normal((xs.shape[1], NV, 128, 128))).astype(np.float32)
        layer.layer.conv_state.copy_(torch.from_numpy(conv0[:, plan.conv_channels()]))
        layer.layer.state.copy_(torch.from_numpy(st0[:, plan.v0:plan.v0 + plan.nv_local]))
        outs = []
        for t in range(xs.shape[0]):
            resid = xs[t].clone()
            outs.append(layer.step(resid).clone())
        if rank == 0:
            torch.save(torch.stack(outs), result_path)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dense", [False, True])  # b|a as tile-rows / dense (from a q4nx file)
def test_tp_deltanet_gloo_matches_single_rank(tmp_path, dense):
    rng = np.random.default_rng(11)
    xs = torch.from_numpy(rng.standard_normal((2, 2, HIDDEN)).astype(np.float32))
    ctx_mp = mp.get_context("spawn")
    paths = {}
    for world in (1, 2):
        paths[world] = tmp_path / f"w{world}.pt"
        port = _free_port()
        procs = [ctx_mp.Process(target=_run_rank, args=(r, world, port, xs, str(paths[world]), dense))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=240)
            assert p.exitcode == 0
    a, b = torch.load(paths[1]), torch.load(paths[2])
    for t in range(2):  # the second step reads the states the first one wrote
        cos, rel = orc.compare(b[t].numpy(), a[t].numpy())
        assert cos >= 0.99999 and rel <= 1e-3, (t, cos, rel)
