"""Tensor-parallel Qwen3.5 stack host logic on CPU: the shard plan's uneven K-tile
split, and 2-rank gloo runs of TPQwen35Decoder (DeltaNet by k head, gated attention
by kv head or replicated, SwiGLU MLP by whole K-tiles split unevenly, vocab-sharded
q8 lm_head) equal to the single-rank stack and to Qwen35Decoder, over two steps.
The GPU ops are the oracle-backed shims: this tests sharding and collectives."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llmnputest_b200.qwen35_decode import Qwen35Config, Qwen35Decoder
from llmnputest_b200.tp_qwen35 import Qwen35ShardPlan, TPQwen35Decoder, shard_qwen35, split_even
from oracle import q4nx_oracle as orc
from tests.test_qwen35_decode_host import Q35Ops
from tests.test_tp_host import _free_port


def cfg_of(nkv: int) -> Qwen35Config:
    return Qwen35Config(hidden=256, n_layers=4, layer_types=("linear_attention",) * 3 + ("full_attention",),
                        n_k_heads=2, n_v_heads=4, n_q_heads=2 * nkv, n_kv_heads=nkv, rot_dim=64,
                        rope_theta=10000.0, intermediate=768, vocab=512)


def test_split_even_covers_every_unit_once():
    for n, w in ((14, 4), (14, 8), (3, 2), (16, 8)):
        parts = [split_even(n, w, r) for r in range(w)]
        assert [u for p in parts for u in p] == list(range(n))
        assert max(map(len, parts)) - min(map(len, parts)) <= 1
    # config 5: 14 intermediate K-tiles over 4 ranks
    assert [len(split_even(14, 4, r)) for r in range(4)] == [4, 4, 3, 3]


def _inputs(cfg, bsz=2):
    rng = np.random.default_rng(21)
    xs = torch.from_numpy(rng.standard_normal((2, bsz, cfg.hidden)).astype(np.float32))
    return xs, torch.from_numpy((np.arange(bsz) % 6 + 3).astype(np.int32))


def _full(cfg):
    return Qwen35Decoder(cfg, 1, 1, device="cpu", seed=7, ops_impl=Q35Ops()).w


def _run_rank(rank, world, port, nkv, result_path, bsz):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = cfg_of(nkv)
        xs, pos = _inputs(cfg, bsz)
        plan = Qwen35ShardPlan(cfg, world, rank)
        dec = TPQwen35Decoder(cfg, xs.shape[1], 12, shard_qwen35(_full(cfg), plan), plan, device="cpu",
                              ops=Q35Ops())
        outs = []
        for t in range(2):
            dec.x_in.copy_(xs[t])
            dec.pos.copy_(pos + t)
            outs.append(dec.step().clone())
        if rank == 0:
            torch.save(torch.stack(outs), result_path)
    finally:
        dist.destroy_process_group()


# attention sharded by kv head / replicated (1 kv head, 2 ranks); GEMV path / tcgen05 GEMM path
@pytest.mark.parametrize("nkv,bsz", [(2, 2), (1, 2), (2, 10)])
def test_tp_qwen35_gloo_matches_single_rank(tmp_path, nkv, bsz):
    ctx_mp = mp.get_context("spawn")
    paths = {}
    for world in (1, 2):
        paths[world] = tmp_path / f"w{world}.pt"
        port = _free_port()
        procs = [ctx_mp.Process(target=_run_rank, args=(r, world, port, nkv, str(paths[world]), bsz))
                 for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=300)
            assert p.exitcode == 0
    a, b = torch.load(paths[1]), torch.load(paths[2])
    for t in range(2):
        cos, rel = orc.compare(b[t].numpy(), a[t].numpy())
        assert cos >= 0.99999 and rel <= 1e-3, (t, cos, rel)
    # and the single-rank TP stack is the plain stack
    cfg = cfg_of(nkv)
    xs, pos = _inputs(cfg, bsz)
    dec = Qwen35Decoder(cfg, xs.shape[1], 12, device="cpu", weights=_full(cfg), ops_impl=Q35Ops())
    for t in range(2):
        dec.x_in.copy_(xs[t])
        dec.pos.copy_(pos + t)
        cos, rel = orc.compare(a[t].numpy(), dec.step().numpy())
        assert cos >= 0.99999 and rel <= 1e-3, ("plain", t, cos, rel)
