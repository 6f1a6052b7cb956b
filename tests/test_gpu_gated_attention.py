"""Qwen3.5 gated full-attention decode on the GPU through the C ABI (b2_gated_attn_decode).

Checked against transformers' own module outputs (tests/golden/gated_attn_golden.npz)
and against the float64 oracle.  The kernel's KV cache is bf16: against the oracle run
on the same bf16 cache values (the appended row included) the gate is the north star's (cos >= 0.99999, max rel
err <= 1e-3, fp32 output); against the module, whose float32 cache the bf16 cache
rounds, cos >= 0.9999 and rel <= 1e-2.  The appended v row is bit-exact (one bf16
rounding of the projection output); the appended k row within one bf16 ulp."""

from pathlib import Path

import numpy as np
import pytest
import torch
from ml_dtypes import bfloat16

from oracle import gated_attention_oracle as ga
from tests.test_gpu_gemv import assert_close

pytestmark = pytest.mark.gpu
NS_COS, NS_REL = 0.99999, 1e-3
GOLDEN = Path(__file__).resolve().parent / "golden" / "gated_attn_golden.npz"
D = 256


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llmnputest_b200 import ops as _ops
    return _ops


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).cuda()


def bf16_cache(c):
    """bf16 device cache from fp32 host values, plus the fp32 image of the rounded values."""
    r = np.ascontiguousarray(np.asarray(c, np.float32).astype(bfloat16))
    return torch.from_numpy(r.view(np.int16)).view(torch.bfloat16).cuda(), r.astype(np.float32)


def inv_freq_of(rot: int, theta: float) -> np.ndarray:
    """transformers' default RoPE frequencies, as Qwen3_5TextRotaryEmbedding forms them."""
    return (1.0 / (theta ** (np.arange(0, rot, 2, dtype=np.int64).astype(np.float32) / rot))).astype(np.float32)


def run(ops, inp, nq, nkv, pos, ctx_max, max_len=None, out_f32=True):
    kc, kc32 = bf16_cache(inp["k_cache"])
    vc, vc32 = bf16_cache(inp["v_cache"])
    out = ops.gated_attn_decode(dev(inp["qg"]), dev(inp["k_new"]), dev(inp["v_new"]), dev(inp["q_norm_w"]),
                                dev(inp["k_norm_w"]), dev(inp["inv_freq"]), kc, vc,
                                torch.tensor(pos, dtype=torch.int32, device="cuda"), nq, nkv, max_len=max_len,
                                out_f32=out_f32)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), kc, vc, kc32, vc32


def synth(rng, bsz, nq, nkv, ctx_max, rot=64, theta=10000.0):
    f = np.float32
    return {
        "qg": rng.standard_normal((bsz, nq * 2 * D), dtype=f),
        "k_new": rng.standard_normal((bsz, nkv * D), dtype=f),
        "v_new": rng.standard_normal((bsz, nkv * D), dtype=f),
        "q_norm_w": f(0.1) * rng.standard_normal(D, dtype=f),
        "k_norm_w": f(0.1) * rng.standard_normal(D, dtype=f),
        "inv_freq": inv_freq_of(rot, theta),
        "k_cache": rng.standard_normal((bsz, nkv, ctx_max, D), dtype=f),
        "v_cache": rng.standard_normal((bsz, nkv, ctx_max, D), dtype=f),
    }


def to_bf16(x):
    """The values the bf16 cache holds for an appended row (the kernel reads the row back)."""
    return np.asarray(x, np.float32).astype(bfloat16).astype(np.float32)


def bf16_ulp_close(got, ref):
    r = np.asarray(ref, np.float32)
    ulp = np.abs(r.astype(bfloat16).astype(np.float32)) * 2.0 ** -7 + 1e-30
    return np.all(np.abs(np.asarray(got, np.float32) - r) <= ulp)


@pytest.mark.parametrize("name", ["g4", "c5", "g2full"])
def test_matches_transformers_golden(ops, name):
    g = np.load(GOLDEN)
    bsz, nq, nkv, d, pos = (int(x) for x in g[f"{name}/dims"])
    ctx_max = pos + 3
    kc0, vc0 = ga.plant_cache(int(g[f"{name}/plant_seed"]), (bsz, nkv, pos, d))
    inp = {k: g[f"{name}/{k}"] for k in ("qg", "k_new", "v_new", "q_norm_w", "k_norm_w", "inv_freq")}
    pad = np.zeros((bsz, nkv, ctx_max - pos, d), np.float32)
    inp["k_cache"], inp["v_cache"] = np.concatenate([kc0, pad], 2), np.concatenate([vc0, pad], 2)
    out, kc, vc, kc32, vc32 = run(ops, inp, nq, nkv, [pos] * bsz, ctx_max)
    assert_close(out, g[f"{name}/out"], 0.9999, 1e-2, f"{name} vs module")
    ref, _, _ = ga.gated_attention_step(inp["qg"], inp["k_new"], inp["v_new"], inp["q_norm_w"], inp["k_norm_w"],
                                        inp["inv_freq"], kc32, vc32, [pos] * bsz, nq, nkv, stored=to_bf16)
    assert_close(out, ref, NS_COS, NS_REL, f"{name} vs oracle on the bf16 cache")
    v_row = vc.float().cpu().numpy()[:, :, pos]
    assert np.array_equal(v_row, g[f"{name}/v_row"].astype(bfloat16).astype(np.float32))
    assert bf16_ulp_close(kc.float().cpu().numpy()[:, :, pos], g[f"{name}/k_row"])


CASES = [  # batch, q heads, kv heads, ctx_max, positions, rotary dims
    (1, 8, 2, 2048, [2047], 64),            # config 5's heads at its context: split + combine
    (3, 4, 1, 700, [699, 10, 355], 64),     # ragged positions across the batch
    (2, 2, 1, 300, [0, 299], 256),          # first position (one key) and full rotary, G = 2
    (5, 2, 2, 130, [129, 64, 1, 100, 17], 64),  # G = 1
    (64, 8, 2, 512, None, 64),              # 128 (kv head, sequence) pairs: splits
    (160, 8, 2, 96, None, 64),              # 320 pairs fill the SMs: one split, no combine
]


@pytest.mark.parametrize("bsz,nq,nkv,ctx,pos,rot", CASES)
def test_vs_oracle(ops, bsz, nq, nkv, ctx, pos, rot):
    rng = np.random.default_rng(bsz * 31 + ctx)
    inp = synth(rng, bsz, nq, nkv, ctx, rot)
    pos = list(rng.integers(0, ctx, bsz)) if pos is None else pos
    out, kc, vc, kc32, vc32 = run(ops, inp, nq, nkv, pos, ctx)
    ref, k_row, v_row = ga.gated_attention_step(inp["qg"], inp["k_new"], inp["v_new"], inp["q_norm_w"],
                                                inp["k_norm_w"], inp["inv_freq"], kc32, vc32, pos, nq, nkv,
                                                stored=to_bf16)
    assert_close(out, ref, NS_COS, NS_REL, "out")
    for b in range(bsz):  # every sequence and head on its own
        for h in range(nq):
            sl = slice(h * D, (h + 1) * D)
            assert_close(out[b, sl], ref[b, sl], NS_COS, NS_REL, f"b{b} h{h}")
    kcn, vcn = kc.float().cpu().numpy(), vc.float().cpu().numpy()
    for b in range(bsz):
        assert np.array_equal(vcn[b, :, pos[b]], v_row[b].astype(np.float32).astype(bfloat16).astype(np.float32))
        assert bf16_ulp_close(kcn[b, :, pos[b]], k_row[b])
        # rows other than pos are untouched
        keep = np.ones(ctx, bool)
        keep[pos[b]] = False
        assert np.array_equal(kcn[b][:, keep], kc32[b][:, keep])


def test_bf16_output_and_chained_steps(ops):
    """Three steps at pos, pos+1, pos+2: each reads the rows the earlier steps appended."""
    bsz, nq, nkv, ctx = 2, 8, 2, 200
    rng = np.random.default_rng(9)
    inp = synth(rng, bsz, nq, nkv, ctx)
    kc, kc32 = bf16_cache(inp["k_cache"])
    vc, vc32 = bf16_cache(inp["v_cache"])
    pos0 = [150, 20]
    prm = {k: dev(inp[k]) for k in ("q_norm_w", "k_norm_w", "inv_freq")}
    for t in range(3):
        step = synth(rng, bsz, nq, nkv, 1)
        pos = [p + t for p in pos0]
        out = ops.gated_attn_decode(dev(step["qg"]), dev(step["k_new"]), dev(step["v_new"]), prm["q_norm_w"],
                                    prm["k_norm_w"], prm["inv_freq"], kc, vc,
                                    torch.tensor(pos, dtype=torch.int32, device="cuda"), nq, nkv)
        ref, k_row, v_row = ga.gated_attention_step(step["qg"], step["k_new"], step["v_new"], inp["q_norm_w"],
                                                    inp["k_norm_w"], inp["inv_freq"], kc32, vc32, pos, nq, nkv,
                                                    stored=to_bf16)
        torch.cuda.synchronize()
        assert_close(out.float().cpu().numpy(), ref, 0.9999, 4e-3, f"step {t} (bf16 out)")
        for b in range(bsz):  # the oracle's cache takes the kernel's appended rows
            kc32[b, :, pos[b]] = kc[b, :, pos[b]].float().cpu().numpy()
            vc32[b, :, pos[b]] = vc[b, :, pos[b]].float().cpu().numpy()


def test_config5_full_batch_sampled(ops):
    """Config 5's size: 256 sequences x 2 kv heads x 2048 positions (1.07 GB of bf16 K/V):
    a sequence's output depends on that sequence alone, so three are checked."""
    bsz, nq, nkv, ctx = 256, 8, 2, 2048
    rng = np.random.default_rng(2048)
    kc = torch.randn(bsz, nkv, ctx, D, device="cuda").to(torch.bfloat16)
    vc = torch.randn(bsz, nkv, ctx, D, device="cuda").to(torch.bfloat16)
    small = synth(rng, bsz, nq, nkv, 1)
    pos = torch.full((bsz,), ctx - 1, dtype=torch.int32, device="cuda")
    out = ops.gated_attn_decode(dev(small["qg"]), dev(small["k_new"]), dev(small["v_new"]), dev(small["q_norm_w"]),
                                dev(small["k_norm_w"]), dev(small["inv_freq"]), kc, vc, pos, nq, nkv, out_f32=True)
    torch.cuda.synchronize()
    out = out.cpu().numpy()
    pick = [0, 131, 255]
    kp = kc[pick].float().cpu().numpy()
    vp = vc[pick].float().cpu().numpy()
    sub = {k: small[k][pick] for k in ("qg", "k_new", "v_new")}
    ref, _, _ = ga.gated_attention_step(sub["qg"], sub["k_new"], sub["v_new"], small["q_norm_w"], small["k_norm_w"],
                                        small["inv_freq"], kp, vp, [ctx - 1] * 3, nq, nkv, stored=to_bf16)
    assert_close(out[pick], ref, NS_COS, NS_REL, "sampled sequences")
    assert np.isfinite(out).all()


def test_rejected_or_flagged(ops):
    """Unbuilt shapes are refused on the host; a position outside max_len is refused by the
    kernel's own check (device error 5, nothing written)."""
    from llmnputest_b200 import _native
    rng = np.random.default_rng(4)
    inp = synth(rng, 1, 8, 1, 64)  # 8 q heads per kv head: not built
    kc, _ = bf16_cache(inp["k_cache"])
    vc, _ = bf16_cache(inp["v_cache"])
    pos = torch.tensor([5], dtype=torch.int32, device="cuda")
    t = {k: dev(inp[k]) for k in ("qg", "k_new", "v_new", "q_norm_w", "k_norm_w", "inv_freq")}
    with pytest.raises(_native.B2Error):
        ops.gated_attn_decode(t["qg"], t["k_new"], t["v_new"], t["q_norm_w"], t["k_norm_w"], t["inv_freq"], kc, vc,
                              pos, 8, 1)
    with pytest.raises(_native.B2Error):  # max_len above ctx_max
        ops.gated_attn_decode(t["qg"], t["k_new"], t["v_new"], t["q_norm_w"], t["k_norm_w"], t["inv_freq"], kc, vc,
                              pos, 4, 1, max_len=65)
    # 4 q heads on the same buffers (qg holds 8 heads' worth, more than needed); pos 40 >= max_len 32
    before = kc.clone()
    assert ops.device_error() == 0
    ops.gated_attn_decode(t["qg"], t["k_new"], t["v_new"], t["q_norm_w"], t["k_norm_w"], t["inv_freq"], kc, vc,
                          torch.tensor([40], dtype=torch.int32, device="cuda"), 4, 1, max_len=32)
    assert ops.device_error() == 5
    assert torch.equal(kc, before)
