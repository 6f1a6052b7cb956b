"""GQA flash-decode attention, RoPE and RMSNorm on the GPU through the C ABI.

Tolerance: the north star's cos >= 0.99999 and max rel err <= 1e-3 on fp32
outputs (float64 metric); bf16 outputs add 2^-9 of storage rounding, so their
gate is the storage floor (4e-3, as granite_rmsnorm.py:117-119 sets it)."""

import numpy as np
import pytest
import torch
from ml_dtypes import bfloat16

from oracle import q4nx_oracle as orc
from tests.conftest import bf16_from_bits
from tests.test_gpu_gemv import assert_close, dev_bf16

pytestmark = pytest.mark.gpu
NS_COS, NS_REL = 0.99999, 1e-3


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llmnputest_b200 import ops as _ops
    return _ops


def f32dev(a):
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).cuda()


@pytest.mark.parametrize("seq", [32, 64, 128, 77])
def test_attention_golden(ops, golden, seq):
    """One q head against the reference's own cases (granite_attention.py:141, 163-167)."""
    q = bf16_from_bits(golden[f"attn{seq}_q"]).astype(np.float32)[None]
    k = bf16_from_bits(golden[f"attn{seq}_k"])
    v = bf16_from_bits(golden[f"attn{seq}_v"])
    kc = dev_bf16(k.astype(np.float32)).view(1, 1, seq, 64)
    vc = dev_bf16(v.astype(np.float32)).view(1, 1, seq, 64)
    pos = torch.tensor([seq - 1], dtype=torch.int32, device="cuda")
    qd = f32dev(q)
    out = ops.gqa_decode(qd, qd, qd, kc, vc, pos, n_q_heads=1, n_kv_heads=1, scale=0.125,
                         append=False, rope=False, out_f32=True)
    assert_close(out.cpu().numpy()[0], golden[f"attn{seq}_ref"], NS_COS, NS_REL, f"seq {seq}")
    outb = ops.gqa_decode(qd, qd, qd, kc, vc, pos, n_q_heads=1, n_kv_heads=1, scale=0.125,
                          append=False, rope=False)
    assert_close(outb.float().cpu().numpy()[0], golden[f"attn{seq}_ref"], NS_COS, 4e-3, f"seq {seq} bf16")


@pytest.mark.parametrize("pos", [0, 17, 4095, 32767])
def test_rope_append_golden(ops, golden, pos):
    """The appended k is the half-split rotation (granite_elementwise.py:136-150) --
    and NOT the interleaved one (granite_elementwise.py:153-162)."""
    x = bf16_from_bits(golden[f"rope{pos}_x"]).astype(np.float32).reshape(1, 40 * 64)
    ref, alt = golden[f"rope{pos}_ref"], golden[f"rope{pos}_alt"]
    ctx = pos + 1
    kc = torch.zeros(1, 40, ctx, 64, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    xd = f32dev(x)
    p = torch.tensor([pos], dtype=torch.int32, device="cuda")
    ops.gqa_decode(xd, xd, xd, kc, vc, p, n_q_heads=40, n_kv_heads=40, theta=10000.0)
    got = kc[0, :, pos].float().cpu().numpy().reshape(-1)
    assert_close(got, ref, NS_COS, 4e-3, "rope")  # bf16 cache: storage floor
    if pos > 0:  # at position 0 both conventions are the identity
        alt_rel = np.abs(got - alt).max() / np.abs(alt).max()
        assert alt_rel > 0.1, "the interleaved convention must not match"
    # v is appended unrotated
    assert np.array_equal(vc[0, :, pos].float().cpu().numpy().reshape(-1),
                          x.astype(bfloat16).astype(np.float32).reshape(-1))


def _gqa_case(ops, bsz, hq, hkv, ctx_max, lens, seed, out_f32=True, prefetch_kv=False):
    rng = np.random.default_rng(seed)
    d = 64
    kc_np = orc.synth_bf16(rng, (bsz, hkv, ctx_max, d))
    vc_np = orc.synth_bf16(rng, (bsz, hkv, ctx_max, d))
    qkv = rng.standard_normal((bsz, (hq + 2 * hkv) * d)).astype(np.float32)
    pos = np.asarray(lens, np.int32) - 1
    kc = dev_bf16(kc_np.astype(np.float32))
    vc = dev_bf16(vc_np.astype(np.float32))
    qkv_d = f32dev(qkv)
    qd, kd, vd = qkv_d[:, :hq * d], qkv_d[:, hq * d:(hq + hkv) * d], qkv_d[:, (hq + hkv) * d:]
    out = ops.gqa_decode(qd, kd, vd, kc, vc, torch.from_numpy(pos).cuda(), n_q_heads=hq, n_kv_heads=hkv,
                         theta=10000.0, max_len=int(max(lens)), out_f32=out_f32, prefetch_kv=prefetch_kv)
    # oracle: rotate the new q/k in float64, narrow to bf16 (the QKV epilogue), append, attend
    kref = kc_np.astype(np.float32).copy()
    vref = vc_np.astype(np.float32).copy()
    qref = np.zeros((bsz, hq, d), np.float32)
    for b in range(bsz):
        p = int(pos[b])
        qh = qkv[b, :hq * d].reshape(hq, d)
        kh = qkv[b, hq * d:(hq + hkv) * d].reshape(hkv, d)
        vh = qkv[b, (hq + hkv) * d:].reshape(hkv, d)
        qref[b] = orc.rope_half_split(qh, p, 10000.0).astype(np.float32).astype(bfloat16).astype(np.float32)
        kref[b, :, p] = orc.rope_half_split(kh, p, 10000.0).astype(np.float32).astype(bfloat16).astype(np.float32)
        vref[b, :, p] = vh.astype(bfloat16).astype(np.float32)
    ref = orc.gqa_decode(qref, kref, vref, lens, d ** -0.5)
    got = out.float().cpu().numpy().reshape(bsz, hq, d)
    # the cache now holds the appended token (bf16 rounding of the fp32 rotation: <= 1 ulp)
    kc_new = kc.float().cpu().numpy()
    for b in range(bsz):
        p = int(pos[b])
        np.testing.assert_allclose(kc_new[b, :, p], kref[b, :, p], rtol=2 ** -7, atol=1e-6)
        assert np.array_equal(vc.float().cpu().numpy()[b, :, p], vref[b, :, p])
    return got, ref


@pytest.mark.parametrize("bsz,ctx,lens", [
    (1, 32, [32]), (1, 77, [77]), (1, 512, [512]), (2, 4096, [4096, 1000]),
    (3, 600, [1, 17, 600]), (1, 32768, [32768]),
])
def test_gqa_vs_oracle(ops, bsz, ctx, lens):
    got, ref = _gqa_case(ops, bsz, 40, 8, ctx, lens, seed=ctx + bsz)
    for b in range(bsz):  # every sequence, every head
        assert_close(got[b], ref[b], NS_COS, NS_REL, f"seq {b} len {lens[b]}")


@pytest.mark.parametrize("bsz,ctx,lens", [(1, 4096, [4096]), (1, 100, [17]), (3, 2048, [2048, 31, 1500]),
                                          (64, 512, None)])
def test_gqa_prefetch_kv(ops, bsz, ctx, lens):
    """B2_ATTN_PREFETCH_KV: K/V chunks read before the wait on the preceding kernel;
    the chunk that reaches the appended row pos is read after it, so the result is
    the oracle's (8-warp and 4-warp launches, appended row in the first or a later chunk)."""
    lens = lens or list(np.random.default_rng(64).integers(1, ctx + 1, bsz))
    got, ref = _gqa_case(ops, bsz, 40, 8, ctx, lens, seed=ctx + 7 * bsz, prefetch_kv=True)
    for b in range(bsz):
        assert_close(got[b], ref[b], NS_COS, NS_REL, f"seq {b} len {lens[b]}")


@pytest.mark.parametrize("bsz,ctx,lens", [
    (32, 4096, None),                                   # the B = 32 decode shape, ragged lengths
    (7, 9000, [9000, 1, 64, 65, 4097, 8999, 128]),      # lengths at and around 64-position edges
    (48, 2048, [2048] * 48),                            # equal lengths, more pairs than CTA slots
])
def test_gqa_large_kv_vs_oracle(ops, bsz, ctx, lens):
    """Launches whose K/V exceed 64 MB: unclustered, capped at one wave of CTAs, merged by
    the combine kernel where a sequence is split.  Every sequence and head against the
    oracle."""
    lens = lens or [int(v) for v in np.random.default_rng(bsz).integers(1, ctx + 1, bsz)]
    got, ref = _gqa_case(ops, bsz, 40, 8, ctx, lens, seed=ctx + 3 * bsz)
    for b in range(bsz):
        assert_close(got[b], ref[b], NS_COS, NS_REL, f"seq {b} len {lens[b]}")
    assert ops.device_error() == 0


def test_gqa_batch16_bf16_out(ops):
    lens = list(np.random.default_rng(5).integers(1, 4097, 16))
    got, ref = _gqa_case(ops, 16, 40, 8, 4096, lens, seed=16, out_f32=False)
    for b in range(16):
        assert_close(got[b], ref[b], NS_COS, 4e-3, f"seq {b}")


def test_rmsnorm_golden(ops, golden):
    x = bf16_from_bits(golden["rms_x"])
    w = bf16_from_bits(golden["rms_w"])
    y = ops.rmsnorm(dev_bf16(x.astype(np.float32)), dev_bf16(w.astype(np.float32)), 1e-6)
    # gate of granite_rmsnorm.py:119 (bf16 output)
    assert_close(y.float().cpu().numpy(), golden["rms_ref"], NS_COS, 4e-3, "rmsnorm")


def test_rmsnorm_f32_batch(ops):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((5, 2560)) * 3).astype(np.float32)
    w = (rng.standard_normal(2560) * 0.1 + 1.0).astype(np.float32).astype(bfloat16)
    y = ops.rmsnorm(f32dev(x), dev_bf16(w.astype(np.float32)), 1e-6).float().cpu().numpy()
    ref = orc.rmsnorm(x, w, 1e-6)
    for b in range(5):
        assert_close(y[b], ref[b], NS_COS, 4e-3, f"row {b}")
