"""The composed decode step (BASELINE config 4 structure) against the numpy
composition of the reference's per-op oracles, two steps in a row, one launch per
op captured in a CUDA graph."""

import numpy as np
import pytest
import torch
from ml_dtypes import bfloat16

from oracle import q4nx_oracle as orc
from tests.test_gpu_gemv import dev_bf16, dev_u8

pytestmark = pytest.mark.gpu


def _bf(a):
    return np.asarray(a, np.float64).astype(np.float32).astype(bfloat16).astype(np.float32)


def _oracle_step(cfg, W, kc, vc, x, pos):
    """fp64/fp32 composition of the oracle ops, mutating the caches like the GPU step."""
    d, hq, hkv = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    bsz = x.shape[0]
    resid = x.astype(np.float64)
    kt_h, kt_q, kt_i = cfg.hidden // 256, hq * d // 256, cfg.intermediate // 256
    for li, L in enumerate(W["layers"]):
        xn = _bf(orc.rmsnorm(resid, L["attn_norm"], cfg.rms_eps))
        qkv = orc.gemv_q4(L["qkv"], xn, cfg.qkv_rows // 32, kt_h).astype(np.float64)
        q = np.zeros((bsz, hq, d), np.float32)
        for b in range(bsz):
            p = int(pos[b])
            q[b] = _bf(orc.rope_half_split(qkv[b, :hq * d].reshape(hq, d), p, cfg.rope_theta))
            kc[li][b, :, p] = _bf(orc.rope_half_split(qkv[b, hq * d:(hq + hkv) * d].reshape(hkv, d), p,
                                                      cfg.rope_theta))
            vc[li][b, :, p] = _bf(qkv[b, (hq + hkv) * d:].reshape(hkv, d))
        attn = _bf(orc.gqa_decode(q, kc[li], vc[li], np.asarray(pos) + 1, d ** -0.5).reshape(bsz, hq * d))
        resid = resid + orc.gemv_q4(L["o"], attn, cfg.hidden // 32, kt_q)
        xn = _bf(orc.rmsnorm(resid, L["mlp_norm"], cfg.rms_eps))
        g32 = orc.gemv_q4(L["gate"], xn, cfg.intermediate // 32, kt_h)
        u32 = orc.gemv_q4(L["up"], xn, cfg.intermediate // 32, kt_h)
        h = _bf(orc.swiglu_from_accumulators(g32, u32))
        resid = resid + orc.gemv_q4(L["down"], h, cfg.hidden // 32, kt_i)
    xf = _bf(orc.rmsnorm(resid, W["final_norm"], cfg.rms_eps))
    return orc.gemv_q8(W["lm_head"], xf, cfg.vocab // 32, kt_h)


@pytest.mark.parametrize("bsz,start", [(1, [40]), (3, [40, 5, 61])])
def test_decode_steps_vs_oracle(bsz, start):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llmnputest_b200.decode import DecoderConfig, Q4Decoder
    cfg = DecoderConfig(n_layers=2, vocab=1024)
    ctx = 64
    rng = np.random.default_rng(100 + bsz)
    kt_h, kt_q, kt_i = cfg.hidden // 256, cfg.n_heads * cfg.head_dim // 256, cfg.intermediate // 256
    W = {"layers": [], "final_norm": (rng.standard_normal(cfg.hidden) * 0.1 + 1).astype(np.float32).astype(bfloat16),
         "lm_head": orc.synth_q8_tiles(rng, cfg.vocab // 32 * kt_h)}
    for _ in range(cfg.n_layers):
        W["layers"].append({
            "qkv": orc.synth_q4_tiles(rng, cfg.qkv_rows // 32 * kt_h),
            "o": orc.synth_q4_tiles(rng, cfg.hidden // 32 * kt_q),
            "gate": orc.synth_q4_tiles(rng, cfg.intermediate // 32 * kt_h),
            "up": orc.synth_q4_tiles(rng, cfg.intermediate // 32 * kt_h),
            "down": orc.synth_q4_tiles(rng, cfg.hidden // 32 * kt_i),
            "attn_norm": (rng.standard_normal(cfg.hidden) * 0.1 + 1).astype(np.float32).astype(bfloat16),
            "mlp_norm": (rng.standard_normal(cfg.hidden) * 0.1 + 1).astype(np.float32).astype(bfloat16),
        })
    dev_w = {"layers": [{k: (dev_u8(v) if v.dtype == np.uint8 else dev_bf16(v.astype(np.float32)))
                         for k, v in L.items()} for L in W["layers"]],
             "final_norm": dev_bf16(W["final_norm"].astype(np.float32)), "lm_head": dev_u8(W["lm_head"])}
    dec = Q4Decoder(cfg, bsz, ctx, weights=dev_w)
    # caches filled with history up to each sequence's position
    kc = [orc.synth_bf16(rng, (bsz, cfg.n_kv_heads, ctx, cfg.head_dim)).astype(np.float32) for _ in range(2)]
    vc = [orc.synth_bf16(rng, (bsz, cfg.n_kv_heads, ctx, cfg.head_dim)).astype(np.float32) for _ in range(2)]
    for li in range(2):
        dec.k_cache[li].copy_(dev_bf16(kc[li]))
        dec.v_cache[li].copy_(dev_bf16(vc[li]))
    graph = dec.capture()
    pos = np.asarray(start, np.int32)
    for step in range(2):
        x = rng.standard_normal((bsz, cfg.hidden)).astype(np.float32)
        dec.x_in.copy_(torch.from_numpy(x))
        dec.pos.copy_(torch.from_numpy(pos))
        graph.replay()
        torch.cuda.synchronize()
        got = dec.logits.cpu().numpy()
        ref = _oracle_step(cfg, W, kc, vc, x, pos)
        for b in range(bsz):
            cos, rel = orc.compare(got[b], ref[b])
            # two layers of bf16 re-roundings on either side: cos >= 0.9999, rel <= 1e-2
            assert cos >= 0.9999 and rel <= 1e-2, (step, b, cos, rel)
        # the appended k/v of every layer match the oracle's cache (bf16, <= 1 ulp for k)
        for li in range(2):
            for b in range(bsz):
                p = int(pos[b])
                got_k = dec.k_cache[li][b, :, p].float().cpu().numpy()
                np.testing.assert_allclose(got_k, kc[li][b, :, p], rtol=2 ** -6, atol=1e-3)
        pos = pos + 1
    from llmnputest_b200 import ops
    assert ops.device_error() == 0
