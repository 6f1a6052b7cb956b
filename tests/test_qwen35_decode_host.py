"""Qwen35Decoder composition on CPU: a 4-layer stack (three gated DeltaNet layers,
one gated attention layer, each with its SwiGLU MLP) and the q8 lm_head, two steps
at advancing positions, against the oracle composition in Qwen3_5DecoderLayer's
order (modeling_qwen3_5.py:744-785).  The GPU ops are the oracle-backed shims of
the host-logic tests: this checks the composition (layer order, residual adds,
norms, shared positions, cache and state carried across steps), not the kernels."""

import numpy as np
import pytest
import torch
from ml_dtypes import bfloat16

from llmnputest_b200.qwen35_decode import Qwen35Config, Qwen35Decoder
from oracle import deltanet_oracle as dn
from oracle import gated_attention_oracle as ga
from oracle import q4nx_oracle as orc
from tests.test_tp_deltanet_host import DeltaOracleOps
from tests.test_tp_gated_attn_host import GatedOracleOps

CFG = Qwen35Config(hidden=256, n_layers=4, layer_types=("linear_attention",) * 3 + ("full_attention",),
                   n_k_heads=2, n_v_heads=4, n_q_heads=2, n_kv_heads=1, rot_dim=64, rope_theta=10000.0,
                   intermediate=512, vocab=256)


class Q35Ops(DeltaOracleOps, GatedOracleOps):
    """Adds the tensor-core GEMM entry points (same arithmetic as the GEMV shim; the
    packing is the identity here: the shims compute on the tiles as stored)."""

    def gemm_workspace_bytes(self, *a):
        return 0

    def q4_gemm_pack(self, tiles, n_t, k_t):
        return tiles

    def q8_gemm_pack(self, tiles, n_t, k_t):
        return tiles

    def q8_gemm(self, tiles, n_t, k_t, x, out=None, accumulate=False, workspace=None, prefetch=False, norm_w=None,
                eps=0.0):
        if norm_w is not None:
            return self.gemv_rmsnorm(tiles, n_t, k_t, x, norm_w, eps, out=out, accumulate=accumulate, q8=True)
        return self.q8_gemv(tiles, n_t, k_t, x, out=out, accumulate=accumulate)

    def q4_gemm(self, tiles, n_t, k_t, x, out=None, accumulate=False, workspace=None, prefetch=False, norm_w=None,
                eps=0.0, packed=False):
        if norm_w is not None:
            return self.gemv_rmsnorm(tiles, n_t, k_t, x, norm_w, eps, out=out, accumulate=accumulate)
        return self.q4_gemv(tiles, n_t, k_t, x, out=out, accumulate=accumulate)

    def q4_swiglu_gemm(self, gate, up, n_t, k_t, x, out=None, workspace=None, prefetch=False, norm_w=None, eps=0.0,
                       packed=False):
        if norm_w is not None:
            return self.swiglu_gemv_rmsnorm(gate, up, n_t, k_t, x, norm_w, eps, out=out)
        return self.q4_swiglu_gemv(gate, up, n_t, k_t, x, out=out)


def _bf(x):
    return np.asarray(x, np.float32).astype(bfloat16).astype(np.float32)


@pytest.mark.parametrize("bsz", [2, 10])  # GEMV path, tensor-core GEMM path
def test_qwen35_decoder_matches_oracle_composition(bsz):
    ctx = 8
    dec = Qwen35Decoder(CFG, bsz, ctx, device="cpu", seed=1, ops_impl=Q35Ops())
    assert dec.use_gemm == (bsz >= 9)
    c = CFG
    W = [{k: (v.float().numpy() if v.dtype != torch.uint8 else v.numpy()) for k, v in L["mixer"].items()}
         for L in dec.w["layers"]]
    mlp = [{k: (v.float().numpy() if v.dtype != torch.uint8 else v.numpy()) for k, v in L.items() if k != "mixer"}
           for L in dec.w["layers"]]
    conv = [np.zeros((bsz, (2 * c.n_k_heads + c.n_v_heads) * 128, 4), np.float32) for _ in range(3)]
    state = [np.zeros((bsz, c.n_v_heads, 128, 128)) for _ in range(3)]
    kc = np.zeros((bsz, c.n_kv_heads, ctx, 256), np.float32)
    vc = np.zeros_like(kc)
    rng = np.random.default_rng(4)
    kt_h, nt_h = c.hidden // 256, c.hidden // 32
    for t in range(2):
        x = rng.standard_normal((bsz, c.hidden)).astype(np.float32)
        pos = (np.arange(bsz) % 5 + 2) + t
        dec.x_in.copy_(torch.from_numpy(x))
        dec.pos.copy_(torch.from_numpy(pos.astype(np.int32)))
        logits = dec.step().numpy().copy()

        r = x.copy()
        for i, kind in enumerate(c.layer_types):
            w = W[i]
            xn = _bf(orc.rmsnorm(r, w["input_norm"], c.eps))
            if kind == "linear_attention":
                m = dec.mixers[i]
                proj = orc.gemv_q4(w["in_proj"], xn, m.nt_in, kt_h)
                o, conv[i], state[i] = dn.gated_delta_step(
                    proj[:, :m.c_z], proj[:, m.c_z:m.c_z + c.n_v_heads * 128], proj[:, m.c_b:m.c_b + c.n_v_heads],
                    proj[:, m.c_a:m.c_a + c.n_v_heads], conv[i], w["conv_w"], w["A_log"], w["dt_bias"], w["norm_w"],
                    state[i], c.n_k_heads, c.n_v_heads, 128, 128, c.eps)
                r = r + orc.gemv_q4(w["out_proj"], _bf(o), nt_h, m.kt_v)
            else:
                m = dec.mixers[i]
                proj = orc.gemv_q4(w["in_proj"], xn, m.nt_in, kt_h)
                o, k_row, v_row = ga.gated_attention_step(
                    proj[:, :m.c_k], proj[:, m.c_k:m.c_v], proj[:, m.c_v:], w["q_norm_w"], w["k_norm_w"],
                    w["inv_freq"], kc, vc, pos, c.n_q_heads, c.n_kv_heads, c.eps, stored=_bf)
                for b in range(bsz):
                    kc[b, :, pos[b]] = _bf(k_row[b])
                    vc[b, :, pos[b]] = _bf(v_row[b])
                r = r + orc.gemv_q4(w["o_proj"], _bf(o), nt_h, m.kt_o)
            L = mlp[i]
            xn2 = _bf(orc.rmsnorm(r, L["post_norm"], c.eps))
            nt_i, kt_i = c.intermediate // 32, c.intermediate // 256
            h = _bf(orc.swiglu_from_accumulators(orc.gemv_q4(L["gate"], xn2, nt_i, kt_h),
                                                 orc.gemv_q4(L["up"], xn2, nt_i, kt_h)))
            r = r + orc.gemv_q4(L["down"], h, nt_h, kt_i)
        xf = _bf(orc.rmsnorm(r, dec.w["final_norm"].float().numpy(), c.eps))
        ref = orc.gemv_q8(dec.w["lm_head"].numpy(), xf, c.vocab // 32, kt_h)
        cos, rel = orc.compare(logits, ref)
        assert cos >= 0.99999 and rel <= 1e-3, (t, cos, rel)
    # the attention layer appended its rows at both steps' positions, in the shared cache
    assert np.array_equal(dec.mixers[3].k_cache.float().numpy(), kc)
