"""Pin the CPU oracle to the reference: every restated function against the
golden vectors that tests/golden/make_golden.py produced by running the
reference's own code.  CPU only."""

import numpy as np
import pytest
from ml_dtypes import bfloat16

from oracle import q4nx_oracle as orc
from tests.conftest import bf16_from_bits


def test_meta_index(golden):
    assert np.array_equal(orc.meta_of_weight(), golden["fmt_meta_index"])


def test_unpack_and_tile_matrix(golden):
    assert np.array_equal(orc.q4_codes(golden["fmt_q4_tiles"][0, 1024:]), golden["fmt_q4_unpack"])
    assert np.array_equal(orc.tile_matrix(np.arange(8192, dtype=np.int32)), golden["fmt_to_matrix"])


def test_dequant_bf16_bit_exact(golden):
    for i, t in enumerate(golden["fmt_q4_tiles"]):
        got = orc.q4_tile_bf16(t).view(np.uint16)
        assert np.array_equal(got, golden["fmt_q4_dequant_bf16"][i]), i
    for i, t in enumerate(golden["fmt_q8_tiles"]):
        got = orc.q8_tile_bf16(t).view(np.uint16)
        assert np.array_equal(got, golden["fmt_q8_dequant_bf16"][i]), i


def test_dequant_f32_and_untile_exact(golden):
    t4, t8 = golden["fmt_q4_tiles"], golden["fmt_q8_tiles"]
    assert np.array_equal(orc.q4_tiles_f32(t4), golden["fmt_q4_f32"])
    assert np.array_equal(orc.q8_tiles_f32(t8), golden["fmt_q8_f32"])
    assert np.array_equal(orc.untile(orc.q4_tiles_f32(t4), 3, 2), golden["fmt_q4_untiled_3x2"])
    assert np.array_equal(orc.untile(orc.q8_tiles_f32(t8), 2, 3), golden["fmt_q8_untiled_2x3"])


@pytest.mark.parametrize("kind", ["q4", "q8"])
def test_gemv_oracle_matches_reference(golden, kind):
    n_t, k_t = (int(v) for v in golden[f"{kind}_shape"])
    w = golden[f"{kind}_w"]
    x = bf16_from_bits(golden[f"{kind}_x"])
    fn = orc.gemv_q4 if kind == "q4" else orc.gemv_q8
    got = fn(w, x, n_t, k_t)
    ref = golden[f"{kind}_y"]
    # same float32 arithmetic in the same order: expected bit-identical
    assert np.array_equal(got, ref)


def test_gemv_onehot_is_a_column(golden):
    """onehot:k isolates one K column, so a layout error is a permutation (README.md:188-190)."""
    n_t, k_t = (int(v) for v in golden["q4_shape"])
    w = orc.q4_matrix(golden["q4_w"], n_t, k_t)
    x = bf16_from_bits(golden["q4_x"]).astype(np.float32)
    hot = np.flatnonzero(x[4])
    assert hot.tolist() == [100]
    assert np.array_equal(golden["q4_y"][4], w[:, 100])


@pytest.mark.parametrize("seq", [32, 64, 128, 77])
def test_attention_oracle(golden, seq):
    q = bf16_from_bits(golden[f"attn{seq}_q"])
    k = bf16_from_bits(golden[f"attn{seq}_k"])
    v = bf16_from_bits(golden[f"attn{seq}_v"])
    got = orc.attention_one_head(q, k, v, 0.125)
    np.testing.assert_allclose(got, golden[f"attn{seq}_ref"], rtol=1e-12, atol=1e-14)
    # and the batched GQA form, with this head as q head 3 of a 5-head group
    qb = np.zeros((1, 5, 64), np.float32)
    qb[0, 3] = q.astype(np.float32)
    kb = k.astype(np.float32)[None, None]
    vb = v.astype(np.float32)[None, None]
    got2 = orc.gqa_decode(qb, kb, vb, [seq], 0.125)[0, 3]
    np.testing.assert_allclose(got2, golden[f"attn{seq}_ref"], rtol=1e-12, atol=1e-14)


@pytest.mark.parametrize("pos", [0, 17, 4095, 32767])
def test_rope_oracle(golden, pos):
    x = bf16_from_bits(golden[f"rope{pos}_x"]).reshape(40, 64)
    got = orc.rope_half_split(x, pos, 10000.0).reshape(-1)
    np.testing.assert_allclose(got, golden[f"rope{pos}_ref"], rtol=0, atol=1e-12)
    alt = orc.rope_interleaved(x, pos, 10000.0).reshape(-1)
    np.testing.assert_allclose(alt, golden[f"rope{pos}_alt"], rtol=0, atol=1e-12)


def test_swiglu_rmsnorm_oracles(golden):
    g = bf16_from_bits(golden["swiglu_g"])
    u = bf16_from_bits(golden["swiglu_u"])
    np.testing.assert_allclose(orc.swiglu(g, u), golden["swiglu_ref"], rtol=1e-13, atol=0)
    x = bf16_from_bits(golden["rms_x"])
    w = bf16_from_bits(golden["rms_w"])
    np.testing.assert_allclose(orc.rmsnorm(x, w, 1e-6), golden["rms_ref"], rtol=1e-13, atol=0)


def test_mlp_oracles(golden):
    tr, kt = (int(v) for v in golden["mlp_shape"])
    x = bf16_from_bits(golden["mlp_x"])
    g32 = orc.gemv_q4(golden["mlp_gate"], x, tr, kt)
    u32 = orc.gemv_q4(golden["mlp_up"], x, tr, kt)
    np.testing.assert_allclose(orc.swiglu_from_accumulators(g32, u32), golden["mlp_ref"],
                               rtol=1e-13, atol=0)
    hidden, inter = (int(v) for v in golden["mlpf_shape"])
    h, out = orc.mlp_block(golden["mlpf_gate"], golden["mlpf_up"], golden["mlpf_down"],
                           bf16_from_bits(golden["mlpf_x"]), hidden, inter)
    assert np.array_equal(h.view(np.uint16), golden["mlpf_h"])
    assert np.array_equal(out, golden["mlpf_ref"])


def test_qkv_rope_oracle(golden):
    cores, q_rows, kv_rows, k_t, pos = (int(v) for v in golden["qkv_meta"])
    x = bf16_from_bits(golden["qkv_x"])
    q = orc.gemv_q4(golden["qkv_q"], x, q_rows, k_t).astype(np.float64)
    k = orc.gemv_q4(golden["qkv_k"], x, kv_rows, k_t).astype(np.float64)
    v = orc.gemv_q4(golden["qkv_v"], x, kv_rows, k_t).astype(np.float64)
    qr = orc.rope_half_split(q.reshape(-1, 64), pos, 10000.0).reshape(cores, -1)
    kr = orc.rope_half_split(k.reshape(-1, 64), pos, 10000.0).reshape(cores, -1)
    ref = np.concatenate([qr, kr, v.reshape(cores, -1)], axis=1)
    np.testing.assert_allclose(ref, golden["qkv_ref"], rtol=0, atol=1e-12)


def test_rope_conventions_differ(golden):
    """The interleaved convention must NOT match the half-split one (granite_elementwise.py:153-162)."""
    ref, alt = golden["rope17_ref"], golden["rope17_alt"]
    assert np.abs(ref - alt).max() / np.abs(alt).max() > 0.1


def test_bf16_rne_matches_ml_dtypes():
    """float32 -> bf16 rounding used throughout is RNE with ties to even."""
    v = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5e-3, 3.3895314e38], np.float32)
    b = v.astype(bfloat16).view(np.uint16)
    assert b[0] == 0x3F80 and b[1] == 0x3F82
