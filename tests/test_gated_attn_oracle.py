"""Pin the gated-attention decode-step oracle to transformers' own module: the
golden vectors tests/golden/make_gated_attn_golden.py recorded from
Qwen3_5Attention.forward (transformers 5.5.0, float32, eager).  CPU only."""

from pathlib import Path

import numpy as np
import pytest

from oracle import gated_attention_oracle as ga
from oracle.q4nx_oracle import compare

GOLDEN = Path(__file__).resolve().parent / "golden" / "gated_attn_golden.npz"
CASES = ["g4", "c5", "g2full", "g1"]


@pytest.fixture(scope="module")
def ggold():
    return np.load(GOLDEN)


def case(g, name):
    bsz, nq, nkv, d, pos = (int(x) for x in g[f"{name}/dims"])
    kc, vc = ga.plant_cache(int(g[f"{name}/plant_seed"]), (bsz, nkv, pos, d))
    return (bsz, nq, nkv, d, pos), kc, vc


def test_rotary_settings_recorded(ggold):
    assert str(ggold["transformers_version"]) == "5.5.0"
    assert ggold["g4/inv_freq"].shape == (32,) and ggold["g2full/inv_freq"].shape == (128,)
    # theta 1e7 decays faster than 1e4 over the same 64 rotary dims
    assert ggold["c5/inv_freq"][-1] < ggold["g4/inv_freq"][-1]


@pytest.mark.parametrize("name", CASES)
def test_step_oracle_matches_transformers(ggold, name):
    (bsz, nq, nkv, d, pos), kc, vc = case(ggold, name)
    g = {k: ggold[f"{name}/{k}"] for k in ("qg", "k_new", "v_new", "q_norm_w", "k_norm_w", "inv_freq")}
    out, k_row, v_row = ga.gated_attention_step(g["qg"], g["k_new"], g["v_new"], g["q_norm_w"], g["k_norm_w"],
                                                g["inv_freq"], kc, vc, np.full(bsz, pos), nq, nkv)
    cos, rel = compare(out, ggold[f"{name}/out"])
    assert cos > 0.9999999 and rel < 1e-5, (name, cos, rel)
    cos, rel = compare(k_row, ggold[f"{name}/k_row"])
    assert cos > 0.9999999 and rel < 1e-5, (name, "k_row", cos, rel)
    assert np.array_equal(v_row.astype(np.float32), ggold[f"{name}/v_row"])


def test_interleaved_rope_must_fail(ggold):
    """Rotating adjacent pairs (the interleaved convention) instead of rotate_half fails the pin."""
    (bsz, nq, nkv, d, pos), kc, vc = case(ggold, "g4")
    g = {k: ggold[f"g4/{k}"] for k in ("qg", "k_new", "v_new", "q_norm_w", "k_norm_w", "inv_freq")}
    good = ga.rope_partial
    try:
        def interleaved(x, p, inv_freq):
            half = inv_freq.shape[0]
            ang = (np.float32(p) * np.asarray(inv_freq, np.float32)).astype(np.float64)
            y = np.array(x, np.float64, copy=True)
            x0, x1 = y[..., 0:2 * half:2].copy(), y[..., 1:2 * half:2].copy()
            y[..., 0:2 * half:2] = x0 * np.cos(ang) - x1 * np.sin(ang)
            y[..., 1:2 * half:2] = x1 * np.cos(ang) + x0 * np.sin(ang)
            return y
        ga.rope_partial = interleaved
        out, _, _ = ga.gated_attention_step(g["qg"], g["k_new"], g["v_new"], g["q_norm_w"], g["k_norm_w"],
                                            g["inv_freq"], kc, vc, np.full(bsz, pos), nq, nkv)
    finally:
        ga.rope_partial = good
    cos, rel = compare(out, ggold["g4/out"])
    assert not (cos > 0.9999999 and rel < 1e-5)
