"""Pin the gated DeltaNet decode-step oracle to transformers' own module: the
golden vectors tests/golden/make_deltanet_golden.py recorded from
Qwen3_5GatedDeltaNet.forward (transformers 5.5.0, float32).  CPU only."""

from pathlib import Path

import numpy as np
import pytest

from oracle import deltanet_oracle as dn
from oracle.q4nx_oracle import compare

GOLDEN = Path(__file__).resolve().parent / "golden" / "deltanet_golden.npz"
CASES = ["d32", "d128", "d128r1", "d32r4"]


@pytest.fixture(scope="module")
def dgold():
    return np.load(GOLDEN)


def case_inputs(g, name):
    """(dims, params, conv_state0, state0) of one golden case."""
    bsz, nk, nv, dk, dv, steps = (int(x) for x in g[f"{name}/dims"])
    conv_dim = 2 * nk * dk + nv * dv
    conv0, state0 = dn.plant_states(int(g[f"{name}/plant_seed"]), (bsz, conv_dim, 4), (bsz, nv, dk, dv))
    params = {k: g[f"{name}/{k}"] for k in ("conv_w", "A_log", "dt_bias", "norm_w")}
    return (bsz, nk, nv, dk, dv, steps), params, conv0, state0


def test_golden_records_transformers_version(dgold):
    assert str(dgold["transformers_version"]) == "5.5.0"


def test_planted_states_regenerate(dgold):
    _, _, conv0, state0 = case_inputs(dgold, "d32")
    assert np.array_equal(conv0, dgold["d32/conv_state0"])
    assert np.array_equal(state0, dgold["d32/state0"])


@pytest.mark.parametrize("name", CASES)
def test_step_oracle_matches_transformers(dgold, name):
    (bsz, nk, nv, dk, dv, steps), prm, conv, state = case_inputs(dgold, name)
    idx = dgold[f"{name}/sample_idx"]
    for t in range(steps):
        out, conv, state = dn.gated_delta_step(
            dgold[f"{name}/qkv{t}"], dgold[f"{name}/z{t}"], dgold[f"{name}/b{t}"], dgold[f"{name}/a{t}"],
            conv, prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["norm_w"], state, nk, nv, dk, dv)
        cos, rel = compare(out, dgold[f"{name}/out{t}"])
        assert cos > 0.9999999 and rel < 1e-5, (name, t, cos, rel)
        # the conv state is a shift register: exact
        assert np.array_equal(conv.astype(np.float32), dgold[f"{name}/conv_state{t + 1}"]), (name, t)
        ref_state = dgold[f"{name}/state{t + 1}"] if f"{name}/state{t + 1}" in dgold \
            else dgold[f"{name}/state{t + 1}_sample"]
        got_state = state if f"{name}/state{t + 1}" in dgold else state.reshape(-1)[idx]
        cos, rel = compare(got_state, ref_state)
        assert cos > 0.9999999 and rel < 1e-5, (name, t, "state", cos, rel)
        # chain the next step from the reference's fp32 state, as the cache would hold it
        if f"{name}/state{t + 1}" in dgold:
            state = dgold[f"{name}/state{t + 1}"]


def test_planted_mistake_is_caught(dgold):
    """A wrong gate (g without the minus sign) must fail the pin."""
    (bsz, nk, nv, dk, dv, _), prm, conv, state = case_inputs(dgold, "d32")
    out, _, _ = dn.gated_delta_step(
        dgold["d32/qkv0"], dgold["d32/z0"], dgold["d32/b0"], dgold["d32/a0"], conv, prm["conv_w"],
        -prm["A_log"] * 0 + np.log(np.float32(1e-9)), prm["dt_bias"], prm["norm_w"], state, nk, nv, dk, dv)
    cos, rel = compare(out, dgold["d32/out0"])
    assert not (cos > 0.9999999 and rel < 1e-5)
