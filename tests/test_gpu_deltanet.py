"""Gated DeltaNet decode step on the GPU through the C ABI (b2_gated_delta_step).

Checked against transformers' own module outputs (tests/golden/deltanet_golden.npz,
head dim 128) and against the float64 oracle on seeded inputs.  Tolerance: the
north star's cos >= 0.99999 and max rel err <= 1e-3 on the fp32 output; the
recurrent state within 1e-4 relative; the conv state bit-exact (a shift
register); bf16 outputs at the storage floor 4e-3."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import deltanet_oracle as dn
from tests.test_gpu_gemv import assert_close

pytestmark = pytest.mark.gpu
NS_COS, NS_REL = 0.99999, 1e-3
GOLDEN = Path(__file__).resolve().parent / "golden" / "deltanet_golden.npz"


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llmnputest_b200 import ops as _ops
    return _ops


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).cuda()


def run_step(ops, inp, nk, nv, **kw):
    """One kernel step on device copies of `inp`; returns (out, conv_state, state) on the host."""
    conv, state = dev(inp["conv_state"]), dev(inp["state"])
    out = ops.gated_delta_step(dev(inp["qkv"]), dev(inp["z"]), dev(inp["b"]), dev(inp["a"]), conv,
                               dev(inp["conv_w"]), dev(inp["A_log"]), dev(inp["dt_bias"]), dev(inp["norm_w"]),
                               state, nk, nv, **kw)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), conv.cpu().numpy(), state.cpu().numpy()


def oracle_step(inp, nk, nv):
    return dn.gated_delta_step(inp["qkv"], inp["z"], inp["b"], inp["a"], inp["conv_state"], inp["conv_w"],
                               inp["A_log"], inp["dt_bias"], inp["norm_w"], inp["state"], nk, nv, 128, 128)


@pytest.mark.parametrize("name", ["d128", "d128r1"])
def test_step_matches_transformers_golden(ops, name):
    g = np.load(GOLDEN)
    bsz, nk, nv, dk, dv, steps = (int(x) for x in g[f"{name}/dims"])
    conv_dim = 2 * nk * dk + nv * dv
    conv0, state0 = dn.plant_states(int(g[f"{name}/plant_seed"]), (bsz, conv_dim, 4), (bsz, nv, dk, dv))
    conv, state = dev(conv0), dev(state0)
    prm = {k: dev(g[f"{name}/{k}"]) for k in ("conv_w", "A_log", "dt_bias", "norm_w")}
    idx = torch.from_numpy(g[f"{name}/sample_idx"]).cuda()
    for t in range(steps):  # chained on the device: the kernel's own state carries to the next step
        out = ops.gated_delta_step(dev(g[f"{name}/qkv{t}"]), dev(g[f"{name}/z{t}"]), dev(g[f"{name}/b{t}"]),
                                   dev(g[f"{name}/a{t}"]), conv, prm["conv_w"], prm["A_log"], prm["dt_bias"],
                                   prm["norm_w"], state, nk, nv, out_f32=True)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), g[f"{name}/out{t}"], NS_COS, NS_REL, f"{name} out step {t}")
        assert np.array_equal(conv.cpu().numpy(), g[f"{name}/conv_state{t + 1}"]), (name, t)
        assert_close(state.reshape(-1)[idx].cpu().numpy(), g[f"{name}/state{t + 1}_sample"], 0.9999999, 1e-4,
                     f"{name} state step {t}")


SHAPES = [(1, 1, 1), (1, 16, 16), (3, 2, 4), (2, 4, 4), (5, 2, 16), (2, 1, 8), (17, 16, 16), (4, 3, 6)]


@pytest.mark.parametrize("bsz,nk,nv", SHAPES)
def test_step_vs_oracle(ops, bsz, nk, nv):
    inp = dn.synth_step_inputs(np.random.default_rng(100 + bsz * 7 + nv), bsz, nk, nv, 128, 128)
    out, conv, state = run_step(ops, inp, nk, nv, out_f32=True)
    r_out, r_conv, r_state = oracle_step(inp, nk, nv)
    assert_close(out, r_out, NS_COS, NS_REL, "out")
    assert np.array_equal(conv, r_conv), "conv state"
    assert_close(state, r_state, 0.9999999, 1e-4, "state")
    # per head: every (sequence, v head) gets its own output, not a neighbour's
    for b in range(bsz):
        for h in range(nv):
            sl = slice(h * 128, (h + 1) * 128)
            assert_close(out[b, sl], r_out[b, sl], NS_COS, NS_REL, f"b{b} h{h}")


def test_bf16_output(ops):
    inp = dn.synth_step_inputs(np.random.default_rng(7), 4, 2, 4, 128, 128)
    out, _, _ = run_step(ops, inp, 2, 4)
    r_out, _, _ = oracle_step(inp, 2, 4)
    assert_close(out, r_out, 0.9999, 4e-3, "bf16 out")


def test_chained_steps_with_prefetch(ops):
    """Three steps in a row on one stream, state read before the PDL wait."""
    nk, nv, bsz = 2, 4, 3
    rng = np.random.default_rng(11)
    inp = dn.synth_step_inputs(rng, bsz, nk, nv, 128, 128)
    conv, state = dev(inp["conv_state"]), dev(inp["state"])
    r_conv, r_state = inp["conv_state"], inp["state"]
    prm = {k: dev(inp[k]) for k in ("conv_w", "A_log", "dt_bias", "norm_w")}
    for t in range(3):
        step = dn.synth_step_inputs(rng, bsz, nk, nv, 128, 128)
        out = ops.gated_delta_step(dev(step["qkv"]), dev(step["z"]), dev(step["b"]), dev(step["a"]), conv,
                                   prm["conv_w"], prm["A_log"], prm["dt_bias"], prm["norm_w"], state, nk, nv,
                                   out_f32=True, prefetch_state=True)
        r_out, r_conv, r_state = dn.gated_delta_step(step["qkv"], step["z"], step["b"], step["a"], r_conv,
                                                     inp["conv_w"], inp["A_log"], inp["dt_bias"], inp["norm_w"],
                                                     r_state, nk, nv, 128, 128)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), r_out, NS_COS, NS_REL, f"step {t}")
    assert np.array_equal(conv.cpu().numpy(), r_conv.astype(np.float32))
    assert_close(state.cpu().numpy(), r_state, 0.9999999, 1e-4, "state after 3 steps")


def test_inputs_sliced_from_one_projection(ops):
    """qkv | z | b | a as column slices of one fused in_proj output (row stride > width)."""
    nk, nv, bsz = 2, 4, 3
    inp = dn.synth_step_inputs(np.random.default_rng(5), bsz, nk, nv, 128, 128)
    conv_dim = 2 * nk * 128 + nv * 128
    fused = np.concatenate([inp["qkv"], inp["z"], inp["b"], inp["a"],
                            np.zeros((bsz, 24), np.float32)], axis=1)  # padded to a multiple of 32
    y = dev(fused)
    c0, c1, c2 = conv_dim, conv_dim + nv * 128, conv_dim + nv * 128 + nv
    conv, state = dev(inp["conv_state"]), dev(inp["state"])
    out = ops.gated_delta_step(y[:, :c0], y[:, c0:c1], y[:, c1:c2], y[:, c2:c2 + nv], conv, dev(inp["conv_w"]),
                               dev(inp["A_log"]), dev(inp["dt_bias"]), dev(inp["norm_w"]), state, nk, nv,
                               out_f32=True)
    torch.cuda.synchronize()
    r_out, _, r_state = oracle_step(inp, nk, nv)
    assert_close(out.cpu().numpy(), r_out, NS_COS, NS_REL, "sliced")
    assert_close(state.cpu().numpy(), r_state, 0.9999999, 1e-4, "sliced state")


def test_rejected_before_launch(ops):
    """Shapes the kernel does not build are refused on the host; nothing launches."""
    from llmnputest_b200 import _native
    inp = dn.synth_step_inputs(np.random.default_rng(3), 1, 1, 2, 128, 128)
    t = {k: dev(v) for k, v in inp.items()}
    with pytest.raises(ValueError):  # conv_state shape of another head count
        ops.gated_delta_step(t["qkv"], t["z"], t["b"], t["a"], t["conv_state"], t["conv_w"], t["A_log"],
                             t["dt_bias"], t["norm_w"], t["state"], 1, 4)
    p = ops._ptr
    args = [p(t["qkv"]), t["qkv"].shape[1], p(t["z"]), 256, p(t["b"]), p(t["a"]), 2, p(t["conv_state"]),
            p(t["conv_w"]), p(t["A_log"]), p(t["dt_bias"]), p(t["norm_w"]), p(t["state"]), 1, 1, 2]
    out = torch.empty(1, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_native.B2Error):  # head dim 64 is not built
        _native.call("b2_gated_delta_step", *args, 64, 1e-6, p(out), 256, 0, ops._stream())
    with pytest.raises(_native.B2Error):  # v heads per k head above 8
        _native.call("b2_gated_delta_step", *args[:14], 1, 9, 128, 1e-6, p(out), 256, 0, ops._stream())
    misaligned = torch.empty(t["state"].numel() + 1, dtype=torch.float32, device="cuda")[1:]
    with pytest.raises(_native.B2Error):  # state not 16-byte aligned
        _native.call("b2_gated_delta_step", *args[:12], p(misaligned), 1, 1, 2, 128, 1e-6, p(out), 256, 0,
                     ops._stream())


def test_config5_full_batch_sampled(ops):
    """Config 5's size, B=256 x 16 v heads (268 MB of state, above L2): the step of a
    sequence depends on that sequence alone, so three sampled sequences are checked
    against the oracle run on those sequences only."""
    bsz, nk, nv = 256, 16, 16
    inp = dn.synth_step_inputs(np.random.default_rng(256), bsz, nk, nv, 128, 128)
    out, conv, state = run_step(ops, inp, nk, nv, out_f32=True)
    pick = [0, 97, 255]
    sub = {k: (v[pick] if k in ("qkv", "z", "b", "a", "conv_state", "state") else v) for k, v in inp.items()}
    r_out, r_conv, r_state = oracle_step(sub, nk, nv)
    assert_close(out[pick], r_out, NS_COS, NS_REL, "out")
    assert np.array_equal(conv[pick], r_conv)
    assert_close(state[pick], r_state, 0.9999999, 1e-4, "state")
    assert np.isfinite(out).all()


@pytest.mark.parametrize("bsz", [3, 12])
def test_layer_step_vs_oracle_composition(ops, bsz):
    """DeltaNetLayer (input RMSNorm -> fused q4 in_proj -> step -> q4 out_proj + residual),
    two chained steps, GEMV path at batch 3 and tcgen05 GEMM path at batch 12, against the
    oracle composition.  Gate: the decode-composition bar (cos >= 0.9999, rel <= 1e-2),
    bf16 re-rounding on both sides of each projection."""
    from ml_dtypes import bfloat16

    from llmnputest_b200.deltanet import DeltaNetLayer
    from oracle import q4nx_oracle as orc
    hidden, nk, nv = 1024, 2, 4
    layer = DeltaNetLayer(hidden, nk, nv, bsz, seed=3)
    w = {k: v.cpu() for k, v in layer.w.items()}
    in_t, out_t = w["in_proj"].numpy(), w["out_proj"].numpy()
    norm_in = w["input_norm"].float().numpy()
    prm = {k: w[k].numpy() for k in ("conv_w", "A_log", "dt_bias", "norm_w")}
    r_conv = np.zeros((bsz, layer.conv_dim, 4), np.float32)
    r_state = np.zeros((bsz, nv, 128, 128), np.float64)
    rng = np.random.default_rng(bsz)
    for t in range(2):
        x = rng.standard_normal((bsz, hidden), dtype=np.float32)
        resid = dev(x)
        layer.step(resid)
        torch.cuda.synchronize()
        xn = orc.rmsnorm(x, norm_in, layer.eps).astype(bfloat16).astype(np.float32)
        proj = orc.gemv_q4(in_t, xn, layer.nt_in, layer.kt_h)
        o, r_conv, r_state = dn.gated_delta_step(
            proj[:, :layer.c_z], proj[:, layer.c_z:layer.c_b], proj[:, layer.c_b:layer.c_a],
            proj[:, layer.c_a:layer.c_a + nv], r_conv, prm["conv_w"], prm["A_log"], prm["dt_bias"],
            prm["norm_w"], r_state, nk, nv, 128, 128)
        h = o.astype(bfloat16).astype(np.float32)
        ref = x + orc.gemv_q4(out_t, h, layer.nt_h, layer.kt_v)
        assert_close(resid.cpu().numpy(), ref, 0.9999, 1e-2, f"resid step {t}")
    assert_close(layer.state.cpu().numpy(), r_state, 0.9999, 1e-2, "state after 2 steps")
    assert ops.device_error() == 0
