"""GEMV / dequant parity on the GPU, through the C ABI (llmnputest_b200.ops -> libb2q4nx.so).

Tolerances: the north star's (cos >= 0.99999, max rel err <= 1e-3) and the
reference's own stricter GEMV gate (cos > 0.9999999, rel < 1e-4,
designs/granite_gemv/granite_gemv.py:335), both in float64.  onehot activations
isolate one K column and must reproduce it bit for bit; dequant is bit-exact.
"""

import numpy as np
import pytest
import torch
from ml_dtypes import bfloat16

from oracle import q4nx_oracle as orc
from tests.conftest import bf16_from_bits

pytestmark = pytest.mark.gpu

NS_COS, NS_REL = 0.99999, 1e-3
REF_COS, REF_REL = 0.9999999, 1e-4  # the reference's own GEMV gate


def dev_u8(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint8).reshape(-1)).cuda()


def dev_bf16(a):
    a = np.ascontiguousarray(np.asarray(a).astype(bfloat16))
    return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()


def assert_close(got, ref, cos_min=REF_COS, rel_max=REF_REL, what=""):
    cos, rel = orc.compare(got, ref)
    assert cos >= cos_min and rel <= rel_max, f"{what}: cos={cos:.10f} rel={rel:.3e}"
    return cos, rel


@pytest.fixture(scope="module")
def ops():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llmnputest_b200 import ops as _ops
    return _ops


def test_q4_golden(ops, golden):
    n_t, k_t = (int(v) for v in golden["q4_shape"])
    w = dev_u8(golden["q4_w"])
    x = dev_bf16(bf16_from_bits(golden["q4_x"]))
    y = ops.q4_gemv(w, n_t, k_t, x).cpu().numpy()
    ref = golden["q4_y"]
    for b in range(x.shape[0]):
        assert_close(y[b], ref[b], what=f"token {b}")
    # tokens 4, 5 are onehot columns: exact
    assert np.array_equal(y[4], ref[4]) and np.array_equal(y[5], ref[5])


def test_q8_golden(ops, golden):
    n_t, k_t = (int(v) for v in golden["q8_shape"])
    w = dev_u8(golden["q8_w"])
    x = dev_bf16(bf16_from_bits(golden["q8_x"]))
    y = ops.q8_gemv(w, n_t, k_t, x).cpu().numpy()
    ref = golden["q8_y"]
    for b in range(x.shape[0]):
        assert_close(y[b], ref[b], what=f"token {b}")
    assert np.array_equal(y[3], ref[3])  # onehot


SHAPES = {  # name: (tile-rows, K-tiles) of the 3B decoder's projections
    "qkv": (112, 10), "o": (80, 10), "gate_up": (512, 10), "down": (80, 32),
}


@pytest.mark.parametrize("shape", list(SHAPES))
@pytest.mark.parametrize("batch", [1, 8, 13])
def test_q4_projection_shapes(ops, shape, batch):
    n_t, k_t = SHAPES[shape]
    rng = np.random.default_rng(hash((shape, batch)) % 2**32)
    w = orc.synth_q4_tiles(rng, n_t * k_t)
    x = orc.synth_bf16(rng, (batch, k_t * 256))
    y = ops.q4_gemv(dev_u8(w), n_t, k_t, dev_bf16(x)).cpu().numpy()
    ref = orc.gemv_q4(w, x, n_t, k_t)
    for b in range(batch):  # every token, not just token 0 (granite_gemv32.py:279-288)
        assert_close(y[b], ref[b], what=f"{shape} b={batch} token {b}")


@pytest.mark.parametrize("n_t,k_t,batch", [(1, 1, 1), (3, 2, 2), (5, 33, 1), (7, 4, 16), (9, 1, 9), (2, 96, 3)])
def test_q4_ragged(ops, n_t, k_t, batch):
    rng = np.random.default_rng(n_t * 1000 + k_t)
    w = orc.synth_q4_tiles(rng, n_t * k_t)
    x = orc.synth_bf16(rng, (batch, k_t * 256))
    y = ops.q4_gemv(dev_u8(w), n_t, k_t, dev_bf16(x)).cpu().numpy()
    ref = orc.gemv_q4(w, x, n_t, k_t)
    for b in range(batch):
        assert_close(y[b], ref[b], what=f"token {b}")


@pytest.mark.parametrize("n_t,k_t,batch", [(7760, 4, 1), (3136, 10, 1), (130, 4, 8), (3, 7, 12)])
def test_q8_shapes(ops, n_t, k_t, batch):
    rng = np.random.default_rng(n_t + 7 * k_t)
    w = orc.synth_q8_tiles(rng, n_t * k_t)
    x = orc.synth_bf16(rng, (batch, k_t * 256))
    y = ops.q8_gemv(dev_u8(w), n_t, k_t, dev_bf16(x)).cpu().numpy()
    ref = orc.gemv_q8(w, x, n_t, k_t)
    for b in range(batch):
        assert_close(y[b], ref[b], what=f"token {b}")


def test_accumulate(ops):
    rng = np.random.default_rng(9)
    n_t, k_t = 20, 10
    w = orc.synth_q4_tiles(rng, n_t * k_t)
    x = orc.synth_bf16(rng, (2, k_t * 256))
    y0 = rng.standard_normal((2, n_t * 32)).astype(np.float32)
    out = torch.from_numpy(y0.copy()).cuda()
    ops.q4_gemv(dev_u8(w), n_t, k_t, dev_bf16(x), out=out, accumulate=True)
    ref = orc.gemv_q4(w, x, n_t, k_t) + y0
    assert_close(out.cpu().numpy(), ref, what="residual add")


def test_swiglu_golden(ops, golden):
    tr, kt = (int(v) for v in golden["mlp_shape"])
    x = dev_bf16(bf16_from_bits(golden["mlp_x"]))
    h = ops.q4_swiglu_gemv(dev_u8(golden["mlp_gate"]), dev_u8(golden["mlp_up"]), tr, kt, x)
    got = h.float().cpu().numpy()
    # output is bf16: the floor is bf16 rounding (2^-9 relative), as in granite_rmsnorm.py:117-119
    assert_close(got, golden["mlp_ref"], cos_min=NS_COS, rel_max=4e-3, what="swiglu")
    assert (np.abs(got) > 0).all()  # whole length processed (granite_elementwise.py:175-177)


@pytest.mark.parametrize("batch", [1, 8])
def test_swiglu_full_shape(ops, batch):
    rng = np.random.default_rng(31 + batch)
    n_t, k_t = 256, 10  # intermediate 8192 from hidden 2560
    g = orc.synth_q4_tiles(rng, n_t * k_t)
    u = orc.synth_q4_tiles(rng, n_t * k_t)
    x = orc.synth_bf16(rng, (batch, k_t * 256))
    h = ops.q4_swiglu_gemv(dev_u8(g), dev_u8(u), n_t, k_t, dev_bf16(x)).float().cpu().numpy()
    for b in range(batch):
        ref = orc.swiglu_from_accumulators(orc.gemv_q4(g, x[b], n_t, k_t), orc.gemv_q4(u, x[b], n_t, k_t))
        assert_close(h[b], ref, cos_min=NS_COS, rel_max=4e-3, what=f"token {b}")


def test_dequant_bit_exact(ops, golden):
    for q8, key in ((False, "q4"), (True, "q8")):
        t = golden[f"fmt_{key}_tiles"]
        got = ops.dequant_tiles(dev_u8(t), q8=q8).view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(got, golden[f"fmt_{key}_dequant_bf16"]), key
    m = ops.dequant_matrix(dev_u8(golden["fmt_q4_tiles"]), 3, 2).cpu().numpy()
    assert np.array_equal(m, golden["fmt_q4_untiled_3x2"])
    m = ops.dequant_matrix(dev_u8(golden["fmt_q8_tiles"]), 2, 3, q8=True).cpu().numpy()
    assert np.array_equal(m, golden["fmt_q8_untiled_2x3"])


def test_dequant_random_bit_exact(ops):
    rng = np.random.default_rng(77)
    t4 = orc.synth_q4_tiles(rng, 300)
    t8 = orc.synth_q8_tiles(rng, 300)
    got4 = ops.dequant_matrix(dev_u8(t4), 30, 10).cpu().numpy()
    assert np.array_equal(got4, orc.q4_matrix(t4, 30, 10))
    got8 = ops.dequant_matrix(dev_u8(t8), 75, 4, q8=True).cpu().numpy()
    assert np.array_equal(got8, orc.q8_matrix(t8, 75, 4))


def test_argument_errors(ops):
    from llmnputest_b200._native import B2Error
    w = torch.zeros(5120, dtype=torch.uint8, device="cuda")
    x = torch.zeros(17, 256, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(17, 32, dtype=torch.float32, device="cuda")
    from llmnputest_b200 import _native
    import ctypes
    with pytest.raises(B2Error):  # batch 17 > 16 straight into the C ABI
        _native.call("b2_q4_gemv", ctypes.c_void_p(w.data_ptr()), 1, 1, ctypes.c_void_p(x.data_ptr()), 17, 256,
                     ctypes.c_void_p(out.data_ptr()), 32, 0, ctypes.c_void_p(0))
    with pytest.raises(B2Error):  # misaligned weights
        _native.call("b2_q4_gemv", ctypes.c_void_p(w.data_ptr() + 4), 1, 1, ctypes.c_void_p(x.data_ptr()), 1, 256,
                     ctypes.c_void_p(out.data_ptr()), 32, 0, ctypes.c_void_p(0))
    with pytest.raises(ValueError):
        ops.q4_gemv(w, 2, 1, x[0])  # wrong byte count
    with pytest.raises(ValueError):
        ops.q4_gemv(w.cpu(), 1, 1, x[0].cpu())  # no CPU fallback


def test_no_device_error(ops):
    torch.cuda.synchronize()
    assert ops.device_error() == 0


@pytest.mark.parametrize("q8,n_t,k_t,batch", [(False, 112, 10, 1), (False, 80, 32, 3), (True, 130, 10, 2)])
def test_gemv_fused_rmsnorm(ops, q8, n_t, k_t, batch):
    """GEMV with RMSNorm fused into its input == rmsnorm (bf16 out) then the GEMV."""
    rng = np.random.default_rng(40 + n_t)
    w = (orc.synth_q8_tiles if q8 else orc.synth_q4_tiles)(rng, n_t * k_t)
    x = (rng.standard_normal((batch, k_t * 256)) * 4).astype(np.float32)
    nw = (rng.standard_normal(k_t * 256) * 0.1 + 1).astype(np.float32).astype(bfloat16)
    y = ops.gemv_rmsnorm(dev_u8(w), n_t, k_t, torch.from_numpy(x).cuda(), dev_bf16(nw.astype(np.float32)), 1e-6,
                         q8=q8).cpu().numpy()
    xn = orc.rmsnorm(x, nw, 1e-6).astype(np.float32).astype(bfloat16)
    ref = (orc.gemv_q8 if q8 else orc.gemv_q4)(w, xn, n_t, k_t)
    for b in range(batch):
        # the fused norm rounds x*inv*w in fp32 rather than fp64: a few bf16 inputs differ by 1 ulp
        assert_close(y[b], ref[b], NS_COS, NS_REL, f"token {b}")


def test_swiglu_fused_rmsnorm(ops):
    rng = np.random.default_rng(71)
    n_t, k_t = 256, 10
    g = orc.synth_q4_tiles(rng, n_t * k_t)
    u = orc.synth_q4_tiles(rng, n_t * k_t)
    x = (rng.standard_normal((2, k_t * 256)) * 3).astype(np.float32)
    nw = (rng.standard_normal(k_t * 256) * 0.1 + 1).astype(np.float32).astype(bfloat16)
    h = ops.swiglu_gemv_rmsnorm(dev_u8(g), dev_u8(u), n_t, k_t, torch.from_numpy(x).cuda(),
                                dev_bf16(nw.astype(np.float32)), 1e-6).float().cpu().numpy()
    xn = orc.rmsnorm(x, nw, 1e-6).astype(np.float32).astype(bfloat16)
    for b in range(2):
        ref = orc.swiglu_from_accumulators(orc.gemv_q4(g, xn[b], n_t, k_t), orc.gemv_q4(u, xn[b], n_t, k_t))
        assert_close(h[b], ref, NS_COS, 4e-3, f"token {b}")


@pytest.mark.parametrize("shape", ["qkv", "down", "gate_up"])
def test_chained_prefetch_plan(ops, shape):
    """The prefetch (chained) launch plan gives the same results as the default plan."""
    n_t, k_t = SHAPES[shape]
    rng = np.random.default_rng(7)
    w = dev_u8(orc.synth_q4_tiles(rng, n_t * k_t))
    x = dev_bf16(orc.synth_bf16(rng, (2, k_t * 256)).astype(np.float32))
    a = ops.q4_gemv(w, n_t, k_t, x).cpu().numpy()
    b = ops.q4_gemv(w, n_t, k_t, x, prefetch=True).cpu().numpy()
    for i in range(2):
        assert_close(b[i], a[i], REF_COS, REF_REL, f"token {i}")
