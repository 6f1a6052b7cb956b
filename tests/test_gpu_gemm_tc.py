"""Tensor-core (tcgen05 / TMEM) W4A16 GEMM for large decode batches against the
numpy oracle (tools/q4nx.py dequant + fp32 matmul, granite_gemv.py:256-272) and
against the mma.sync GEMV on the same inputs.

The weights reach the tensor core as fp16 (w = code*d + m rounded once), so the
bar is the north-star tolerance: cosine >= 0.99999 and max rel <= 1e-3 per
token, fp32 accumulation."""

import numpy as np
import pytest
import torch
from ml_dtypes import bfloat16

from oracle import q4nx_oracle as orc
from tests.test_gpu_gemv import dev_bf16, dev_u8

pytestmark = pytest.mark.gpu

COS, REL = 0.99999, 1e-3


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _check(got, ref, cos_min=COS, rel_max=REL, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    for b in range(ref.shape[0]):
        cos, rel = orc.compare(got[b], ref[b])
        assert cos >= cos_min and rel <= rel_max, (what, b, cos, rel)


@pytest.mark.parametrize("n_t,k_t,bsz", [(4, 1, 17), (7, 3, 32), (12, 10, 100), (5, 2, 256), (4, 4, 1)])
def test_gemm_vs_oracle(cuda, n_t, k_t, bsz):
    from llmnputest_b200 import ops
    rng = np.random.default_rng(1000 + n_t * 37 + k_t * 5 + bsz)
    w = orc.synth_q4_tiles(rng, n_t * k_t)
    x = orc.synth_bf16(rng, (bsz, k_t * 256)).astype(np.float32)
    y = ops.q4_gemm(dev_u8(w), n_t, k_t, dev_bf16(x))
    torch.cuda.synchronize()
    ref = np.stack([orc.gemv_q4(w, x[b], n_t, k_t) for b in range(bsz)])
    _check(y.cpu().numpy(), ref, what=(n_t, k_t, bsz))
    assert ops.device_error() == 0


@pytest.mark.parametrize("name,n_t,k_t", [("qkv", 112, 10), ("down", 80, 32)])
@pytest.mark.parametrize("bsz", [32, 64])
def test_gemm_matches_gemv_at_decode_shapes(cuda, name, n_t, k_t, bsz):
    """Config-4 projection shapes at batch 32/64: same weights and x through the
    GEMV (16 tokens per pass) and the tensor-core GEMM, plus accumulate mode."""
    from llmnputest_b200 import ops
    from llmnputest_b200.decode import synth_q4
    g = torch.Generator(device=cuda)
    g.manual_seed(n_t + bsz)
    w = synth_q4(n_t * k_t, g, cuda)
    x = torch.randn(bsz, k_t * 256, device=cuda, generator=g).to(torch.bfloat16)
    ref = ops.q4_gemv(w, n_t, k_t, x)
    y = ops.q4_gemm(w, n_t, k_t, x)
    base = torch.randn(bsz, n_t * 32, device=cuda, generator=g)
    acc = ops.q4_gemm(w, n_t, k_t, x, out=base.clone(), accumulate=True)
    torch.cuda.synchronize()
    _check(y.cpu().numpy(), ref.cpu().numpy(), what=name)
    _check((acc - base).cpu().numpy(), ref.cpu().numpy(), what=(name, "acc"))
    assert ops.device_error() == 0


@pytest.mark.parametrize("n_t,k_t,bsz", [(8, 4, 32), (512, 10, 48)])
def test_swiglu_gemm_matches_gemv(cuda, n_t, k_t, bsz):
    """Fused gate/up + SiLU*up: both paths narrow g and u to bf16 before SiLU, so
    an accumulator on a bf16 rounding boundary may land one bf16 ulp apart."""
    from llmnputest_b200 import ops
    from llmnputest_b200.decode import synth_q4
    g = torch.Generator(device=cuda)
    g.manual_seed(77 + bsz)
    gate = synth_q4(n_t * k_t, g, cuda)
    up = synth_q4(n_t * k_t, g, cuda)
    x = torch.randn(bsz, k_t * 256, device=cuda, generator=g).to(torch.bfloat16)
    ref = ops.q4_swiglu_gemv(gate, up, n_t, k_t, x)
    h = ops.q4_swiglu_gemm(gate, up, n_t, k_t, x)
    torch.cuda.synchronize()
    _check(h.float().cpu().numpy(), ref.float().cpu().numpy(), 0.9999, 1e-2, "swiglu")
    assert ops.device_error() == 0


@pytest.mark.parametrize("n_t,k_t,bsz", [(8, 2, 256), (6, 3, 192), (10, 1, 128), (112, 4, 256)])
def test_swiglu_gemm_column_split_vs_oracle(cuda, n_t, k_t, bsz):
    """Large batches split the token columns of the SwiGLU GEMM over CTAs (each CTA
    one column block of one row tile): every token against the numpy oracle
    (gate/up GEMVs in fp32, both narrowed to bf16 before SiLU, granite_mlp.py:172-181)."""
    from llmnputest_b200 import ops
    rng = np.random.default_rng(500 + n_t * 7 + bsz)
    gate = orc.synth_q4_tiles(rng, n_t * k_t)
    up = orc.synth_q4_tiles(rng, n_t * k_t)
    x = orc.synth_bf16(rng, (bsz, k_t * 256)).astype(np.float32)
    h = ops.q4_swiglu_gemm(dev_u8(gate), dev_u8(up), n_t, k_t, dev_bf16(x))
    torch.cuda.synchronize()
    bf = lambda a: torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16).float().numpy()
    g = bf(orc.gemv_q4(gate, x, n_t, k_t))
    u = bf(orc.gemv_q4(up, x, n_t, k_t))
    ref = g / (1.0 + np.exp(-g.astype(np.float64))) * u
    # fp16 weights vs exact ones, then two bf16 roundings before SiLU: a token can
    # move a bf16 ulp on both g and u (2 x 2^-8)
    _check(h.float().cpu().numpy(), ref, 0.9999, 2e-2, ("swiglu split", bsz))
    # the column blocks compute exactly what one unsplit CTA computes for the same
    # tokens (batches of <= 48 are never split): bit-identical
    hd = h.cpu()
    for t0 in range(0, bsz, 48):
        sub = ops.q4_swiglu_gemm(dev_u8(gate), dev_u8(up), n_t, k_t, dev_bf16(x[t0:t0 + 48]))
        assert torch.equal(sub.cpu(), hd[t0:t0 + 48]), ("column block differs", t0)
    assert ops.device_error() == 0


def test_gemm_argument_errors(cuda):
    from llmnputest_b200 import _native, ops
    w = torch.zeros(4 * 5120, dtype=torch.uint8, device=cuda)
    x = torch.zeros(257, 256, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(_native.B2Error):
        ops.q4_gemm(w, 4, 1, x)  # batch above 256
    small = torch.empty(256, dtype=torch.uint8, device=cuda)
    with pytest.raises((_native.B2Error, ValueError)):
        ops.q4_gemm(w, 4, 1, x[:32], workspace=small)


@pytest.mark.parametrize("bsz,ctx", [(32, 512), (20, 300)])
def test_decode_step_gemm_matches_gemv(cuda, bsz, ctx):
    """A two-layer decode step at batch 20/32: projections on the tensor-core GEMM
    against the same step on the GEMV path (same weights, caches and inputs)."""
    from llmnputest_b200 import ops
    from llmnputest_b200.decode import DecoderConfig, Q4Decoder
    cfg = DecoderConfig(n_layers=2, vocab=2048)
    a = Q4Decoder(cfg, bsz, ctx, seed=31, gemm_min_batch=10 ** 9)  # GEMV path
    b = Q4Decoder(cfg, bsz, ctx, weights=a.w)
    assert b.use_gemm and not a.use_gemm
    g = torch.Generator(device=cuda)
    g.manual_seed(9)
    for li in range(cfg.n_layers):
        kc = torch.randn(a.k_cache[li].shape, device=cuda, generator=g).to(torch.bfloat16)
        vc = torch.randn(a.v_cache[li].shape, device=cuda, generator=g).to(torch.bfloat16)
        for dec in (a, b):
            dec.k_cache[li].copy_(kc)
            dec.v_cache[li].copy_(vc)
    pos = torch.randint(0, ctx - 2, (bsz,), device=cuda, generator=g, dtype=torch.int32)
    for step in range(2):
        x = torch.randn(bsz, cfg.hidden, device=cuda, generator=g)
        for dec in (a, b):
            dec.x_in.copy_(x)
            dec.pos.copy_(pos)
        la, lb = a.step().clone(), b.step().clone()
        torch.cuda.synchronize()
        # fp16 weights on one side, exact products on the other, re-rounded to bf16 between ops
        _check(lb.cpu().numpy(), la.cpu().numpy(), 0.9999, 1e-2, ("step", step))
        pos = pos + 1
    assert ops.device_error() == 0


@pytest.mark.parametrize("n_t,k_t,bsz,swiglu", [(112, 10, 32, False), (80, 32, 10, False), (256, 10, 32, True),
                                                (7, 3, 17, False), (14, 4, 256, True)])
def test_gemm_fused_rmsnorm_and_prefetch(cuda, n_t, k_t, bsz, swiglu):
    """The GEMM with its RMSNorm fused into the x pre-pass (and the weights streamed before
    the PDL wait) against b2_rmsnorm followed by the plain GEMM, and against the oracle (the
    norm in float64).  The two norms sum their squares in different fp32 orders, so a few
    bf16 inputs may differ by one ulp: the bar is the GEMM's own."""
    from ml_dtypes import bfloat16
    from llmnputest_b200 import ops
    rng = np.random.default_rng(7000 + n_t + k_t + bsz)
    g = orc.synth_q4_tiles(rng, n_t * k_t)
    u = orc.synth_q4_tiles(rng, n_t * k_t) if swiglu else None
    x = (rng.standard_normal((bsz, k_t * 256)) * 3).astype(np.float32)
    nw = (rng.standard_normal(k_t * 256) * 0.1 + 1).astype(np.float32).astype(bfloat16)
    xd, nwd = torch.from_numpy(x).to(cuda), dev_bf16(nw.astype(np.float32))
    xn = ops.rmsnorm(xd, nwd, 1e-6)
    if swiglu:
        fused = ops.q4_swiglu_gemm(dev_u8(g), dev_u8(u), n_t, k_t, xd, prefetch=True, norm_w=nwd, eps=1e-6)
        plain = ops.q4_swiglu_gemm(dev_u8(g), dev_u8(u), n_t, k_t, xn)
    else:
        fused = ops.q4_gemm(dev_u8(g), n_t, k_t, xd, prefetch=True, norm_w=nwd, eps=1e-6)
        plain = ops.q4_gemm(dev_u8(g), n_t, k_t, xn)
    torch.cuda.synchronize()
    # SwiGLU outputs are bf16 products of two bf16-rounded accumulators: a one-ulp flip of
    # g or u moves h by up to ~3 ulps (2^-8 each); the bars of the other SwiGLU checks here
    bar, bar_oracle = (1e-2, 2e-2) if swiglu else (REL, REL)
    _check(fused.float().cpu().numpy(), plain.float().cpu().numpy(), COS, bar, "fused vs rmsnorm + GEMM")
    xr = orc.rmsnorm(x, nw, 1e-6).astype(np.float32).astype(bfloat16)
    if swiglu:
        ref = np.stack([orc.swiglu_from_accumulators(orc.gemv_q4(g, xr[b], n_t, k_t), orc.gemv_q4(u, xr[b], n_t, k_t))
                        for b in range(bsz)])
        _check(fused.float().cpu().numpy(), ref, 0.9999, bar_oracle, "swiglu vs oracle")
    else:
        _check(fused.cpu().numpy(), orc.gemv_q4(g, xr, n_t, k_t), what="vs oracle")
    assert ops.device_error() == 0


# ------------------------------------------------------------ packed form
def test_device_pack_matches_layout(cuda):
    """b2_q4_gemm_pack against the numpy statement of the packed layout, byte for byte."""
    from llmnputest_b200 import ops
    from tests import gemm_pack_layout as gpl
    rng = np.random.default_rng(5)
    for n_t, k_t in ((7, 5), (4, 1), (1, 3)):
        tiles = orc.synth_q4_tiles(rng, n_t * k_t)
        got = ops.q4_gemm_pack(dev_u8(tiles), n_t, k_t)
        torch.cuda.synchronize()
        assert np.array_equal(got.cpu().numpy().reshape(tiles.shape), gpl.pack(tiles, n_t, k_t)), (n_t, k_t)


# (n_t, k_t, batch, form): split-K, odd shapes, one token, 256 tokens (one accumulator
# buffer of 256 TMEM columns), accumulate, fused norm, SwiGLU with and without the
# column split
@pytest.mark.parametrize("n_t,k_t,bsz,form", [
    (112, 10, 32, "f32"), (80, 32, 32, "acc"), (7, 3, 17, "f32"), (4, 4, 1, "f32"), (12, 10, 256, "f32"),
    (112, 10, 32, "norm"), (256, 10, 32, "swiglu"), (14, 4, 256, "swiglu"), (30, 10, 9, "swiglu_norm")])
def test_packed_gemm_equals_gemm(cuda, n_t, k_t, bsz, form):
    """The packed form (A dequantised into tensor memory) multiplies the same fp16 weights
    and x as the shared-memory form; it sums the K-tile's MMAs in up to four partial
    accumulators, so the fp32 sums differ only in grouping (bf16 SwiGLU outputs then by a
    rounding flip at most); and both against the oracle."""
    from llmnputest_b200 import ops
    rng = np.random.default_rng(9000 + n_t + k_t + bsz)
    swiglu = form.startswith("swiglu")
    g = orc.synth_q4_tiles(rng, n_t * k_t)
    u = orc.synth_q4_tiles(rng, n_t * k_t) if swiglu else None
    norm = form.endswith("norm")
    if norm:
        x = (rng.standard_normal((bsz, k_t * 256)) * 3).astype(np.float32)
        xd = torch.from_numpy(x).to(cuda)
        nw = (rng.standard_normal(k_t * 256) * 0.1 + 1).astype(np.float32)
        kw = dict(norm_w=dev_bf16(nw), eps=1e-6)
    else:
        x = orc.synth_bf16(rng, (bsz, k_t * 256)).astype(np.float32)
        xd = dev_bf16(x)
        kw = {}
    gd = dev_u8(g)
    gp = ops.q4_gemm_pack(gd, n_t, k_t)
    if swiglu:
        ud = dev_u8(u)
        up = ops.q4_gemm_pack(ud, n_t, k_t)
        plain = ops.q4_swiglu_gemm(gd, ud, n_t, k_t, xd, **kw)
        packed = ops.q4_swiglu_gemm(gp, up, n_t, k_t, xd, packed=True, prefetch=True, **kw)
    else:
        acc = form == "acc"
        y0 = torch.from_numpy(rng.standard_normal((bsz, n_t * 32)).astype(np.float32)).to(cuda)
        plain = ops.q4_gemm(gd, n_t, k_t, xd, out=y0.clone(), accumulate=acc, **kw)
        packed = ops.q4_gemm(gp, n_t, k_t, xd, out=y0.clone(), accumulate=acc, packed=True, prefetch=True, **kw)
    torch.cuda.synchronize()
    a, b = packed.float().cpu().numpy(), plain.float().cpu().numpy()
    if swiglu:  # bf16 outputs: the other SwiGLU checks' bar
        _check(a, b, 0.9999, 1e-2, ("packed swiglu", n_t, k_t, bsz))
    else:  # fp32 sums of other grouping (and split-K partials meeting in atomics of either order)
        assert np.abs(a - b).max() <= 1e-5 * max(1.0, float(np.abs(b).max())), float(np.abs(a - b).max())
    if not norm and not swiglu and form != "acc":
        _check(a, np.stack([orc.gemv_q4(g, x[i], n_t, k_t) for i in range(bsz)]), what=("packed", n_t, k_t, bsz))
    assert ops.device_error() == 0


def test_device_pack8_matches_layout(cuda):
    from llmnputest_b200 import ops
    from tests import gemm_pack_layout as gpl
    rng = np.random.default_rng(6)
    for n_t, k_t in ((5, 3), (2, 1)):
        tiles = orc.synth_q8_tiles(rng, n_t * k_t)
        got = ops.q8_gemm_pack(dev_u8(tiles), n_t, k_t)
        torch.cuda.synchronize()
        assert np.array_equal(got.cpu().numpy().reshape(tiles.shape), gpl.pack8(tiles, n_t, k_t)), (n_t, k_t)


# q8 (the lm_head): decode batches, 256 tokens, odd shapes, the fused RMSNorm
@pytest.mark.parametrize("n_t,k_t,bsz,norm", [(40, 10, 32, False), (9, 4, 256, False), (7, 3, 17, False),
                                              (40, 10, 32, True), (3, 2, 1, False)])
def test_q8_gemm_vs_oracle(cuda, n_t, k_t, bsz, norm):
    """q8 GEMM on packed tiles: w = fp16(code * scale) rounded once (relative 2^-11), fp32
    accumulation: the north-star bar against the oracle's float32 GEMV."""
    from llmnputest_b200 import ops
    rng = np.random.default_rng(8000 + n_t + k_t + bsz)
    w = orc.synth_q8_tiles(rng, n_t * k_t)
    pk = ops.q8_gemm_pack(dev_u8(w), n_t, k_t)
    if norm:
        from ml_dtypes import bfloat16
        x = (rng.standard_normal((bsz, k_t * 256)) * 3).astype(np.float32)
        nw = (rng.standard_normal(k_t * 256) * 0.1 + 1).astype(np.float32)
        y = ops.q8_gemm(pk, n_t, k_t, torch.from_numpy(x).to(cuda), prefetch=True, norm_w=dev_bf16(nw), eps=1e-6)
        xr = orc.rmsnorm(x, nw.astype(bfloat16), 1e-6).astype(np.float32).astype(bfloat16).astype(np.float32)
    else:
        xr = orc.synth_bf16(rng, (bsz, k_t * 256)).astype(np.float32)
        y = ops.q8_gemm(pk, n_t, k_t, dev_bf16(xr), prefetch=True)
    torch.cuda.synchronize()
    ref = np.stack([orc.gemv_q8(w, xr[b], n_t, k_t) for b in range(bsz)])
    _check(y.cpu().numpy(), ref, what=("q8", n_t, k_t, bsz, norm))
    assert ops.device_error() == 0


@pytest.mark.parametrize("nt_i,kt_h,nt_h,bsz", [(16, 2, 4, 32), (64, 3, 8, 100), (32, 10, 20, 256)])
def test_swiglu_in_gemm_vs_oracle(cuda, nt_i, kt_h, nt_h, bsz):
    """The split MLP: gate and up as one split-K GEMM over their stacked tile-rows (fp32
    outputs), then the down GEMM whose x pre-pass forms bf16(silu(bf16 g) * bf16 u)
    (granite_mlp.py:172-181).  Against the numpy oracle and against the fused SwiGLU GEMM
    feeding the plain down GEMM; the bars are the SwiGLU bars (a token may move a bf16 ulp
    on g and u before SiLU)."""
    from llmnputest_b200 import ops
    rng = np.random.default_rng(9100 + nt_i + kt_h + bsz)
    kt_i = nt_i * 32 // 256
    gate = orc.synth_q4_tiles(rng, nt_i * kt_h)
    up = orc.synth_q4_tiles(rng, nt_i * kt_h)
    down = orc.synth_q4_tiles(rng, nt_h * kt_i)
    x = orc.synth_bf16(rng, (bsz, kt_h * 256)).astype(np.float32)
    gu_w = ops.q4_gemm_pack(dev_u8(np.concatenate([gate.reshape(-1), up.reshape(-1)])), 2 * nt_i, kt_h)
    down_p = ops.q4_gemm_pack(dev_u8(down), nt_h, kt_i)
    gu = ops.q4_gemm(gu_w, 2 * nt_i, kt_h, dev_bf16(x), packed=True, prefetch=True)
    y = ops.q4_gemm(down_p, nt_h, kt_i, gu, packed=True, prefetch=True, swiglu_in=True)
    h = ops.q4_swiglu_gemm(ops.q4_gemm_pack(dev_u8(gate), nt_i, kt_h), ops.q4_gemm_pack(dev_u8(up), nt_i, kt_h),
                           nt_i, kt_h, dev_bf16(x), packed=True)
    y_fused = ops.q4_gemm(down_p, nt_h, kt_i, h, packed=True)
    torch.cuda.synchronize()
    bf = lambda a: np.asarray(a, np.float32).astype(bfloat16).astype(np.float32)
    g = bf(np.stack([orc.gemv_q4(gate, x[b], nt_i, kt_h) for b in range(bsz)]))
    u = bf(np.stack([orc.gemv_q4(up, x[b], nt_i, kt_h) for b in range(bsz)]))
    hb = bf(g / (1.0 + np.exp(-g.astype(np.float64))) * u)
    ref = np.stack([orc.gemv_q4(down, hb[b], nt_h, kt_i) for b in range(bsz)])
    _check(y.cpu().numpy(), ref, 0.9999, 2e-2, ("swiglu_in", nt_i, kt_h, bsz))
    _check(y.cpu().numpy(), y_fused.cpu().numpy(), 0.9999, 2e-2, ("swiglu_in vs fused", nt_i, kt_h, bsz))
    # the gate/up GEMM alone is the plain GEMM on the stacked rows
    _check(gu[:, :nt_i * 32].cpu().numpy(), np.stack([orc.gemv_q4(gate, x[b], nt_i, kt_h) for b in range(bsz)]),
           what="gate half")
    assert ops.device_error() == 0


def test_swiglu_in_argument_errors(cuda):
    from llmnputest_b200 import _native, ops
    w = torch.zeros(4 * 2 * 5120, dtype=torch.uint8, device=cuda)
    with pytest.raises(ValueError):
        ops.q4_gemm(w, 4, 2, torch.zeros(32, 512, device=cuda), swiglu_in=True)  # needs [B, 2K]
    ws = torch.empty(ops.gemm_workspace_bytes(32, 2), dtype=torch.uint8, device=cuda)
    y = torch.zeros(32, 128, device=cuda)
    gu = torch.zeros(32, 1024, device=cuda)
    with pytest.raises(_native.B2Error):  # ldgu below 2K
        _native.call("b2_q4_gemm_swiglu_in", w.data_ptr(), 4, 2, gu.data_ptr(), 32, 512, y.data_ptr(), 128, 0,
                     ws.data_ptr(), ws.numel(), None)
