"""The persistent decode program (b2_program_*) against the one-launch-per-op
entry points: a chain of plain q4 GEMVs, and full decode steps at a context
long enough that attention runs in many splits merged by the O projection."""

import pytest
import torch

from oracle import q4nx_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _compare_rows(got, ref, cos_min, rel_max, what):
    g, r = got.double().cpu().numpy(), ref.double().cpu().numpy()
    for b in range(g.shape[0]):
        cos, rel = orc.compare(g[b], r[b])
        assert cos >= cos_min and rel <= rel_max, (what, b, cos, rel)


@pytest.mark.parametrize("bsz", [1, 5, 8])
def test_gemv_chain_matches_per_op(cuda, bsz):
    """Eight GEMVs of the config-2 shapes (and ragged ones), bf16 x; every output
    is the per-op GEMV's up to fp32 summation order."""
    from llmnputest_b200 import ops
    from llmnputest_b200 import program as pg
    from llmnputest_b200.decode import synth_q4
    g = torch.Generator(device=cuda)
    g.manual_seed(7 + bsz)
    shapes = [(112, 10), (80, 10), (512, 10), (80, 32), (7, 3), (112, 10), (80, 32), (3, 9)]
    ws, xs = [], []
    for n_t, k_t in shapes:
        ws.append(synth_q4(n_t * k_t, g, cuda))
        xs.append(torch.randn(bsz, k_t * 256, device=cuda, generator=g).to(torch.bfloat16))
    sizes = [n_t * 32 for n_t, _ in shapes]
    ybuf = torch.full((bsz, sum(sizes)), float("nan"), device=cuda)
    dummy_pos = torch.zeros(bsz, dtype=torch.int32, device=cuda)
    phases = [pg.prep_phase(zero0=ybuf, zero0_n=ybuf.numel())]
    off = 0
    for (n_t, k_t), w, x, n in zip(shapes, ws, xs, sizes):
        phases.append(pg.gemv_phase(w, n_t, k_t, pg.X_BF16, x, x.shape[1], ybuf.data_ptr() + off * 4, ybuf.shape[1]))
        off += n
    prog = pg.Program(phases, bsz, cuda)
    for _ in range(2):  # a second launch re-zeroes and re-accumulates
        prog.launch(dummy_pos)
    torch.cuda.synchronize()
    off = 0
    for (n_t, k_t), w, x, n in zip(shapes, ws, xs, sizes):
        ref = ops.q4_gemv(w, n_t, k_t, x)
        _compare_rows(ybuf[:, off:off + n], ref, 0.9999999, 1e-5, (n_t, k_t))
        off += n
    assert ops.device_error() == 0


@pytest.mark.parametrize("bsz,ctx,start", [(1, 4096, [4000]), (2, 4096, [4094, 1200]),
                                           (8, 2048, list(range(100, 2048, 250)))])
def test_program_step_matches_per_op_step(cuda, bsz, ctx, start):
    """Two decode steps (2 layers, real widths) through both paths on the same
    weights and caches: logits and appended cache rows agree."""
    from llmnputest_b200 import ops
    from llmnputest_b200.decode import DecoderConfig, Q4Decoder
    cfg = DecoderConfig(n_layers=2, vocab=2048)
    a = Q4Decoder(cfg, bsz, ctx, seed=21)
    b = Q4Decoder(cfg, bsz, ctx, weights=a.w)
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    for li in range(cfg.n_layers):
        kc = torch.randn(a.k_cache[li].shape, device=cuda, generator=g).to(torch.bfloat16)
        vc = torch.randn(a.v_cache[li].shape, device=cuda, generator=g).to(torch.bfloat16)
        for dec in (a, b):
            dec.k_cache[li].copy_(kc)
            dec.v_cache[li].copy_(vc)
    ga, gb = a.capture(), b.capture(program=True)
    pos = torch.tensor(start, dtype=torch.int32, device=cuda)
    for step in range(2):
        x = torch.randn(bsz, cfg.hidden, device=cuda, generator=g)
        for dec in (a, b):
            dec.x_in.copy_(x)
            dec.pos.copy_(pos)
        ga.replay()
        gb.replay()
        torch.cuda.synchronize()
        # same arithmetic per element; fp32 summation order differs and is re-rounded to bf16 between ops
        _compare_rows(b.logits, a.logits, 0.9999, 1e-2, ("logits", step))
        # appended cache rows: the two paths compute 1/rms in different fp32 orders, so a normed
        # input that lands on a bf16 midpoint can round differently (one x element moves by an
        # ulp and every projection row by w * ulp); compare each row by the logits metric
        for li in range(cfg.n_layers):
            for s in range(bsz):
                p = int(pos[s])
                for cache in ("k_cache", "v_cache"):
                    got = getattr(b, cache)[li][s, :, p].reshape(1, -1)
                    ref = getattr(a, cache)[li][s, :, p].reshape(1, -1)
                    _compare_rows(got, ref, 0.9999, 1e-2, (cache, li, s, step))
        pos = pos + 1
    assert ops.device_error() == 0


def test_upload_rejects_bad_phases(cuda):
    from llmnputest_b200 import _native
    from llmnputest_b200 import program as pg
    w = torch.zeros(4 * 10 * 5120, dtype=torch.uint8, device=cuda)
    x = torch.zeros(1, 2560, dtype=torch.bfloat16, device=cuda)
    y = torch.zeros(1, 128, device=cuda)
    bad = [
        pg.gemv_phase(w, 4, 10, pg.X_BF16, x, 2560, y, 64),                       # ldy < rows
        pg.gemv_phase(w.data_ptr() + 8, 4, 10, pg.X_BF16, x, 2560, y, 128),       # tiles misaligned
        pg.gemv_phase(w, 4, 10, 9, x, 2560, y, 128),                              # unknown x source
        pg.gemv_phase(w, 4, 10, pg.X_RMSNORM, y, 2560, y, 128),                   # no norm weight
        pg.gemv_phase(w, 4, 10, pg.X_SWIGLU, y, 2560, y, 128, half=100),          # half < K
    ]
    for ph in bad:
        with pytest.raises(_native.B2Error):
            pg.Program([pg.prep_phase(), ph], 1, cuda)
    with pytest.raises(_native.B2Error):
        pg.Program([pg.prep_phase()], 9, cuda)  # batch above 8
