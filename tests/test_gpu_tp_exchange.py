"""The tensor-parallel exchange kernels (b2_tp_gather / b2_tp_allreduce) and the pulled
seam (b2_gemm_rmsnorm_seam) on one GPU.

World 1 exercises the whole push / signal / wait / consume path against torch.  The
timeout tests give a rank-0 exchange, and a rank-0 seam pre-pass, a second region whose
rank never runs: its signal never comes, the bounded wait runs out after the short
limit set here, the kernel records device error 6 and returns, and the context stays
usable.  No two kernels that wait on each other ever run on the one GPU.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV_ERR_PEER_TIMEOUT = 6
CTL = 65536  # B2_PEER_CTL_BYTES


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llmnputest_b200 import _native
    return _native.lib()


def _region(lib, nbytes):
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    assert lib.b2_peer_alloc(ctypes.c_size_t(nbytes), ctypes.byref(ptr), handle) == 0, lib.b2_last_error_message()
    return ptr.value


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


# 16-byte units in several chunks; single elements (width not a multiple of 4 floats);
# more units than one per thread of 256 CTAs; a block smaller than one unit
@pytest.mark.parametrize("rows,cols", [(5, 3000), (3, 1001), (64, 8192), (1, 2)])
def test_world1_gather_and_allreduce(lib, rows, cols):
    from llmnputest_b200.peer import wrap
    base = _region(lib, CTL + 3 * rows * cols * 4 + 4096)
    try:
        peers = torch.tensor([base], dtype=torch.int64, device="cuda")
        dst = wrap(base + CTL, (rows, cols), torch.float32, "cuda")
        slots = CTL + (rows * cols * 4 + 255) // 256 * 256
        g = torch.Generator(device="cuda")
        g.manual_seed(0)
        src = torch.randn(rows, cols, device="cuda", generator=g)
        for _ in range(3):  # repeated exchanges: the signal counters advance together
            assert lib.b2_tp_gather(ctypes.c_void_p(peers.data_ptr()), 1, 0, ctypes.c_void_p(src.data_ptr()), rows,
                                    cols, cols, 4, CTL, cols, None, _stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(dst, src)
        base_before = dst.clone()
        assert lib.b2_tp_gather(ctypes.c_void_p(peers.data_ptr()), 1, 0, ctypes.c_void_p(src.data_ptr()), rows, cols,
                                cols, 4, CTL, cols, ctypes.c_void_p(dst.data_ptr()), _stream()) == 0  # add mode
        torch.cuda.synchronize()
        assert torch.equal(dst, base_before + src)
        y = torch.randn(rows, cols + 8, device="cuda", generator=g)
        y0 = y.clone()
        assert lib.b2_tp_allreduce(ctypes.c_void_p(peers.data_ptr()), 1, 0, ctypes.c_void_p(src.data_ptr()), rows,
                                   cols, cols, slots, ctypes.c_void_p(y.data_ptr()), y.stride(0), _stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(y[:, :cols], y0[:, :cols] + src) and torch.equal(y[:, cols:], y0[:, cols:])
        h = torch.randn(rows, cols, device="cuda", generator=g).to(torch.bfloat16)  # 2-byte elements
        hd = wrap(base + CTL, (rows, cols), torch.bfloat16, "cuda")
        assert lib.b2_tp_gather(ctypes.c_void_p(peers.data_ptr()), 1, 0, ctypes.c_void_p(h.data_ptr()), rows, cols,
                                cols, 2, CTL, cols, None, _stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(hd, h)
        from llmnputest_b200 import ops
        assert ops.device_error() == 0
    finally:
        lib.b2_peer_free(ctypes.c_void_p(base))


def test_exchange_wait_runs_out(lib):
    """Rank 0 of a 2-rank exchange whose other rank never runs: device error 6, no hang."""
    from llmnputest_b200 import ops
    rows, cols = 2, 256
    r0, r1 = _region(lib, CTL + rows * cols * 4 * 2), _region(lib, CTL + rows * cols * 4 * 2)
    try:
        assert ops.device_error() == 0
        assert lib.b2_set_peer_timeout_ms(50) == 0
        peers = torch.tensor([r0, r1], dtype=torch.int64, device="cuda")
        src = torch.ones(rows, cols, device="cuda")
        assert lib.b2_tp_gather(ctypes.c_void_p(peers.data_ptr()), 2, 0, ctypes.c_void_p(src.data_ptr()), rows, cols,
                                cols, 4, CTL, 2 * cols, None, _stream()) == 0
        torch.cuda.synchronize()  # returns: the wait gave up after 50 ms
        assert ops.device_error() == DEV_ERR_PEER_TIMEOUT
        assert ops.device_error() == 0  # read and cleared
        x = torch.arange(10.0, device="cuda")
        assert float((x * 2).sum()) == 90.0  # the context is still usable
    finally:
        lib.b2_set_peer_timeout_ms(2000)
        lib.b2_peer_free(ctypes.c_void_p(r0))
        lib.b2_peer_free(ctypes.c_void_p(r1))


def test_exchange_argument_errors(lib):
    peers = torch.zeros(2, dtype=torch.int64, device="cuda")
    src = torch.zeros(4, 4, device="cuda")
    s = _stream()
    p = ctypes.c_void_p(peers.data_ptr())
    sp = ctypes.c_void_p(src.data_ptr())
    assert lib.b2_tp_gather(p, 2, 2, sp, 4, 4, 4, 4, CTL, 8, None, s) != 0          # rank out of range
    assert lib.b2_tp_gather(p, 17, 0, sp, 4, 4, 4, 4, CTL, 68, None, s) != 0        # more ranks than the limit
    assert lib.b2_tp_gather(p, 2, 0, sp, 4, 4, 4, 4, CTL - 16, 8, None, s) != 0     # inside the control words
    assert lib.b2_tp_gather(p, 2, 0, sp, 4, 4, 4, 4, CTL, 7, None, s) != 0          # ld_dst < cols*world
    assert lib.b2_tp_gather(p, 2, 0, sp, 4, 4, 4, 3, CTL, 8, None, s) != 0          # element size
    assert lib.b2_tp_gather(p, 2, 0, sp, 4, 4, 4, 2, CTL, 8, sp, s) != 0            # add needs fp32
    assert lib.b2_tp_allreduce(p, 2, 0, sp, 4, 4, 4, CTL + 4, sp, 4, s) != 0        # slots misaligned
    assert lib.b2_set_peer_timeout_ms(0) != 0


def _seam_gemm_args(lib):
    """A small packed q4 GEMM (4 tile-rows, K = 512, batch 16) for b2_gemm_rmsnorm_seam."""
    from llmnputest_b200 import ops
    from llmnputest_b200.decode import synth_q4
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    w = ops.q4_gemm_pack(synth_q4(4 * 2, g, torch.device("cuda")), 4, 2)
    x = torch.randn(16, 512, device="cuda", generator=g)
    nw = torch.ones(512, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(16, 128, device="cuda")
    ws = torch.empty(ops.gemm_workspace_bytes(16, 2) + 256, dtype=torch.uint8, device="cuda")
    off = (256 - ws.data_ptr() % 256) % 256
    return w, x, nw, y, ctypes.c_void_p(ws.data_ptr() + off), ws.numel() - 256, ws


def test_seam_wait_runs_out(lib):
    """A pulled seam (the all-reduce in a GEMM's x pre-pass) whose other rank never posts:
    the pre-pass's bounded wait gives up, device error 6, the GEMM completes, no hang."""
    from llmnputest_b200 import ops
    r0, r1 = _region(lib, CTL + 16 * 512 * 4), _region(lib, CTL + 16 * 512 * 4)
    try:
        assert ops.device_error() == 0
        assert lib.b2_set_peer_timeout_ms(50) == 0
        peers = torch.tensor([r0, r1], dtype=torch.int64, device="cuda")
        w, x, nw, y, wsp, wsn, _ws = _seam_gemm_args(lib)
        st = lib.b2_gemm_rmsnorm_seam(0, ctypes.c_void_p(w.data_ptr()), None, 4, 2, ctypes.c_void_p(x.data_ptr()), 16,
                                      512, ctypes.c_void_p(nw.data_ptr()), ctypes.c_float(1e-6),
                                      ctypes.c_void_p(y.data_ptr()), 128, 4 | 2, wsp, wsn,
                                      ctypes.c_void_p(peers.data_ptr()), 2, 0, CTL, 512, 0, _stream())
        assert st == 0, lib.b2_last_error_message().decode()
        torch.cuda.synchronize()  # returns: the wait gave up after 50 ms
        assert ops.device_error() == DEV_ERR_PEER_TIMEOUT
        assert ops.device_error() == 0  # read and cleared
        v = torch.arange(10.0, device="cuda")
        assert float((v * 2).sum()) == 90.0  # the context is still usable
    finally:
        lib.b2_set_peer_timeout_ms(2000)
        lib.b2_peer_free(ctypes.c_void_p(r0))
        lib.b2_peer_free(ctypes.c_void_p(r1))


def test_seam_argument_errors(lib):
    w, x, nw, y, wsp, wsn, _ws = _seam_gemm_args(lib)
    peers = torch.zeros(2, dtype=torch.int64, device="cuda")
    s = _stream()

    def call(form=0, world=2, rank=0, off=CTL, ld=512, seam=0, k_t=2):
        return lib.b2_gemm_rmsnorm_seam(form, ctypes.c_void_p(w.data_ptr()), None, 4, k_t,
                                        ctypes.c_void_p(x.data_ptr()), 16, 512, ctypes.c_void_p(nw.data_ptr()),
                                        ctypes.c_float(1e-6), ctypes.c_void_p(y.data_ptr()), 128, 4 | 2, wsp, wsn,
                                        ctypes.c_void_p(peers.data_ptr()), world, rank, off, ld, seam, s)

    assert call(form=7) != 0            # unknown form
    assert call(form=1) != 0            # SwiGLU form without the up weight
    assert call(rank=2) != 0            # rank out of range
    assert call(world=17) != 0          # more ranks than the limit
    assert call(off=CTL - 256) != 0     # partials inside the control words
    assert call(off=CTL + 4) != 0       # partials misaligned
    assert call(ld=256) != 0            # ld_part < K
    assert call(seam=8) != 0            # seam counters out of range
