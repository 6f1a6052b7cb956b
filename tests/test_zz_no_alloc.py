"""b2_gqa_decode_static: attention for callers that cannot allocate device memory.

Some callers only receive input and output buffers from a host framework that
owns the GPU allocator, or run in a service that forbids device allocation once
it has started; they cannot hand the library a workspace.  This entry point
uses a fixed scratch array inside the library instead.  These tests call it
through the C ABI and check it against b2_gqa_decode (which takes a caller
workspace) on the same inputs, several calls in a row with different shapes, so
the shared scratch is reused with a different split layout each time.

This file is named to run last, after every other GPU test.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import q4nx_oracle as orc

pytestmark = pytest.mark.gpu

NS_COS, NS_REL = 0.99999, 1e-3   # the attention tolerance of the other GPU tests
B2_ERR_WORKSPACE = -6
OUT_F32_NO_APPEND = 4 | 1        # B2_ATTN_OUT_F32 | B2_ATTN_NO_APPEND: caches stay as they are


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llmnputest_b200 import _native
    return _native.lib()


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def _case(bsz, hq, hkv, ctx, lens, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    d = 64
    qkv = torch.randn(bsz, (hq + 2 * hkv) * d, device="cuda", generator=g)
    kc = torch.randn(bsz, hkv, ctx, d, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(bsz, hkv, ctx, d, device="cuda", generator=g).to(torch.bfloat16)
    pos = torch.tensor([n - 1 for n in lens], dtype=torch.int32, device="cuda")
    return qkv, kc, vc, pos


def _static(lib, qkv, kc, vc, pos, hq, hkv, max_len):
    bsz, _, ctx, d = kc.shape
    out = torch.full((bsz, hq * d), float("nan"), device="cuda")
    st = lib.b2_gqa_decode_static(
        _vp(qkv), ctypes.c_void_p(qkv.data_ptr() + hq * d * 4), ctypes.c_void_p(qkv.data_ptr() + (hq + hkv) * d * 4),
        qkv.stride(0), _vp(kc), _vp(vc), _vp(pos), bsz, hq, hkv, d, ctx, max_len, 10000.0, d ** -0.5,
        _vp(out), out.stride(0), OUT_F32_NO_APPEND, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return st, out


def _with_workspace(qkv, kc, vc, pos, hq, hkv, max_len):
    from llmnputest_b200 import ops
    d = kc.shape[-1]
    return ops.gqa_decode(qkv[:, :hq * d], qkv[:, hq * d:(hq + hkv) * d], qkv[:, (hq + hkv) * d:], kc, vc, pos,
                          n_q_heads=hq, n_kv_heads=hkv, max_len=max_len, append=False, out_f32=True)


def test_static_scratch_matches_workspace_entry_point(lib):
    from llmnputest_b200 import ops
    # Long contexts with more than 16 splits: the split partials go through the scratch
    # (b2_gqa_decode_workspace_size is this entry point's own scratch need, both plan alike).
    # Up to 16 splits merge inside a thread-block cluster and need no scratch at all.
    cases = [(2, 40, 8, 32768, [32768, 20000], 11, True), (1, 40, 8, 32768, [32768], 12, True),
             (3, 40, 8, 32768, [32768, 100, 5000], 14, False), (1, 40, 8, 512, [512], 13, False)]
    for bsz, hq, hkv, ctx, lens, seed, uses_scratch in cases:  # calls in a row through the shared scratch
        assert (ops.gqa_decode_workspace_bytes(bsz, hq, hkv, 64, max(lens)) > 0) == uses_scratch
        qkv, kc, vc, pos = _case(bsz, hq, hkv, ctx, lens, seed)
        st, got = _static(lib, qkv, kc, vc, pos, hq, hkv, max(lens))
        assert st == 0, lib.b2_last_error_message().decode()
        ref = _with_workspace(qkv, kc, vc, pos, hq, hkv, max(lens))
        torch.cuda.synchronize()
        g, r = got.cpu().numpy(), ref.cpu().numpy()
        for b in range(bsz):
            cos, rel = orc.compare(g[b], r[b])
            assert cos >= NS_COS and rel <= NS_REL, (bsz, ctx, b, cos, rel)
    assert ops.device_error() == 0


_OVERSIZE = r"""
import ctypes, sys, torch
from llmnputest_b200 import _native, ops
lib = _native.lib()
bsz, hq, hkv, ctx, d = 64, 64, 8, 4096, 64
need = ops.gqa_decode_workspace_bytes(bsz, hq, hkv, d, ctx)
if need <= (2 << 20):
    print("SKIP plan needs only", need)
    sys.exit(0)
# buffers of the full shape the call describes: a refusal that went missing would only compute
qkv = torch.zeros(bsz, (hq + 2 * hkv) * d, device="cuda")
kc = torch.zeros(bsz, hkv, ctx, d, dtype=torch.bfloat16, device="cuda")
vc = torch.zeros_like(kc)
pos = torch.full((bsz,), ctx - 1, dtype=torch.int32, device="cuda")
out = torch.zeros(bsz, hq * d, device="cuda")
vp = lambda t, off=0: ctypes.c_void_p(t.data_ptr() + off)
st = lib.b2_gqa_decode_static(vp(qkv), vp(qkv, hq * d * 4), vp(qkv, (hq + hkv) * d * 4), qkv.stride(0), vp(kc),
                              vp(vc), vp(pos), bsz, hq, hkv, d, ctx, ctx, 10000.0, 0.125, vp(out), out.stride(0),
                              5, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
torch.cuda.synchronize()
print("STATUS", st, lib.b2_last_error_message().decode())
"""


def test_static_scratch_rejects_oversize(lib):
    # With the default plan (at most one wave of resident CTAs) no call on a 148-SM part needs
    # more than the 2 MiB.  A plan without that cap does: 64 sequences x 8 kv heads x 8 q heads
    # per group in two splits need 2,162,688 bytes.  The plan knob is read once per process, so
    # the refusal is checked in a child process that sets it.
    import os
    import subprocess
    import sys
    from pathlib import Path
    env = dict(os.environ, B2Q4NX_ATTN_WAVE="0")
    root = Path(__file__).resolve().parents[1]
    r = subprocess.run([sys.executable, "-c", _OVERSIZE], env=env, cwd=root, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    if "SKIP" in r.stdout:
        pytest.skip(r.stdout.strip())
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("STATUS")][0]
    assert line.split()[1] == str(B2_ERR_WORKSPACE), line
    assert "static scratch" in line
