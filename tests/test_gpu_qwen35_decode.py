"""Qwen35Decoder (config 5's stack: gated DeltaNet and gated attention token mixers,
SwiGLU MLPs, q8 lm_head) on the GPU against the same stack on the CPU oracle shims,
with the same weights: two steps at advancing positions (recurrent states and the
KV cache carried), the GEMV path at batch 2 and the tensor-core GEMM path at batch
10.  Gate: the decode-composition bar (cos >= 0.9999, rel <= 1e-2; measured on a
B200: cos >= 0.99999994, rel <= 6.5e-4)."""

import pytest
import torch

from oracle import q4nx_oracle as orc
from tests.test_qwen35_decode_host import CFG, Q35Ops

pytestmark = pytest.mark.gpu


def _to_dev(w):
    if isinstance(w, dict):
        return {k: _to_dev(v) for k, v in w.items()}
    if isinstance(w, list):
        return [_to_dev(v) for v in w]
    return w.cuda()


@pytest.mark.parametrize("bsz", [2, 10])
def test_qwen35_decoder_gpu_matches_oracle_stack(bsz):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llmnputest_b200 import ops
    from llmnputest_b200.qwen35_decode import Qwen35Decoder
    cpu = Qwen35Decoder(CFG, bsz, 8, device="cpu", seed=1, ops_impl=Q35Ops())
    gpu = Qwen35Decoder(CFG, bsz, 8, device="cuda", weights=_to_dev(cpu.w))
    assert gpu.use_gemm == (bsz >= 9)
    x = torch.randn(bsz, CFG.hidden, generator=torch.Generator().manual_seed(2))
    pos = torch.arange(bsz, dtype=torch.int32) % 5 + 2
    for t in range(2):
        cpu.x_in.copy_(x)
        cpu.pos.copy_(pos + t)
        gpu.x_in.copy_(x)
        gpu.pos.copy_(pos + t)
        a = cpu.step().numpy()
        b = gpu.step().cpu().numpy()
        cos, rel = orc.compare(b, a)
        assert cos >= 0.9999 and rel <= 1e-2, (t, cos, rel)
    assert ops.device_error() == 0
