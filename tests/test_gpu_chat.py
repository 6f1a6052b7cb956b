"""chat.py's turn (chat.py:37-42, 64-91) driven end to end with this package's
attach_lm_head: a small random-init transformers Qwen3.5 (hidden 1024, vocab 64, one
gated-DeltaNet and one gated-attention layer) in bf16 on the CPU, its lm_head read
from the synthetic q4nx container (tests/golden/container.q4nx, a 64 x 1024 q8 head)
and computed on the GPU; greedy generation of 16 tokens from a 5-token prompt (prefill
of 5 positions, then one position per token), with chat.py's accounting line.

Against the same model under chat.py's --cpu path: everything in torch, the lm_head a
bf16 Linear over the reference's dequantisation of the same container bytes
(chat.py:26-28, reference/npu.py:138-140).  Gate: the same greedy tokens, each step's
logits within the decode bar (cos >= 0.9999, rel <= 1e-2), every lm_head call on the
GPU (no CPU fallback)."""

import numpy as np
import pytest
import torch

from oracle import q4nx_oracle as orc

pytestmark = pytest.mark.gpu

MAX_NEW = 16


@pytest.fixture
def cpu_torch_qwen35(monkeypatch):
    """transformers' Qwen3.5 modules on their torch path: with a GPU present they bind
    flash-linear-attention's and causal-conv1d's Triton kernels, which cannot take the CPU
    tensors of chat.py's model (the model stays on the CPU, as in the reference)."""
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mq
    for name in ("FusedRMSNormGated", "chunk_gated_delta_rule", "fused_recurrent_gated_delta_rule",
                 "causal_conv1d_fn", "causal_conv1d_update"):
        if hasattr(mq, name):
            monkeypatch.setattr(mq, name, None)


def _model():
    from transformers.models.qwen3_5 import configuration_qwen3_5 as conf
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mq
    torch.manual_seed(0)
    cfg = conf.Qwen3_5TextConfig(vocab_size=64, hidden_size=1024, intermediate_size=512, num_hidden_layers=2,
                                 num_attention_heads=4, num_key_value_heads=1, head_dim=256, linear_num_key_heads=2,
                                 linear_num_value_heads=4, linear_key_head_dim=128, linear_value_head_dim=128,
                                 layer_types=["linear_attention", "full_attention"], tie_word_embeddings=False,
                                 max_position_embeddings=256, pad_token_id=0, eos_token_id=63)
    return mq.Qwen3_5ForCausalLM(cfg).to(torch.bfloat16).eval()


def _turn(model, ids, head):
    """chat.py:64-91: reset the head's counters, generate greedily, report the line."""
    import time
    if head is not None:
        head.design.seconds = head.design.calls = head.npu_calls = 0
    t = time.time()
    with torch.no_grad():
        out = model.generate(ids, max_new_tokens=MAX_NEW, do_sample=False, pad_token_id=0, output_scores=True,
                             return_dict_in_generate=True)
    new = out.sequences[0, ids.shape[-1]:]
    dt = time.time() - t
    line = f"[{len(new)} tokens, {dt:.1f}s, {len(new) / dt:.2f} tok/s"
    if head is not None:
        per = head.design.seconds / max(head.design.calls, 1) * 1e3
        line += (f"; lm_head on npu {head.npu_calls}x at {per:.1f} ms, "
                 f"{100 * head.design.seconds / dt:.0f}% of wall")
    return new, torch.stack(out.scores, 0)[:, 0].float().numpy(), line + "]"


def test_chat_turn_with_gpu_lm_head(container_path, golden, cpu_torch_qwen35):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from llmnputest_b200 import format as fmt
    from llmnputest_b200 import npu
    ids = torch.tensor([[1, 5, 9, 12, 3]])
    # --cpu: the reference's dequantised head as a bf16 Linear
    cpu_model = _model()
    cpu_model.lm_head.weight.data.copy_(torch.from_numpy(golden["ctr_lm_head_f32"]).to(torch.bfloat16))
    tok_cpu, logit_cpu, _ = _turn(cpu_model, ids, None)
    # the GPU head attached the way chat.py attaches the NPU one
    model = _model()
    design = {"kind": "q8_gemv", "n_rows": 64, "k": 1024}
    saved = npu.DESIGNS["lm_head"]
    npu.DESIGNS["lm_head"] = design
    try:
        head = npu.attach_lm_head(model, fmt.Q4NX(container_path))
    finally:
        npu.DESIGNS["lm_head"] = saved
    assert model.lm_head is head and head.n_rows == 64 and head.k == 1024
    tok, logit, line = _turn(model, ids, head)
    head.design.close()
    assert torch.equal(tok, tok_cpu), (tok.tolist(), tok_cpu.tolist())
    for step in range(MAX_NEW):
        cos, rel = orc.compare(logit[step], logit_cpu[step])
        assert cos >= 0.9999 and rel <= 1e-2, (step, cos, rel)
    # one prefill call of 5 positions, then one call per generated token, all on the GPU
    assert head.npu_calls == MAX_NEW and head.cpu_calls == 0 and head.design.calls == MAX_NEW
    assert f"lm_head on npu {MAX_NEW}x" in line
