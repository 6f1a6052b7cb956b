"""Golden vectors for one decode step of Qwen3.5's gated full-attention layer.

    python tests/golden/make_gated_attn_golden.py

The reference has no code of its own for this layer: its Qwen3.5 path builds
transformers' `Qwen3_5ForCausalLM` in float32 (reference/from_q4nx.py:140-171)
and steps it token by token (chat.py:74-78).  This script runs transformers
5.5.0's `Qwen3_5Attention.forward` (models/qwen3_5/modeling_qwen3_5.py:647-692,
eager attention) with its `Qwen3_5TextRotaryEmbedding`, seeded random
parameters and a `DynamicCache` whose prefilled keys and values are replaced by
seeded ones, then records one decode step: the q/k/v_proj outputs (hooks), the
o_proj input (the gated attention output) and the rows the step appended to the
cache.  Nothing in the product or the tests imports it: the tests read only
`gated_attn_golden.npz`.  Re-running it reproduces that file bit for bit.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle.gated_attention_oracle import plant_cache  # noqa: E402  (the seeded caches only)

HIDDEN = 64
EPS = 1e-6
# (name, batch, q heads, kv heads, prefill length = pos of the step, rope theta, partial rotary factor)
CASES = [
    ("g4", 2, 4, 1, 37, 10000.0, 0.25),
    ("c5", 1, 8, 2, 45, 10000000.0, 0.25),   # config 5's heads: 8 q / 2 kv, head_dim 256
    ("g2full", 1, 2, 1, 20, 10000.0, 1.0),   # rotary over the whole head
    ("g1", 2, 2, 2, 30, 10000.0, 0.25),       # one q head per kv head
]


def run_case(name, batch, nq, nkv, t_pre, theta, partial, seed):
    from transformers.cache_utils import DynamicCache
    from transformers.models.qwen3_5 import configuration_qwen3_5 as conf
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mq

    torch.manual_seed(seed)
    cfg = conf.Qwen3_5TextConfig(
        hidden_size=HIDDEN, num_hidden_layers=1, layer_types=["full_attention"], num_attention_heads=nq,
        num_key_value_heads=nkv, head_dim=256, rms_norm_eps=EPS,
        rope_parameters={"rope_type": "default", "rope_theta": theta, "partial_rotary_factor": partial})
    cfg._attn_implementation = "eager"
    attn = mq.Qwen3_5Attention(cfg, 0).float().eval()
    rope = mq.Qwen3_5TextRotaryEmbedding(cfg)
    with torch.no_grad():
        attn.q_norm.weight.normal_(0.0, 0.1)
        attn.k_norm.weight.normal_(0.0, 0.1)
        for lin in (attn.q_proj, attn.k_proj, attn.v_proj, attn.o_proj):
            lin.weight.normal_(0.0, 1.0 / HIDDEN ** 0.5)
    cache = DynamicCache(config=cfg)
    got: dict[str, torch.Tensor] = {}
    with torch.no_grad():
        h = torch.randn(batch, t_pre, HIDDEN)
        pe = rope(h, torch.arange(t_pre)[None].expand(batch, t_pre))
        causal = torch.full((t_pre, t_pre), float("-inf")).triu(1)[None, None]
        attn(h, pe, causal, past_key_values=cache)
        layer = cache.layers[0]
        k0, v0 = plant_cache(seed, tuple(layer.keys.shape))
        layer.keys.copy_(torch.from_numpy(k0))
        layer.values.copy_(torch.from_numpy(v0))
        hooks = [getattr(attn, p).register_forward_hook(
            lambda m, i, o, p=p: got.__setitem__(p, o.detach().clone())) for p in ("q_proj", "k_proj", "v_proj")]
        hooks.append(attn.o_proj.register_forward_pre_hook(
            lambda m, i: got.__setitem__("core", i[0].detach().clone())))
        h1 = torch.randn(batch, 1, HIDDEN)
        attn(h1, rope(h1, torch.full((batch, 1), t_pre)), None, past_key_values=cache)
        for hk in hooks:
            hk.remove()
    out = {
        "dims": np.array([batch, nq, nkv, 256, t_pre], np.int32),
        "plant_seed": np.array(seed, np.int64),
        "q_norm_w": attn.q_norm.weight.detach().numpy().copy(),
        "k_norm_w": attn.k_norm.weight.detach().numpy().copy(),
        "inv_freq": rope.inv_freq.numpy().copy(),
        "qg": got["q_proj"][:, 0].numpy().copy(),
        "k_new": got["k_proj"][:, 0].numpy().copy(),
        "v_new": got["v_proj"][:, 0].numpy().copy(),
        "out": got["core"][:, 0].numpy().copy(),
        "k_row": layer.keys[:, :, t_pre].numpy().copy(),
        "v_row": layer.values[:, :, t_pre].numpy().copy(),
    }
    return {f"{name}/{k}": v for k, v in out.items()}


def main() -> None:
    import transformers

    blobs: dict[str, np.ndarray] = {"transformers_version": np.array(transformers.__version__)}
    for i, case in enumerate(CASES):
        blobs.update(run_case(*case, seed=2000 + i))
    path = HERE / "gated_attn_golden.npz"
    np.savez_compressed(path, **blobs)
    print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
