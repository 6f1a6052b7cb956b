"""Golden vectors for one decode step of the gated DeltaNet (linear-attention) layer.

    python tests/golden/make_deltanet_golden.py

The reference has no DeltaNet code of its own: its Qwen3.5 path builds
transformers' `Qwen3_5ForCausalLM` in float32 (reference/from_q4nx.py:140-171,
no dtype given, so the torch default) and steps it token by token
(chat.py:74-78).  The arithmetic is therefore transformers 5.5.0's
`Qwen3_5GatedDeltaNet.forward` (models/qwen3_5/modeling_qwen3_5.py:422-533) on
its decode branch (seq_len 1, a cache with a previous state): the torch
`torch_causal_conv1d_update` (:210-225), `l2norm` (:228-231),
`torch_recurrent_gated_delta_rule` (:314-353) and `Qwen3_5RMSNormGated`
(:175-190), the torch fallbacks that run on a CPU (no fla / causal-conv1d).

This script runs that module itself with seeded random parameters, plants
seeded conv and recurrent states in a `DynamicCache`, and records, per decode
step, what the fused step kernel consumes (the in_proj_qkv / z / b / a outputs,
captured by hooks) and produces (the out_proj input, the new conv and recurrent
states).  Nothing in the product or the tests imports it: the tests read only
`deltanet_golden.npz`.  Re-running it reproduces that file bit for bit on the
same torch build.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle.deltanet_oracle import plant_states  # noqa: E402  (the seeded step-0 states only)

# (name, batch, k heads, v heads, head dim, steps, state entries kept)
CASES = [
    ("d32", 2, 1, 2, 32, 3, "all"),        # every tensor, three chained steps
    ("d128", 2, 1, 2, 128, 2, "sample"),   # the kernel's head dim, GQA ratio 2
    ("d128r1", 1, 2, 2, 128, 1, "sample"),  # ratio 1
    ("d32r4", 1, 1, 4, 32, 2, "all"),      # four v heads per k head
]
SAMPLE_STRIDE = 61  # recurrent-state entries kept for the head-dim-128 cases
HIDDEN = 64
EPS = 1e-6


def build(batch: int, nk: int, nv: int, d: int, seed: int):
    from transformers.cache_utils import DynamicCache
    from transformers.models.qwen3_5 import configuration_qwen3_5 as conf
    from transformers.models.qwen3_5 import modeling_qwen3_5 as mq

    torch.manual_seed(seed)
    cfg = conf.Qwen3_5TextConfig(
        hidden_size=HIDDEN, num_hidden_layers=1, layer_types=["linear_attention"],
        linear_num_key_heads=nk, linear_num_value_heads=nv, linear_key_head_dim=d,
        linear_value_head_dim=d, linear_conv_kernel_dim=4, rms_norm_eps=EPS,
        num_attention_heads=2, num_key_value_heads=1, head_dim=32)
    mod = mq.Qwen3_5GatedDeltaNet(cfg, 0).float().eval()
    with torch.no_grad():
        mod.conv1d.weight.normal_(0.0, 0.5)
        mod.A_log.copy_(torch.log(torch.empty(nv).uniform_(1.0, 16.0)))
        mod.dt_bias.normal_(0.0, 1.0)
        mod.norm.weight.normal_(1.0, 0.1)
        for lin in (mod.in_proj_qkv, mod.in_proj_z, mod.in_proj_b, mod.in_proj_a, mod.out_proj):
            lin.weight.normal_(0.0, 1.0 / HIDDEN ** 0.5)
    cache = DynamicCache(config=cfg)
    with torch.no_grad():  # a 2-token prefill creates the cache layer's tensors
        mod(torch.randn(batch, 2, HIDDEN), cache_params=cache)
        layer = cache.layers[0]
        conv0, state0 = plant_states(seed, tuple(layer.conv_states.shape), tuple(layer.recurrent_states.shape))
        layer.conv_states.copy_(torch.from_numpy(conv0))
        layer.recurrent_states.copy_(torch.from_numpy(state0))
    assert cache.has_previous_state(0)
    return mod, cache


def run_case(name, batch, nk, nv, d, steps, keep, seed):
    mod, cache = build(batch, nk, nv, d, seed)
    layer = cache.layers[0]
    got: dict[str, torch.Tensor] = {}
    hooks = [getattr(mod, p).register_forward_hook(
        lambda m, i, o, p=p: got.__setitem__(p, o.detach().clone()))
        for p in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")]
    hooks.append(mod.out_proj.register_forward_pre_hook(
        lambda m, i: got.__setitem__("core", i[0].detach().clone())))
    out: dict[str, np.ndarray] = {
        "conv_w": mod.conv1d.weight.detach()[:, 0, :].numpy().copy(),   # [conv_dim][4]
        "A_log": mod.A_log.detach().numpy().copy(),
        "dt_bias": mod.dt_bias.detach().numpy().copy(),
        "norm_w": mod.norm.weight.detach().numpy().copy(),
        "plant_seed": np.array(seed, np.int64),  # plant_states(seed, ...) gives the step-0 states
        "dims": np.array([batch, nk, nv, d, d, steps], np.int32),
    }
    if keep == "all":
        out["conv_state0"] = layer.conv_states.numpy().copy()       # [B][conv_dim][4]
        out["state0"] = layer.recurrent_states.numpy().copy()       # [B][nv][dk][dv]
    flat = np.arange(layer.recurrent_states.numel())[::SAMPLE_STRIDE]
    out["sample_idx"] = flat
    with torch.no_grad():
        for t in range(steps):
            mod(torch.randn(batch, 1, HIDDEN), cache_params=cache)
            out[f"qkv{t}"] = got["in_proj_qkv"][:, 0].numpy().copy()   # [B][2*nk*d + nv*d]
            out[f"z{t}"] = got["in_proj_z"][:, 0].numpy().copy()       # [B][nv*d]
            out[f"b{t}"] = got["in_proj_b"][:, 0].numpy().copy()       # [B][nv]
            out[f"a{t}"] = got["in_proj_a"][:, 0].numpy().copy()       # [B][nv]
            out[f"out{t}"] = got["core"][:, 0].numpy().copy()          # [B][nv*d]
            out[f"conv_state{t + 1}"] = layer.conv_states.numpy().copy()
            st = layer.recurrent_states.numpy()
            if keep == "all":
                out[f"state{t + 1}"] = st.copy()
            else:
                out[f"state{t + 1}_sample"] = st.reshape(-1)[flat].copy()
    for h in hooks:
        h.remove()
    return {f"{name}/{k}": v for k, v in out.items()}


def main() -> None:
    import transformers

    blobs: dict[str, np.ndarray] = {"transformers_version": np.array(transformers.__version__)}
    for i, case in enumerate(CASES):
        blobs.update(run_case(*case, seed=1000 + i))
    path = HERE / "deltanet_golden.npz"
    np.savez_compressed(path, **blobs)
    print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
