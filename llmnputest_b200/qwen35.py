"""Qwen3.5 layer weights from a q4nx file, for DeltaNetLayer and GatedAttentionLayer.

The file uses FastFlowLM's tensor names and conventions that differ from
transformers (reference/from_q4nx.py:46-95, the reference's own loader):

  * q_proj of a full-attention layer stores all query rows, then all gate rows;
    transformers (and GatedAttentionLayer) want them per head, [q_h | gate_h].
    Each head's block is 256 rows, whole tile-rows, so the regroup is an order of
    tile-rows (`q_gate_tile_rows`): no tile byte changes.
  * q_norm / k_norm store 1 + w (transformers' Qwen3_5RMSNorm multiplies by 1 + w):
    the gated attention kernel takes w, so 1 is subtracted.  The layer input norms
    are passed as stored: the decode path's RMSNorm multiplies by the weight as is.
  * ssm_a stores -exp(A_log): A_log = log(-ssm_a).
  * The conv weight is stored [kernel][channels]; the step kernel wants [channels][4].
  * in_proj_b / in_proj_a are plain bf16 matrices (`.bf16.weight`), not tiles: they
    stay dense ("ba_dense", fp32 [2*nv][hidden]) and DeltaNetLayer runs them as one
    small fp32 GEMM beside the q4 in_proj.
Tiled weights are uploaded once through the reader's pinned staging
(`Q4NX.tile_segments` / `upload_segments`); dense ones are small.
"""

from __future__ import annotations

import numpy as np
import torch

from .format import TILE_ROWS, Q4NX, _device, upload_segments

# DeltaNetLayer key -> FLM name suffix of a linear-attention layer (reference/from_q4nx.py:46-56)
LINEAR_ATTN = {
    "qkv": "linear_attn.qkv_proj.weight",
    "z": "self_attn.gate_proj.weight",
    "b": "linear_attn.ssm_beta_proj.bf16.weight",
    "a": "linear_attn.ssm_alpha_proj.bf16.weight",
    "out_proj": "linear_attn.ssm_out_proj.weight",
    "conv": "linear_attn.ssm_conv1d.weight",
    "ssm_a": "linear_attn.ssm_a",
    "dt_bias": "linear_attn.ssm_dt.bias",
    "norm": "linear_attn.ssm_norm.weight",
}


def q_gate_tile_rows(n_heads: int, head_dim: int = 256) -> list[int]:
    """Tile-rows of the stored q_proj ([all q | all gate]) in transformers' order, per
    head q_h then gate_h (reference/from_q4nx.py:121-126 does the same on rows)."""
    tph = head_dim // TILE_ROWS
    rows: list[int] = []
    for i in range(n_heads):
        rows += range(i * tph, (i + 1) * tph)
        rows += range((n_heads + i) * tph, (n_heads + i + 1) * tph)
    return rows


def _f32(f: Q4NX, name: str) -> np.ndarray:
    return np.asarray(f.tensor(name), np.float32)


def _bf16_t(a: np.ndarray, device) -> torch.Tensor:
    from ml_dtypes import bfloat16
    b = np.ascontiguousarray(np.asarray(a, np.float32).astype(bfloat16))
    return torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).to(device)


def deltanet_weights(f: Q4NX, layer: int, n_k_heads: int, n_v_heads: int, hidden: int, device=None,
                     head_dim: int = 128) -> dict:
    """DeltaNetLayer weights of linear-attention layer `layer` (with "ba_dense")."""
    device = torch.device(device) if device is not None else _device()
    p = f"model.layers.{layer}."
    n = {k: p + v for k, v in LINEAR_ATTN.items()}
    conv_dim = (2 * n_k_heads + n_v_heads) * head_dim
    segs = (f.tile_segments(n["qkv"], n=conv_dim, k=hidden)
            + f.tile_segments(n["z"], n=n_v_heads * head_dim, k=hidden))
    ba = np.concatenate([_f32(f, n["b"]).reshape(n_v_heads, hidden), _f32(f, n["a"]).reshape(n_v_heads, hidden)])
    t = lambda a: torch.from_numpy(np.array(a, np.float32, order="C")).to(device)  # a C-order copy (file views are read-only)
    return {
        "in_proj": upload_segments(segs, device),
        "ba_dense": t(ba),
        "out_proj": f.device_tiles(n["out_proj"], device, n=hidden, k=n_v_heads * head_dim),
        "conv_w": t(_f32(f, n["conv"]).reshape(4, conv_dim).T),
        "A_log": t(np.log(-_f32(f, n["ssm_a"]).reshape(n_v_heads))),
        "dt_bias": t(_f32(f, n["dt_bias"]).reshape(n_v_heads)),
        "norm_w": t(_f32(f, n["norm"]).reshape(head_dim)),
        "input_norm": _bf16_t(_f32(f, p + "input_layernorm.weight"), device),
    }


def gated_attention_weights(f: Q4NX, layer: int, n_q_heads: int, n_kv_heads: int, hidden: int, inv_freq,
                            device=None, head_dim: int = 256) -> dict:
    """GatedAttentionLayer weights of full-attention layer `layer`; inv_freq: the rotary
    frequencies (llmnputest_b200.gated_attention.rope_inv_freq of the config's theta and
    partial rotary factor)."""
    device = torch.device(device) if device is not None else _device()
    p = f"model.layers.{layer}.self_attn."
    segs = (f.tile_segments(p + "q_proj.weight", tile_rows=q_gate_tile_rows(n_q_heads, head_dim),
                            n=2 * n_q_heads * head_dim, k=hidden)
            + f.tile_segments(p + "k_proj.weight", n=n_kv_heads * head_dim, k=hidden)
            + f.tile_segments(p + "v_proj.weight", n=n_kv_heads * head_dim, k=hidden))
    t = lambda a: torch.from_numpy(np.array(a, np.float32, order="C")).to(device)  # a C-order copy (file views are read-only)
    return {
        "in_proj": upload_segments(segs, device),
        "o_proj": f.device_tiles(p + "o_proj.weight", device, n=hidden, k=n_q_heads * head_dim),
        "q_norm_w": t(_f32(f, p + "q_norm.weight").reshape(head_dim) - 1.0),
        "k_norm_w": t(_f32(f, p + "k_norm.weight").reshape(head_dim) - 1.0),
        "inv_freq": inv_freq.to(device) if isinstance(inv_freq, torch.Tensor) else t(inv_freq),
        "input_norm": _bf16_t(_f32(f, f"model.layers.{layer}.input_layernorm.weight"), device),
    }
