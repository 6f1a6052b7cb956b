"""numpy restatement of one decode step of the gated DeltaNet (linear-attention) layer.

TEST INFRASTRUCTURE ONLY (see the package docstring).  The reference has no
DeltaNet code of its own: its Qwen3.5 path runs transformers' model in float32
(reference/from_q4nx.py:140-171; chat.py:74-78), so the algorithm is
transformers 5.5.0's `Qwen3_5GatedDeltaNet.forward` decode branch
(models/qwen3_5/modeling_qwen3_5.py:422-533) with its torch fallbacks
`torch_causal_conv1d_update` (:210-225), `l2norm` (:228-231),
`torch_recurrent_gated_delta_rule` (:314-353) and `Qwen3_5RMSNormGated`
(:175-190).  Pinned against that module's own outputs by
tests/golden/deltanet_golden.npz (made by tests/golden/make_deltanet_golden.py).

Evaluated in float64 on float32 inputs.  Layouts are transformers' cache and
projection layouts:
  qkv         [B][2*nk*dk + nv*dv]   in_proj_qkv output before the conv: q | k | v
  z           [B][nv*dv]             in_proj_z output (the norm gate)
  b, a        [B][nv]                in_proj_b / in_proj_a outputs
  conv_state  [B][conv_dim][W]       the last W conv inputs per channel, oldest first
  conv_w      [conv_dim][W]          depthwise conv1d weight, no bias
  state       [B][nv][dk][dv]        recurrent state
"""

from __future__ import annotations

import numpy as np


def plant_states(seed: int, conv_shape, state_shape) -> tuple[np.ndarray, np.ndarray]:
    """The seeded step-0 conv / recurrent states the golden script plants in the cache."""
    rng = np.random.default_rng(seed)
    conv0 = rng.standard_normal(conv_shape, dtype=np.float32)
    state0 = np.float32(0.5) * rng.standard_normal(state_shape, dtype=np.float32)
    return conv0, state0


def _silu(x: np.ndarray) -> np.ndarray:
    return x / (1.0 + np.exp(-x))


def _softplus(x: np.ndarray) -> np.ndarray:
    """torch.nn.functional.softplus (beta 1, threshold 20): x above the threshold."""
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


def conv_update(x: np.ndarray, conv_state: np.ndarray, conv_w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """torch_causal_conv1d_update for one new position (modeling_qwen3_5.py:210-225).

    The window is the state's last W-1 entries and the new input; the new state
    drops the oldest entry.  Returns (silu(conv), new_state)."""
    new_state = np.concatenate([conv_state[:, :, 1:], x[:, :, None]], axis=2)
    y = np.einsum("bcw,cw->bc", new_state.astype(np.float64), conv_w.astype(np.float64))
    return _silu(y), new_state


def l2norm(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """modeling_qwen3_5.py:228-231: x * rsqrt(sum(x^2) + eps) over the last axis."""
    return x / np.sqrt((x * x).sum(-1, keepdims=True) + eps)


def gated_delta_step(qkv, z, b, a, conv_state, conv_w, A_log, dt_bias, norm_w, state,
                     nk: int, nv: int, dk: int, dv: int, eps: float = 1e-6):
    """One decode step.  Returns (out [B][nv*dv] float64, conv_state', state').

    Follows modeling_qwen3_5.py:446-533 with seq_len 1 and a previous state:
    conv + silu over q|k|v, split, beta = sigmoid(b), g = -exp(A_log) *
    softplus(a + dt_bias), k heads repeated to the v heads (repeat_interleave),
    then torch_recurrent_gated_delta_rule with the q/k l2norm inside and
    Qwen3_5RMSNormGated over each head's dv outputs."""
    bsz = qkv.shape[0]
    key_dim = nk * dk
    mixed, conv_new = conv_update(np.asarray(qkv, np.float32), np.asarray(conv_state, np.float32),
                                  np.asarray(conv_w, np.float32))
    q = mixed[:, :key_dim].reshape(bsz, nk, dk)
    k = mixed[:, key_dim:2 * key_dim].reshape(bsz, nk, dk)
    v = mixed[:, 2 * key_dim:].reshape(bsz, nv, dv)
    beta = 1.0 / (1.0 + np.exp(-np.asarray(b, np.float64)))                       # [B][nv]
    g = -np.exp(np.asarray(A_log, np.float64)) * _softplus(np.asarray(a, np.float64) + dt_bias)
    rep = nv // nk
    q = np.repeat(q, rep, axis=1)
    k = np.repeat(k, rep, axis=1)
    q = l2norm(q) / np.sqrt(dk)
    k = l2norm(k)
    s = np.asarray(state, np.float64) * np.exp(g)[:, :, None, None]             # [B][nv][dk][dv]
    kv_mem = np.einsum("bhkv,bhk->bhv", s, k)
    delta = (v - kv_mem) * beta[:, :, None]
    s = s + k[:, :, :, None] * delta[:, :, None, :]
    o = np.einsum("bhkv,bhk->bhv", s, q)                                         # [B][nv][dv]
    zz = np.asarray(z, np.float64).reshape(bsz, nv, dv)
    o = o / np.sqrt((o * o).mean(-1, keepdims=True) + eps) * np.asarray(norm_w, np.float64) * _silu(zz)
    return o.reshape(bsz, nv * dv), conv_new, s


def synth_step_inputs(rng: np.random.Generator, batch: int, nk: int, nv: int, dk: int, dv: int,
                      width: int = 4) -> dict:
    """Seeded step inputs at the magnitudes of the golden module (unit-scale projections)."""
    conv_dim = 2 * nk * dk + nv * dv
    f = np.float32
    return {
        "qkv": rng.standard_normal((batch, conv_dim), dtype=f),
        "z": rng.standard_normal((batch, nv * dv), dtype=f),
        "b": rng.standard_normal((batch, nv), dtype=f),
        "a": rng.standard_normal((batch, nv), dtype=f),
        "conv_state": rng.standard_normal((batch, conv_dim, width), dtype=f),
        "conv_w": (f(0.5) * rng.standard_normal((conv_dim, width), dtype=f)),
        "A_log": np.log(rng.uniform(1.0, 16.0, nv)).astype(f),
        "dt_bias": rng.standard_normal(nv, dtype=f),
        "norm_w": (f(1.0) + f(0.1) * rng.standard_normal(dv, dtype=f)),
        "state": (f(0.5) * rng.standard_normal((batch, nv, dk, dv), dtype=f)),
    }
