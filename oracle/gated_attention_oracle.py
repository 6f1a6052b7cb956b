"""numpy restatement of one decode step of Qwen3.5's gated full-attention layer.

TEST INFRASTRUCTURE ONLY (see the package docstring).  The reference has no
code of its own for it: its Qwen3.5 path runs transformers' model in float32
(reference/from_q4nx.py:140-171; chat.py:74-78), so the algorithm is
transformers 5.5.0's `Qwen3_5Attention.forward` (models/qwen3_5/
modeling_qwen3_5.py:647-692) between q/k/v_proj and o_proj, with
`Qwen3_5RMSNorm` (:711-725, weight applied as 1 + w), `apply_rotary_pos_emb`
(:544-579, rotate_half on the first rotary dims only), the default RoPE
frequencies of `Qwen3_5TextRotaryEmbedding` (:85-155; text positions make the
interleaved MRoPE the plain one) and `eager_attention_forward` (:594-617).
Pinned against that module's own outputs by tests/golden/gated_attn_golden.npz
(made by tests/golden/make_gated_attn_golden.py).

Float64 arithmetic on float32 inputs, except the RoPE angle, which is the float32
product pos * inv_freq as torch forms it.  Layouts:
  qg          [B][nq * 2 * D]   q_proj output; head h is [q_h (D) | gate_h (D)]
  k_new, v_new[B][nkv * D]      k_proj / v_proj outputs
  k_cache     [B][nkv][>= pos][D] keys after q/k-norm and RoPE; v_cache alike
"""

from __future__ import annotations

import numpy as np


def plant_cache(seed: int, shape) -> tuple[np.ndarray, np.ndarray]:
    """The seeded K / V cache contents the golden script plants before the step."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal(shape, dtype=np.float32), rng.standard_normal(shape, dtype=np.float32)


def rmsnorm_plus_one(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """Qwen3_5RMSNorm (modeling_qwen3_5.py:711-725): x * rsqrt(mean(x^2) + eps) * (1 + w)."""
    xf = np.asarray(x, np.float64)
    return xf / np.sqrt((xf * xf).mean(-1, keepdims=True) + eps) * (1.0 + np.asarray(w, np.float64))


def rope_partial(x: np.ndarray, pos: int, inv_freq: np.ndarray) -> np.ndarray:
    """apply_rotary_pos_emb on the first 2*len(inv_freq) dims (rotate_half), the rest unchanged."""
    half = inv_freq.shape[0]
    ang = (np.float32(pos) * np.asarray(inv_freq, np.float32)).astype(np.float64)   # torch's fp32 product
    c, s = np.cos(ang), np.sin(ang)
    y = np.array(x, np.float64, copy=True)
    x0, x1 = y[..., :half].copy(), y[..., half:2 * half].copy()
    y[..., :half] = x0 * c - x1 * s
    y[..., half:2 * half] = x1 * c + x0 * s
    return y


def gated_attention_step(qg, k_new, v_new, q_norm_w, k_norm_w, inv_freq, k_cache, v_cache, pos,
                         nq: int, nkv: int, eps: float = 1e-6, stored=None):
    """One decode token per sequence at positions pos[b] (cache rows 0..pos-1 valid).

    Returns (out [B][nq*D] float64 = attention * sigmoid(gate), k_row, v_row [B][nkv][D]),
    k_row / v_row being what the step appends to the cache at pos.  `stored` (None:
    transformers' float32 cache) maps the appended rows to the values a cache of
    another precision holds, which the attention at pos then reads."""
    qg = np.asarray(qg, np.float64)
    bsz = qg.shape[0]
    d = qg.shape[1] // (2 * nq)
    grp = nq // nkv
    q = qg.reshape(bsz, nq, 2, d)[:, :, 0]
    gate = qg.reshape(bsz, nq, 2, d)[:, :, 1]
    qn = rmsnorm_plus_one(q, q_norm_w, eps)
    kn = rmsnorm_plus_one(np.asarray(k_new, np.float64).reshape(bsz, nkv, d), k_norm_w, eps)
    vr = np.asarray(v_new, np.float64).reshape(bsz, nkv, d)
    out = np.zeros((bsz, nq, d))
    k_row = np.zeros((bsz, nkv, d))
    for b in range(bsz):
        p = int(pos[b])
        qr = rope_partial(qn[b], p, inv_freq)
        kr = rope_partial(kn[b], p, inv_freq)
        k_row[b] = kr
        for g in range(nkv):
            k_at = kr[g] if stored is None else np.asarray(stored(kr[g]), np.float64)
            v_at = vr[b, g] if stored is None else np.asarray(stored(vr[b, g]), np.float64)
            keys = np.concatenate([np.asarray(k_cache[b, g, :p], np.float64), k_at[None]], 0)
            vals = np.concatenate([np.asarray(v_cache[b, g, :p], np.float64), v_at[None]], 0)
            for j in range(grp):
                h = g * grp + j
                s = keys @ qr[h] * d ** -0.5
                w = np.exp(s - s.max())
                out[b, h] = (w / w.sum()) @ vals
    out = out / (1.0 + np.exp(-gate))
    return out.reshape(bsz, nq * d), k_row, vr
