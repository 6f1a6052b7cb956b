"""numpy restatement of the reference's CPU implementation of the decode path.

TEST INFRASTRUCTURE ONLY (see the package docstring).  Each function names the
reference file:line whose behaviour it restates; those line numbers are into
the vegah/LLMNpuTest tree.  The q4nx index equations are the file format and
are necessarily the same as the reference's; the code around them is written
for this checker.

Float conventions follow the reference oracles exactly:
  * dequantised weights are float32, `code*d + m` (q4) / `code*s` (q8), and the
    `dequant_*` single-tile forms round that to bf16 with RNE
    (tools/q4nx.py:97-111, 127-143);
  * GEMV is float32 `W @ x` over the float32 weights (lm_head.py:129-144,
    granite_gemv.py:256-272);
  * attention, RoPE, SwiGLU and RMSNorm are evaluated in float64
    (granite_attention.py:163-167, granite_elementwise.py:328-366,
    granite_rmsnorm.py:112-113).
"""

from __future__ import annotations

import numpy as np
from ml_dtypes import bfloat16

# ----------------------------------------------------------------- format
TILE_ROWS = 32          # output rows per tile            (tools/q4nx.py:48)
TILE_K = 256            # K per tile                      (tools/q4nx.py:49)
ROW_BLOCK = 16          # rows per row-block, 2 per tile  (tools/q4nx.py:50)
GROUP = 32              # K per quantisation block        (tools/q4nx.py:47)
N_WEIGHTS = TILE_ROWS * TILE_K                  # 8192
N_META = TILE_ROWS * (TILE_K // GROUP)          # 256 scale entries per plane
Q4_TILE_BYTES = 2 * 2 * N_META + N_WEIGHTS // 2  # 5120: d | m | nibbles
Q8_TILE_BYTES = 2 * N_META + N_WEIGHTS           # 8704: scale | int8 codes


def meta_of_weight() -> np.ndarray:
    """Scale-plane index of each weight-index position (tools/q4nx.py:89-94).

    Weight i sits at row-block rb = i // 4096, k = (i % 4096) // 16 and row
    r = i % 16 inside the block; its scale is entry (k // 32)*32 + rb*16 + r.
    """
    i = np.arange(N_WEIGHTS)
    rb = i >> 12
    k = (i >> 4) & 255
    r = i & 15
    return (k >> 5) * TILE_ROWS + rb * ROW_BLOCK + r


_META = meta_of_weight()


def q4_codes(nibbles: np.ndarray) -> np.ndarray:
    """[..., 4096] packed bytes -> [..., 8192] codes 0..15 (tools/q4nx.py:80-86).

    Byte j holds weight 2j in its low nibble and weight 2j+1 in its high one.
    """
    nib = np.asarray(nibbles, dtype=np.uint8)
    out = np.empty(nib.shape[:-1] + (nib.shape[-1] * 2,), dtype=np.uint8)
    out[..., 0::2] = nib & 0x0F
    out[..., 1::2] = nib >> 4
    return out


def _bf16_plane(b: np.ndarray, lo: int, hi: int) -> np.ndarray:
    return np.ascontiguousarray(b[..., lo:hi]).view(bfloat16).astype(np.float32)


def q4_tiles_f32(tiles: np.ndarray) -> np.ndarray:
    """[T, 5120] uint8 -> [T, 8192] float32 in weight-index order.

    w = code*d + m in float32, as tools/q4nx.py:127-137 (`_q4_tiles`).
    """
    b = np.asarray(tiles, dtype=np.uint8).reshape(-1, Q4_TILE_BYTES)
    d = _bf16_plane(b, 0, 512)
    m = _bf16_plane(b, 512, 1024)
    codes = q4_codes(b[:, 1024:]).astype(np.float32)
    return codes * d[:, _META] + m[:, _META]


def q8_tiles_f32(tiles: np.ndarray) -> np.ndarray:
    """[T, 8704] uint8 -> [T, 8192] float32: w = code*scale (tools/q4nx.py:140-143)."""
    b = np.asarray(tiles, dtype=np.uint8).reshape(-1, Q8_TILE_BYTES)
    s = _bf16_plane(b, 0, 512)
    return b[:, 512:].view(np.int8).astype(np.float32) * s[:, _META]


def q4_tile_bf16(tile: bytes | np.ndarray) -> np.ndarray:
    """One q4 tile -> bf16[8192], the RNE rounding of `code*d + m` (tools/q4nx.py:97-101)."""
    return q4_tiles_f32(np.frombuffer(bytes(tile), np.uint8))[0].astype(bfloat16)


def q8_tile_bf16(tile: bytes | np.ndarray) -> np.ndarray:
    """One q8 tile -> bf16[8192] (tools/q4nx.py:104-111)."""
    return q8_tiles_f32(np.frombuffer(bytes(tile), np.uint8))[0].astype(bfloat16)


def tile_matrix(flat: np.ndarray) -> np.ndarray:
    """Weight-index order [8192] -> [32 rows][256 k] (tools/q4nx.py:114-116).

    Row rb*16 + r, column k holds weight rb*4096 + k*16 + r.
    """
    return np.asarray(flat).reshape(2, TILE_K, ROW_BLOCK).swapaxes(1, 2).reshape(TILE_ROWS, TILE_K)


def untile(flat: np.ndarray, n_t: int, k_t: int) -> np.ndarray:
    """[n_t*k_t, 8192] -> [n_t*32, k_t*256] (tools/q4nx.py:146-149).

    Tile (tr, kt) is stored at flat row tr*k_t + kt; inside it row rb*16 + r and
    column k come from weight index rb*4096 + k*16 + r.
    """
    a = np.asarray(flat).reshape(n_t, k_t, 2, TILE_K, ROW_BLOCK)
    # -> [tr][rb][r][kt][k]
    a = a.transpose(0, 2, 4, 1, 3)
    return a.reshape(n_t * TILE_ROWS, k_t * TILE_K)


def q4_matrix(raw, n_t: int, k_t: int) -> np.ndarray:
    """Whole q4 tensor -> float32 [N, K] (Q4NX.tensor, tools/q4nx.py:175-197)."""
    b = np.frombuffer(bytes(raw), np.uint8) if not isinstance(raw, np.ndarray) else raw
    return untile(q4_tiles_f32(b), n_t, k_t)


def q8_matrix(raw, n_t: int, k_t: int) -> np.ndarray:
    b = np.frombuffer(bytes(raw), np.uint8) if not isinstance(raw, np.ndarray) else raw
    return untile(q8_tiles_f32(b), n_t, k_t)


# ------------------------------------------------------------------ GEMV
def _gemv(raw, x, n_t: int, k_t: int, tile_bytes: int, decode, chunk: int) -> np.ndarray:
    b_all = (np.frombuffer(bytes(raw), np.uint8) if not isinstance(raw, np.ndarray)
             else np.asarray(raw, np.uint8)).reshape(n_t * k_t, tile_bytes)
    xf = np.asarray(x).astype(np.float32)
    single = xf.ndim == 1
    xb = xf[None, :] if single else xf
    assert xb.shape[1] == k_t * TILE_K, (xb.shape, k_t)
    out = np.empty((xb.shape[0], n_t * TILE_ROWS), np.float32)
    for lo in range(0, n_t, chunk):
        n = min(chunk, n_t - lo)
        w = untile(decode(b_all[lo * k_t:(lo + n) * k_t]), n, k_t)
        # one float32 GEMV per token, as the reference does it per call
        for t in range(xb.shape[0]):
            out[t, lo * TILE_ROWS:(lo + n) * TILE_ROWS] = w @ xb[t]
    return out[0] if single else out


def gemv_q4(raw, x, n_t: int, k_t: int, chunk: int = 256) -> np.ndarray:
    """y = W @ x, W q4nx q4 (granite_gemv.py:256-272).  x [K] or [B][K] -> fp32."""
    return _gemv(raw, x, n_t, k_t, Q4_TILE_BYTES, q4_tiles_f32, chunk)


def gemv_q8(raw, x, n_t: int, k_t: int, chunk: int = 256) -> np.ndarray:
    """y = W @ x, W q4nx q8 (lm_head.py:129-144, there with k_t fixed at 4)."""
    return _gemv(raw, x, n_t, k_t, Q8_TILE_BYTES, q8_tiles_f32, chunk)


def cpu_baseline_x(k: int) -> np.ndarray:
    """The fixed activation the reference's cpu_baseline.cpp uses (cpu_baseline.cpp:143)."""
    i = np.arange(k, dtype=np.int64)
    return (((i * 37) % 101) - 50).astype(np.float32) / np.float32(50.0)


# ------------------------------------------------------------ elementwise
def rope_cos_sin(pos: int, head_dim: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    """float64 cos/sin of pos * theta^(-2i/hd), i < hd/2 (granite_elementwise.py:328-331)."""
    half = head_dim // 2
    inv = 1.0 / (float(theta) ** (np.arange(half, dtype=np.float64) * 2.0 / head_dim))
    ang = float(pos) * inv
    return np.cos(ang), np.sin(ang)


def rope_half_split(x: np.ndarray, pos: int, theta: float) -> np.ndarray:
    """Half-split (rotate_half) RoPE over [..., hd], float64 (granite_elementwise.py:339-343)."""
    xh = np.asarray(x).astype(np.float64)
    hd = xh.shape[-1]
    half = hd // 2
    c, s = rope_cos_sin(pos, hd, theta)
    out = np.empty_like(xh)
    out[..., :half] = xh[..., :half] * c - xh[..., half:] * s
    out[..., half:] = xh[..., half:] * c + xh[..., :half] * s
    return out


def rope_interleaved(x: np.ndarray, pos: int, theta: float) -> np.ndarray:
    """The WRONG (interleaved-pair) convention, for the negative test (granite_elementwise.py:348-351)."""
    xh = np.asarray(x).astype(np.float64)
    c, s = rope_cos_sin(pos, xh.shape[-1], theta)
    out = np.empty_like(xh)
    e, o = xh[..., 0::2], xh[..., 1::2]
    out[..., 0::2] = e * c - o * s
    out[..., 1::2] = e * s + o * c
    return out


def swiglu(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """silu(g)*u in float64 (granite_elementwise.py:365-366)."""
    gf = np.asarray(g).astype(np.float64)
    return gf / (1.0 + np.exp(-gf)) * np.asarray(u).astype(np.float64)


def swiglu_from_accumulators(g32: np.ndarray, u32: np.ndarray) -> np.ndarray:
    """SwiGLU of fp32 GEMV outputs narrowed to bf16 first (granite_mlp.py:172-181)."""
    gb = np.asarray(g32, np.float32).astype(bfloat16).astype(np.float64)
    ub = np.asarray(u32, np.float32).astype(bfloat16).astype(np.float64)
    return gb / (1.0 + np.exp(-gb)) * ub


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """x * rsqrt(mean(x^2) + eps) * w over the last axis, float64 (granite_rmsnorm.py:112-113)."""
    xf = np.asarray(x).astype(np.float64)
    wf = np.asarray(w).astype(np.float64)
    ms = (xf * xf).mean(axis=-1, keepdims=True)
    return xf * (1.0 / np.sqrt(ms + eps)) * wf


# -------------------------------------------------------------- attention
def attention_one_head(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """softmax(K q * scale) V for one head in float64 (granite_attention.py:163-167)."""
    qf = np.asarray(q).astype(np.float64)
    kf = np.asarray(k).astype(np.float64)
    vf = np.asarray(v).astype(np.float64)
    s = (kf @ qf) * scale
    p = np.exp(s - s.max())
    return (p / p.sum()) @ vf


def gqa_decode(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
               lengths, scale: float) -> np.ndarray:
    """GQA decode for a batch, float64: the one-head oracle applied per q head.

    q [B][Hq][D]; caches [B][Hkv][T][D]; q head h reads kv head h // (Hq/Hkv);
    sequence b attends to positions [0, lengths[b]).  Returns [B][Hq][D].
    """
    q = np.asarray(q)
    bsz, hq, d = q.shape
    hkv = k_cache.shape[1]
    grp = hq // hkv
    out = np.zeros((bsz, hq, d), np.float64)
    for b in range(bsz):
        n = int(lengths[b])
        for kvh in range(hkv):
            kf = np.asarray(k_cache[b, kvh, :n]).astype(np.float64)
            vf = np.asarray(v_cache[b, kvh, :n]).astype(np.float64)
            qf = np.asarray(q[b, kvh * grp:(kvh + 1) * grp]).astype(np.float64)
            s = (qf @ kf.T) * scale                      # [grp][n]
            p = np.exp(s - s.max(axis=1, keepdims=True))
            out[b, kvh * grp:(kvh + 1) * grp] = (p / p.sum(axis=1, keepdims=True)) @ vf
    return out


# ------------------------------------------------------------ composition
def mlp_block(gate_raw, up_raw, down_raw, x, hidden: int, inter: int) -> tuple[np.ndarray, np.ndarray]:
    """gate+up -> SwiGLU -> bf16 h -> down (granite_mlp_full.py:231-237).

    Returns (h bf16 [inter], out float64 [hidden]).
    """
    g32 = gemv_q4(gate_raw, x, inter // TILE_ROWS, hidden // TILE_K)
    u32 = gemv_q4(up_raw, x, inter // TILE_ROWS, hidden // TILE_K)
    h = swiglu_from_accumulators(g32, u32).astype(np.float32).astype(bfloat16)
    out = gemv_q4(down_raw, h, hidden // TILE_ROWS, inter // TILE_K).astype(np.float64)
    return h, out


# --------------------------------------------------------------- synthetic
def synth_q4_tiles(rng: np.random.Generator, n_tiles: int) -> np.ndarray:
    """Seeded q4 tiles: codes uniform 0..15, d = bf16|N(0,.02)|, m = -bf16|N(0,.02)|.

    Q4_1 stores d > 0 and m < 0 (tools/q4nx.py:22-26), hence the sign of m.
    """
    t = np.empty((n_tiles, Q4_TILE_BYTES), np.uint8)
    d = (np.abs(rng.standard_normal((n_tiles, N_META))) * 0.02).astype(np.float32).astype(bfloat16)
    m = (-np.abs(rng.standard_normal((n_tiles, N_META))) * 0.02).astype(np.float32).astype(bfloat16)
    t[:, 0:512] = d.view(np.uint8).reshape(n_tiles, 512)
    t[:, 512:1024] = m.view(np.uint8).reshape(n_tiles, 512)
    t[:, 1024:] = rng.integers(0, 256, (n_tiles, N_WEIGHTS // 2), dtype=np.uint8)
    return t


def synth_q8_tiles(rng: np.random.Generator, n_tiles: int) -> np.ndarray:
    """Seeded q8 tiles: codes uniform int8 [-127, 127], scales bf16|N(0,.02)|."""
    t = np.empty((n_tiles, Q8_TILE_BYTES), np.uint8)
    s = (np.abs(rng.standard_normal((n_tiles, N_META))) * 0.02).astype(np.float32).astype(bfloat16)
    t[:, 0:512] = s.view(np.uint8).reshape(n_tiles, 512)
    t[:, 512:] = rng.integers(-127, 128, (n_tiles, N_WEIGHTS), dtype=np.int16).astype(np.int8).view(np.uint8)
    return t


def synth_bf16(rng: np.random.Generator, shape) -> np.ndarray:
    """Seeded N(0,1) values rounded to bf16."""
    return rng.standard_normal(shape).astype(np.float32).astype(bfloat16)


# ----------------------------------------------------------------- metrics
def compare(got, ref) -> tuple[float, float]:
    """(cosine, max-rel-err) in float64, the metric of granite_gemv.py:326-334."""
    g = np.asarray(got, dtype=np.float64).reshape(-1)
    r = np.asarray(ref, dtype=np.float64).reshape(-1)
    rel = float(np.abs(g - r).max() / (np.abs(r).max() + 1e-30))
    cos = float(g @ r / (np.linalg.norm(g) * np.linalg.norm(r) + 1e-30))
    return cos, rel
