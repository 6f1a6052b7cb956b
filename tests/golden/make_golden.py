"""Generate the golden vectors in tests/golden/ by running the REFERENCE's own code.

    python tests/golden/make_golden.py --reference <path to a vegah/LLMNpuTest checkout>

The reference is an NPU project, but its CPU oracles are plain numpy:

  * tools/q4nx.py imports directly (the q4nx reader and the dequantisers);
  * designs/lm_head/lm_head.py and designs/granite_gemv/granite_gemv.py hold the
    GEMV oracles `reference()`; they import the NPU toolchain (`aie`) at module
    level only, so a stub module with an identity `iron.jit` lets them import;
  * the attention / RoPE / SwiGLU / RMSNorm / MLP / QKV oracles are written
    inline in each design's `main()`.  Those exact source lines are executed
    here, in a namespace holding this script's seeded inputs, so the fixture
    is the reference's own arithmetic and not a restatement of it.

Nothing here is imported by the product or by the tests: the tests read only
the .npz / .bin files this writes.  Re-running it reproduces them bit for bit.
"""

from __future__ import annotations

import argparse
import json
import struct
import sys
import textwrap
import types
from pathlib import Path

import numpy as np
from ml_dtypes import bfloat16

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle import q4nx_oracle as orc  # noqa: E402  (only for the seeded generators)


# ---------------------------------------------------------------- aie stub
class _Anything:
    """Stands in for every toolchain object the design modules touch at import."""

    def __init__(self, *a, **k):
        pass

    def __call__(self, *a, **k):
        return _Anything()

    def __getattr__(self, name):
        return _Anything()

    def __getitem__(self, item):
        return _Anything()


def _stub_module(name: str) -> types.ModuleType:
    mod = types.ModuleType(name)
    mod.__getattr__ = lambda attr: _Anything()  # type: ignore[attr-defined]
    mod.__path__ = []  # mark as package so submodules resolve
    return mod


def install_aie_stub() -> None:
    for name in ("aie", "aie.iron", "aie.iron.controlflow", "aie.iron.device",
                 "aie.iron.kernel", "aie.helpers", "aie.helpers.taplib",
                 "aie.utils", "aie.utils.benchmark", "aie.iron.kernels",
                 "aie.iron.kernels._common"):
        sys.modules[name] = _stub_module(name)
    # `@iron.jit(...)` must leave the design function alone.
    sys.modules["aie.iron"].jit = lambda *a, **k: (lambda f: f)  # type: ignore[attr-defined]
    sys.modules["aie"].iron = sys.modules["aie.iron"]  # type: ignore[attr-defined]


def run_lines(path: Path, first: int, last: int, ns: dict, must_contain: list[str]) -> dict:
    """Execute lines first..last (1-based, inclusive) of a reference file in `ns`."""
    lines = path.read_text(encoding="utf-8").splitlines()[first - 1:last]
    src = textwrap.dedent("\n".join(lines))
    for token in must_contain:
        if token not in src:
            raise SystemExit(f"{path.name}:{first}-{last} no longer contains {token!r}; "
                             f"the reference moved, update the line range")
    exec(compile(src, f"{path.name}:{first}-{last}", "exec"), ns)
    return ns


def bf16_bits(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a).astype(bfloat16)).view(np.uint16)


# ------------------------------------------------------------- generators
def gen_format(q4nx, out: dict) -> None:
    rng = np.random.default_rng(101)
    t4 = orc.synth_q4_tiles(rng, 6)
    t8 = orc.synth_q8_tiles(rng, 6)
    out["fmt_q4_tiles"] = t4
    out["fmt_q8_tiles"] = t8
    out["fmt_meta_index"] = q4nx.meta_index().astype(np.int32)
    # single-tile dequant, bf16 (tools/q4nx.py:97-111)
    out["fmt_q4_dequant_bf16"] = np.stack([
        bf16_bits(q4nx.dequant_q4(*q4nx.split_q4_tile(t.tobytes()))) for t in t4])
    out["fmt_q8_dequant_bf16"] = np.stack([bf16_bits(q4nx.dequant_q8(t.tobytes())) for t in t8])
    out["fmt_q4_unpack"] = q4nx.unpack_nibbles(t4[0, 1024:])
    out["fmt_to_matrix"] = q4nx.to_matrix(np.arange(8192, dtype=np.int32))
    # whole-tensor float32 dequant + un-tiling, 3 tile-rows x 2 K-tiles
    out["fmt_q4_f32"] = q4nx._q4_tiles(t4)
    out["fmt_q8_f32"] = q4nx._q8_tiles(t8)
    out["fmt_q4_untiled_3x2"] = q4nx._untile(q4nx._q4_tiles(t4), 3, 2)
    out["fmt_q8_untiled_2x3"] = q4nx._untile(q4nx._q8_tiles(t8), 2, 3)


def write_container(path: Path, q4nx) -> dict:
    """A tiny .q4nx (safetensors) holding both tiled-shape conventions seen in FLM files."""
    rng = np.random.default_rng(202)
    tensors = {
        # Qwen-style 3-D tiled shape [n_t, k_t, tile_bytes]
        "lm_head.weight": ("I8", [2, 4, 8704], orc.synth_q8_tiles(rng, 8)),
        "model.layers.0.mlp.gate_proj.weight": ("I8", [3, 2, 5120], orc.synth_q4_tiles(rng, 6)),
        # granite-style 2-D tiled shape [n_t*k_t, tile_bytes]
        "model.layers.0.mlp.down_proj.weight": ("I8", [6, 5120], orc.synth_q4_tiles(rng, 6)),
        "model.norm.weight": ("BF16", [64], bf16_bits(rng.standard_normal(64) * 0.1 + 1.0)),
    }
    header, blobs, off = {"__metadata__": {"format": "q4nx-golden"}}, [], 0
    for name, (dt, shape, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    path.write_bytes(struct.pack("<Q", len(hj)) + hj + b"".join(blobs))

    f = q4nx.Q4NX(path)
    res = {
        "ctr_names": np.array(f.names()),
        "ctr_lm_head_f32": f.tensor("lm_head.weight"),
        "ctr_gate_f32": f.tensor("model.layers.0.mlp.gate_proj.weight"),
        "ctr_gate_f32_trim": f.tensor("model.layers.0.mlp.gate_proj.weight", (80, 300)),
        "ctr_norm": bf16_bits(f.tensor("model.norm.weight")),
        "ctr_down_raw": np.frombuffer(f.raw("model.layers.0.mlp.down_proj.weight"), np.uint8),
    }
    return res


def gen_gemv(lm_head, granite_gemv, out: dict) -> None:
    rng = np.random.default_rng(303)
    # q4: 6 tile-rows (not a multiple of 4 -- exercises a ragged row group) x 3 K-tiles
    n4, k4 = 6, 3
    w4 = orc.synth_q4_tiles(rng, n4 * k4)
    xs = [orc.synth_bf16(rng, k4 * 256) for _ in range(3)]
    xs.append(np.ones(k4 * 256, np.float32).astype(bfloat16))
    for hot in (100, 700):
        e = np.zeros(k4 * 256, np.float32)
        e[hot] = 1.0
        xs.append(e.astype(bfloat16))
    x4 = np.stack(xs)
    out["q4_w"], out["q4_x"] = w4, bf16_bits(x4)
    out["q4_shape"] = np.array([n4, k4])
    out["q4_y"] = np.stack([granite_gemv.reference(w4.tobytes(), x, n4, k4) for x in x4])

    # q8: lm_head.reference hard-codes K = 1024 (4 K-tiles); 5 tile-rows
    n8 = 5
    w8 = orc.synth_q8_tiles(rng, n8 * 4)
    xs = [orc.synth_bf16(rng, 1024) for _ in range(2)]
    xs.append(np.ones(1024, np.float32).astype(bfloat16))
    e = np.zeros(1024, np.float32)
    e[513] = 1.0
    xs.append(e.astype(bfloat16))
    x8 = np.stack(xs)
    out["q8_w"], out["q8_x"] = w8, bf16_bits(x8)
    out["q8_shape"] = np.array([n8, 4])
    out["q8_y"] = np.stack([lm_head.reference(w8.tobytes(), x, n8) for x in x8])


def gen_inline(ref: Path, granite_gemv, out: dict) -> None:
    gdir = ref / "designs" / "granite_gemv"
    rng = np.random.default_rng(404)

    # attention (granite_attention.py:163-167), seq lengths of its own test + a ragged one
    for seq in (32, 64, 128, 77):
        q_real = orc.synth_bf16(rng, 64)
        K = orc.synth_bf16(rng, (seq, 64))
        V = orc.synth_bf16(rng, (seq, 64))
        ns = run_lines(gdir / "granite_attention.py", 163, 167,
                       {"np": np, "q_real": q_real, "K": K, "V": V, "scale": 0.125},
                       ["Kf @ qf", "np.exp(s - s.max())"])
        out[f"attn{seq}_q"], out[f"attn{seq}_k"], out[f"attn{seq}_v"] = (
            bf16_bits(q_real), bf16_bits(K), bf16_bits(V))
        out[f"attn{seq}_ref"] = ns["ref"]

    # RoPE (granite_elementwise.py:136-138, 146-150, 155-158)
    heads, hd, theta = 40, 64, 10000.0
    for pos in (0, 17, 4095, 32767):
        x = orc.synth_bf16(rng, heads * hd)
        ns = {"np": np, "bfloat16": bfloat16, "theta": theta, "half": hd // 2, "hd": hd,
              "pos": pos, "x": x, "heads": heads}
        run_lines(gdir / "granite_elementwise.py", 136, 138, ns, ["inv = 1.0 / (theta"])
        run_lines(gdir / "granite_elementwise.py", 146, 150, ns, ["half-split"])
        run_lines(gdir / "granite_elementwise.py", 155, 158, ns, ["alt[:, 0::2]"])
        out[f"rope{pos}_x"] = bf16_bits(x)
        out[f"rope{pos}_ref"] = ns["ref"].reshape(-1)
        out[f"rope{pos}_alt"] = ns["alt"].reshape(-1)

    # SwiGLU (granite_elementwise.py:172-173)
    g = orc.synth_bf16(rng, 8192)
    u = orc.synth_bf16(rng, 8192)
    ns = run_lines(gdir / "granite_elementwise.py", 172, 173,
                   {"np": np, "g": g, "u": u}, ["ref2 ="])
    out["swiglu_g"], out["swiglu_u"], out["swiglu_ref"] = bf16_bits(g), bf16_bits(u), ns["ref2"]

    # RMSNorm (granite_rmsnorm.py:112-113), non-uniform weight as in :130-133
    x = orc.synth_bf16(rng, 2560)
    w = (rng.standard_normal(2560) * 0.1 + 1.0).astype(np.float32).astype(bfloat16)
    ns = run_lines(gdir / "granite_rmsnorm.py", 112, 113,
                   {"np": np, "x": x, "w": w, "eps": 1e-6}, ["np.sqrt((xf * xf).mean() + eps)"])
    out["rms_x"], out["rms_w"], out["rms_ref"] = bf16_bits(x), bf16_bits(w), ns["ref"]

    # fused gate+up+SwiGLU (granite_mlp.py:172-181)
    tile_rows, k_tiles = 8, 2
    raws = [orc.synth_q4_tiles(rng, tile_rows * k_tiles).tobytes() for _ in range(2)]
    x = orc.synth_bf16(rng, k_tiles * 256)
    ns = run_lines(ref / "designs" / "granite_gemv" / "granite_mlp.py", 172, 181,
                   {"np": np, "bfloat16": bfloat16, "reference": granite_gemv.reference,
                    "raws": raws, "x": x, "tile_rows": tile_rows, "k_tiles": k_tiles},
                   ["g32.astype(bfloat16)", "ref = (g / (1.0 + np.exp(-g))) * u"])
    out["mlp_gate"] = np.frombuffer(raws[0], np.uint8)
    out["mlp_up"] = np.frombuffer(raws[1], np.uint8)
    out["mlp_x"], out["mlp_shape"], out["mlp_ref"] = bf16_bits(x), np.array([tile_rows, k_tiles]), ns["ref"]

    # whole MLP block (granite_mlp_full.py:231-237): hidden 512, inter 1024
    hidden, inter = 512, 1024
    gu_rows, dn_rows = inter // 32, hidden // 32
    raws = [orc.synth_q4_tiles(rng, gu_rows * (hidden // 256)).tobytes(),
            orc.synth_q4_tiles(rng, gu_rows * (hidden // 256)).tobytes(),
            orc.synth_q4_tiles(rng, dn_rows * (inter // 256)).tobytes()]
    xfull = np.zeros(inter, np.float32)
    xfull[:hidden] = rng.standard_normal(hidden)
    xfull = xfull.astype(bfloat16)
    ns = run_lines(ref / "designs" / "granite_gemv" / "granite_mlp_full.py", 231, 237,
                   {"np": np, "bfloat16": bfloat16, "reference": granite_gemv.reference,
                    "raws": raws, "x": xfull, "hidden": hidden, "inter": inter,
                    "gu_rows": gu_rows, "dn_rows": dn_rows, "TILE_K": 256},
                   ["xh = x[:hidden]", "ref = reference(raws[2], h"])
    out["mlpf_gate"], out["mlpf_up"], out["mlpf_down"] = (np.frombuffer(r, np.uint8) for r in raws)
    out["mlpf_x"] = bf16_bits(xfull[:hidden])
    out["mlpf_shape"] = np.array([hidden, inter])
    out["mlpf_h"], out["mlpf_ref"] = bf16_bits(ns["h"]), ns["ref"]

    # q + k + v + RoPE (granite_qkv.py:157-159, 167-168, 176-194), 2 "cores" of 1 q head + 1 kv head
    cores, q_rows, kv_rows, k_tiles = 2, 4, 4, 2
    raws = [orc.synth_q4_tiles(rng, n * k_tiles).tobytes() for n in (q_rows, kv_rows, kv_rows)]
    kdim = k_tiles * 256
    x = np.concatenate([orc.synth_bf16(rng, kdim).astype(np.float32),
                        np.zeros(64, np.float32)]).astype(bfloat16)
    ns = {"np": np, "HD": 64, "theta": 10000.0, "pos": 1234, "x": x, "k": kdim,
          "reference": granite_gemv.reference, "raws": raws, "q_rows": q_rows,
          "kv_rows": kv_rows, "k_tiles": k_tiles, "q_per": q_rows // cores,
          "kv_per": kv_rows // cores, "ROWS_PER_TILE": 32, "CORES": cores}
    run_lines(gdir / "granite_qkv.py", 157, 159, ns, ["ang = pos * inv"])
    run_lines(gdir / "granite_qkv.py", 167, 168, ns, ["slice_f = rows_per * ROWS_PER_TILE"])
    run_lines(gdir / "granite_qkv.py", 176, 194, ns, ["def rope(y)", "rope(kk[c * kn:(c + 1) * kn])"])
    out["qkv_q"], out["qkv_k"], out["qkv_v"] = (np.frombuffer(r, np.uint8) for r in raws)
    out["qkv_x"] = bf16_bits(x[:kdim])
    out["qkv_meta"] = np.array([cores, q_rows, kv_rows, k_tiles, 1234])
    out["qkv_ref"] = ns["ref"]


def main(argv: list[str]) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path,
                    help="root of a vegah/LLMNpuTest checkout (read-only)")
    a = ap.parse_args(argv[1:])
    ref = a.reference.resolve()

    install_aie_stub()
    sys.path.insert(0, str(ref / "tools"))
    sys.path.insert(0, str(ref / "designs" / "lm_head"))
    sys.path.insert(0, str(ref / "designs" / "granite_gemv"))
    import q4nx  # noqa: E402  the reference's reader
    import lm_head  # noqa: E402
    import granite_gemv  # noqa: E402

    out: dict = {}
    gen_format(q4nx, out)
    gen_gemv(lm_head, granite_gemv, out)
    gen_inline(ref, granite_gemv, out)
    ctr_path = HERE / "container.q4nx"
    out.update(write_container(ctr_path, q4nx))
    np.savez_compressed(HERE / "golden.npz", **out)
    total = sum(v.nbytes for v in out.values())
    print(f"wrote {len(out)} arrays ({total / 1e6:.2f} MB raw) to {HERE / 'golden.npz'} "
          f"and {ctr_path.name} ({ctr_path.stat().st_size} B)")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
