"""Benchmark of the decode hot path on B200 (one JSON line on rank 0).

Value (the metric's "decode tokens/s at 1/2/4/8 B200"): one
full random-init decode step of the dense GQA 3B -- 40 layers of RMSNorm, q4nx QKV,
RoPE + GQA flash-decode, q4nx O, RMSNorm + fused SwiGLU gate/up, q4nx down; final
RMSNorm and q8 lm_head -- at batch 32 (--batch) and context 4096, one CUDA graph per
step, tensor-parallel over the ranks at N > 1 (kv heads, O input columns, FFN rows /
down K-tiles, vocab rows; the O and down all-reduces summed over NVLink by the next
GEMM's x pre-pass, the logits gathered by a peer-memory exchange).  Strong
scaling: the same step, split over more GPUs.  tokens/s = batch / step time (max over
ranks).  `roofline` is the step's dominant kernel, timed alone on the step's own
buffers; `e2e` is the same step with its inputs copied in from pinned host memory and
its logits copied out, every step.

Extra keys: the GEMV sweep (the 160 q4nx GEMVs of a step's weight
stream, batch 1 and 8, GB/s against HBM), the q8 lm_head GEMV, GQA
flash-decode, the decode step at batch 1 and 8, config 5's kernels and
step, and the CPU baselines of configs 1-4 timed on this host; at N > 1 the tensor-
parallel parity checks (config 4 and config 5 against one GPU) and config 5's
tensor-parallel step.  Synthetic seeded data with the BASELINE distributions.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

`--impl reference` times config 4's step composed from the reference's own CPU parts
(its cpu_baseline.cpp GEMV, compiled unmodified into oracle/_ref/, its attention oracle,
its --cpu torch lm_head) on this host's cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "q4/q8 GEMV HBM GB/s (% of peak); decode tokens/s at 1/2/4/8 B200"
SHAPES = [("qkv", 112, 10), ("o", 80, 10), ("gate_up", 512, 10), ("down", 80, 32)]  # (tile-rows, K-tiles)
Q4_TILE, Q8_TILE = 5120, 8704
# dram__bytes_read.sum + dram__bytes_write.sum over tile bytes for the GEMV launches
# that stream from DRAM (one ncu capture of a layer's four GEMVs)
GEMV_DRAM_RATIO = 1.003
# the same ratio for the step's kernels (one ncu capture each of bench.py --profile-case):
# attention at B=32 ctx 4096 (268.94 MB read + 4.18 MB written
# over 268.44 MB of K/V), the packed SwiGLU GEMM (26.44 over 26.21 MB of tiles), the q8
# lm_head GEMM (273.19 + 9.50 over 273.11 MB of tiles; the logits are written)
DRAM_RATIO = {"gqa_decode": 1.0175, "q4_swiglu_gemm": 1.009, "lm_head_q8_gemm": 1.035}
LAYERS = 40


def peaks() -> dict:
    try:
        p = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p.get("bf16_tflops", 1590.0)), "src": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


# ------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.lines: list[str] = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", self.gpu_id], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_uuid(torch) -> str:
    try:
        u = str(torch.cuda.get_device_properties(torch.cuda.current_device()).uuid)
        return u if u.startswith("GPU-") else f"GPU-{u}"
    except Exception:
        return str(torch.cuda.current_device())


# -------------------------------------------------------------- CPU baselines
def _write_sample_file(path: Path, n_tiles: int, rng) -> None:
    import numpy as np
    from oracle import q4nx_oracle as orc
    with path.open("wb") as f:
        left = n_tiles
        while left:
            n = min(left, 4096)
            f.write(orc.synth_q4_tiles(rng, n).tobytes())
            left -= n


def run_reference_gemv(iters: int, layers: int = 8) -> dict:
    """The reference's cpu_baseline.cpp (oracle/_ref) over `layers` layers' projections, all cores.

    Falls back to the numpy oracle port when the compiled reference is absent.
    Returns {"gbs", "cores", "kind", "sample", "seconds"}.
    """
    import numpy as np
    exe = ROOT / "oracle" / "_ref" / "cpu_baseline"
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(1234)
    k2560_rows = sum(n for name, n, k in SHAPES if k == 10) * layers
    k8192_rows = sum(n for name, n, k in SHAPES if k == 32) * layers
    groups = [(k2560_rows, 10), (k8192_rows, 32)]
    total_bytes = sum(r * k * Q4_TILE for r, k in groups)
    t0 = time.time()
    if exe.exists():
        tot_ms = 0.0
        with tempfile.TemporaryDirectory() as td:
            for rows, kt in groups:
                p = Path(td) / f"w{kt}.bin"
                _write_sample_file(p, rows * kt, rng)
                r = subprocess.run([str(exe), str(p), "0", str(rows), str(kt), str(cores), str(iters)],
                                   capture_output=True, text=True, timeout=900)
                if r.returncode != 0:
                    raise RuntimeError(f"cpu_baseline failed: {r.stderr}")
                line = next(ln for ln in r.stdout.splitlines() if ln.startswith("GEMV"))
                tot_ms += float(line.split()[1])
        gbs = total_bytes / (tot_ms * 1e-3) / 1e9
        kind = "reference"
    else:
        from oracle import q4nx_oracle as orc
        w = orc.synth_q4_tiles(rng, 80 * 10)
        x = orc.synth_bf16(rng, 2560)
        n = 0
        t1 = time.time()
        while time.time() - t1 < 5.0:
            orc.gemv_q4(w, x, 80, 10)
            n += 1
        gbs = n * w.nbytes / (time.time() - t1) / 1e9
        kind, cores = "port", 1
    return {"gbs": gbs, "cores": cores, "kind": kind, "seconds": time.time() - t0,
            "sample": (f"{layers} layers of the 4 projection shapes ({total_bytes / 1e6:.0f} MB of q4 tiles), "
                       f"batch 1, {iters} passes each" if kind == "reference"
                       else "one 80x10-tile O projection, numpy oracle, 5 s")}


def cpu_lm_head(n_t: int = 7760, k_t: int = 4, seconds: float = 4.0) -> dict:
    """Config 1 (q8 lm_head, batch 1) on the host cores, two ways:
    numpy   the restatement of lm_head.reference (designs/lm_head/lm_head.py:129-144: chunked
            float32 dequant, then a float32 matmul) over the whole head, once;
    torch   the reference's --cpu path: torch bf16 F.linear on the dequantised weight
            (chat.py:26-28, reference/npu.py:138-140) on all threads, the dequant not timed.
    GB/s against the head's algorithmic bytes (tiles + x + y)."""
    import numpy as np
    import torch
    from oracle import q4nx_oracle as orc
    rng = np.random.default_rng(77)
    w = orc.synth_q8_tiles(rng, n_t * k_t)
    x = orc.synth_bf16(rng, k_t * 256)
    nbytes = w.nbytes + k_t * 256 * 2 + n_t * 32 * 4
    t0 = time.perf_counter()
    orc.gemv_q8(w, x, n_t, k_t)
    t_np = time.perf_counter() - t0
    wd = torch.from_numpy(orc.q8_matrix(w, n_t, k_t)).to(torch.bfloat16)
    xt = torch.from_numpy(x.astype(np.float32)).to(torch.bfloat16)[None, :]
    torch.nn.functional.linear(xt, wd)
    n, t1 = 0, time.perf_counter()
    while time.perf_counter() - t1 < seconds:
        torch.nn.functional.linear(xt, wd)
        n += 1
    t_t = (time.perf_counter() - t1) / n
    return {"numpy_ms": round(t_np * 1e3, 1), "numpy_gbs": round(nbytes / t_np / 1e9, 2),
            "torch_bf16_ms": round(t_t * 1e3, 2), "torch_bf16_gbs": round(nbytes / t_t / 1e9, 2),
            "threads": torch.get_num_threads(), "cores": os.cpu_count(),
            "sample": f"{n_t * 32}x{k_t * 256} q8 head, batch 1; numpy once, torch {n} calls"}


def cpu_attention(bsz: int, ctx: int, hq: int = 40, hkv: int = 8, d: int = 64, seconds: float = 2.0) -> dict:
    """Config 3 on the host cores: the reference's attention oracle (designs/granite_gemv/
    granite_attention.py:163-167: scores, softmax, weighted sum) vectorised over sequences and
    kv heads in float32 numpy, and torch's CPU scaled_dot_product_attention (float32, GQA), one
    new query token per sequence over ctx cached positions.  GB/s against the bf16 K/V bytes
    the GPU kernel reads (B*ctx*Hkv*D*2*2)."""
    import numpy as np
    import torch
    rng = np.random.default_rng(ctx + bsz)
    grp = hq // hkv
    q = rng.standard_normal((bsz, hkv, grp, d), dtype=np.float32)
    k = rng.standard_normal((bsz, hkv, ctx, d), dtype=np.float32)
    v = rng.standard_normal((bsz, hkv, ctx, d), dtype=np.float32)

    def numpy_attn():
        s = (q @ k.transpose(0, 1, 3, 2)) * np.float32(d ** -0.5)
        p = np.exp(s - s.max(axis=-1, keepdims=True))
        return (p / p.sum(axis=-1, keepdims=True)) @ v

    def timed(fn):
        fn()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds or n < 2:
            fn()
            n += 1
        return (time.perf_counter() - t0) / n

    t_np = timed(numpy_attn)
    qt = torch.from_numpy(q.reshape(bsz, hq, 1, d))
    kt, vt = torch.from_numpy(k), torch.from_numpy(v)
    t_sdpa = timed(lambda: torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, enable_gqa=True))
    nbytes = bsz * ctx * hkv * d * 2 * 2
    return {"batch": bsz, "ctx": ctx, "numpy_ms": round(t_np * 1e3, 3), "numpy_gbs": round(nbytes / t_np / 1e9, 2),
            "sdpa_ms": round(t_sdpa * 1e3, 3), "sdpa_gbs": round(nbytes / t_sdpa / 1e9, 2),
            "threads": torch.get_num_threads(), "cores": os.cpu_count()}


def cpu_decode_step(bsz: int, ctx: int, gemv: dict | None = None) -> dict:
    """Config 4's decode step on the host cores, composed from the reference's CPU parts as the
    layer runs them (designs/granite_gemv/granite_layer.py:54-59), one layer timed and counted
    40 times:
      projections  the reference's own cpu_baseline.cpp GEMV (oracle/_ref, its batch-1 kernel run
                   once per token) at the GB/s it reaches on the four projection shapes;
      attention    the reference's attention oracle, vectorised float32 numpy, at (bsz, ctx);
      lm_head      the reference's --cpu path, torch bf16 F.linear over all tokens at once
                   (chat.py:26-28), the 100352 x 2560 head;
    RMSNorm, RoPE and SwiGLU add < 1 % and are left out.  Returns tok/s and the parts."""
    import numpy as np
    import torch
    from llmnputest_b200.decode import GRANITE_3B as cfg
    gemv = gemv or run_reference_gemv(iters=10, layers=2)
    wb = cfg.weight_bytes()
    t_proj = bsz * wb["per_layer"] / (gemv["gbs"] * 1e9)
    att = cpu_attention(bsz, ctx, seconds=1.0)
    t_att = att["numpy_ms"] * 1e-3
    rng = np.random.default_rng(5)
    wd = torch.from_numpy(rng.standard_normal((cfg.vocab, cfg.hidden), dtype=np.float32)).to(torch.bfloat16)
    xt = torch.from_numpy(rng.standard_normal((bsz, cfg.hidden), dtype=np.float32)).to(torch.bfloat16)
    torch.nn.functional.linear(xt, wd)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 1.0 or n < 2:
        torch.nn.functional.linear(xt, wd)
        n += 1
    t_lm = (time.perf_counter() - t0) / n
    step = cfg.n_layers * (t_proj + t_att) + t_lm
    return {"tok_s": round(bsz / step, 3), "ms_per_step": round(step * 1e3, 1), "batch": bsz, "ctx": ctx,
            "cores": gemv["cores"], "kind": gemv["kind"],
            "parts_ms": {"projections_per_layer": round(t_proj * 1e3, 2), "attention_per_layer": round(t_att * 1e3, 2),
                         "lm_head": round(t_lm * 1e3, 2)},
            "sample": f"one layer's parts timed, x {cfg.n_layers} layers + lm_head; projections: {gemv['sample']} "
                      f"at {gemv['gbs']:.1f} GB/s, once per token; attention: numpy float32 at batch {bsz}, ctx {ctx}; "
                      "lm_head: torch bf16 F.linear"}


# --------------------------------------------------------------------- B200
def make_q4_tiles(torch, n_tiles: int, gen, device):
    w = torch.randint(0, 256, (n_tiles, Q4_TILE), dtype=torch.uint8, device=device, generator=gen)
    d = (torch.randn(n_tiles, 256, device=device, generator=gen) * 0.02).abs().to(torch.bfloat16)
    m = -(torch.randn(n_tiles, 256, device=device, generator=gen) * 0.02).abs().to(torch.bfloat16)
    w[:, 0:512] = d.view(torch.uint8)
    w[:, 512:1024] = m.view(torch.uint8)
    return w.reshape(-1)


def make_q8_tiles(torch, n_tiles: int, gen, device):
    w = torch.randint(-127, 128, (n_tiles, Q8_TILE), dtype=torch.int16, device=device, generator=gen)
    w = w.to(torch.int8).view(torch.uint8)
    s = (torch.randn(n_tiles, 256, device=device, generator=gen) * 0.02).abs().to(torch.bfloat16)
    w[:, 0:512] = s.view(torch.uint8)
    return w.reshape(-1)


def build_sweep(torch, ops, batch: int, layers: int, gen, device):
    """Weights, inputs and outputs of the 40-layer sweep; returns (calls, bytes)."""
    calls, nbytes = [], 0
    for _ in range(layers):
        for name, n_t, k_t in SHAPES:
            w = make_q4_tiles(torch, n_t * k_t, gen, device)
            x = torch.randn(batch, k_t * 256, device=device, generator=gen).to(torch.bfloat16)
            y = torch.empty(batch, n_t * 32, device=device, dtype=torch.float32)
            calls.append((name, w, n_t, k_t, x, y))
            nbytes += w.numel()
    return calls, nbytes


def graph_of(torch, fn):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()  # warm the launch plans outside capture
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


def time_graph(torch, g, steps: int, warmup: int) -> float:
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        g.replay()
    b.record()
    b.synchronize()
    return a.elapsed_time(b) / steps  # ms per replay


def measure_tc_gemm(torch, ops, gen, device, tensor_peak: float, steps: int, hbm_peak: float) -> list:
    """Tensor-core GEMM (b2_q4_gemm / b2_q4_swiglu_gemm): config-5 MLP shapes at batch 256
    (hidden 1024, intermediate 3584) and config-4 projections at batch 32, on packed tiles
    (A dequantised into TMEM, the decoders' form) and on the tiles as stored (A through
    shared memory).  A weight pool above L2 is rotated; algorithmic bytes = the q4 tiles,
    flops = 2*B*N*K."""
    cases = [("c5_gate_up_swiglu", 112, 4, 256, True), ("c5_down", 32, 14, 256, False),
             ("c4_qkv", 112, 10, 32, False), ("c4_gate_up_swiglu", 256, 10, 32, True), ("c4_down", 80, 32, 32, False)]
    out = []
    for name, n_t, k_t, bsz, swiglu in cases:
        per = n_t * k_t * Q4_TILE * (2 if swiglu else 1)
        pool = max(1, min(64, -(-300_000_000 // per)))
        ws_ = [(make_q4_tiles(torch, n_t * k_t, gen, device), make_q4_tiles(torch, n_t * k_t, gen, device) if swiglu
                else None) for _ in range(pool)]
        x = torch.randn(bsz, k_t * 256, device=device, generator=gen).to(torch.bfloat16)
        y = torch.empty(bsz, n_t * 32, device=device, dtype=torch.bfloat16 if swiglu else torch.float32)
        nb = ops.gemm_workspace_bytes(bsz, k_t)
        raw = torch.empty(nb + 256, dtype=torch.uint8, device=device)
        wsb = raw[(256 - raw.data_ptr() % 256) % 256:][:nb]

        def calls(pool_=ws_, packed=False, x=x, y=y, wsb=wsb, n_t=n_t, k_t=k_t, swiglu=swiglu):
            for g_, u_ in pool_:
                if swiglu:
                    ops.q4_swiglu_gemm(g_, u_, n_t, k_t, x, out=y, workspace=wsb, prefetch=True, packed=packed)
                else:
                    ops.q4_gemm(g_, n_t, k_t, x, out=y, workspace=wsb, prefetch=True, packed=packed)

        flops = 2 * bsz * n_t * 32 * k_t * 256 * (2 if swiglu else 1)
        g = graph_of(torch, calls)
        t_smem = time_graph(torch, g, max(5, steps // 50), 3) / pool
        del g
        pk = [(ops.q4_gemm_pack(g_, n_t, k_t), ops.q4_gemm_pack(u_, n_t, k_t) if u_ is not None else None)
              for g_, u_ in ws_]
        g = graph_of(torch, lambda: calls(pk, True))
        t_ms = time_graph(torch, g, max(5, steps // 50), 3) / pool
        out.append({"case": name, "batch": bsz, "us": round(t_ms * 1e3, 2), "gbs": round(per / (t_ms * 1e-3) / 1e9, 1),
                    "frac_of_measured_hbm": round(per / (t_ms * 1e-3) / 1e9 / hbm_peak, 3),
                    "tflops": round(flops / (t_ms * 1e-3) / 1e12, 1),
                    "frac_of_measured_tensor": round(flops / (t_ms * 1e-3) / 1e12 / tensor_peak, 3),
                    "form": "packed tiles, A in TMEM", "us_tiles_as_stored": round(t_smem * 1e3, 2)})
        del g, ws_, pk
        torch.cuda.empty_cache()
    return out


def graph_kernel_nodes(g) -> int | None:
    """Kernel nodes in a CUDA graph captured with keep_graph=True (cuda-python), else None."""
    try:
        from cuda.bindings import runtime as rt
        h = rt.cudaGraph_t(init_value=g.raw_cuda_graph())
        err, _, n = rt.cudaGraphGetNodes(h, 0)
        err, nodes, n = rt.cudaGraphGetNodes(h, n)
        kern = rt.cudaGraphNodeType.cudaGraphNodeTypeKernel
        return sum(1 for nd in nodes if rt.cudaGraphNodeGetType(nd)[1] == kern)
    except Exception:
        return None


def build_decoder(torch, world: int, rank: int, batch: int, ctx: int, seed: int = 11, cfg=None):
    """Config 4's decoder on this rank: decode.Q4Decoder on one GPU, else tp.TPDecoder on this
    rank's shard (every rank draws the same seeded full weights, then keeps its shard), with
    the peer exchanges."""
    from llmnputest_b200.decode import GRANITE_3B, Q4Decoder
    from llmnputest_b200.tp import ShardPlan, TPDecoder, shard_weights
    cfg = cfg or GRANITE_3B
    if world == 1:
        return Q4Decoder(cfg, batch, ctx, seed=seed)
    full = Q4Decoder(cfg, 1, 1, seed=seed)  # weights only; the KV cache lives in the TP decoder
    plan = ShardPlan(cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.hidden, cfg.intermediate, cfg.vocab, world, rank)
    dec = TPDecoder(cfg, batch, ctx, shard_weights(full.w, plan), plan)
    del full
    torch.cuda.empty_cache()
    return dec


def capture_step(torch, dec):
    """The decoder's step in one CUDA graph (kept, so its kernel nodes can be counted)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        dec.step()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph(keep_graph=True)
    with torch.cuda.graph(g):
        dec.step()
    return g


def step_bytes(cfg, batch: int, ctx: int) -> int:
    """Algorithmic HBM bytes of one config-4 step: every weight byte and every K/V byte once."""
    wb = cfg.weight_bytes()
    return wb["layers"] + wb["lm_head"] + batch * ctx * cfg.n_kv_heads * cfg.head_dim * 4 * cfg.n_layers


def _max_over_ranks(torch, world: int, v: float) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measure_decode(torch, world: int, rank: int, batch: int, ctx: int, steps: int, warmup: int) -> dict:
    """Config 4: the full 40-layer decode step at `batch` tokens, context `ctx`, TP over `world` ranks."""
    import torch.distributed as dist
    from llmnputest_b200.decode import GRANITE_3B as cfg
    dec = build_decoder(torch, world, rank, batch, ctx)
    dec.pos.fill_(ctx - 1)  # attend over the full context
    dec.x_in.normal_()
    g = capture_step(torch, dec)
    how = "tcgen05 GEMM, cuda graph" if getattr(dec, "use_gemm", False) else "GEMV, cuda graph"
    if world > 1:
        how += ", peer exchanges"
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        g.replay()
    b.record()
    b.synchronize()
    ms = _max_over_ranks(torch, world, a.elapsed_time(b) / steps)
    nbytes = step_bytes(cfg, batch, ctx)
    out = {"batch": batch, "ctx": ctx, "tp": world, "ms_per_step": round(ms, 4),
           "tok_s": round(batch / (ms * 1e-3), 1), "how": how,
           "hbm_gbs_per_gpu": round(nbytes / world / (ms * 1e-3) / 1e9, 1)}
    torch.cuda.synchronize()
    del g
    if hasattr(dec, "close"):
        dec.close()
    del dec
    torch.cuda.empty_cache()
    return out


def decode_kernel_split(torch, dec, hbm_peak: float, reps: int = 10) -> dict:
    """Time, with CUDA events, each kind of kernel of a decoder's step on its own buffers:
    the 40 layers' attention calls, and their projection launches by kind (one graph each,
    replayed `reps` times).  Algorithmic bytes per launch: attention the bf16 K/V read,
    projections their q4 tiles."""
    from llmnputest_b200 import ops
    c = dec.cfg
    d = c.head_dim
    p = getattr(dec, "plan", None)
    hq = p.q_local if p else c.n_heads
    hkv = p.kv_local if p else c.n_kv_heads
    qd, kd = hq * d, hkv * d
    n_l = len(dec.w["layers"])
    attn_out = dec.attn_local[:, :qd] if hasattr(dec, "attn_local") else dec.attn
    out = {}

    def timed(fn, nbytes, launches, name):
        g = graph_of(torch, fn)
        t_ms = time_graph(torch, g, reps, 2)
        del g
        us = t_ms * 1e3 / launches
        gbs = nbytes / launches / (us * 1e-6) / 1e9
        out[name] = {"launches_per_step": launches, "us_per_launch": round(us, 2), "bytes_per_launch": nbytes // launches,
                     "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / hbm_peak, 4),
                     "ms_per_step": round(t_ms, 4)}

    kv = dec.batch * dec.ctx_max * hkv * d * 4 * n_l
    timed(lambda: [ops.gqa_decode(dec.qkv[:, :qd], dec.qkv[:, qd:qd + kd], dec.qkv[:, qd + kd:], dec.k_cache[li],
                                  dec.v_cache[li], dec.pos, n_q_heads=hq, n_kv_heads=hkv, theta=c.rope_theta,
                                  scale=d ** -0.5, max_len=dec.ctx_max, out=attn_out,
                                  workspace=dec.attn_ws, prefetch_kv=True) for li in range(n_l)],
          kv, n_l, "gqa_decode")
    if getattr(dec, "use_gemm", False):
        ws = dec.gemm_ws
        kt_i = getattr(dec, "kt_i_local", dec.kt_i)
        nt_qkv = getattr(dec, "nt_qkv_local", getattr(dec, "nt_qkv", None))
        nt_i = getattr(dec, "nt_i_local", getattr(dec, "nt_i", None))
        tp = hasattr(dec, "o_part")  # tensor-parallel: O by input columns into fp32 partials
        kt_o = dec.kt_o_local if tp else dec.kt_q
        o_in = dec.attn_local if tp else dec.attn
        down_out = getattr(dec, "down", None)
        # the step's own calls: packed weights (A in TMEM), RMSNorm fused, weights prefetched
        L, G = dec.w["layers"], dec.wg
        pk = getattr(dec, "packed", True)
        qkv_b = sum(g["qkv"].numel() for g in G)
        timed(lambda: [ops.q4_gemm(g["qkv"], nt_qkv, dec.kt_h, dec.resid, out=dec.qkv, workspace=ws, prefetch=True,
                                   norm_w=l["attn_norm"], eps=c.rms_eps, packed=pk) for g, l in zip(G, L)],
              qkv_b, n_l, "q4_gemm_qkv")
        timed(lambda: [ops.q4_gemm(g["o"], c.hidden // 32, kt_o, o_in, out=dec.o_part if tp else dec.resid,
                                   accumulate=not tp, workspace=ws, prefetch=True, packed=pk) for g in G],
              sum(g["o"].numel() for g in G), n_l, "q4_gemm_o")
        if getattr(dec, "swiglu_split", False):
            # gate+up as one split-K GEMM, the SwiGLU in the down GEMM's x pre-pass
            timed(lambda: [ops.q4_gemm(g["gu"], 2 * nt_i, dec.kt_h, dec.resid, out=dec.gu, workspace=ws,
                                       prefetch=True, norm_w=l["mlp_norm"], eps=c.rms_eps, packed=pk)
                           for g, l in zip(G, L)], sum(g["gu"].numel() for g in G), n_l, "q4_gemm_gate_up")
            timed(lambda: [ops.q4_gemm(g["down"], c.hidden // 32, kt_i, dec.gu, out=down_out, workspace=ws,
                                       prefetch=True, packed=pk, swiglu_in=True) for g in G],
                  sum(g["down"].numel() for g in G), n_l, "q4_gemm_down_swiglu_in")
        else:
            timed(lambda: [ops.q4_swiglu_gemm(g["gate"], g["up"], nt_i, dec.kt_h, dec.resid, out=dec.h, workspace=ws,
                                              prefetch=True, norm_w=l["mlp_norm"], eps=c.rms_eps, packed=pk)
                           for g, l in zip(G, L)], sum(g["gate"].numel() + g["up"].numel() for g in G), n_l,
                  "q4_swiglu_gemm")
            timed(lambda: [ops.q4_gemm(g["down"], c.hidden // 32, kt_i, dec.h,
                                       out=down_out if down_out is not None else dec.resid,
                                       accumulate=down_out is None, workspace=ws, prefetch=True, packed=pk)
                           for g in G], sum(g["down"].numel() for g in G), n_l, "q4_gemm_down")
    # the lm_head (q8, RMSNorm fused) once per step: the q8 GEMM on the packed head at GEMM
    # batches, else the GEMV
    nt_v = getattr(dec, "nt_v_local", getattr(dec, "nt_v", None))
    lg = getattr(dec, "logits_local", dec.logits)
    lmp = getattr(dec, "lm_packed", None)
    if lmp is not None:
        timed(lambda: ops.q8_gemm(lmp, nt_v, dec.kt_h, dec.resid, out=lg, workspace=dec.gemm_ws, prefetch=True,
                                  norm_w=dec.w["final_norm"], eps=c.rms_eps), lmp.numel(), 1, "lm_head_q8_gemm")
    else:
        timed(lambda: ops.gemv_rmsnorm(dec.w["lm_head"], nt_v, dec.kt_h, dec.resid, dec.w["final_norm"], c.rms_eps,
                                       out=lg, q8=True), dec.w["lm_head"].numel(), 1, "lm_head_q8")
    return out


PROFILE_CASES = ("attention_b32", "swiglu_b32", "lm_head_b32", "step_b32")


def profile_case(torch, name: str) -> None:
    """One small workload for an ncu capture (`--profile-case`), a few launches of it:
      attention_b32  one config-4 layer's GQA attention, batch 32, ctx 4096 (268 MB of K/V), 4 calls
      swiglu_b32     config-4 gate+up SwiGLU then down GEMMs, batch 32, packed, 8 layers' weights, x2
      lm_head_b32    config-4 q8 lm_head GEMM (100352 x 2560, packed), batch 32, 4 calls
      step_b32       the config-4 batch-32 decode step (one CUDA graph), 3 replays
    Prints "ok" after checking the device error word."""
    from llmnputest_b200 import ops
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    if name == "attention_b32":
        B, H, HKV, D, CTX = 32, 40, 8, 64, HEAD_CTX
        qkv = torch.randn(B, (H + 2 * HKV) * D, device=dev, generator=gen)
        kc = torch.randn(B, HKV, CTX, D, device=dev, generator=gen).to(torch.bfloat16)
        vc = torch.randn(B, HKV, CTX, D, device=dev, generator=gen).to(torch.bfloat16)
        pos = torch.full((B,), CTX - 1, dtype=torch.int32, device=dev)
        out = torch.empty(B, H * D, device=dev, dtype=torch.bfloat16)
        ws = torch.empty(max(ops.gqa_decode_workspace_bytes(B, H, HKV, D, CTX), 16), dtype=torch.uint8, device=dev)
        qd, kd = H * D, HKV * D
        for _ in range(4):
            ops.gqa_decode(qkv[:, :qd], qkv[:, qd:qd + kd], qkv[:, qd + kd:], kc, vc, pos, n_q_heads=H,
                           n_kv_heads=HKV, theta=10000.0, scale=D ** -0.5, max_len=CTX, out=out, workspace=ws,
                           prefetch_kv=True)
    elif name == "swiglu_b32":
        B = 32
        resid = torch.randn(B, 2560, device=dev, generator=gen)
        norm = (torch.randn(2560, device=dev, generator=gen) * 0.1 + 1).to(torch.bfloat16)
        h = torch.randn(B, 8192, device=dev, generator=gen).to(torch.bfloat16)
        ws = torch.empty(64 << 20, device=dev, dtype=torch.uint8)
        W = [{k: ops.q4_gemm_pack(make_q4_tiles(torch, n * kt, gen, dev), n, kt)
              for k, n, kt in (("gate", 256, 10), ("up", 256, 10), ("down", 80, 32))} for _ in range(8)]
        for _ in range(2):
            for L in W:
                ops.q4_swiglu_gemm(L["gate"], L["up"], 256, 10, resid, out=h, workspace=ws, norm_w=norm, eps=1e-5,
                                   prefetch=True, packed=True)
                ops.q4_gemm(L["down"], 80, 32, h, out=resid, accumulate=True, workspace=ws, prefetch=True,
                            packed=True)
    elif name == "lm_head_b32":
        pk = ops.q8_gemm_pack(make_q8_tiles(torch, 3136 * 10, gen, dev), 3136, 10)
        resid = torch.randn(32, 2560, device=dev, generator=gen)
        norm = (torch.randn(2560, device=dev, generator=gen) * 0.1 + 1).to(torch.bfloat16)
        out = torch.empty(32, 100352, device=dev)
        for _ in range(4):
            ops.q8_gemm(pk, 3136, 10, resid, out=out, prefetch=True, norm_w=norm, eps=1e-5)
    elif name == "step_b32":
        dec = build_decoder(torch, 1, 0, 32, HEAD_CTX)
        dec.pos.fill_(HEAD_CTX - 1)
        dec.x_in.normal_()
        g = capture_step(torch, dec)
        for _ in range(3):
            g.replay()
    else:
        raise ValueError(f"unknown profile case {name!r}: {PROFILE_CASES}")
    torch.cuda.synchronize()
    assert ops.device_error() == 0, "a kernel recorded a device-side error"
    print("ok")


def measure_headline(torch, world: int, rank: int, batch: int, ctx: int, steps: int, warmup: int,
                     hbm_peak: float) -> dict:
    """The bench line's value: config 4's decode step (tokens/s over all ranks), K timed graph
    replays between a barrier and a synchronize on both sides, max over ranks, clocks sampled
    during the timed region; then the same step end to end with host buffers (the step's input
    rows and positions copied in, its logits copied out, inside the timed region); then the
    per-kernel split that names the dominant kernel."""
    import torch.distributed as dist
    from llmnputest_b200.decode import GRANITE_3B as cfg
    dec = build_decoder(torch, world, rank, batch, ctx)
    dec.pos.fill_(ctx - 1)
    dec.x_in.normal_()
    g = capture_step(torch, dec)
    kernels_per_step = graph_kernel_nodes(g)
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(gpu_uuid(torch)) as clk:
        time.sleep(0.15)  # let the sampler start
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            g.replay()
        b.record()
        b.synchronize()
    ms = _max_over_ranks(torch, world, a.elapsed_time(b) / steps)
    # end to end: the step's inputs from pinned host memory, its logits back, every step
    x_host = torch.randn(batch, cfg.hidden).pin_memory()
    pos_host = torch.full((batch,), ctx - 1, dtype=torch.int32).pin_memory()
    logits_host = torch.empty(batch, cfg.vocab).pin_memory()

    def e2e_step():
        dec.x_in.copy_(x_host, non_blocking=True)
        dec.pos.copy_(pos_host, non_blocking=True)
        g.replay()
        logits_host.copy_(dec.logits, non_blocking=True)

    for _ in range(max(2, warmup // 2)):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_steps = max(5, steps // 2)
    a.record()
    for _ in range(e2e_steps):
        e2e_step()
    b.record()
    b.synchronize()
    e2e_ms = _max_over_ranks(torch, world, a.elapsed_time(b) / e2e_steps)
    del g
    torch.cuda.synchronize()
    split = decode_kernel_split(torch, dec, hbm_peak)
    if hasattr(dec, "close"):
        dec.close()
    del dec
    torch.cuda.empty_cache()
    nbytes = step_bytes(cfg, batch, ctx)
    return {"ms": ms, "tok_s": batch / (ms * 1e-3), "e2e_ms": e2e_ms, "e2e_tok_s": batch / (e2e_ms * 1e-3),
            "h2d": x_host.numel() * 4 + pos_host.numel() * 4, "d2h": logits_host.numel() * 4,
            "kernels_per_step": kernels_per_step, "bytes_per_step": nbytes, "clocks": clk.summary(),
            "split": split}


def _compare(torch, got, ref) -> tuple[float, float]:
    """(cosine, max rel err) in float64 over every token, as the tests measure."""
    g, r = got.double().flatten(), ref.double().flatten()
    cos = float((g @ r) / (g.norm() * r.norm() + 1e-30))
    rel = float((g - r).abs().max() / (r.abs().max() + 1e-30))
    return cos, rel


def tp_parity(torch, world: int, rank: int) -> dict:
    """Before the timed region at N > 1: the tensor-parallel steps against the one-GPU steps
    on the same weights, two steps each (every rank draws the same seeded full weights and
    cache history and keeps its shard; rank 0 also runs the one-GPU decoder and compares the
    full logits, every token, float64; the worst step is reported).
      config 4: 2 layers of the 3B's real widths (vocab 100352), batch 1 (GEMVs) and 32
                (tcgen05 GEMMs), peer exchanges, ctx 256 with a random history;
      config 5: one gated DeltaNet and one gated attention layer of config 5's widths
                (vocab 248320, the logits gathered), batch 1 and 256, from zero states."""
    import torch.distributed as dist
    from llmnputest_b200.decode import DecoderConfig, Q4Decoder
    from llmnputest_b200.qwen35_decode import Qwen35Config, Qwen35Decoder
    from llmnputest_b200.tp import ShardPlan, TPDecoder, shard_weights
    from llmnputest_b200.tp_qwen35 import Qwen35ShardPlan, TPQwen35Decoder, shard_qwen35
    out = {"config4": {}, "config5": {}}
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = DecoderConfig(n_layers=2)
    ctx = 256
    for bsz in (1, 32):
        try:
            full = Q4Decoder(cfg, 1, 1, seed=23)
            plan = ShardPlan(cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.hidden, cfg.intermediate, cfg.vocab,
                             world, rank)
            tp = TPDecoder(cfg, bsz, ctx, shard_weights(full.w, plan), plan)
            one = Q4Decoder(cfg, bsz, ctx, weights=full.w) if rank == 0 else None
            gen = torch.Generator(device=dev)
            gen.manual_seed(5)
            h0 = rank * plan.kv_local
            for li in range(cfg.n_layers):
                kc = torch.randn(bsz, cfg.n_kv_heads, ctx, cfg.head_dim, device=dev, generator=gen).to(torch.bfloat16)
                vc = torch.randn(bsz, cfg.n_kv_heads, ctx, cfg.head_dim, device=dev, generator=gen).to(torch.bfloat16)
                tp.k_cache[li].copy_(kc[:, h0:h0 + plan.kv_local])
                tp.v_cache[li].copy_(vc[:, h0:h0 + plan.kv_local])
                if one is not None:
                    one.k_cache[li].copy_(kc)
                    one.v_cache[li].copy_(vc)
            g = tp.capture()
            worst = (1.0, 0.0)
            pos = (torch.arange(bsz, dtype=torch.int32, device=dev) * 7 + 100) % (ctx - 4)
            for _ in range(2):
                x = torch.randn(bsz, cfg.hidden, device=dev, generator=gen)
                tp.x_in.copy_(x)
                tp.pos.copy_(pos)
                g.replay()
                if one is not None:
                    one.x_in.copy_(x)
                    one.pos.copy_(pos)
                    ref = one.step()
                    cos, rel = _compare(torch, tp.logits, ref)
                    worst = (min(worst[0], cos), max(worst[1], rel))
                pos = pos + 1
                torch.cuda.synchronize()
                dist.barrier()  # rank 0's extra work stays on the host side of the next exchange
            torch.cuda.synchronize()
            dist.barrier()
            del g
            tp.close()
            out["config4"][f"b{bsz}"] = {"cos": round(worst[0], 9), "rel": float(f"{worst[1]:.3e}"),
                                         "how": "tcgen05 GEMM" if tp.use_gemm else "GEMV",
                                         "mlp": "split (gate+up GEMM, SwiGLU in the down pre-pass)"
                                         if tp.swiglu_split else "fused SwiGLU"} if rank == 0 else None
            del tp, one, full
            torch.cuda.empty_cache()
        except Exception as e:  # recorded in the line; every rank raises alike or the barrier times out
            out["config4"][f"b{bsz}"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    cfg5 = Qwen35Config(n_layers=2, layer_types=("linear_attention", "full_attention"))
    for bsz in (1, 256):
        try:
            full = Qwen35Decoder(cfg5, 1, 1, seed=29)
            plan5 = Qwen35ShardPlan(cfg5, world, rank)
            tp = TPQwen35Decoder(cfg5, bsz, 64, shard_qwen35(full.w, plan5), plan5)
            one = Qwen35Decoder(cfg5, bsz, 64, weights=full.w) if rank == 0 else None
            gen = torch.Generator(device=dev)
            gen.manual_seed(6)
            worst = (1.0, 0.0)
            for step in range(2):
                x = torch.randn(bsz, cfg5.hidden, device=dev, generator=gen)
                tp.x_in.copy_(x)
                tp.pos.fill_(step)
                got = tp.step()
                if one is not None:
                    one.x_in.copy_(x)
                    one.pos.fill_(step)
                    cos, rel = _compare(torch, got, one.step())
                    worst = (min(worst[0], cos), max(worst[1], rel))
            torch.cuda.synchronize()
            dist.barrier()
            out["config5"][f"b{bsz}"] = {"cos": round(worst[0], 9), "rel": float(f"{worst[1]:.3e}"),
                                         "how": "tcgen05 GEMM" if tp.use_gemm else "GEMV",
                                         "attention": "kv-head shards" if plan5.attn() is not None
                                         else "replicated (2 kv heads)"} if rank == 0 else None
            del tp, one, full
            torch.cuda.empty_cache()
        except Exception as e:
            out["config5"][f"b{bsz}"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    return out


def measure_qwen35_tp(torch, world: int, rank: int, steps: int, warmup: int) -> list:
    """Config 5 on `world` GPUs (tp_qwen35.TPQwen35Decoder: DeltaNet by k head, attention by kv
    head or replicated, MLP by down K-tiles, the q8 lm_head by vocab rows with the fp32 logits
    all-gathered), ctx 2048, batch 1 and 256, one CUDA graph per step, max over ranks.  The
    lm_head and the logits all-gather are also timed alone, each in its own graph."""
    import torch.distributed as dist
    from llmnputest_b200 import ops
    from llmnputest_b200.qwen35_decode import Qwen35Config, Qwen35Decoder
    from llmnputest_b200.tp_qwen35 import Qwen35ShardPlan, TPQwen35Decoder, shard_qwen35
    out = []
    cfg = Qwen35Config()
    try:
        full = Qwen35Decoder(cfg, 1, 1, seed=11)
        plan = Qwen35ShardPlan(cfg, world, rank)
        shard = shard_qwen35(full.w, plan)
        del full
        torch.cuda.empty_cache()
        for bsz in (1, 256):
            dec = TPQwen35Decoder(cfg, bsz, GATED_CTX, shard, plan)
            dec.pos.fill_(GATED_CTX - 1)
            dec.x_in.normal_()
            g = graph_of(torch, dec.step)
            for _ in range(warmup):
                g.replay()
            torch.cuda.synchronize()
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n = max(5, steps // 2)
            a.record()
            for _ in range(n):
                g.replay()
            b.record()
            b.synchronize()
            ms = _max_over_ranks(torch, world, a.elapsed_time(b) / n)
            del g
            # the lm_head alone (the q8 GEMM on the packed shard at GEMM batches, else the
            # GEMV), and the logits all-gather alone
            if dec.use_gemm:
                gl = graph_of(torch, lambda: ops.q8_gemm(dec.lm_packed, dec.nt_v_local, dec.kt_h, dec.resid,
                                                          out=dec.logits_local, workspace=dec.gemm_ws, prefetch=True,
                                                          norm_w=dec.w["final_norm"], eps=cfg.eps))
            else:
                gl = graph_of(torch, lambda: ops.gemv_rmsnorm(dec.w["lm_head"], dec.nt_v_local, dec.kt_h, dec.resid,
                                                               dec.w["final_norm"], cfg.eps, out=dec.logits_local,
                                                               prefetch=True, q8=True))
            dist.barrier()
            t_lm = _max_over_ranks(torch, world, time_graph(torch, gl, 10, 2))
            del gl
            ga = graph_of(torch, lambda: dist.all_gather_into_tensor(dec.logits_all, dec.logits_local))
            dist.barrier()
            t_ag = _max_over_ranks(torch, world, time_graph(torch, ga, 10, 2))
            del ga
            torch.cuda.synchronize()
            dist.barrier()
            out.append({"batch": bsz, "ctx": GATED_CTX, "tp": world, "ms_per_step": round(ms, 4),
                        "tok_s": round(bsz / (ms * 1e-3), 1), "lm_head_ms": round(t_lm, 4),
                        "lm_head_how": "q8 tcgen05 GEMM" if dec.use_gemm else "q8 GEMV",
                        "logits_all_gather_ms": round(t_ag, 4),
                        "logits_all_gather_mb": round(bsz * cfg.vocab * 4 / 1e6, 1),
                        "how": ("tcgen05 GEMM" if dec.use_gemm else "GEMV") + ", cuda graph, NCCL collectives",
                        "attention": "kv-head shards" if plan.attn() is not None else "replicated (2 kv heads)"})
            del dec
            torch.cuda.empty_cache()
    except Exception as e:
        out.append({"error": f"{type(e).__name__}: {str(e)[:300]}"})
    return out


def measure_attention(torch, ops, gen, device, hbm_peak: float, steps: int) -> list:
    """Config 3: GQA flash-decode (40/8 heads, D 64, RoPE fused, new k/v appended at pos = ctx-1).

    Algorithmic bytes per call: B*ctx*8*64*2*2 (the bf16 K and V read once).  Each graph
    replay rotates over a pool of caches whose total is above L2, so every call reads HBM.
    Calls use B2_ATTN_PREFETCH_KV as the decoders do: pos is constant and a call writes
    only row pos of its cache, so rows before pos are final when the next call launches.
    """
    hq, hkv, d = 40, 8, 64
    out = []
    for ctx in (512, 4096, 32768):
        for bsz in (1, 16, 64):
            kv_bytes = bsz * ctx * hkv * d * 2 * 2
            n_pool = max(1, min(512, -(-300_000_000 // kv_bytes)))
            pool = []
            for _ in range(n_pool):
                kc = torch.randn(bsz, hkv, ctx, d, device=device, generator=gen).to(torch.bfloat16)
                vc = torch.randn(bsz, hkv, ctx, d, device=device, generator=gen).to(torch.bfloat16)
                pool.append((kc, vc))
            qkv = torch.randn(bsz, (hq + 2 * hkv) * d, device=device, generator=gen)
            pos = torch.full((bsz,), ctx - 1, dtype=torch.int32, device=device)
            o = torch.empty(bsz, hq * d, dtype=torch.bfloat16, device=device)
            ws = torch.empty(max(1, ops.gqa_decode_workspace_bytes(bsz, hq, hkv, d, ctx)), dtype=torch.uint8,
                             device=device)

            def calls(pool=pool, qkv=qkv, pos=pos, o=o, ws=ws, ctx=ctx):
                for kc, vc in pool:
                    ops.gqa_decode(qkv[:, :hq * d], qkv[:, hq * d:(hq + hkv) * d], qkv[:, (hq + hkv) * d:], kc, vc,
                                   pos, n_q_heads=hq, n_kv_heads=hkv, max_len=ctx, out=o, workspace=ws,
                                   prefetch_kv=True)

            g = graph_of(torch, calls)
            reps = max(3, min(200, int(steps * 2e6 / (kv_bytes * n_pool) + 1)))
            t_ms = time_graph(torch, g, reps, 3) / n_pool
            gbs = kv_bytes / (t_ms * 1e-3) / 1e9
            out.append({"batch": bsz, "ctx": ctx, "us": round(t_ms * 1e3, 2), "gbs": round(gbs, 1),
                        "frac_of_measured_hbm": round(gbs / hbm_peak, 3), "pool": n_pool})
            del g, pool, ws
            torch.cuda.empty_cache()
    return out


DELTA_KH, DELTA_VH, DELTA_D = 16, 16, 128  # config 5's linear-attention heads (synthetic dims)


def delta_bytes(bsz: int) -> int:
    """Algorithmic bytes of one gated DeltaNet decode step: the fp32 recurrent state and
    conv state read and written, the fp32 qkv / z / b / a read, the bf16 output written."""
    conv_dim = (2 * DELTA_KH + DELTA_VH) * DELTA_D
    per_seq = (DELTA_VH * DELTA_D * DELTA_D * 4 * 2 + conv_dim * 16 * 2 + conv_dim * 4
               + DELTA_VH * DELTA_D * 4 + DELTA_VH * 8 + DELTA_VH * DELTA_D * 2)
    return bsz * per_seq + conv_dim * 16 + DELTA_VH * 8 + DELTA_D * 4


def measure_deltanet(torch, ops, gen, device, hbm_peak: float, steps: int) -> list:
    """Config 5's linear-attention layers: one fused gated DeltaNet decode step
    (16 k / 16 v heads of 128, conv width 4) at batch 1, 16 and 256.  Each graph
    replay rotates over a pool of recurrent states whose total is above L2; a call
    reads its state before the PDL wait (B2_DELTA_PREFETCH_STATE): a pool entry's
    state was last written one replay earlier."""
    conv_dim = (2 * DELTA_KH + DELTA_VH) * DELTA_D
    out = []
    for bsz in (1, 16, 256):
        nbytes = delta_bytes(bsz)
        n_pool = max(1, min(512, -(-300_000_000 // nbytes)))
        pool = [(0.1 * torch.randn(bsz, DELTA_VH, DELTA_D, DELTA_D, device=device, generator=gen),
                 torch.randn(bsz, conv_dim, 4, device=device, generator=gen)) for _ in range(n_pool)]
        proj = torch.randn(bsz, conv_dim + DELTA_VH * DELTA_D + 2 * DELTA_VH, device=device, generator=gen)
        c0, c1 = conv_dim, conv_dim + DELTA_VH * DELTA_D
        conv_w = 0.5 * torch.randn(conv_dim, 4, device=device, generator=gen)
        a_log = torch.log(torch.rand(DELTA_VH, device=device, generator=gen) * 15 + 1)
        dt_bias = torch.randn(DELTA_VH, device=device, generator=gen)
        norm_w = 1 + 0.1 * torch.randn(DELTA_D, device=device, generator=gen)
        o = torch.empty(bsz, DELTA_VH * DELTA_D, dtype=torch.bfloat16, device=device)

        def calls(pool=pool, proj=proj, o=o):
            for st, cs in pool:
                ops.gated_delta_step(proj[:, :c0], proj[:, c0:c1], proj[:, c1:c1 + DELTA_VH],
                                     proj[:, c1 + DELTA_VH:], cs, conv_w, a_log, dt_bias, norm_w, st,
                                     DELTA_KH, DELTA_VH, out=o, prefetch_state=True)

        g = graph_of(torch, calls)
        reps = max(3, min(200, int(steps * 2e6 / (nbytes * n_pool) + 1)))
        t_ms = time_graph(torch, g, reps, 3) / n_pool
        gbs = nbytes / (t_ms * 1e-3) / 1e9
        out.append({"batch": bsz, "heads": f"{DELTA_KH}k/{DELTA_VH}v x {DELTA_D}", "us": round(t_ms * 1e3, 2),
                    "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / hbm_peak, 3), "pool": n_pool})
        del g, pool
        torch.cuda.empty_cache()
    return out


def measure_deltanet_layers(torch, device, hbm_peak: float, steps: int, n_layers: int = 18) -> list:
    """Config 5's 18 linear-attention layers as one graph: per layer input RMSNorm, the
    fused q4 in_proj (q|k|v|z|b|a, 8224 rows x 1024), the gated DeltaNet step and the q4
    out_proj (1024 x 2048) added into the residual (llmnputest_b200.deltanet), at batch
    1 (GEMV) and 256 (tcgen05 GEMM).  Each layer's states were last written one graph
    replay earlier, so its step reads them before its PDL wait."""
    from llmnputest_b200.deltanet import DeltaNetLayer
    out = []
    for bsz in (1, 256):
        layers = [DeltaNetLayer(1024, DELTA_KH, DELTA_VH, bsz, device=device, seed=50 + i) for i in range(n_layers)]
        resid = torch.randn(bsz, 1024, device=device)

        def chain(layers=layers, resid=resid):
            for layer in layers:
                layer.step(resid, prefetch_state=True)

        g = graph_of(torch, chain)
        nbytes = sum(layer.bytes_per_step() for layer in layers)
        reps = max(5, min(100, int(steps * 4e6 / nbytes + 1)))
        t_ms = time_graph(torch, g, reps, 3)
        gbs = nbytes / (t_ms * 1e-3) / 1e9
        out.append({"batch": bsz, "layers": n_layers, "ms": round(t_ms, 4), "gbs": round(gbs, 1),
                    "frac_of_measured_hbm": round(gbs / hbm_peak, 3), "bytes_per_step": nbytes,
                    "how": "tcgen05 GEMM" if layers[0].use_gemm else "GEMV (RMSNorm fused)",
                    "us_per_layer": round(t_ms * 1e3 / n_layers, 2),
                    # the reference's CPU path for the same layer (transformers, float32), beside it
                    "cpu_reference": cpu_reference_qwen35("linear_attention", bsz)})
        del g, layers
        torch.cuda.empty_cache()
    return out


GATED_Q, GATED_KV, GATED_D, GATED_CTX = 8, 2, 256, 2048  # config 5's gated full-attention layers


def measure_gated_attention(torch, ops, gen, device, hbm_peak: float, steps: int) -> list:
    """Config 5's gated full-attention decode (8 q / 2 kv heads, head_dim 256, q/k RMSNorm,
    partial RoPE over 64 dims, sigmoid output gate) at ctx 2048, pos 2047.  Algorithmic bytes
    per call: B*2*2048*256*2*2 (the bf16 K and V read once).  Each graph replay rotates over
    a pool of caches whose total is above L2."""
    out = []
    inv_freq = (1.0 / (10000.0 ** (torch.arange(0, 64, 2, device=device).float() / 64))).contiguous()
    qn = 0.1 * torch.randn(GATED_D, device=device, generator=gen)
    kn = 0.1 * torch.randn(GATED_D, device=device, generator=gen)
    for bsz in (1, 16, 256):
        kv_bytes = bsz * GATED_KV * GATED_CTX * GATED_D * 2 * 2
        n_pool = max(1, min(512, -(-300_000_000 // kv_bytes)))
        pool = [(torch.randn(bsz, GATED_KV, GATED_CTX, GATED_D, device=device, generator=gen).to(torch.bfloat16),
                 torch.randn(bsz, GATED_KV, GATED_CTX, GATED_D, device=device, generator=gen).to(torch.bfloat16))
                for _ in range(n_pool)]
        proj = torch.randn(bsz, (2 * GATED_Q + 2 * GATED_KV) * GATED_D, device=device, generator=gen)
        c0, c1 = 2 * GATED_Q * GATED_D, (2 * GATED_Q + GATED_KV) * GATED_D
        pos = torch.full((bsz,), GATED_CTX - 1, dtype=torch.int32, device=device)
        o = torch.empty(bsz, GATED_Q * GATED_D, dtype=torch.bfloat16, device=device)
        ws_n = ops.gated_attn_workspace_bytes(bsz, GATED_Q, GATED_KV, GATED_CTX)
        ws = torch.empty(max(ws_n, 16), dtype=torch.uint8, device=device)

        def calls(pool=pool, proj=proj, pos=pos, o=o, ws=ws):
            for kc, vc in pool:
                ops.gated_attn_decode(proj[:, :c0], proj[:, c0:c1], proj[:, c1:], qn, kn, inv_freq, kc, vc, pos,
                                      GATED_Q, GATED_KV, out=o, workspace=ws)

        g = graph_of(torch, calls)
        reps = max(3, min(200, int(steps * 2e6 / (kv_bytes * n_pool) + 1)))
        t_ms = time_graph(torch, g, reps, 3) / n_pool
        gbs = kv_bytes / (t_ms * 1e-3) / 1e9
        row = {"batch": bsz, "ctx": GATED_CTX, "heads": "8q/2kv x 256", "us": round(t_ms * 1e3, 2),
               "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / hbm_peak, 3), "pool": n_pool}
        if bsz <= 16:  # the reference's CPU path (transformers, float32; a whole layer: projections included)
            row["cpu_reference"] = cpu_reference_qwen35("full_attention", bsz)
        out.append(row)
        del g, pool, ws
        torch.cuda.empty_cache()
    return out


def measure_qwen35_step(torch, device, hbm_peak: float, steps: int) -> list:
    """Config 5 as one decode step (llmnputest_b200.qwen35_decode.Qwen35Decoder: 18 gated
    DeltaNet + 6 gated attention layers of hidden 1024, SwiGLU MLPs of 3584, the q8
    lm_head 248320 x 1024) at ctx 2048 (pos 2047), batch 1 (GEMVs) and 256 (tcgen05 GEMMs;
    the lm_head GEMV in passes of 16 tokens), one CUDA graph per step.  Algorithmic bytes:
    every weight tile once, the DeltaNet states read and written, each attention layer's
    bf16 K/V read.  Measured last: an exception is recorded instead of a number."""
    from llmnputest_b200 import ops
    from llmnputest_b200.qwen35_decode import Qwen35Config, Qwen35Decoder
    out = []
    try:
        cfg = Qwen35Config()
        for bsz in (1, 256):
            dec = Qwen35Decoder(cfg, bsz, GATED_CTX, device=device, seed=11)
            dec.pos.fill_(GATED_CTX - 1)
            dec.x_in.normal_()
            nbytes = dec.w["lm_head"].numel()
            for m, L in zip(dec.mixers, dec.w["layers"]):
                nbytes += L["gate"].numel() + L["up"].numel() + L["down"].numel()
                if hasattr(m, "state"):  # DeltaNetLayer: its weights, states, projection, residual
                    nbytes += m.bytes_per_step()
                else:
                    nbytes += (m.w["in_proj"].numel() + m.w["o_proj"].numel()
                               + bsz * cfg.n_kv_heads * GATED_CTX * GATED_D * 2 * 2)
            g = graph_of(torch, dec.step)
            t_ms = time_graph(torch, g, max(5, min(50, steps // 4)), 3)
            gbs = nbytes / (t_ms * 1e-3) / 1e9
            out.append({"batch": bsz, "ctx": GATED_CTX, "ms_per_step": round(t_ms, 4),
                        "tok_s": round(bsz / (t_ms * 1e-3), 1), "gbs": round(gbs, 1),
                        "frac_of_measured_hbm": round(gbs / hbm_peak, 3), "bytes_per_step": nbytes,
                        "how": "tcgen05 GEMM, cuda graph" if dec.use_gemm else "GEMV, cuda graph"})
            del g, dec
            torch.cuda.empty_cache()
        if ops.device_error() != 0:
            out.append({"error": "a kernel recorded a device-side error"})
    except Exception as e:  # recorded, so the rest of the line stands
        out.append({"error": f"{type(e).__name__}: {str(e)[:300]}"})
    return out


def cpu_reference_qwen35(kind: str, bsz: int, ctx: int = GATED_CTX, steps: int = 3) -> dict:
    """The reference's own CPU path for a config-5 layer: transformers 5.5.0's module
    (Qwen3_5GatedDeltaNet or Qwen3_5Attention, float32, as reference/from_q4nx.py:140-171
    builds the model) stepping one decode token with a filled cache, on all host threads.
    Returns {"us_per_layer", "threads", "sample"} or {"error"}."""
    saved = {}
    try:
        import torch
        from transformers.cache_utils import DynamicCache
        from transformers.models.qwen3_5 import configuration_qwen3_5 as conf
        from transformers.models.qwen3_5 import modeling_qwen3_5 as mq
        # With a GPU present transformers binds flash-linear-attention's Triton kernels (and
        # causal-conv1d's), which cannot take CPU tensors: the CPU path is the module's
        # torch implementation, so its fast-path hooks are cleared while it is built.
        for name in ("FusedRMSNormGated", "chunk_gated_delta_rule", "fused_recurrent_gated_delta_rule",
                     "causal_conv1d_fn", "causal_conv1d_update"):
            if hasattr(mq, name):
                saved[name] = getattr(mq, name)
                setattr(mq, name, None)
        torch.manual_seed(0)
        linear = kind == "linear_attention"
        cfg = conf.Qwen3_5TextConfig(
            hidden_size=1024, num_hidden_layers=1, layer_types=[kind], linear_num_key_heads=DELTA_KH,
            linear_num_value_heads=DELTA_VH, linear_key_head_dim=DELTA_D, linear_value_head_dim=DELTA_D,
            num_attention_heads=GATED_Q, num_key_value_heads=GATED_KV, head_dim=GATED_D,
            rope_parameters={"rope_type": "default", "rope_theta": 1e7, "partial_rotary_factor": 0.25})
        cfg._attn_implementation = "eager"
        cache = DynamicCache(config=cfg)
        with torch.no_grad():
            if linear:
                mod = mq.Qwen3_5GatedDeltaNet(cfg, 0).float().eval()
                mod(torch.randn(bsz, 2, 1024), cache_params=cache)  # creates the conv / recurrent states
                run = lambda: mod(torch.randn(bsz, 1, 1024), cache_params=cache)
            else:
                mod = mq.Qwen3_5Attention(cfg, 0).float().eval()
                rope = mq.Qwen3_5TextRotaryEmbedding(cfg)
                layer = cache.layers[0]
                layer.lazy_initialization(torch.zeros(bsz, GATED_KV, 1, GATED_D), torch.zeros(bsz, GATED_KV, 1, GATED_D))
                layer.keys = torch.randn(bsz, GATED_KV, ctx - 1, GATED_D)
                layer.values = torch.randn(bsz, GATED_KV, ctx - 1, GATED_D)
                pos = torch.full((bsz, 1), ctx - 1)

                def run():
                    h = torch.randn(bsz, 1, 1024)
                    out = mod(h, rope(h, pos), None, past_key_values=cache)
                    layer.keys, layer.values = layer.keys[:, :, :ctx - 1], layer.values[:, :, :ctx - 1]
                    return out
            run()
            t0 = time.perf_counter()
            for _ in range(steps):
                run()
            dt = (time.perf_counter() - t0) / steps
        return {"us_per_layer": round(dt * 1e6, 1), "threads": torch.get_num_threads(), "cores": os.cpu_count(),
                "sample": f"transformers {kind} module (its torch implementation), float32, batch {bsz}"
                          + ("" if linear else f", ctx {ctx}") + f", {steps} decode steps"}
    except Exception as e:
        return {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    finally:
        if saved:
            from transformers.models.qwen3_5 import modeling_qwen3_5 as mq
            for name, v in saved.items():
                setattr(mq, name, v)


def gemv_sweep(torch, ops, args, rank: int, world: int, gen, device, pk: dict) -> dict:
    """Config 2: the q4nx W4A16 GEMV sweep -- the 160 GEMVs of a 40-layer 3B step's weight
    stream (QKV, O, gate+up, down; 1.966 GB, above L2) at batch 1 from one CUDA graph with
    PDL, K replays timed with CUDA events (max over ranks; at N > 1 every rank streams its
    own copy, weak scaling).  Also, on rank 0 of one GPU: GB/s per shape, batch 8, and the
    sweep end to end with host buffers."""
    import torch.distributed as dist
    calls, nbytes = build_sweep(torch, ops, 1, args.layers, gen, device)

    def sweep():
        for _, w, n_t, k_t, x, y in calls:
            ops.q4_gemv(w, n_t, k_t, x, out=y, prefetch=True)

    g = graph_of(torch, sweep)
    steps = max(20, args.steps)
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        g.replay()
    b.record()
    b.synchronize()
    ms = _max_over_ranks(torch, world, a.elapsed_time(b) / steps)
    per_gpu = nbytes / (ms * 1e-3) / 1e9
    out = {"gbs": round(world * per_gpu, 1), "gbs_per_gpu": round(per_gpu, 1),
           "frac_of_measured_hbm": round(per_gpu / pk["hbm_gbs"], 4), "ms_per_step": round(ms, 4),
           "launches_per_step": len(calls), "bytes_per_step_per_gpu": nbytes, "batch": 1, "layers": args.layers,
           "kernel": "q4nx_gemv_kernel<q4,NB=1,f32>",
           "traffic_per_launch": int(nbytes / len(calls) * GEMV_DRAM_RATIO),
           "parallelism": f"replicas x{world} (each rank streams its own weights, no collective)"}
    if rank == 0 and world == 1 and not args.quick:
        per_shape = {}
        for name, n_t, k_t in SHAPES:
            sub = [c for c in calls if c[0] == name]
            gs = graph_of(torch, lambda sub=sub: [ops.q4_gemv(w, n, k, x, out=y, prefetch=True)
                                                  for _, w, n, k, x, y in sub])
            t_ms = time_graph(torch, gs, max(20, args.steps // 10), 3)
            per_shape[name] = round(sum(c[1].numel() for c in sub) / (t_ms * 1e-3) / 1e9, 1)
            del gs
        out["per_shape_gbs_b1"] = per_shape
        calls8 = [(n, w, nt, kt, torch.randn(8, kt * 256, device=device, generator=gen).to(torch.bfloat16),
                   torch.empty(8, nt * 32, device=device)) for n, w, nt, kt, _, _ in calls]
        g8 = graph_of(torch, lambda: [ops.q4_gemv(w, n, k, x, out=y, prefetch=True) for _, w, n, k, x, y in calls8])
        t8 = time_graph(torch, g8, max(20, args.steps // 10), 3)
        out["batch8_gbs"] = round(nbytes / (t8 * 1e-3) / 1e9, 1)
        del g8, calls8
        # end to end: every call's x from pinned host memory, every y back, inside the timed region
        xs_host = torch.cat([c[4].reshape(-1) for c in calls]).cpu().pin_memory()
        ys_host = torch.empty(sum(c[5].numel() for c in calls), dtype=torch.float32).pin_memory()
        x_dev = torch.empty_like(xs_host, device=device)
        y_dev = torch.empty(ys_host.numel(), dtype=torch.float32, device=device)
        views, off_x, off_y = [], 0, 0
        for _, w, n_t, k_t, x, y in calls:
            views.append((w, n_t, k_t, x_dev[off_x:off_x + x.numel()].view(x.shape),
                          y_dev[off_y:off_y + y.numel()].view(y.shape)))
            off_x += x.numel()
            off_y += y.numel()
        ge = graph_of(torch, lambda: [ops.q4_gemv(w, n, k, x, out=y, prefetch=True) for w, n, k, x, y in views])

        def e2e_step():
            x_dev.copy_(xs_host, non_blocking=True)
            ge.replay()
            ys_host.copy_(y_dev, non_blocking=True)

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize()
        n_e = max(10, args.steps // 2)
        a.record()
        for _ in range(n_e):
            e2e_step()
        b.record()
        b.synchronize()
        e2e_ms = a.elapsed_time(b) / n_e
        out["e2e"] = {"gbs": round(nbytes / (e2e_ms * 1e-3) / 1e9, 1), "h2d_bytes_per_step": int(xs_host.numel() * 2),
                      "d2h_bytes_per_step": int(ys_host.numel() * 4)}
        del ge
    del g, calls
    torch.cuda.empty_cache()
    return out


HEAD_CTX = 4096


def run_b200(args, rank: int, world: int) -> dict | None:
    import torch
    from llmnputest_b200 import ops
    from llmnputest_b200.decode import GRANITE_3B

    device = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=device)
    gen.manual_seed(1000 + rank)
    pk = peaks()
    extras = {}

    # ---- N > 1: the tensor-parallel results against one GPU's, before anything is timed
    if world > 1 and not args.quick:
        extras["tp_parity"] = tp_parity(torch, world, rank)

    # ---- the value: config 4's decode step, tensor-parallel over the ranks
    head = measure_headline(torch, world, rank, args.batch, HEAD_CTX, args.steps, args.warmup, pk["hbm_gbs"])

    if not args.quick:
        extras["decode"] = [measure_decode(torch, world, rank, b, HEAD_CTX, max(10, args.steps // 2), 3)
                            for b in (1, 8)]
        if world > 1:
            extras["qwen35_tp"] = measure_qwen35_tp(torch, world, rank, args.steps, args.warmup)
        extras["gemv_sweep"] = gemv_sweep(torch, ops, args, rank, world, gen, device, pk)
        if world == 1:  # the single-GPU kernel lines (configs 1, 3, 5)
            w8 = make_q8_tiles(torch, 7760 * 4, gen, device)
            x8 = torch.randn(1, 1024, device=device, generator=gen).to(torch.bfloat16)
            y8 = torch.empty(1, 248320, device=device)
            gl = graph_of(torch, lambda: ops.q8_gemv(w8, 7760, 4, x8, out=y8))
            tl = time_graph(torch, gl, max(50, args.steps), 5)
            extras["q8_lm_head"] = {"us": round(tl * 1e3, 2), "gbs": round(w8.numel() / (tl * 1e-3) / 1e9, 1),
                                    "frac_of_measured_hbm": round(w8.numel() / (tl * 1e-3) / 1e9 / pk["hbm_gbs"], 3)}
            del gl, w8
            extras["attention"] = measure_attention(torch, ops, gen, device, pk["hbm_gbs"], args.steps)
            extras["tc_gemm"] = measure_tc_gemm(torch, ops, gen, device, pk["bf16_tflops"], args.steps, pk["hbm_gbs"])
            extras["deltanet"] = measure_deltanet(torch, ops, gen, device, pk["hbm_gbs"], args.steps)
            extras["deltanet_layers"] = measure_deltanet_layers(torch, device, pk["hbm_gbs"], args.steps)
            extras["gated_attention"] = measure_gated_attention(torch, ops, gen, device, pk["hbm_gbs"], args.steps)
            extras["qwen35_step"] = measure_qwen35_step(torch, device, pk["hbm_gbs"], args.steps)
    assert ops.device_error() == 0, "a kernel recorded a device-side error"
    if rank != 0:
        return None

    cfg = GRANITE_3B
    split = head["split"]
    dom_name, dom = max(split.items(), key=lambda kv: kv[1]["ms_per_step"])
    step_gbs = head["bytes_per_step"] / world / (head["ms"] * 1e-3) / 1e9
    out = {
        "metric": METRIC,
        "value": round(head["tok_s"], 1),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(head["ms"], 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random-init q4nx/q8 weights with BASELINE distributions, KV cache and inputs ~ N(0,1))",
        "config": {
            "workload": f"config 4: full random-init decode step of the dense GQA 3B ({cfg.n_layers} layers, hidden "
                        f"{cfg.hidden}, {cfg.n_heads}/{cfg.n_kv_heads} heads, intermediate {cfg.intermediate}, vocab "
                        f"{cfg.vocab}; q4nx projections, q8 lm_head), batch {args.batch}, context {HEAD_CTX}, one CUDA "
                        "graph per step",
            "batch": args.batch, "ctx": HEAD_CTX, "layers": cfg.n_layers,
            "bytes_per_step": head["bytes_per_step"],
            "l2": f"inputs larger than L2 ({head['bytes_per_step'] / 1e9:.1f} GB of weights and KV cache per step)",
            "parallelism": "1 GPU" if world == 1 else
                           f"tp{world}: kv heads, O input columns, FFN rows / down K-tiles, vocab rows; all-reduces "
                           "summed over NVLink in the next GEMM's x pre-pass",
        },
        "gpu_launches": head["kernels_per_step"] * args.steps if head["kernels_per_step"] else None,
        "e2e": {"value": round(head["e2e_tok_s"], 1), "unit": "tok/s", "h2d_bytes_per_step": int(head["h2d"]),
                "d2h_bytes_per_step": int(head["d2h"])},
        "roofline": {"bound": "hbm", "achieved": dom["gbs"], "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": dom["frac_of_measured_hbm"],
                     "traffic": (int(dom["bytes_per_launch"] * DRAM_RATIO[dom_name]) if dom_name in DRAM_RATIO
                                 else None),
                     "kernel": dom_name,
                     "bytes_per_launch": dom["bytes_per_launch"], "us_per_launch": dom["us_per_launch"],
                     "peak_src": pk["src"],
                     "step": {"gbs_per_gpu": round(step_gbs, 1), "frac": round(step_gbs / pk["hbm_gbs"], 4)}},
        "kernel_split": split,
        "clocks": head["clocks"],
    }
    if world == 1 and not args.no_cpu_baseline:
        gemv = run_reference_gemv(iters=20)
        cb = cpu_decode_step(args.batch, HEAD_CTX, gemv)
        out["cpu_baseline"] = {"value": cb["tok_s"], "unit": "tok/s", "cores": cb["cores"], "kind": cb["kind"],
                               "sample": cb["sample"], "parts_ms": cb["parts_ms"]}
        if not args.quick:
            extras["cpu_baselines"] = {
                "config1_lm_head": cpu_lm_head(),
                "config2_gemv": {"gbs": round(gemv["gbs"], 2), "cores": gemv["cores"], "kind": gemv["kind"],
                                 "sample": gemv["sample"]},
                "config3_attention": [cpu_attention(b, c) for b, c in ((1, 4096), (1, 32768), (16, 4096))],
                "config4_step_b1": cpu_decode_step(1, HEAD_CTX, gemv),
            }
    out.update(extras)
    return out


def run_reference(args, rank: int) -> dict | None:
    """The reference arm: config 4's decode step composed from the reference's own CPU parts
    (bench.cpu_decode_step: its compiled cpu_baseline.cpp GEMV for the projections, its
    attention oracle, its --cpu torch lm_head) on all of this host's cores, at the batch and
    context of the B200 arm.  Rank 0 alone runs; the other ranks exit without work."""
    if rank != 0:
        return None
    t0 = time.time()
    gemv = run_reference_gemv(iters=max(5, args.steps // 2), layers=4)
    cb = cpu_decode_step(args.batch, HEAD_CTX, gemv)
    sec = time.time() - t0
    return {
        "impl": "reference", "metric": METRIC, "value": cb["tok_s"], "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp32 projections and attention, bf16 lm_head (the reference's CPU paths)",
        "data": "synthetic",
        "config": {"workload": f"config 4: decode step of the dense GQA 3B, batch {args.batch}, context {HEAD_CTX} "
                               "(reference CPU parts, one layer timed x 40 + lm_head)",
                   "batch": args.batch, "ctx": HEAD_CTX},
        "cpu_baseline": {"value": cb["tok_s"], "unit": "tok/s", "cores": cb["cores"], "kind": cb["kind"],
                         "sample": cb["sample"]},
        "e2e": {"value": cb["tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "parts_ms": cb["parts_ms"], "wall_s": round(sec, 1),
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--batch", type=int, default=32, help="decode batch of the headline step")
    ap.add_argument("--layers", type=int, default=LAYERS, help="layers of the GEMV sweep")
    ap.add_argument("--quick", action="store_true", help="the headline step only")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-case", choices=PROFILE_CASES,
                    help="run one small workload for an ncu capture and exit (no timing, no JSON line)")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.profile_case:
        import torch
        torch.cuda.set_device(local)
        profile_case(torch, args.profile_case)
        return 0
    if args.impl == "reference":
        res = run_reference(args, rank)
    else:
        import torch
        torch.cuda.set_device(local)
        if world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                    device_id=torch.device("cuda", local))
        res = run_b200(args, rank, world)
        if world > 1:
            import torch.distributed as dist
            torch.cuda.synchronize()
            dist.barrier()
            dist.destroy_process_group()
    if res is not None:
        print(json.dumps(res), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
